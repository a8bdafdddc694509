"""GPU: the sequence split of the raw-row page decode
(zkv_page_decode_raw_split, seqsplit.RawSplitGroup).

World size 1 on one GPU runs the four split kernels with the exchanges
looped back into the own buffer: the selection must equal the oracle's bit
for bit and the output must be within the north-star bar of the oracle's
fp64 softmax over the same raw rows, eager and replayed in a CUDA graph.
Two ranks on two GPUs (skipped with fewer) check the real exchange over
NVLink at the config-3 shape.  A rank that never arrives is made on the
host side: a world-2 call whose second rank is never launched gives up its
bounded waits and reports ZKV_ERR_TIMEOUT, with the context still usable.
No test here runs launches of two ranks on one GPU."""
import ctypes
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle as O
from conftest import to_u16
from test_gpu_raw import close, oracle_raw
from zoomkv_revision_b200 import _lib, ops
from zoomkv_revision_b200 import seqsplit as S
from zoomkv_revision_b200 import workload as W

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _split_call(grp, rc, q, nk, **kw):
    lay, near_start = S.local_raw_layer(rc, grp.lo, grp.hi, grp.rank)
    return grp.decode(q, lay, nk, rc.n_near, n_sink=rc.n_sink, near_start=near_start, **kw)


@pytest.mark.parametrize("bs,H,G,n_c,nk,n_sink,n_near", [
    (2, 2, 4, 300, 24, 0, 37),     # ragged near window
    (2, 2, 4, 130, 16, 64, 128),   # sink 64
    (1, 2, 8, 3000, 200, 16, 40),  # G = 8
    (1, 2, 1, 500, 31, 3, 17),     # G = 1, odd sizes
    (1, 8, 4, 8184, 256, 0, 128),  # the config-3 shape
    (1, 1, 2, 8193, 256, 0, 16),   # the radix select path
])
def test_world1_matches_oracle(bs, H, G, n_c, nk, n_sink, n_near):
    rc = W.build_raw_cache(21 + n_c, bs, H, 16 * n_c, n_near, DEV, n_sink=n_sink)
    q = W.synth_query(torch.Generator(device=DEV).manual_seed(9 + nk), bs, H * G, DEV)
    R = bs * H
    grp = S.RawSplitGroup(R, G, n_c, 1, 0, DEV)
    try:
        sel = torch.full((R, nk), -7, dtype=torch.int64, device=DEV)
        lse = torch.empty(R, G, device=DEV)
        out = _split_call(grp, rc, q, nk, sel_out=sel, lse=lse)
        torch.cuda.synchronize()
        grp.check()
        ro, rl, rsel = oracle_raw(rc, q, nk)
        assert np.array_equal(sel.cpu().numpy(), rsel), "selected pages differ from the oracle"
        close(O.bf16_to_f32(to_u16(out)).reshape(R, G, 128), O.bf16_to_f32(ro))
        assert np.abs(lse.cpu().numpy() - rl).max() < 1e-3
    finally:
        grp.close()


def test_world1_invalid_pages_and_ties():
    """Validity is applied in the split's score kernel (-inf scores): an
    invalid page never beats a valid one and equal keys tie to the lowest
    page ids, exactly as the oracle's select."""
    bs, H, G, n_c, nk = 1, 2, 4, 200, 20
    rc = W.build_raw_cache(3, bs, H, 16 * n_c, 8, DEV)
    rc.keys[0, 0, :16 * n_c] = rc.keys[0, 0, :1]
    cmin, cmax = torch.zeros_like(rc.chunk_min), torch.zeros_like(rc.chunk_max)
    valid = torch.zeros_like(rc.valid)
    packed = torch.empty(bs, H, n_c, 16, 16, dtype=torch.int32, device=DEV)
    ops.kivi_encode_chunks(rc.keys[:, :, :16 * n_c], cmin, cmax, None, valid, packed, 0)
    valid[0, 1, ::3] = False
    rc = W.RawCache(cmin, cmax, valid, rc.keys, rc.values, 0, n_c, 16 * n_c, 8)
    q = W.synth_query(torch.Generator(device=DEV).manual_seed(2), bs, H * G, DEV)
    grp = S.RawSplitGroup(bs * H, G, n_c, 1, 0, DEV)
    try:
        sel = torch.empty(bs * H, nk, dtype=torch.int64, device=DEV)
        out = _split_call(grp, rc, q, nk, sel_out=sel)
        torch.cuda.synchronize()
        grp.check()
        ro, _, rsel = oracle_raw(rc, q, nk)
        s = sel.cpu().numpy()
        assert np.array_equal(s, rsel)
        assert np.array_equal(s[0], np.arange(nk))
        assert not np.any(s[1] % 3 == 0)
        close(O.bf16_to_f32(to_u16(out)).reshape(bs * H, G, 128), O.bf16_to_f32(ro))
    finally:
        grp.close()


def test_world1_repeated_calls_and_graph_replay():
    """The device epochs advance once per call: many eager calls over two
    layers, then the same calls captured in a CUDA graph and replayed, give
    bit-identical outputs every time."""
    bs, H, G, n_c, nk, n_near = 1, 8, 4, 2047, 128, 128
    rcs = [W.build_raw_cache(40 + i, bs, H, 16 * n_c, n_near, DEV) for i in range(2)]
    qs = [W.synth_query(torch.Generator(device=DEV).manual_seed(50 + i), bs, H * G, DEV) for i in range(2)]
    grp = S.RawSplitGroup(bs * H, G, n_c, 1, 0, DEV)
    try:
        lays = [S.local_raw_layer(rc, grp.lo, grp.hi, 0) for rc in rcs]
        outs = [torch.empty(bs, 1, H * G, 128, dtype=torch.bfloat16, device=DEV) for _ in rcs]

        def loop():
            for (lay, ns), q, o in zip(lays, qs, outs):
                grp.decode(q, lay, nk, n_near, near_start=ns, out=o)

        first = []
        for it in range(5):
            loop()
            torch.cuda.synchronize()
            if it == 0:
                first = [o.clone() for o in outs]
            for o, f in zip(outs, first):
                assert torch.equal(o, f)
        stream = torch.cuda.Stream()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            loop()
        for _ in range(4):
            for o in outs:
                o.zero_()
            graph.replay()
            torch.cuda.synchronize()
            for o, f in zip(outs, first):
                assert torch.equal(o, f)
        grp.check()
        del graph
        for rc, q, f in zip(rcs, qs, first):
            ref = ops.page_decode_raw(q, rc.layer(), n_c, nk, n_near, near_start=rc.near_start)
            err = (f.float() - ref.float()).abs()
            assert err.max().item() <= 2e-2
    finally:
        grp.close()


def test_split_wait_expires_on_a_missing_rank():
    """Failure detection without a GPU fault: world 2 is declared but only
    rank 0 runs (both buffer slots are rank 0's own buffer, so nothing ever
    writes rank 1's words).  The select and merge waits give up after the
    limit, ZKV_ERR_TIMEOUT lands in the status word, the call returns and
    the context stays usable."""
    L = _lib.lib()
    bs, H, G, n_c, nk, n_near = 1, 2, 4, 96, 8, 16
    rc = W.build_raw_cache(5, bs, H, 16 * n_c, n_near, DEV)
    q = W.synth_query(torch.Generator(device=DEV).manual_seed(6), bs, H * G, DEV)
    R = bs * H
    nbytes = int(L.zkv_raw_split_buffer_bytes(R, G, n_c, 2))
    base, _, _ = S._share_buffer(nbytes, 1, 0)
    bases = (ctypes.c_void_p * 2)(base, base)

    class Split:
        rank, world = 0, 2
        struct = _lib.ZkvRawSplit(ctypes.cast(bases, ctypes.POINTER(ctypes.c_void_p)), nbytes, 0, 2)

    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    S.set_peer_wait_ms(300)
    try:
        lo, hi = ops.raw_split_range(n_c, 2, 0)
        lay, ns = S.local_raw_layer(rc, lo, hi, 0)
        t0 = time.perf_counter()
        ops.page_decode_raw_split(q, lay, Split, n_c, nk, n_near, near_start=ns, status=status)
        torch.cuda.synchronize()
        waited = time.perf_counter() - t0
        assert int(status.item()) == _lib.ZKV_ERR_TIMEOUT
        assert 0.25 < waited < 30.0, f"waited {waited:.3f} s; each wait's limit was 0.3 s on the GPU timer"
        x = torch.arange(16, device=DEV, dtype=torch.float32)
        assert float(x.sum().item()) == 120.0
    finally:
        S.set_peer_wait_ms(5000)
        torch.cuda.synchronize()
        L.zkv_peer_free(ctypes.c_void_p(base))


def _rank_main(rank, world, port, path):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    # gloo carries only the IPC handles and barriers; the data path is P2P
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    grp = None
    try:
        bs, H, G, n_c, nk, n_near = 1, 8, 4, 8184, 256, 128
        rcs = [W.build_raw_cache(70 + i, bs, H, 16 * n_c, n_near, dev, n_sink=16 * i) for i in range(2)]
        qs = [W.synth_query(torch.Generator(device=dev).manual_seed(80 + i), bs, H * G, dev) for i in range(2)]
        grp = S.RawSplitGroup(bs * H, G, n_c, world, rank, dev)
        lays = [S.local_raw_layer(rc, grp.lo, grp.hi, rank) for rc in rcs]
        res = {}
        outs = [torch.empty(bs, 1, H * G, 128, dtype=torch.bfloat16, device=dev) for _ in rcs]
        sels = [torch.empty(bs * H, nk, dtype=torch.int64, device=dev) for _ in rcs]

        def loop():
            for (lay, ns), rc, q, o, s in zip(lays, rcs, qs, outs, sels):
                grp.decode(q, lay, nk, n_near, n_sink=rc.n_sink, near_start=ns, out=o, sel_out=s)

        for _ in range(3):
            loop()
        torch.cuda.synchronize()
        for i, rc in enumerate(rcs):
            ref_sel = torch.empty(bs * H, nk, dtype=torch.int64, device=dev)
            ref = ops.page_decode_raw(qs[i], rc.layer(), n_c, nk, n_near, n_sink=rc.n_sink,
                                      near_start=rc.near_start, sel_out=ref_sel)
            torch.cuda.synchronize()
            res[f"out{i}"], res[f"ref{i}"] = outs[i].float().cpu().numpy(), ref.float().cpu().numpy()
            res[f"sel{i}"], res[f"ref_sel{i}"] = sels[i].cpu().numpy(), ref_sel.cpu().numpy()
        stream = torch.cuda.Stream(device=dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            loop()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        for i in range(len(rcs)):
            res[f"graph{i}"] = outs[i].float().cpu().numpy()
        res["status"] = np.array([int(grp.status.item())])
        del graph
        np.savez(os.path.join(path, f"s{rank}.npz"), **res)
    finally:
        if grp is not None:
            grp.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_world2_config3_shape(tmp_path):
    """Two ranks, one per GPU, at the config-3 shape (131072 context, budget
    4096): the selection equals the single-GPU selection exactly on both
    ranks, both ranks hold the same output, within the north-star bar of the
    single-GPU decode, eager and replayed as a CUDA graph."""
    mp.start_processes(_rank_main, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn", join=True)
    res = [np.load(os.path.join(tmp_path, f"s{r}.npz")) for r in range(2)]
    for r in res:
        assert int(r["status"][0]) == 0
        for i in range(2):
            assert np.array_equal(r[f"sel{i}"], r[f"ref_sel{i}"])
            assert np.array_equal(r[f"out{i}"], res[0][f"out{i}"])
            assert np.array_equal(r[f"graph{i}"], r[f"out{i}"])
            err = np.abs(r[f"out{i}"] - r[f"ref{i}"])
            assert err.max() <= 2e-2 and err.mean() / np.abs(r[f"ref{i}"]).mean() <= 1e-2
