"""GPU: sequence-split page decode (zoomkv_revision_b200.seqsplit) against
the single-device fused page decode: same selected pages (exact), output
within the attention tolerance (bit-identical at world size 1).  Ranks are
emulated on one GPU; a real NCCL run needs >= 2 GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from zoomkv_revision_b200 import ops
from zoomkv_revision_b200 import seqsplit as S
from zoomkv_revision_b200 import workload as W

pytestmark = pytest.mark.gpu
G = 4


def _setup(seed, bs, H, n_c, n_near, dev):
    pc, _ = W.build_page_cache(seed, bs, H, n_c * 16, n_near, dev)
    q = W.synth_query(torch.Generator(device=dev).manual_seed(seed + 7), bs, H * G, dev)
    return pc, q


def _close(out, ref):
    o, r = out.float(), ref.float()
    err = (o - r).abs()
    assert err.max() <= 2e-2 and err.mean() / r.abs().mean() <= 1e-2, (float(err.max()), float(err.mean()))


def test_world1_bit_identical_to_page_decode():
    dev = torch.device("cuda", 0)
    bs, H, n_c, nk, n_near = 2, 4, 700, 96, 64
    pc, q = _setup(1, bs, H, n_c, n_near, dev)
    sel = torch.empty(bs * H, nk, dtype=torch.int64, device=dev)
    ref = ops.page_decode(q, pc.layer(), n_c, nk, n_near, sel_out=sel)
    bufs = S.SplitBuffers.alloc(bs, H, G, n_c, nk, 1, dev)
    out, s = S.decode_step(q, pc.layer(), n_c, nk, bufs, rank=0, world=1, n_near=n_near)
    torch.cuda.synchronize()
    assert torch.equal(s.view(bs * H, nk), sel)
    assert torch.equal(out, ref)
    assert int(bufs.status.item()) == 0


@pytest.mark.parametrize("world,bs,H,n_c,nk,n_near", [(2, 1, 8, 1001, 64, 128), (3, 2, 2, 500, 120, 16),
                                                      (4, 1, 8, 8184, 256, 128), (8, 1, 8, 8184, 256, 128)])
def test_emulated_ranks_match_page_decode(world, bs, H, n_c, nk, n_near):
    """Each emulated rank scores only its own pages and attends only the
    selected pages it owns; the merge of the partials equals the fused
    single-device decode (config-3 shape: 131072 context, budget 4096)."""
    dev = torch.device("cuda", 0)
    pc, q = _setup(world * 10 + nk, bs, H, n_c, n_near, dev)
    sel_ref = torch.empty(bs * H, nk, dtype=torch.int64, device=dev)
    ref = ops.page_decode(q, pc.layer(), n_c, nk, n_near, sel_out=sel_ref)
    be = S.CudaBackend()
    per = S.split_range(n_c, world, 0)[2]
    raw_q = be.raw_q(q, H)
    rows = []
    layers = []
    for r in range(world):
        lo, hi, _ = S.split_range(n_c, world, r)
        lay = S.local_layer(pc.layer(), lo, hi)
        layers.append((lo, hi, lay))
        sc = torch.full((bs, H, per), -float("inf"), device=dev)
        be.local_scores(raw_q, lay, hi - lo, torch.empty(bs * H * per, device=dev), sc)
        rows.append(sc)
    row = torch.cat(rows, dim=2)
    sel = be.global_topk(row, nk, torch.empty(bs, H, nk, dtype=torch.int64, device=dev))
    parts = torch.empty(world, bs * H * G, 128, device=dev)
    lses = torch.empty(world, bs * H * G, device=dev)
    for r, (lo, hi, lay) in enumerate(layers):
        part = torch.empty(bs, H * G, 128, device=dev)
        lse = torch.empty(bs, H * G, device=dev)
        be.attend(q, lay, sel, lo, hi, 0, 0, n_near if r == 0 else 0, part, lse, None)
        parts[r] = part.view(-1, 128)
        lses[r] = lse.view(-1)
    out = torch.empty(bs, 1, H * G, 128, dtype=torch.bfloat16, device=dev)
    be.merge(parts, lses, out.view(-1, 128))
    torch.cuda.synchronize()
    assert torch.equal(sel.view(bs * H, nk), sel_ref)
    _close(out, ref)


@pytest.mark.parametrize("world,n_c,nk,parts", [(2, 1001, 64, 1), (2, 8184, 256, 4), (4, 8184, 256, 2),
                                                 (8, 8184, 256, 4)])
def test_scored_select_attend_own_ranges(world, n_c, nk, parts):
    """zkv_page_decode_scored, as each rank of a sequence split runs it (ranks
    emulated one after another; nothing waits): the top nk of the whole
    score row, attention over the own selected pages only, partials of every
    rank and cluster merged -> the single-device selection exactly and its
    output within tolerance."""
    dev = torch.device("cuda", 0)
    bs, H, n_near = 1, 8, 128
    pc, q = _setup(world * 100 + n_c, bs, H, n_c, n_near, dev)
    sel_ref = torch.empty(bs * H, nk, dtype=torch.int64, device=dev)
    ref = ops.page_decode(q, pc.layer(), n_c, nk, n_near, sel_out=sel_ref)
    per = S.split_range(n_c, world, 0)[2]
    row = torch.full((bs, H, world * per), -float("inf"), device=dev)
    local = torch.empty(bs * H * n_c, device=dev)
    lay = pc.layer()
    ops.quest_chunk_score_gqa(q, lay.tensors[0], lay.tensors[1], local, n_c, lay.tensors[2])
    row[:, :, :n_c] = local.view(bs, H, n_c)
    rows = bs * H
    parts_all = torch.empty(world * parts, rows * G, 128, device=dev)
    lses_all = torch.empty(world * parts, rows * G, device=dev)
    for r in range(world):
        lo, hi, _ = S.split_range(n_c, world, r)
        sel = torch.empty(bs, H, nk, dtype=torch.int64, device=dev)
        ops.page_decode_scored(q, S.local_layer(lay, lo, hi), row, world * per, nk, lo, hi, parts,
                               parts_all[r * parts:(r + 1) * parts], lses_all[r * parts:(r + 1) * parts],
                               n_near=n_near if r == 0 else 0, sel_out=sel)
        torch.cuda.synchronize()
        assert torch.equal(sel.view(rows, nk), sel_ref)
    out = torch.empty(bs, 1, H * G, 128, dtype=torch.bfloat16, device=dev)
    ops.lse_merge_n(parts_all, lses_all, out.view(-1, 128))
    torch.cuda.synchronize()
    _close(out, ref)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank, world, port, path):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        bs, H, n_c, nk, n_near = 1, 8, 2047, 128, 128
        pc, q = _setup(3, bs, H, n_c, n_near, dev)
        lo, hi, per = S.split_range(n_c, world, rank)
        bufs = S.SplitBuffers.alloc(bs, H, G, per, nk, world, dev)
        out, sel = S.decode_step(q, S.local_layer(pc.layer(), lo, hi), n_c, nk, bufs, rank=rank, world=world,
                                 n_near=n_near)
        ref_sel = torch.empty(bs * H, nk, dtype=torch.int64, device=dev)
        ref = ops.page_decode(q, pc.layer(), n_c, nk, n_near, sel_out=ref_sel)
        torch.cuda.synchronize()
        np.savez(os.path.join(path, f"r{rank}.npz"), out=out.float().cpu().numpy(), ref=ref.float().cpu().numpy(),
                 sel=sel.cpu().numpy(), ref_sel=ref_sel.cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_nccl_world2(tmp_path):
    env = {"NCCL_NVLS_ENABLE": "0"}
    os.environ.update(env)
    mp.start_processes(_nccl_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn", join=True)
    res = [np.load(os.path.join(tmp_path, f"r{r}.npz")) for r in range(2)]
    for r in res:
        assert np.array_equal(r["sel"].reshape(r["ref_sel"].shape), r["ref_sel"])
        assert np.array_equal(r["out"], res[0]["out"])
        _close(torch.from_numpy(r["out"]), torch.from_numpy(r["ref"]))


def test_p2p_world1_matches_nccl_form_and_replays_in_a_graph():
    """The peer-memory transport at world size 1 (put into the own buffer,
    wait on the own flag): the same selection as the collective form, the
    output within tolerance of the fused single-device decode (the select +
    attend kernel spreads a row over several clusters, merged by LSE), and
    correct across repeated steps and CUDA-graph replays (device-resident
    epochs)."""
    dev = torch.device("cuda", 0)
    bs, H, n_c, nk, n_near = 1, 8, 1500, 128, 64
    pcs = [_setup(40 + i, bs, H, n_c, n_near, dev) for i in range(3)]
    pg = S.PeerGroup(bs, H, G, n_c, nk, 1, 0, dev)
    try:
        refs = []
        for pc, q in pcs:
            bufs = S.SplitBuffers.alloc(bs, H, G, n_c, nk, 1, dev)
            _, s = S.decode_step(q, pc.layer(), n_c, nk, bufs, rank=0, world=1, n_near=n_near)
            ref = ops.page_decode(q, pc.layer(), n_c, nk, n_near)
            refs.append((ref, s.clone()))
        first = []
        for it in range(2):  # eager, twice (epochs advance)
            for i, ((pc, q), (ref, rs)) in enumerate(zip(pcs, refs)):
                o, s = S.decode_step_p2p(q, pc.layer(), pg, n_near=n_near)
                torch.cuda.synchronize()
                assert torch.equal(s, rs)
                _close(o, ref)
                if it == 0:
                    first.append(o.clone())
                else:
                    assert torch.equal(o, first[i])
        stream = torch.cuda.Stream(device=dev)
        outs = [torch.empty_like(first[0]) for _ in pcs]

        def loop():
            for i, (pc, q) in enumerate(pcs):
                o, _ = S.decode_step_p2p(q, pc.layer(), pg, n_near=n_near)
                outs[i].copy_(o)

        with torch.cuda.stream(stream):
            loop()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            loop()
        for _ in range(3):
            graph.replay()
            torch.cuda.synchronize()
            for o, f in zip(outs, first):
                assert torch.equal(o, f)
        del graph
        assert int(pg.status.item()) == 0
    finally:
        pg.close()


def test_peer_wait_expires_on_a_missing_rank():
    """Failure detection without a GPU fault: a wait for a rank that never
    puts (world 2 declared, one process, nothing sets rank 1's flag) gives up
    after its bounded poll, reports ZKV_ERR_TIMEOUT in the status word and
    returns; the context stays usable and the epoch still advances."""
    import time
    from zoomkv_revision_b200 import _lib
    dev = torch.device("cuda", 0)
    pg = S.PeerGroup(1, 2, G, 64, 8, 1, 0, dev)  # one real buffer; its flag array has room for 8 ranks
    S.set_peer_wait_ms(300)
    try:
        stream = torch.cuda.current_stream(dev).cuda_stream
        L = _lib.lib()
        t0 = time.perf_counter()
        # the own flag of rank 0 is raised by a put; rank 1's never is
        pg._put(pg._seg_scores, 1, 0, stream)
        _lib.check(L.zkv_peer_wait(pg.flags_a, pg.epoch, 2, pg.status.data_ptr(), stream), "zkv_peer_wait")
        torch.cuda.synchronize()
        waited = time.perf_counter() - t0
        assert int(pg.status.item()) == _lib.ZKV_ERR_TIMEOUT
        assert 0.25 < waited < 30.0, f"waited {waited:.3f} s; the limit was 0.3 s on the GPU timer"
        with pytest.raises(RuntimeError, match="rebuilt"):
            pg.check()
        # the context is still usable: a normal world-1 step afterwards succeeds
        pg.status.zero_()
        x = torch.arange(16, device=dev, dtype=torch.float32)
        torch.cuda.synchronize()
        assert float(x.sum().item()) == 120.0
    finally:
        S.set_peer_wait_ms(5000)
        pg.close()


def _p2p_rank(rank, world, port, path):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    # gloo only carries the IPC handles and barriers; the data path is P2P
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    pg = None
    try:
        bs, H, n_c, nk, n_near = 1, 8, 8184, 256, 128
        pcs = [_setup(60 + i, bs, H, n_c, n_near, dev) for i in range(2)]
        pg = S.PeerGroup(bs, H, G, n_c, nk, world, rank, dev)
        lo, hi = pg.lo, pg.hi
        res = {}
        for i, (pc, q) in enumerate(pcs):
            out, sel = S.decode_step_p2p(q, S.local_layer(pc.layer(), lo, hi), pg, n_near=n_near)
            ref_sel = torch.empty(bs * H, nk, dtype=torch.int64, device=dev)
            ref = ops.page_decode(q, pc.layer(), n_c, nk, n_near, sel_out=ref_sel)
            torch.cuda.synchronize()
            res[f"out{i}"], res[f"ref{i}"] = out.float().cpu().numpy(), ref.float().cpu().numpy()
            res[f"sel{i}"], res[f"ref_sel{i}"] = sel.cpu().numpy(), ref_sel.cpu().numpy()
        # the two layers as one CUDA graph, replayed
        stream = torch.cuda.Stream(device=dev)
        outs = [torch.empty(bs, 1, H * G, 128, dtype=torch.bfloat16, device=dev) for _ in pcs]

        def loop():
            for i, (pc, q) in enumerate(pcs):
                o, _ = S.decode_step_p2p(q, S.local_layer(pc.layer(), lo, hi), pg, n_near=n_near)
                outs[i].copy_(o)

        with torch.cuda.stream(stream):
            loop()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            loop()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        for i in range(len(pcs)):
            res[f"graph{i}"] = outs[i].float().cpu().numpy()
        res["status"] = np.array([int(pg.status.item())])
        del graph
        np.savez(os.path.join(path, f"p{rank}.npz"), **res)
    finally:
        if pg is not None:
            pg.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_p2p_world2(tmp_path):
    """Two ranks, one per GPU, exchanging scores and partials through peer
    memory: the selection equals the single-device selection exactly, the
    output is the same on both ranks and within tolerance of the fused
    single-device decode, eager and replayed as a CUDA graph."""
    mp.start_processes(_p2p_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn", join=True)
    res = [np.load(os.path.join(tmp_path, f"p{r}.npz")) for r in range(2)]
    for r in res:
        assert int(r["status"][0]) == 0
        for i in range(2):
            assert np.array_equal(r[f"sel{i}"].reshape(r[f"ref_sel{i}"].shape), r[f"ref_sel{i}"])
            assert np.array_equal(r[f"out{i}"], res[0][f"out{i}"])
            assert np.array_equal(r[f"graph{i}"], r[f"out{i}"])
            _close(torch.from_numpy(r[f"out{i}"]), torch.from_numpy(r[f"ref{i}"]))
