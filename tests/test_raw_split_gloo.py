"""CPU, world size 2 and 3 (gloo): the protocol of the raw-row sequence
split (zkv_page_decode_raw_split) restated over the oracle, against the
single-device oracle page decode over raw rows.

Each rank scores only the pages the library's split rule gives it
(zkv_raw_split_range, a host function), writing -inf for its invalid pages
(the kernel applies validity there, not in the select); the score rows are
all-gathered; every rank takes the top nk of the whole row; the own pages
are the selection positions whose ids fall in the rank's range; each rank
attends those pages (rank 0 also the sink and near rows) into an
unnormalised partial (M, L, O); the partials are all-gathered and combined
in rank order.  The selection must equal the single-device selection
exactly (so validity as -inf keys picks the same pages, ties included), the
output must be within the attention tolerance and the same on every rank."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O

G, D = 4, 128
SCALE = 1 / np.sqrt(D)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def make_raw(seed, R, n_c, n_sink, n_near, invalid_every):
    """A raw layer: keys with 4 outlier channels x10, values, q (bf16); the
    Quest min / max of the retrieval pages; every `invalid_every`-th page of
    odd rows invalid; row 0's retrieval keys all equal (every page ties)."""
    rng = np.random.default_rng(seed)
    T = 16 * n_c
    cap = n_sink + T + n_near
    k = rng.standard_normal((R, cap, D)).astype(np.float32)
    k[:, :, rng.choice(D, 4, replace=False)] *= 10
    k[0, n_sink:n_sink + T] = k[0, n_sink]
    v = rng.standard_normal((R, cap, D)).astype(np.float32)
    q = rng.standard_normal((R, G, D)).astype(np.float32)
    kb, vb, qb = O.f32_to_bf16(k), O.f32_to_bf16(v), O.f32_to_bf16(q)
    mn, mx, _, _ = O.kivi_encode_chunks(np.ascontiguousarray(kb[:, n_sink:n_sink + T]))
    valid = np.ones((R, n_c), np.uint8)
    if invalid_every:
        valid[1::2, ::invalid_every] = 0
    return dict(k=kb, v=vb, q=qb, mn=mn, mx=mx, valid=valid, n_sink=n_sink, n_near=n_near,
                near_start=n_sink + T)


def gqa_mean(qb):
    """bf16(fp32 sum of the G heads in head order / G), as the score kernel."""
    qf = O.bf16_to_f32(qb)
    acc = np.zeros((qf.shape[0], D), np.float32)
    for g in range(qf.shape[1]):
        acc = (acc + qf[:, g]).astype(np.float32)
    return O.f32_to_bf16(acc / np.float32(qf.shape[1]))


def _rank_main(rank, world, port, case, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from zoomkv_revision_b200 import ops
        R, n_c, nk, n_sink, n_near, inv, seed = case
        d = make_raw(seed, R, n_c, n_sink, n_near, inv)
        lo, hi = ops.raw_split_range(n_c, world, rank)
        # 1. own scores (invalid -> -inf) into the whole row
        own = O.quest_score(gqa_mean(d["q"]), np.ascontiguousarray(d["mn"][:, lo:hi]),
                            np.ascontiguousarray(d["mx"][:, lo:hi]), np.ascontiguousarray(d["valid"][:, lo:hi]),
                            hi - lo)
        spans = [ops.raw_split_range(n_c, world, r) for r in range(world)]
        width = max(b - a for a, b in spans)
        mine = torch.full((R, width), float("nan"))
        mine[:, :hi - lo] = torch.from_numpy(own)
        rows = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(rows, mine)
        row = np.concatenate([rows[r][:, :b - a].numpy() for r, (a, b) in enumerate(spans)], axis=1)
        # 2. the top nk of the whole row; the own pages are a run of it
        sel = O.topk_f32(row, nk)
        part = np.zeros((R, G, D + 2), np.float64)
        qf = O.bf16_to_f32(d["q"])
        kf, vf = O.bf16_to_f32(d["k"]), O.bf16_to_f32(d["v"])
        for r in range(R):
            pos = [p for p in range(nk) if lo <= sel[r, p] < hi]
            assert not pos or pos == list(range(pos[0], pos[-1] + 1)), "own pages are not one run"
            toks = [d["n_sink"] + 16 * int(sel[r, p]) + t for p in pos for t in range(16)]
            if rank == 0:
                toks = list(range(d["n_sink"])) + toks + list(range(d["near_start"], d["near_start"] + n_near))
            if not toks:
                part[r, :, D] = -np.inf
                continue
            s = (qf[r].astype(np.float64) @ kf[r, toks].T.astype(np.float64)) * SCALE   # [G, n]
            m = s.max(axis=1)
            p = np.exp(s - m[:, None])
            part[r, :, :D] = p @ vf[r, toks].astype(np.float64)
            part[r, :, D] = m
            part[r, :, D + 1] = p.sum(axis=1)
        # 3. every rank's partial, combined in rank order
        parts = [torch.empty(R, G, D + 2, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(part))
        P = np.stack([x.numpy() for x in parts])               # [world, R, G, D + 2]
        M = P[..., D].max(axis=0)
        w = np.where(np.isfinite(P[..., D]), np.exp(P[..., D] - M), 0.0)
        Ls = (w * P[..., D + 1]).sum(axis=0)
        out = (w[..., None] * P[..., :D]).sum(axis=0) / Ls[..., None]
        lse = M + np.log(Ls)
        np.savez(os.path.join(result_dir, f"r{rank}.npz"), out=out, lse=lse, sel=sel)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,case", [
    (2, (4, 37, 9, 5, 24, 3, 0)),      # ragged ownership (rank 1 holds 5 pages), sink, invalid pages, ties
    (2, (2, 80, 80 - 1, 0, 16, 0, 1)), # all but one page selected
    (3, (3, 61, 20, 16, 0, 2, 2)),     # three ranks, no near rows
])
def test_raw_split_protocol_matches_single_device(tmp_path, world, case):
    mp.start_processes(_rank_main, args=(world, _free_port(), case, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    R, n_c, nk, n_sink, n_near, inv, seed = case
    d = make_raw(seed, R, n_c, n_sink, n_near, inv)
    ro, rl, rsel = O.page_decode_raw(d["q"], d["mn"], d["mx"], d["valid"], d["k"], d["v"], n_c, nk,
                                     page_base=n_sink, n_sink=n_sink, near_start=d["near_start"], n_near=n_near,
                                     scale=SCALE)
    res = [np.load(os.path.join(tmp_path, f"r{r}.npz")) for r in range(world)]
    for r in res:
        assert np.array_equal(r["sel"], rsel), "the split selection differs from the single-device one"
        assert np.array_equal(r["out"], res[0]["out"])
    ref = O.bf16_to_f32(ro).astype(np.float64)
    err = np.abs(res[0]["out"] - ref)
    assert err.max() <= 2e-2 and err.mean() / np.abs(ref).mean() <= 1e-2, (err.max(), err.mean())
    assert np.abs(res[0]["lse"] - rl).max() < 1e-3


@pytest.mark.parametrize("n_c,world", [(8184, 1), (8184, 2), (8184, 8), (2040, 4), (37, 2), (100, 7), (17, 2)])
def test_split_range_rule(n_c, world):
    """Ranks hold contiguous ascending ranges covering every page once, each
    starting on a multiple of 16 pages (16-page aligned score slices)."""
    from zoomkv_revision_b200 import ops
    spans = [ops.raw_split_range(n_c, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] <= n_c
    assert sum(b - a for a, b in spans) == n_c
    for (a, b), (c, _) in zip(spans, spans[1:]):
        assert b == c
    for a, _ in spans:
        assert a % 16 == 0


def test_split_buffer_and_workspace_sizes():
    """Host-side sizes: the exchange buffer holds the epochs, the tagged score
    row (8 bytes per page, rows padded to 32 pages) and world tagged partials
    per (row, head); bad shapes give 0."""
    from zoomkv_revision_b200 import _lib
    L = _lib.lib()
    R, G, n_c, world = 8, 4, 8184, 2
    n = int(L.zkv_raw_split_buffer_bytes(R, G, n_c, world))
    assert n % 256 == 0 and n >= R * 8192 * 8 + world * R * G * 130 * 8
    assert L.zkv_raw_split_buffer_bytes(R, G, n_c, 9) == 0
    assert L.zkv_raw_split_buffer_bytes(-1, G, n_c, 2) == 0
    ws0 = int(L.zkv_page_decode_raw_split_ws_bytes(R, n_c, world, 0, 256, 0, 128))
    ws1 = int(L.zkv_page_decode_raw_split_ws_bytes(R, n_c, world, 1, 256, 0, 128))
    assert ws0 >= ws1 > R * 8192 * 4 and ws0 % 256 == 0
    assert L.zkv_page_decode_raw_split_ws_bytes(R, n_c, world, 2, 256, 0, 128) == 0
    # argument checks run before any launch
    assert L.zkv_page_decode_raw_split(None, None, None, R, G, 1, n_c, 256, 0, 0, 0, 1.0, None, None, None,
                                       None, None, 0, None) == 1  # ZKV_ERR_ARG


def test_split_rejects_undersized_exchange_buffers():
    """The call checks the declared size of the exchange buffers against its
    shape before any device work: a group built for fewer rows (or a shorter
    row) gets ZKV_ERR_CAPACITY (3) instead of stores past a peer's buffer.
    The pointers are never dereferenced by these host-side checks."""
    import ctypes
    from zoomkv_revision_b200 import _lib
    L = _lib.lib()
    R, G, n_c, nk, world = 8, 4, 8184, 256, 2
    need = int(L.zkv_raw_split_buffer_bytes(R, G, n_c, world))
    fake = 1 << 20                                   # 256-byte aligned, never dereferenced here
    bases = (ctypes.c_void_p * world)(fake, fake + (1 << 24))
    lo, hi = ctypes.c_int(), ctypes.c_int()
    assert L.zkv_raw_split_range(n_c, world, 0, ctypes.byref(lo), ctypes.byref(hi)) == 0
    lay = _lib.ZkvRawLayer(fake, fake, None, fake, fake, 128 * (16 * hi.value + 128), 0)
    ws = int(L.zkv_page_decode_raw_split_ws_bytes(R, n_c, world, 0, nk, 0, 128))

    def call(nbytes):
        sp = _lib.ZkvRawSplit(ctypes.cast(bases, ctypes.POINTER(ctypes.c_void_p)), nbytes, 0, world)
        return L.zkv_page_decode_raw_split(fake, ctypes.byref(lay), ctypes.byref(sp), R, G, hi.value, n_c, nk, 0,
                                           16 * hi.value, 128, 1.0, fake, None, None, None, fake, ws, None)

    assert call(need - 256) == 3   # ZKV_ERR_CAPACITY
    assert call(int(L.zkv_raw_split_buffer_bytes(R // 2, G, n_c, world))) == 3
