"""GPU parity of the page mode over raw bf16 rows (zkv_page_decode_raw).

The reference's page mode attends the raw K/V rows of the Quest-selected
chunks together with the sink and near rows
(cache_hub/polar_cache_quest_density_single_layer_kivi.py:1589-1775,
:1734-1750).  The selected chunk ids must equal the oracle's bit for bit
(lowest index on ties, ascending order); the output must be within max-abs
2e-2 / mean-rel 1e-2 of an fp64 softmax over the same raw rows."""
import numpy as np
import pytest
import torch

import oracle as O
from conftest import to_u16
from zoomkv_revision_b200 import ops
from zoomkv_revision_b200 import workload as W

pytestmark = pytest.mark.gpu
DEV = "cuda"
ATOL, MEAN_REL = 2e-2, 1e-2   # attention output tolerance (bf16)
SCALE = 1 / np.sqrt(128)


def close(out, ref):
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(out - ref)
    mean_rel = err.mean() / max(np.abs(ref).mean(), 1e-12)
    assert err.max() <= ATOL, f"max abs err {err.max():.3e}"
    assert mean_rel <= MEAN_REL, f"mean rel err {mean_rel:.3e}"
    return err.max(), mean_rel


def run_raw(rc, q, nk, **kw):
    bs, H = rc.keys.shape[:2]
    G = q.shape[2] // H
    R = bs * H
    nsel = nk if rc.n_c > 0 else 0
    sel = torch.full((R, max(nsel, 1)), -7, dtype=torch.int64, device=DEV)
    lse = torch.empty(R, G, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = ops.page_decode_raw(q, rc.layer(), rc.n_c, nk, rc.n_near, n_sink=rc.n_sink, near_start=rc.near_start,
                              lse=lse, sel_out=sel if nsel else None, status=status, **kw)
    torch.cuda.synchronize()
    assert int(status.item()) == 0, f"device status {int(status.item())}"
    return out, lse, sel[:, :nsel]


def oracle_raw(rc, q, nk, rows=None):
    bs, H, cap, D = rc.keys.shape
    G = q.shape[2] // H
    R = bs * H
    rows = np.arange(R) if rows is None else np.asarray(rows)
    ri = torch.as_tensor(rows, device=DEV)
    kk = to_u16(rc.keys.reshape(R, cap, D)[ri])
    vv = to_u16(rc.values.reshape(R, cap, D)[ri])
    qq = to_u16(q).reshape(R, G, D)[rows]
    mn = to_u16(rc.chunk_min).reshape(R, -1, D)[rows]
    mx = to_u16(rc.chunk_max).reshape(R, -1, D)[rows]
    va = rc.valid.cpu().numpy().astype(np.uint8).reshape(R, -1)[rows]
    return O.page_decode_raw(qq, mn, mx, va, kk, vv, rc.n_c, nk, page_base=rc.n_sink, n_sink=rc.n_sink,
                             near_start=rc.near_start, n_near=rc.n_near, scale=SCALE, threads=8)


@pytest.mark.parametrize("bs,H,G,n_c,nk,n_sink,n_near", [
    (2, 2, 4, 300, 24, 0, 37),     # ragged near window, no sink
    (1, 3, 4, 97, 97, 5, 0),       # every chunk selected (no select runs), partial sink page
    (2, 2, 4, 130, 16, 64, 128),   # reference default sink 64
    (1, 2, 8, 3000, 200, 16, 40),  # G = 8, shared-memory select
    (1, 2, 1, 500, 31, 3, 17),     # G = 1, odd sizes
    (3, 1, 2, 64, 8, 0, 0),        # pages only
    (1, 1, 4, 4096, 128, 0, 128),  # shared-memory select at its largest n_c
    (1, 1, 4, 5001, 300, 64, 64),  # 4096 < n_c <= 8192: 8 keys per select thread
    (1, 1, 4, 8192, 256, 0, 16),   # the 8-keys path at its largest n_c
    (1, 1, 2, 8193, 256, 0, 16),   # n_c > 8192: the radix select over global scores
    (1, 1, 4, 16384, 64, 0, 8),    # the largest n_c the entry accepts
    (8, 8, 4, 300, 24, 5, 37),     # 64 rows: a few attend CTAs per row
    (4, 8, 2, 200, 100, 0, 16),    # 32 rows, 13 entries per attend CTA
])
def test_raw_matches_oracle(bs, H, G, n_c, nk, n_sink, n_near):
    rc = W.build_raw_cache(11 + n_c, bs, H, 16 * n_c, n_near, DEV, n_sink=n_sink)
    q = W.synth_query(torch.Generator(device=DEV).manual_seed(5 + nk), bs, H * G, DEV)
    out, lse, sel = run_raw(rc, q, nk)
    ro, rl, rsel = oracle_raw(rc, q, nk)
    R = bs * H
    assert np.array_equal(sel.cpu().numpy(), rsel), "selected chunk ids differ from the oracle"
    close(O.bf16_to_f32(to_u16(out)).reshape(R, G, 128), O.bf16_to_f32(ro))
    assert np.abs(lse.cpu().numpy() - rl).max() < 1e-3


def test_raw_ties_invalid_chunks_and_empty_rows():
    """All-equal keys tie every chunk (lowest ids win); invalid chunks score
    -inf and lose to every valid one; a row set with no pages and no raw rows
    gives zeros and lse -inf."""
    bs, H, G, n_c, nk = 1, 2, 4, 200, 20
    rc = W.build_raw_cache(3, bs, H, 16 * n_c, 8, DEV)
    rc.keys[0, 0, :16 * n_c] = rc.keys[0, 0, :1]          # row 0: every chunk identical -> ties
    rc.keys[0, 1, :16 * n_c] = rc.keys[0, 1, :16 * n_c].abs()
    cmin = torch.zeros_like(rc.chunk_min)
    cmax = torch.zeros_like(rc.chunk_max)
    valid = torch.zeros_like(rc.valid)
    packed = torch.empty(bs, H, n_c, 16, 16, dtype=torch.int32, device=DEV)
    ops.kivi_encode_chunks(rc.keys[:, :, :16 * n_c], cmin, cmax, None, valid, packed, 0)
    valid[0, 1, ::3] = False                                  # row 1: every third chunk invalid
    rc = W.RawCache(cmin, cmax, valid, rc.keys, rc.values, 0, n_c, 16 * n_c, 8)
    q = W.synth_query(torch.Generator(device=DEV).manual_seed(2), bs, H * G, DEV)
    out, lse, sel = run_raw(rc, q, nk)
    ro, rl, rsel = oracle_raw(rc, q, nk)
    s = sel.cpu().numpy()
    assert np.array_equal(s, rsel)
    assert np.array_equal(s[0], np.arange(nk)), "ties must go to the lowest chunk ids"
    assert not np.any(s[1] % 3 == 0), "an invalid chunk was selected over valid ones"
    close(O.bf16_to_f32(to_u16(out)).reshape(bs * H, G, 128), O.bf16_to_f32(ro))
    # no pages, no raw rows: nothing to attend
    empty = W.build_raw_cache(4, 1, 2, 0, 0, DEV)
    out_e, lse_e, _ = run_raw(empty, q, 0)
    assert torch.count_nonzero(out_e).item() == 0
    assert torch.isneginf(lse_e).all().item()


def test_raw_workspace_reuse_across_shapes_and_repeats():
    """The workspace is scratch only (no state carries between calls, no zero
    fill): one workspace full of garbage bytes serves different shapes back
    to back and repeats bit-exactly."""
    ws = torch.full((ops.page_decode_raw_ws_bytes(16, 3000, 256, 64, 128),), 0x7F, dtype=torch.uint8, device=DEV)
    cases = []
    for bs, H, n_c, nk, s, nn in [(2, 8, 700, 64, 0, 128), (1, 2, 3000, 256, 64, 33), (2, 8, 700, 64, 0, 128)]:
        rc = W.build_raw_cache(40 + n_c, bs, H, 16 * n_c, nn, DEV, n_sink=s)
        q = W.synth_query(torch.Generator(device=DEV).manual_seed(8), bs, H * 4, DEV)
        outs = [run_raw(rc, q, nk, workspace=ws) for _ in range(3)]
        for o, _, sl in outs[1:]:
            assert torch.equal(o, outs[0][0]) and torch.equal(sl, outs[0][2])
        cases.append((rc, q, nk, outs[0]))
    assert torch.equal(cases[0][3][0], cases[2][3][0])
    rc, q, nk, (out, _, sel) = cases[1]
    ro, _, rsel = oracle_raw(rc, q, nk)
    assert np.array_equal(sel.cpu().numpy(), rsel)
    close(O.bf16_to_f32(to_u16(out)).reshape(-1, 4, 128), O.bf16_to_f32(ro))


def test_raw_config0_shape_and_sparse_vs_dense_error(capsys):
    """Config 0 at its stated shape: batch 1, 32 q / 8 KV heads, context 4096
    = 3968 retrieval tokens (248 pages) + 128 residual rows, top 64 pages.
    Parity against the oracle, and the sparse result compared against dense
    attention over all 4096 tokens (reported, not bounded: it is the quality
    of the sparse approximation, not a kernel error)."""
    bs, H, G, ctx, res, nk = 1, 8, 4, 4096, 128, 64
    rc = W.build_raw_cache(0, bs, H, ctx - res, res, DEV)
    q = W.synth_query(torch.Generator(device=DEV).manual_seed(0), bs, H * G, DEV)
    out, lse, sel = run_raw(rc, q, nk)
    ro, rl, rsel = oracle_raw(rc, q, nk)
    R = bs * H
    assert np.array_equal(sel.cpu().numpy(), rsel)
    err, rel = close(O.bf16_to_f32(to_u16(out)).reshape(R, G, 128), O.bf16_to_f32(ro))
    Kf = O.bf16_to_f32(to_u16(rc.keys)).reshape(R, ctx, 128)
    Vf = O.bf16_to_f32(to_u16(rc.values)).reshape(R, ctx, 128)
    qf = O.bf16_to_f32(to_u16(q)).reshape(R, G, 128)
    o = O.bf16_to_f32(to_u16(out)).reshape(R, G, 128)
    d_err, d_ref = [], []
    for r in range(R):
        dense, _ = O.attn_dense(qf[r], Kf[r], Vf[r], SCALE)
        d_err.append(np.abs(o[r] - dense))
        d_ref.append(np.abs(dense))
    d_err, d_ref = np.stack(d_err), np.stack(d_ref)
    with capsys.disabled():
        print(f"\nconfig0: kernel vs oracle max-abs {err:.2e} mean-rel {rel:.2e}; sparse (64 of 248 pages + 128 "
              f"residual) vs dense over 4096 tokens: max-abs {d_err.max():.3e}, "
              f"mean-rel {d_err.mean() / d_ref.mean():.3e}")
    assert np.isfinite(d_err).all()


def test_raw_config1_launch_shape():
    """The exact launch the bench times: 64 rows (batch 8 x 8 KV heads) x 2040
    chunks, nk = 128, 128 residual rows, G = 4.  Selection checked for every
    row, attention output for 8 sampled rows."""
    bs, H, G, n_ret, res, nk = 8, 8, 4, 32768 - 128, 128, 128
    rc = W.build_raw_cache(1000, bs, H, n_ret, res, DEV)
    q = W.synth_query(torch.Generator(device=DEV).manual_seed(77), bs, H * G, DEV)
    out, lse, sel = run_raw(rc, q, nk)
    R = bs * H
    qf = O.bf16_to_f32(to_u16(q)).reshape(R, G, 128)
    acc = np.zeros((R, 128), np.float32)
    for g in range(G):
        acc = (acc + qf[:, g]).astype(np.float32)
    raw_q = O.f32_to_bf16((acc / np.float32(G)).astype(np.float32))
    sc = O.quest_score(raw_q, to_u16(rc.chunk_min).reshape(R, -1, 128), to_u16(rc.chunk_max).reshape(R, -1, 128),
                       rc.valid.cpu().numpy().astype(np.uint8).reshape(R, -1), rc.n_c)
    assert np.array_equal(sel.cpu().numpy(), O.topk_f32(sc, nk))
    rows = [0, 9, 18, 27, 36, 45, 54, 63]
    ro, rl, rsel = oracle_raw(rc, q, nk, rows=rows)
    assert np.array_equal(sel.cpu().numpy()[rows], rsel)
    close(O.bf16_to_f32(to_u16(out)).reshape(R, G, 128)[rows], O.bf16_to_f32(ro))
    assert np.abs(lse.cpu().numpy()[rows] - rl).max() < 1e-3


def test_raw_cuda_graph_replay_matches_eager():
    bs, H, G, n_c, nk = 2, 4, 4, 900, 64
    rc = W.build_raw_cache(21, bs, H, 16 * n_c, 100, DEV, n_sink=4)
    q = W.synth_query(torch.Generator(device=DEV).manual_seed(3), bs, H * G, DEV)
    eager, _, _ = run_raw(rc, q, nk)
    out = torch.empty_like(eager)
    layer = rc.layer()
    ws = torch.zeros(ops.page_decode_raw_ws_bytes(bs * H, n_c, nk, 4, 100), dtype=torch.uint8, device=DEV)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        ops.page_decode_raw(q, layer, n_c, nk, 100, n_sink=4, near_start=rc.near_start, out=out, workspace=ws)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for _ in range(3):
            ops.page_decode_raw(q, layer, n_c, nk, 100, n_sink=4, near_start=rc.near_start, out=out, workspace=ws)
    out.zero_()
    g.replay()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)


def test_raw_rejects_bad_arguments():
    rc = W.build_raw_cache(1, 1, 2, 16 * 40, 8, DEV)
    q = W.synth_query(torch.Generator(device=DEV).manual_seed(1), 1, 8, DEV)
    with pytest.raises(RuntimeError):
        ops.page_decode_raw(q, rc.layer(), rc.n_c, rc.n_c + 1, 8, near_start=rc.near_start)   # nk > n_c
    with pytest.raises(RuntimeError):
        ops.page_decode_raw(q, rc.layer(), rc.n_c, 4, 8, near_start=rc.near_start + 1)        # near past cap
    small = torch.zeros(64, dtype=torch.uint8, device=DEV)
    with pytest.raises(RuntimeError):
        ops.page_decode_raw(q, rc.layer(), rc.n_c, 4, 8, near_start=rc.near_start, workspace=small)
