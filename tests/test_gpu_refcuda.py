"""The library's kernels against the reference's own CUDA kernels.

tests/golden/ref_cuda.npz holds outputs of the reference's production
kernels (built from its sources by oracle/build_ref.py, run on a B200 by
tests/golden/make_ref_cuda_golden.py).  Scores must be equal bit for bit,
index sets exactly (top-k ties compared by the multiset of selected scores,
as the reference's own top-k test does)."""
import numpy as np
import pytest
import torch

from conftest import from_u16, golden, to_u16
from zoomkv_revision_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"
G = golden("ref_cuda.npz")


def test_quest_scores_bit_exact_vs_reference_kernel():
    bs, kv, n_max, D = G["quest_min"].shape
    n_c = int(G["quest_n_chunks"])
    q, mn, mx = (from_u16(G[k]) for k in ("quest_q", "quest_min", "quest_max"))
    for v in (0, 1):
        sc = torch.empty(bs, kv, n_c, dtype=torch.float32, device=DEV)
        valid = torch.from_numpy(G["quest_valid"].astype(bool)).to(DEV) if v else None
        ops.quest_chunk_score(q, mn, mx, sc, n_c, valid)
        torch.cuda.synchronize()
        assert np.array_equal(sc.cpu().numpy().view(np.uint32), G[f"quest_scores_v{v}"].view(np.uint32)), v


def test_kivi_stage2_bit_exact_vs_reference_kernel():
    g = golden("kivi_qk.npz")
    ids = torch.from_numpy(g["chunk_ids"]).to(DEV)
    dense = torch.from_numpy(g["dense"].astype(bool)).to(DEV)
    packed = torch.from_numpy(g["packed"]).to(DEV)
    mn, mx, q = (from_u16(g[k]) for k in ("chunk_min", "chunk_max", "raw_q"))
    bs, kv, nk = g["chunk_ids"].shape
    for dt, st in ((16, 16), (16, 8), (8, 8), (8, 4)):
        sc = torch.empty(bs, kv, nk * 16, dtype=torch.float32, device=DEV)
        ix = torch.empty(bs, kv, nk * 16, dtype=torch.int64, device=DEV)
        ops.partial_chunk_kivi_qk_dense_sparse_cuda(ids, dense, packed, mn, mx, q, dt, st, 16, sc, ix)
        torch.cuda.synchronize()
        rs, ri = G[f"kivi_scores_{dt}_{st}"], G[f"kivi_idx_{dt}_{st}"]
        assert np.array_equal(sc.cpu().numpy().view(np.uint32), rs.view(np.uint32)), (dt, st)
        kept = rs > -1e29
        assert np.array_equal(ix.cpu().numpy()[kept], ri[kept]), (dt, st)


def test_density_and_mask_vs_reference_kernel():
    g = golden("quest_density.npz")
    ids = torch.from_numpy(g["density_ids"]).to(DEV)
    out = torch.empty(ids.shape, dtype=torch.float32, device=DEV)
    ops.partial_chunk_density_scores_cuda(ids, from_u16(g["centroid"]), from_u16(g["raw_q"]), out)
    mask = torch.ones(ids.shape, dtype=torch.bool, device=DEV)
    ops.dense_mask_from_topk_cuda(torch.from_numpy(G["mask_pos"]).to(DEV), mask)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), G["density"].view(np.uint32))
    assert np.array_equal(mask.cpu().numpy().astype(np.uint8), G["mask"])


def test_float_topk_vs_reference_kernel():
    s, k = G["topk_scores"], int(G["topk_k"])
    idx = ops.float_topk_3d(torch.from_numpy(s).to(DEV), k).cpu().numpy()
    ref = G["topk_idx"]
    for r in np.ndindex(*s.shape[:-1]):
        assert np.array_equal(np.sort(s[r][idx[r]]), np.sort(s[r][ref[r]])), r


def test_rerank4_bit_exact_vs_reference_kernel():
    g = golden("rerank4.npz")
    cen = from_u16(g["centers"])
    for i in range(3):
        cand = torch.from_numpy(g[f"c{i}_cand"]).to(DEV)
        p4 = torch.from_numpy(np.ascontiguousarray(g[f"c{i}_packed"].transpose(0, 1, 3, 2, 4))).to(DEV)
        w = from_u16(np.ascontiguousarray(g[f"c{i}_weight"].transpose(0, 1, 3, 2)))
        lay = ops.RqLayout.from_reference(torch.zeros(1, 2, 16, p4.shape[3], dtype=torch.uint8, device=DEV), p4, w)
        H, C = cand.shape[1], cand.shape[2]
        sc, _ = ops.partial_rerank_cuda(cand.reshape(H, C), lay, from_u16(g[f"c{i}_q_blocks"]).reshape(H, 128),
                                        from_u16(g[f"c{i}_q_norm"]).reshape(H), cen, final_topk=1)
        torch.cuda.synchronize()
        assert np.array_equal(to_u16(sc), G[f"rerank_c{i}"].reshape(H, C)), i


def test_coarse2bit_vs_reference_kernel():
    bs, kv, B, L, _ = G["c2_packed"].shape
    p4 = torch.from_numpy(G["c2_packed"]).to(DEV)
    lay = ops.RqLayout.from_reference(torch.zeros(bs, kv, B, L, dtype=torch.uint8, device=DEV), p4)
    out = ops.coarse_2bit_score_cuda(lay, torch.from_numpy(G["c2_qs"]).to(DEV), torch.from_numpy(G["c2_qm"]).to(DEV),
                                     L)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().reshape(bs, kv, L), G["c2_scores"])


def test_hierarchical_pick_vs_reference_kernels():
    """zkv_page_decode_raw_hier's pick against the reference's hierarchical
    Quest chain run on the GPU (ref_cuda_hier.npz): large min/max rebuilt by
    zkv_quest_large_minmax bit-exact, the picked chunk ids equal as sets.
    One query head per KV head, so the GQA mean is the fixture's raw q."""
    H = golden("ref_cuda_hier.npz")
    f, n_c = int(H["hier_factor"]), int(H["hier_n_c"])
    nkl, nks = int(H["hier_nk_large"]), int(H["hier_nk_small"])
    bs, kv, n_max, D = H["hier_min"].shape
    mn, mx = from_u16(H["hier_min"]), from_u16(H["hier_max"])
    nml = H["hier_lmin"].shape[2]
    lmn = torch.zeros(bs, kv, nml, D, dtype=torch.bfloat16, device=DEV)
    lmx = torch.zeros_like(lmn)
    lv = torch.zeros(bs, kv, nml, dtype=torch.uint8, device=DEV)
    ops.quest_large_minmax(mn, mx, n_c, f, lmn, lmx, lv)
    torch.cuda.synchronize()
    ref_v = H["hier_lvalid"].astype(bool)
    ref_v_built = ref_v.copy()
    ref_v_built[1 // kv, 1 % kv, 5] = True          # the fixture invalidated one group after building
    assert np.array_equal(lv.cpu().numpy().astype(bool), ref_v_built)
    assert np.array_equal(to_u16(lmn)[ref_v_built], H["hier_lmin"][ref_v_built])
    assert np.array_equal(to_u16(lmx)[ref_v_built], H["hier_lmax"][ref_v_built])
    lv.copy_(torch.from_numpy(H["hier_lvalid"].astype(np.uint8)))
    g = torch.Generator(device=DEV).manual_seed(3)
    keys = torch.randn(bs, kv, n_max * 16, D, generator=g, device=DEV).to(torch.bfloat16)
    layer = ops.RawLayer(mn, mx, None, keys, keys)
    q = from_u16(H["hier_q"]).reshape(bs, 1, kv, D)
    sel = torch.empty(bs * kv, nks, dtype=torch.int64, device=DEV)
    ops.page_decode_raw_hier(q, layer, ops.LargeLayer(lmn, lmx, lv), n_c, f, nkl, nks, 0, near_start=n_c * 16,
                             sel_out=sel)
    torch.cuda.synchronize()
    ref = H["hier_chunk_idx"].reshape(bs * kv, -1)
    got = sel.cpu().numpy()
    for r in range(bs * kv):
        assert set(got[r]) == set(ref[r]), r
