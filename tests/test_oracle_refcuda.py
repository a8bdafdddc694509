"""The oracle against the reference's own CUDA kernels (CPU).

tests/golden/ref_cuda.npz holds outputs of the reference's production
kernels, built from the reference sources (oracle/build_ref.py) and run on a
B200 by tests/golden/make_ref_cuda_golden.py.  Where the reference's CUDA
and PyTorch paths differ in rounding, these fixtures pin the CUDA semantics:
scores bit for bit, index sets exactly (top-k ties compared as the
reference's own test does, by the multiset of selected scores)."""
import os

import numpy as np

import oracle as O
from conftest import golden

G = golden("ref_cuda.npz")


def test_quest_scores_bit_exact_vs_reference_kernel():
    bs, kv, n_max, D = G["quest_min"].shape
    R = bs * kv
    n_c = int(G["quest_n_chunks"])
    for v in (0, 1):
        valid = G["quest_valid"].reshape(R, n_max) if v else None
        sc = O.quest_score(G["quest_q"].reshape(R, D), G["quest_min"].reshape(R, n_max, D),
                           G["quest_max"].reshape(R, n_max, D), valid, n_c)
        ref = G[f"quest_scores_v{v}"].reshape(R, n_c)
        assert np.array_equal(sc.view(np.uint32), ref.view(np.uint32)), f"valid={v}"


def test_kivi_stage2_bit_exact_vs_reference_kernel():
    g = golden("kivi_qk.npz")
    for dt, st in ((16, 16), (16, 8), (8, 8), (8, 4)):
        sc, ix = O.kivi_qk(g["chunk_ids"], g["dense"], g["packed"], g["chunk_min"], g["chunk_max"], g["raw_q"], dt,
                           st)
        rs, ri = G[f"kivi_scores_{dt}_{st}"], G[f"kivi_idx_{dt}_{st}"]
        assert np.array_equal(sc.view(np.uint32), rs.view(np.uint32)), (dt, st)
        # kept slots: identical token ids; dropped slots carry only the fill score
        kept = rs > -1e29
        assert np.array_equal(ix[kept], ri[kept]), (dt, st)


def test_density_and_mask_vs_reference_kernel():
    g = golden("quest_density.npz")
    d = O.chunk_density(g["density_ids"], g["centroid"], g["raw_q"])
    assert np.array_equal(d.view(np.uint32), G["density"].view(np.uint32))
    nk = G["mask"].shape[-1]
    m = O.mask_from_topk(G["mask_pos"], nk)
    assert np.array_equal(m, G["mask"])


def test_float_topk_sets_vs_reference_kernel():
    s, k = G["topk_scores"], int(G["topk_k"])
    ours = O.topk_f32(s, k)
    ref = G["topk_idx"]
    for r in np.ndindex(*s.shape[:-1]):
        a, b = s[r][ours[r]], s[r][ref[r]]
        # same multiset of selected scores (ties may pick different indices)
        assert np.array_equal(np.sort(a), np.sort(b)), r
        # and exactly the reference set wherever the k-th score is not tied
        kth = np.sort(s[r])[-k]
        if np.count_nonzero(s[r] == kth) == 1:
            assert set(ours[r].tolist()) == set(ref[r].tolist()), r


def test_collision_counts_vs_reference_kernel():
    g = golden("collision_ref.npz")
    sid = g["sorted_ids"].astype(np.int64)[0]
    cnt = O.update_cache_cnt_sorted(sid, g["hist"][0], g["codes"][0].astype(np.int32), g["targets"])
    assert np.array_equal(cnt, G["collision_cnt"][0])


def test_rerank4_bit_exact_vs_reference_kernel():
    g = golden("rerank4.npz")
    for i in range(3):
        cand = g[f"c{i}_cand"][0]
        packed = g[f"c{i}_packed"][0]
        H, kv = packed.shape[:2]
        sc = O.rerank4(cand, packed.reshape(H, kv, 64), g[f"c{i}_weight"][0], g[f"c{i}_q_blocks"][0].reshape(H, 128),
                       g[f"c{i}_q_norm"][0], g["centers"])
        assert np.array_equal(sc, G[f"rerank_c{i}"][0]), i


def test_coarse2bit_vs_reference_kernel():
    bs, kv, B, L, _ = G["c2_packed"].shape
    R = bs * kv
    packed = G["c2_packed"].transpose(0, 1, 3, 2, 4).reshape(R, L, B * 4)
    out = O.coarse2bit(packed, G["c2_qs"].reshape(R, B), G["c2_qm"].reshape(R, B))
    assert np.array_equal(out, G["c2_scores"].reshape(R, L))


def test_hierarchical_quest_vs_reference_kernels():
    """Hierarchical Quest as the separate-kernel cache runs it on the GPU
    (quest_chunk_score over large chunks, float_topk_3d, quest_sub_chunk_score,
    float_topk_3d, quest_map_back; tests/golden/ref_cuda_hier.npz): the oracle's
    stage scores are bit-exact, its picks equal as sets."""
    d = np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_cuda_hier.npz"))
    f, n_c = int(d["hier_factor"]), int(d["hier_n_c"])
    nkl, nks = int(d["hier_nk_large"]), int(d["hier_nk_small"])
    assert O.hier_plan(n_c, f)[1:] == (nkl, nks)
    q = d["hier_q"].reshape(-1, 128)
    R = q.shape[0]
    mn, mx = d["hier_min"].reshape(R, -1, 128), d["hier_max"].reshape(R, -1, 128)
    lmn, lmx, lv = d["hier_lmin"].reshape(R, -1, 128), d["hier_lmax"].reshape(R, -1, 128), \
        d["hier_lvalid"].reshape(R, -1)
    ls = O.quest_score(q, lmn, lmx, lv, n_c // f)
    assert np.array_equal(ls.view(np.uint32), d["hier_large_scores"].reshape(R, -1).view(np.uint32))
    # sub-chunk scores of the reference's own large picks, in its order
    ref_li = d["hier_large_idx"].reshape(R, -1)
    sub = O.sub_chunk_score(q, mn, mx, ref_li, f)
    assert np.array_equal(sub.view(np.uint32), d["hier_sub_scores"].reshape(R, -1).view(np.uint32))
    assert np.array_equal(O.map_back(ref_li, d["hier_sub_pos"].reshape(R, -1), f, n_c),
                          d["hier_chunk_idx"].reshape(R, -1))
    out, li, _ = O.hier_select(q, mn, mx, lmn, lmx, lv, n_c, f, nkl, nks)
    for r in range(R):
        assert set(li[r]) == set(ref_li[r])
        assert set(out[r]) == set(d["hier_chunk_idx"].reshape(R, -1)[r])
