"""Hierarchical Quest: the oracle against the reference's PyTorch path
(tests/golden/hier_quest.npz, made by tests/golden/make_hier_golden.py from
polar_cache_kivi_quest_density_seperate_kernel.py:1762-1798, :1852-1940).

The PyTorch path scores in bf16 (products and the sum rounded to bf16), the
production CUDA kernels and the oracle in fp32, so scores are compared within
bf16 rounding and the selections by overlap; the integer steps (large
min/max, the plan arithmetic, map-back) are exact."""
import os

import numpy as np

import oracle as O

FIX = np.load(os.path.join(os.path.dirname(__file__), "golden", "hier_quest.npz"))


def test_large_minmax_bit_exact():
    f = int(FIX["factor"])
    lmn, lmx, lv = O.large_minmax(FIX["chunk_min"], FIX["chunk_max"], int(FIX["n_chunks"]), f,
                                  FIX["large_min"].shape[-2])
    assert np.array_equal(lv, FIX["large_valid"])
    v = FIX["large_valid"].astype(bool)
    assert np.array_equal(lmn[v], FIX["large_min"][v])
    assert np.array_equal(lmx[v], FIX["large_max"][v])


def test_plan_arithmetic():
    assert O.hier_plan(int(FIX["n_chunks"]), int(FIX["factor"]))[1:] == (int(FIX["nk_large"]), int(FIX["nk_small"]))
    assert O.hier_plan(15, 16) == (0, 0, 0)
    assert O.hier_plan(16, 16) == (1, 1, 5)


def test_stage_scores_within_bf16_rounding():
    q = FIX["raw_q"].reshape(-1, 128)
    R = q.shape[0]
    n_large = int(FIX["n_chunks"]) // int(FIX["factor"])
    ls = O.quest_score(q, FIX["large_min"].reshape(R, -1, 128), FIX["large_max"].reshape(R, -1, 128),
                       FIX["large_valid"].reshape(R, -1), n_large)
    ref = FIX["large_scores"].reshape(R, -1)
    scale = np.abs(ref).max(axis=1, keepdims=True)
    assert (np.abs(ls - ref) <= scale * 2.0 ** -6).all()
    sub = O.sub_chunk_score(q, FIX["chunk_min"], FIX["chunk_max"], FIX["large_idx"], int(FIX["factor"]))
    ref = FIX["sub_scores"].reshape(R, -1)
    scale = np.abs(ref).max(axis=1, keepdims=True)
    assert (np.abs(sub - ref) <= scale * 2.0 ** -6).all()


def test_map_back_exact():
    out = O.map_back(FIX["large_idx"], FIX["sub_pos"], int(FIX["factor"]), int(FIX["n_chunks"]))
    assert np.array_equal(out, FIX["chunk_idx"])
    li = np.array([[3, 0]], np.int64)
    pos = np.array([[0, 17, 31, 32, -1]], np.int64)
    assert O.map_back(li, pos, 16, 60).tolist() == [[48, 1, 15, -1, -1]]
    assert O.map_back(li, np.array([[15]], np.int64), 16, 60).tolist() == [[59]]   # clamped to n_chunks - 1


def test_selection_overlaps_reference():
    R = FIX["raw_q"].reshape(-1, 128).shape[0]
    out, li, _ = O.hier_select(FIX["raw_q"], FIX["chunk_min"], FIX["chunk_max"], FIX["large_min"],
                               FIX["large_max"], FIX["large_valid"], int(FIX["n_chunks"]), int(FIX["factor"]),
                               int(FIX["nk_large"]), int(FIX["nk_small"]))
    ref = FIX["chunk_idx"].reshape(R, -1)
    ref_l = FIX["large_idx"].reshape(R, -1)
    for r in range(R):
        assert len(set(li[r]) & set(ref_l[r])) >= len(ref_l[r]) - 1
        assert len(set(out[r]) & set(ref[r])) >= 0.8 * ref.shape[1]
        assert (np.diff(out[r]) > 0).all()   # ascending chunk ids


def test_drop_in_plan_matches_oracle():
    from zoomkv_revision_b200 import polar_cache as P
    for n_c in (0, 15, 16, 17, 100, 290, 2040, 8184):
        for f in (4, 8, 16):
            assert P.hier_plan(n_c, f, 0.3, 0.3) == O.hier_plan(n_c, f), (n_c, f)
    assert P.hier_plan(2040, 16, 0.5, 0.1) == O.hier_plan(2040, 16, 0.5, 0.1)


def test_drop_in_knobs(monkeypatch):
    import pytest
    from zoomkv_revision_b200 import polar_cache as P
    monkeypatch.setenv("POLAR_QUEST_HIERARCHICAL", "1")
    monkeypatch.setenv("ZKV_ATTENTION_MODE", "page")
    cfg = P.env_config()
    assert cfg["hierarchical"] and cfg["large_chunk"] == 256 and cfg["large_ratio"] == 0.3
    monkeypatch.setenv("POLAR_QUEST_LARGE_CHUNK", "512")
    with pytest.raises(ValueError):
        P.env_config()
    monkeypatch.setenv("POLAR_QUEST_LARGE_CHUNK", "128")
    monkeypatch.setenv("ZKV_ATTENTION_MODE", "reference")
    with pytest.raises(ValueError):
        P.env_config()
