"""CPU tests of the drop-in cache's host logic against the reference's own
code (fixtures from tests/golden/make_golden.py): candidate budget, chunk
plan, region arithmetic and the full offload-bookkeeping flush schedule."""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN
from zoomkv_revision_b200 import polar_cache as P


def zoomkv_cfg(force=None, monkeypatch=None):
    env = {"POLAR_QUEST_CHUNK": "16", "POLAR_QUEST_CAND_RATIO": "0.4", "POLAR_QUEST_DYNAMIC_CAND_RATIO": "1",
           "POLAR_QUEST_DYNAMIC_CAND_THRESHOLDS": "5000,10001", "POLAR_QUEST_DYNAMIC_CAND_RATIOS": "0.7,0.5,0.4",
           "POLAR_CDS_DENSE_RATIO": "0.3", "POLAR_CDS_DENSE_TOPK": "8", "POLAR_CDS_SPARSE_TOPK": "8"}
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    if force is None:
        monkeypatch.delenv("POLAR_FORCE_CAND_TOKENS", raising=False)
    else:
        monkeypatch.setenv("POLAR_FORCE_CAND_TOKENS", str(force))
    return P.env_config()


def test_candidate_budget_matches_reference(monkeypatch):
    with open(os.path.join(GOLDEN, "host_logic.json")) as f:
        rows = json.load(f)
    for r in rows:
        cfg = zoomkv_cfg(r["force"], monkeypatch)
        assert P.quest_aligned_candidate_tokens(r["kv_len"], cfg) == r["cand_tokens"], r
        n_chunks, nk, n_dense, skipped = P.quest_chunk_plan(r["kv_len"], cfg)
        assert (n_chunks, nk, n_dense, skipped) == (r["n_chunks"], r["nk"], r["n_dense"], r["skipped"]), r


def test_flush_schedule_replays_reference_trace(monkeypatch):
    """CacheSchedule reproduces the reference's prefill zones, flush points,
    retrieval lengths, nk and skipped tails step by step."""
    cfg = zoomkv_cfg(None, monkeypatch)
    g = np.load(os.path.join(GOLDEN, "schedule.npz"))
    L, bs, H, sink, local, interval, prefill, steps, max_new = (int(x) for x in g["params"])
    with open(os.path.join(GOLDEN, "schedule_trace.json")) as f:
        trace = json.load(f)
    s = P.CacheSchedule(L, sink, local, interval, prefill, cfg, offload=True)
    for l in range(L):
        s.prefill(l, prefill, 0)
    it = iter(trace)
    flushes = 0
    for t in range(steps):
        for l in range(L):
            if s.flush_due(l):
                lo, hi, num_new = s.flush()
                flushes += 1
                assert lo % 16 == 0 and hi % 16 == 0 and num_new == interval
            s.append(l)
            r = next(it)
            r_len, local_start, local_len = s.region(l)
            n_chunks, nk, n_dense, skipped = s.plan
            assert (r["step"], r["layer"]) == (t, l)
            assert s.current_seq_len[l] == r["total_len"]
            assert (r_len, local_len) == (r["retrieval_length"], r["local_len"]), r
            assert s.cpu_valid_end[l] == r["cpu_valid_end"] and s.actual_retrieval == r["actual"], r
            assert (nk, n_chunks, skipped) == (r["nk"], r["n_chunks"], r["skipped"]), r
            assert r["carry"] == s.actual_retrieval % 16
    assert flushes == 4
    # encoded chunks after the run == the reference's valid chunk mask
    n_valid = (s.actual_retrieval // 16)
    assert (g["valid"][:, :, :, :n_valid] == 1).all() and not g["valid"][:, :, :, n_valid:].any()


def test_region_non_offload_arithmetic(monkeypatch):
    """All-GPU bookkeeping: local window from the update-buffer arithmetic."""
    for total in (10, 40, 300, 301, 1000):
        r_len, ls, ll = P.region(total, None, 200, 4, 64, 32)
        assert ls == P.compute_local_start(total, 200, 4, 64, 32)
        assert r_len == max(0, ls - 4) and (ll == total - ls if ls < total else ll == 0)


def test_env_rejects_unsupported(monkeypatch):
    monkeypatch.setenv("POLAR_QUEST_CHUNK", "8")
    with pytest.raises(ValueError):
        P.env_config()
    monkeypatch.setenv("POLAR_QUEST_CHUNK", "16")
    monkeypatch.setenv("ZKV_ATTENTION_MODE", "bogus")
    with pytest.raises(ValueError):
        P.env_config()


def test_skipped_overflow_raises(monkeypatch):
    cfg = zoomkv_cfg(None, monkeypatch)
    cfg = dict(cfg, max_skipped=4)
    with pytest.raises(RuntimeError):
        P.quest_chunk_plan(16 * 3 + 9, cfg)


@pytest.mark.parametrize("sink,local,interval,prefill,steps", [
    (4, 32, 24, 107, 300),      # the reference trace's shape, long
    (4, 128, 512, 4000, 2000),  # production-like local / interval
    (0, 64, 64, 500, 600),      # no sink
    (16, 256, 256, 100, 900),   # prompt shorter than sink + local
    (4, 40, 24, 77, 500),       # odd sizes: ragged chunk tails at every flush
])
def test_offload_window_invariants(monkeypatch, sink, local, interval, prefill, steps):
    """The offload tier's HBM window, replayed through the real schedule:
    the window base (first unencoded token) is where every flush's encode
    range starts, the local window never starts before it, every appended
    token fits the near part, and the gathered selection fits the staging
    rows (the arithmetic polar_cache uses with ZKV_HOST_RETRIEVAL=1)."""
    cfg = zoomkv_cfg(None, monkeypatch)
    F = 100
    cap = prefill + steps
    stage, near_cap = P.offload_window(sink, local, interval, F, cfg["max_skipped"], 2000, cap)
    s = P.CacheSchedule(1, sink, local, interval, prefill, cfg, offload=True)
    _, r_len, (lo, hi) = s.prefill(0, prefill, 0)
    base = sink + hi
    assert lo == 0 and prefill - base <= near_cap or prefill <= sink
    for _ in range(steps):
        if s.flush_due(0):
            lo, hi, _ = s.flush()
            assert sink + lo == base           # the completed chunks start at the window base
            base = sink + hi
        pos = s.append(0)
        if pos >= sink:
            assert 0 <= pos - base < near_cap  # the appended token has a window row
        r_len, local_start, _ = s.region(0)
        assert local_start >= base or r_len == 0
        n_chunks, nk, _, skipped = s.plan
        assert min(F, nk * 16) + skipped <= stage
