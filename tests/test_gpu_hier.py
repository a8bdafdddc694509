"""GPU parity of hierarchical Quest (zkv_quest_large_minmax,
zkv_page_decode_raw_hier) against the oracle restatement of
polar_cache_kivi_quest_density_seperate_kernel.py:1762-1798 (large-chunk
min/max) and :1852-1940 (the two-level pick), and of the attention over the
picked pages' raw rows (fp64 softmax, 2e-2 / 1e-2)."""
import numpy as np
import pytest
import torch

import oracle as O
from conftest import to_u16
from zoomkv_revision_b200 import ops
from zoomkv_revision_b200 import workload as W

pytestmark = pytest.mark.gpu
DEV = "cuda"
SCALE = 1 / np.sqrt(128)


def large_of(rc, factor, valid_end=None):
    bs, H, n_max, _ = rc.chunk_min.shape
    nml = (n_max + factor - 1) // factor
    lmn = torch.zeros(bs, H, nml, 128, dtype=torch.bfloat16, device=DEV)
    lmx = torch.zeros_like(lmn)
    lv = torch.zeros(bs, H, nml, dtype=torch.uint8, device=DEV)
    ops.quest_large_minmax(rc.chunk_min, rc.chunk_max, rc.n_c if valid_end is None else valid_end, factor,
                           lmn, lmx, lv)
    return lmn, lmx, lv


def gqa_raw_q(q, R, G):
    qf = O.bf16_to_f32(to_u16(q)).reshape(R, G, 128)
    acc = np.zeros((R, 128), np.float32)
    for g in range(G):
        acc = (acc + qf[:, g]).astype(np.float32)
    return O.f32_to_bf16((acc / np.float32(G)).astype(np.float32))


@pytest.mark.parametrize("factor,n_c", [(16, 290), (16, 2040), (8, 333), (5, 101)])
def test_large_minmax_bit_exact(factor, n_c):
    rc = W.build_raw_cache(n_c, 2, 2, 16 * n_c, 0, DEV)
    lmn, lmx, lv = large_of(rc, factor)
    torch.cuda.synchronize()
    R = 4
    omn, omx, olv = O.large_minmax(to_u16(rc.chunk_min).reshape(R, -1, 128), to_u16(rc.chunk_max).reshape(R, -1, 128),
                                   rc.n_c, factor, lmn.shape[2])
    assert np.array_equal(lv.cpu().numpy().reshape(R, -1), olv)
    v = olv.astype(bool)
    assert np.array_equal(to_u16(lmn).reshape(R, -1, 128)[v], omn[v])
    assert np.array_equal(to_u16(lmx).reshape(R, -1, 128)[v], omx[v])


def test_large_minmax_group_range_leaves_others():
    rc = W.build_raw_cache(7, 1, 2, 16 * 100, 0, DEV)
    lmn, lmx, lv = large_of(rc, 16, valid_end=40)   # groups 0..2 valid, group 2 partial
    before = (lmn.clone(), lv.clone())
    ops.quest_large_minmax(rc.chunk_min, rc.chunk_max, 100, 16, lmn, lmx, lv, g_lo=2, g_hi=7)
    torch.cuda.synchronize()
    assert torch.equal(lmn[:, :, :2], before[0][:, :, :2])
    R = 2
    omn, omx, olv = O.large_minmax(to_u16(rc.chunk_min).reshape(R, -1, 128), to_u16(rc.chunk_max).reshape(R, -1, 128),
                                   100, 16, lmn.shape[2])
    assert np.array_equal(lv.cpu().numpy().reshape(R, -1), olv)
    assert np.array_equal(to_u16(lmn).reshape(R, -1, 128)[olv.astype(bool)], omn[olv.astype(bool)])


def attend_ref(rc, q, sel, R, G):
    cap = rc.keys.shape[2]
    K = O.bf16_to_f32(to_u16(rc.keys)).reshape(R, cap, 128)
    V = O.bf16_to_f32(to_u16(rc.values)).reshape(R, cap, 128)
    qf = O.bf16_to_f32(to_u16(q)).reshape(R, G, 128)
    out = np.zeros((R, G, 128))
    for r in range(R):
        tok = list(range(rc.n_sink))
        for c in sel[r]:
            tok += list(range(rc.n_sink + 16 * int(c), rc.n_sink + 16 * int(c) + 16))
        tok += list(range(rc.near_start, rc.near_start + rc.n_near))
        o, _ = O.attn_dense(qf[r], K[r][tok], V[r][tok], SCALE)
        out[r] = o
    return out


@pytest.mark.parametrize("bs,H,G,n_c,factor,n_sink,n_near,invalid", [
    (2, 2, 4, 290, 16, 0, 37, False),
    (1, 4, 4, 2040, 16, 16, 128, True),   # config-1 row length, some large chunks invalid
    (2, 1, 8, 333, 8, 3, 20, False),
    (4, 8, 4, 600, 16, 0, 128, False),    # 128 rows
])
def test_hier_decode_matches_oracle(bs, H, G, n_c, factor, n_sink, n_near, invalid):
    rc = W.build_raw_cache(31 + n_c, bs, H, 16 * n_c, n_near, DEV, n_sink=n_sink)
    lmn, lmx, lv = large_of(rc, factor)
    if invalid:
        lv[:, :, 3] = 0
        lv[0, 1, 10:14] = 0
    n_large, nk_large, nk_small = O.hier_plan(n_c, factor)
    q = W.synth_query(torch.Generator(device=DEV).manual_seed(12), bs, H * G, DEV)
    R = bs * H
    sel = torch.full((R, nk_small), -7, dtype=torch.int64, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    lse = torch.empty(R, G, device=DEV)
    out = ops.page_decode_raw_hier(q, rc.layer(), ops.LargeLayer(lmn, lmx, lv), n_c, factor, nk_large, nk_small,
                                   n_near, n_sink=n_sink, near_start=rc.near_start, sel_out=sel, lse=lse,
                                   status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    raw_q = gqa_raw_q(q, R, G)
    osel, oli, _ = O.hier_select(raw_q, to_u16(rc.chunk_min).reshape(R, -1, 128),
                                 to_u16(rc.chunk_max).reshape(R, -1, 128), to_u16(lmn).reshape(R, -1, 128),
                                 to_u16(lmx).reshape(R, -1, 128), lv.cpu().numpy().reshape(R, -1), n_c, factor,
                                 nk_large, nk_small)
    assert np.array_equal(sel.cpu().numpy(), osel), "hierarchical selection differs from the oracle"
    ref = attend_ref(rc, q, osel, R, G)
    o = O.bf16_to_f32(to_u16(out)).reshape(R, G, 128).astype(np.float64)
    err = np.abs(o - ref)
    assert err.max() <= 2e-2 and err.mean() / np.abs(ref).mean() <= 1e-2, (err.max(), err.mean())


def test_hier_rejects_bad_arguments():
    rc = W.build_raw_cache(3, 1, 2, 16 * 64, 8, DEV)
    lmn, lmx, lv = large_of(rc, 16)
    q = W.synth_query(torch.Generator(device=DEV).manual_seed(1), 1, 8, DEV)
    big = ops.LargeLayer(lmn, lmx, lv)
    with pytest.raises(RuntimeError):   # nk_large > n_large
        ops.page_decode_raw_hier(q, rc.layer(), big, 64, 16, 5, 8, 8, near_start=rc.near_start)
    with pytest.raises(RuntimeError):   # nk_small > nk_large * factor
        ops.page_decode_raw_hier(q, rc.layer(), big, 64, 16, 2, 33, 8, near_start=rc.near_start)
    with pytest.raises(RuntimeError):   # factor > 16
        ops.page_decode_raw_hier(q, rc.layer(), big, 64, 32, 1, 8, 8, near_start=rc.near_start)


def test_drop_in_hierarchical_page_mode(monkeypatch):
    """polar_cache with POLAR_QUEST_HIERARCHICAL=1 in page mode: the large-chunk
    boxes follow prefill and flushes (bit-exact against the oracle rebuilt
    from the cache's chunk boxes), and compute() attends the hierarchical
    pick + sink + every token from the first partial large chunk on."""
    from zoomkv_revision_b200 import polar_cache as P
    env = {"ZKV_ATTENTION_MODE": "page", "POLAR_QUEST_HIERARCHICAL": "1", "POLAR_QUEST_LARGE_CHUNK": "128",
           "POLAR_QUEST_CHUNK": "16", "ZKV_HOST_RETRIEVAL": "0"}
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    bs, H, G, sink, local, interval, prefill, steps = 1, 2, 4, 4, 32, 32, 1100, 70
    c = P.polar_cache(valid_start=[0] * bs, layer_num=1, batch_size=bs, max_length=prefill + steps + 16,
                      num_key_value_heads=H, num_heads=G * H, head_dim=128, dtype=torch.bfloat16,
                      layer_mapping={"0": DEV}, max_new_length=steps + 16, sink_size=sink, local_size=local,
                      final_topk=64, dynamic_update_interval=interval, full_attention_threshold=0,
                      enable_offload=True)
    g = torch.Generator(device=DEV).manual_seed(5)
    kk = torch.randn(bs, prefill + steps, H, 128, generator=g, device=DEV).to(torch.bfloat16)
    vv = torch.randn(bs, prefill + steps, H, 128, generator=g, device=DEV).to(torch.bfloat16)
    c.prefill_update_kv_cache(None, kk[:, :prefill].contiguous(), vv[:, :prefill].contiguous(), 0, 0)
    for t in range(steps):
        pos = prefill + t
        c.decode_update_kv_cache(kk[:, pos:pos + 1].contiguous(), vv[:, pos:pos + 1].contiguous(), 0)
    q = W.synth_query(torch.Generator(device=DEV).manual_seed(6), bs, G * H, DEV)
    out = c.compute(q, 0)
    torch.cuda.synchronize()
    R, f = bs * H, c.hq_factor
    n_c = c.sched.plan[0]
    omn, omx, olv = O.large_minmax(to_u16(c.chunk_min[0]).reshape(R, -1, 128), to_u16(c.chunk_max[0]).reshape(R, -1, 128),
                                   n_c, f, c.large_min[0].shape[2])
    v = olv.astype(bool)
    assert np.array_equal(c.large_valid[0].cpu().numpy().reshape(R, -1), olv)
    assert np.array_equal(to_u16(c.large_min[0]).reshape(R, -1, 128)[v], omn[v])
    assert np.array_equal(to_u16(c.large_max[0]).reshape(R, -1, 128)[v], omx[v])
    n_large, nk_large, nk_small = O.hier_plan(n_c, f)
    assert n_large > 0
    raw_q = gqa_raw_q(q, R, G)
    osel, _, _ = O.hier_select(raw_q, to_u16(c.chunk_min[0]).reshape(R, -1, 128),
                               to_u16(c.chunk_max[0]).reshape(R, -1, 128), omn, omx, olv, n_c, f, nk_large, nk_small)
    total = c.current_seq_len[0]
    K = O.bf16_to_f32(to_u16(c.keys[0])).reshape(R, -1, 128)
    V = O.bf16_to_f32(to_u16(c.values[0])).reshape(R, -1, 128)
    qf = O.bf16_to_f32(to_u16(q)).reshape(R, G, 128)
    o = O.bf16_to_f32(to_u16(out)).reshape(R, G, 128).astype(np.float64)
    for r in range(R):
        tok = list(range(sink))
        for ch in osel[r]:
            tok += list(range(sink + 16 * int(ch), sink + 16 * int(ch) + 16))
        tok += list(range(sink + n_large * f * 16, total))
        ref, _ = O.attn_dense(qf[r], K[r][tok], V[r][tok], SCALE)
        err = np.abs(o[r] - ref)
        assert err.max() <= 2e-2 and err.mean() / np.abs(ref).mean() <= 1e-2, (r, err.max())
