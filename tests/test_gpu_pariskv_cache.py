"""GPU: the drop-in ParisKV cache (zoomkv_revision_b200.pariskv_cache)
replays the reference's own prefill / decode / flush trace
(tests/golden/pariskv_schedule.npz) with bit-exact retrieval codes, and its
compute() equals an oracle restatement of the retrieval pipeline."""
import math
import os

import numpy as np
import pytest
import torch

import oracle as O
from conftest import GOLDEN, from_u16, to_u16
from zoomkv_revision_b200 import ops
from zoomkv_revision_b200 import pariskv_cache as PK

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _make(g, final_topk=16, threshold=0):
    L, bs, H, sink, local, interval, prefill, steps, max_new = (int(x) for x in g["params"])
    c = PK.polar_cache(valid_start=[0] * bs, layer_num=L, batch_size=bs, max_length=prefill + max_new,
                       num_key_value_heads=H, num_heads=4 * H, head_dim=128, dtype=torch.bfloat16,
                       layer_mapping={str(l): "cuda:0" for l in range(L)}, max_new_length=max_new, sink_size=sink,
                       local_size=local, final_topk=final_topk, dynamic_update_interval=interval,
                       full_attention_threshold=threshold, enable_offload=True)
    # the reference fixture was encoded with the CPU generator's SRHT signs
    c.quantizer.srht_diagonal_signs[0] = from_u16(g["signs"]).to(DEV)
    return c


def _oracle_compute(c, l, q, signs):
    """sink + RaBitQ-selected retrieval + local attention on the oracle."""
    bs, H = c.batch_size, c.kv_head
    R = bs * H
    s = c.sink_size
    total, valid = c.current_seq_len[l], c.cpu_valid_end[l]
    cand_ratio, coll_ratio = PK._adaptive_ratios(valid)
    C = min(valid, max(1, int(math.ceil(valid * cand_ratio))))
    keys = to_u16(c.keys[l][:, :, :total]).reshape(R, total, 128)
    vals = to_u16(c.values[l][:, :, :total]).reshape(R, total, 128)
    codes, packed, weight, factor, hist = O.rq_encode(np.ascontiguousarray(keys[:, s:s + valid]), signs)
    qb, qn, qm = O.rq_query(to_u16(q).reshape(R, 4, 128), signs)
    targets = [int(math.ceil(valid * coll_ratio * r)) for r in (0.05, 0.15, 0.30, 0.50, 0.75, 1.0)]
    cnt = O.collision_count(O.collision_weights(qb, hist, targets), codes)
    cand = O.topk_i32(cnt, C)
    F = min(c.final_topk, C)
    sc = O.rerank4(cand, packed, weight, qb, qn)
    final = np.take_along_axis(cand, O.topk_f32(O.bf16_to_f32(sc) + np.float32(0.0), F), 1) if F < C else cand
    qf = O.bf16_to_f32(to_u16(q)).reshape(R, 4, 128)
    Kf, Vf = O.bf16_to_f32(keys), O.bf16_to_f32(vals)
    local_start = min(total, s + valid)
    outs = []
    for r in range(R):
        idx = np.concatenate([np.arange(0, min(s, total)), final[r] + s, np.arange(local_start, total)])
        o, _ = O.attn_dense(qf[r], Kf[r][idx], Vf[r][idx], 1 / np.sqrt(128))
        outs.append(o)
    return np.stack(outs), final, hist


def _close(out, ref):
    err = np.abs(out - ref)
    assert err.max() <= 2e-2 and err.mean() / np.abs(ref).mean() <= 1e-2, (err.max(), err.mean())


def test_pariskv_replays_reference_schedule_and_codes():
    g = np.load(os.path.join(GOLDEN, "pariskv_schedule.npz"))
    L, bs, H, sink, local, interval, prefill, steps, max_new = (int(x) for x in g["params"])
    c = _make(g)
    keys = from_u16(g["keys"]).to(DEV)       # [L, bs, H, T, D]
    vals = from_u16(g["values"]).to(DEV)
    signs = g["signs"]
    for l in range(L):
        c.prefill_update_kv_cache(None, keys[l, :, :, :prefill].transpose(1, 2).contiguous(),
                                  vals[:, :, :prefill].transpose(1, 2).contiguous(), l, 0)
    trace = g["trace"]
    i = 0
    checked = 0
    gen = torch.Generator(device=DEV).manual_seed(9)
    for t in range(steps):
        pos = prefill + t
        for l in range(L):
            c.decode_update_kv_cache(keys[l, :, :, pos:pos + 1].transpose(1, 2).contiguous(),
                                     vals[:, :, pos:pos + 1].transpose(1, 2).contiguous(), l)
            reg = c.get_region_indices(l)
            got = [t, l, reg["total_len"], reg["retrieval_length"], reg["local_len"], c.cpu_valid_end[l],
                   c._actual_retrieval_length]
            assert got == [int(x) for x in trace[i]], (got, trace[i])
            i += 1
            if l == 1 and t in (0, 30, 99):
                q = torch.randn(bs, 1, 4 * H, 128, generator=gen, device=DEV).to(torch.bfloat16)
                out = c.compute(q, l)
                torch.cuda.synchronize()
                ref, final, _ = _oracle_compute(c, l, q, signs)
                assert np.array_equal(c._last_topk_indices.cpu().numpy(), final)
                _close(O.bf16_to_f32(to_u16(out)).reshape(ref.shape), ref)
                checked += 1
    assert checked == 3
    n = c._actual_retrieval_length
    R = bs * H
    for l in range(L):
        lay = c.layouts[l]
        assert np.array_equal(lay.codes[:, sink:sink + n].cpu().numpy(), g["codes"][l].reshape(R, n, 16))
        assert np.array_equal(lay.packed[:, sink:sink + n].cpu().view(torch.uint8).numpy(),
                              g["packed"][l].reshape(R, n, 64))
        assert np.array_equal(to_u16(lay.weight[:, sink:sink + n]), g["weight"][l].reshape(R, n, 16))
        assert np.array_equal(lay.hist.cpu().numpy(), g["hist"][l].reshape(R, 16, 256))
    assert c.context == prefill + steps


def test_pariskv_full_attention_below_threshold():
    g = np.load(os.path.join(GOLDEN, "pariskv_schedule.npz"))
    L, bs, H, sink, local, interval, prefill, steps, max_new = (int(x) for x in g["params"])
    c = _make(g, final_topk=16, threshold=10 ** 6)
    keys = from_u16(g["keys"]).to(DEV)
    vals = from_u16(g["values"]).to(DEV)
    c.prefill_update_kv_cache(None, keys[0, :, :, :prefill].transpose(1, 2).contiguous(),
                              vals[:, :, :prefill].transpose(1, 2).contiguous(), 0, 0)
    q = torch.randn(bs, 1, 4 * H, 128, device=DEV).to(torch.bfloat16)
    out = c.compute(q, 0)
    torch.cuda.synchronize()
    R = bs * H
    qf = O.bf16_to_f32(to_u16(q)).reshape(R, 4, 128)
    Kf = O.bf16_to_f32(to_u16(keys[0, :, :, :prefill])).reshape(R, prefill, 128)
    Vf = O.bf16_to_f32(to_u16(vals[:, :, :prefill])).reshape(R, prefill, 128)
    ref = np.stack([O.attn_dense(qf[r], Kf[r], Vf[r], 1 / np.sqrt(128))[0] for r in range(R)])
    _close(O.bf16_to_f32(to_u16(out)).reshape(R, 4, 128), ref)


def test_srht_signs_follow_reference_recipe_and_keep_rng_state():
    torch.manual_seed(123)
    before = torch.cuda.get_rng_state()
    s = PK.srht_signs(torch.device(DEV))
    assert torch.equal(torch.cuda.get_rng_state(), before)
    torch.manual_seed(42)
    ref = torch.randint(0, 2, (128,), device=DEV, dtype=torch.bfloat16) * 2 - 1
    assert torch.equal(s, ref)


@pytest.mark.parametrize("threshold", [0, 10 ** 6])
def test_pariskv_host_tier_equals_hbm_cache(monkeypatch, threshold):
    """The offload tier of the ParisKV drop-in (ZKV_HOST_RETRIEVAL=1: raw
    retrieval rows in host-pinned memory, the final rows gathered over the
    host link) returns the same output, selects the same rows and writes the
    same codes as the HBM-resident cache, step for step across flushes --
    through the retrieval branch (threshold 0) and the full-attention branch
    (threshold above every length)."""
    g = np.load(os.path.join(GOLDEN, "pariskv_schedule.npz"))
    L, bs, H, sink, local, interval, prefill, steps, max_new = (int(x) for x in g["params"])
    caches = {}
    for mode in ("0", "1"):
        monkeypatch.setenv("ZKV_HOST_RETRIEVAL", mode)
        caches[mode] = _make(g, threshold=threshold)
    hb, ho = caches["0"], caches["1"]
    assert ho.host_tier and not hb.host_tier and ho.keys[0].is_pinned()
    keys = from_u16(g["keys"]).to(DEV)
    vals = from_u16(g["values"]).to(DEV)
    for c in (hb, ho):
        for l in range(L):
            c.prefill_update_kv_cache(None, keys[l, :, :, :prefill].transpose(1, 2).contiguous(),
                                      vals[:, :, :prefill].transpose(1, 2).contiguous(), l, 0)
    gen = torch.Generator(device=DEV).manual_seed(5)
    for t in range(steps):
        pos = prefill + t
        for l in range(L):
            for c in (hb, ho):
                c.decode_update_kv_cache(keys[l, :, :, pos:pos + 1].transpose(1, 2).contiguous(),
                                         vals[:, :, pos:pos + 1].transpose(1, 2).contiguous(), l)
            if t % 9 == 0:
                q = torch.randn(bs, 1, 4 * H, 128, generator=gen, device=DEV).to(torch.bfloat16)
                a, b = hb.compute(q, l), ho.compute(q, l)
                torch.cuda.synchronize()
                assert torch.equal(a, b), (t, l)
                if threshold == 0 and hb._last_topk_indices is not None:
                    assert torch.equal(hb._last_topk_indices, ho._last_topk_indices)
    for s in (hb._status.values(), ho._status.values()):
        assert all(int(x.item()) == 0 for x in s)
    n = ho._actual_retrieval_length
    for l in range(L):
        assert torch.equal(ho.keys[l][:, :, sink:sink + n], keys[l, :, :, sink:sink + n].cpu())
        assert torch.equal(ho.values[l][:, :, sink:sink + n], vals[:, :, sink:sink + n].cpu())
        for name in ("codes", "packed", "weight", "hist"):
            assert torch.equal(getattr(hb.layouts[l], name), getattr(ho.layouts[l], name)), name
