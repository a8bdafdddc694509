"""GPU tests of the drop-in `polar_cache` (reference interface): the token
stream of the reference trace (tests/golden/schedule.npz, produced by the
reference's own prefill / decode / flush code) is replayed through the cache;
its chunk metadata must equal the reference's bit for bit, and `compute()`
must equal an oracle restatement of the production pipeline."""
import os

import numpy as np
import pytest
import torch

import oracle as O
from conftest import GOLDEN, from_u16, to_u16
from zoomkv_revision_b200 import polar_cache as P

pytestmark = pytest.mark.gpu
DEV = "cuda"


def set_env(monkeypatch, mode):
    """mode: 'reference', 'page', 'page4', or 'host' (reference attention
    with the retrieval zone in host-pinned memory).  Page mode is the
    reference run with dense_topk = sparse_topk = 16 (every token of a
    selected chunk survives stage 2)."""
    monkeypatch.setenv("ZKV_HOST_RETRIEVAL", "1" if mode == "host" else "0")
    mode = "reference" if mode == "host" else mode
    env = {"POLAR_QUEST_CHUNK": "16", "POLAR_QUEST_CAND_RATIO": "0.4", "POLAR_QUEST_DYNAMIC_CAND_RATIO": "1",
           "POLAR_QUEST_DYNAMIC_CAND_THRESHOLDS": "5000,10001", "POLAR_QUEST_DYNAMIC_CAND_RATIOS": "0.7,0.5,0.4",
           "POLAR_CDS_DENSE_RATIO": "0.3", "POLAR_CDS_DENSE_TOPK": "16",
           "POLAR_CDS_SPARSE_TOPK": "16" if mode == "page" else "8", "ZKV_ATTENTION_MODE": mode}
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    monkeypatch.delenv("POLAR_FORCE_CAND_TOKENS", raising=False)


def make_cache(g, final_topk=16):
    L, bs, H, sink, local, interval, prefill, steps, max_new = (int(x) for x in g["params"])
    return P.polar_cache(valid_start=[0] * bs, layer_num=L, batch_size=bs, max_length=prefill + max_new,
                         num_key_value_heads=H, num_heads=4 * H, head_dim=128, dtype=torch.bfloat16,
                         layer_mapping={str(l): "cuda:0" for l in range(L)}, max_new_length=max_new, sink_size=sink,
                         local_size=local, core=0, nprobe=0, cache_unit_size=0, cache_cluster_num=0, num_gpus=1,
                         model_size=8, final_topk=final_topk, dynamic_update_interval=interval,
                         full_attention_threshold=0, enable_offload=True)


def oracle_reference_compute(cache, l, q, keys, values, F):
    """Production pipeline restated on the oracle: Quest -> top-nk -> CDS ->
    KIVI stage-2 -> global top-k + skipped -> attention over raw rows."""
    bs, H = cache.batch_size, cache.kv_head
    R = bs * H
    s = cache.sink_size
    total = cache.current_seq_len[l]
    r_len, local_start, _ = cache.sched.region(l)
    n_chunks, nk, n_dense, skipped = cache.sched.plan
    qf = O.bf16_to_f32(to_u16(q)).reshape(bs, 4 * H, 128)
    raw_q = O.f32_to_bf16(qf.reshape(R, 4, 128).sum(axis=1) / 4.0)
    mn = to_u16(cache.chunk_min[l]).reshape(R, -1, 128)
    mx = to_u16(cache.chunk_max[l]).reshape(R, -1, 128)
    ce = to_u16(cache.chunk_centroid[l]).reshape(R, -1, 128)
    valid = cache.chunk_valid[l].cpu().numpy().astype(np.uint8).reshape(R, -1)
    pk = cache.kivi_packed[l].cpu().numpy().reshape(R, -1, 16, 16)
    sc = O.quest_score(raw_q, mn, mx, valid, n_chunks)
    cidx = O.topk_f32(sc, nk)
    dens = O.chunk_density(cidx, ce, raw_q)
    mask = O.mask_from_topk(O.topk_f32(dens, n_dense), nk)
    n_valid = r_len // 16
    osc, oix = O.kivi_qk(cidx, mask, np.ascontiguousarray(pk[:, :n_valid]), mn, mx, raw_q,
                         min(cache.cfg["dense_topk"], 16), min(cache.cfg["sparse_topk"], 16))
    k = min(F, nk * 16)
    skip = np.tile(np.arange(n_chunks * 16, r_len, dtype=np.int64), (R, 1))
    final = O.topk_gather_concat(osc, oix, skip, k)
    Kf = O.bf16_to_f32(keys).reshape(R, -1, 128)
    Vf = O.bf16_to_f32(values).reshape(R, -1, 128)
    outs = []
    for r in range(R):
        idx = np.concatenate([np.arange(0, s), final[r] + s, np.arange(local_start, total)])
        o, _ = O.attn_dense(qf[r // H, (r % H) * 4:(r % H + 1) * 4], Kf[r][idx], Vf[r][idx], 1 / np.sqrt(128))
        outs.append(o)
    return np.stack(outs).reshape(bs, H * 4, 128), final


def close(out, ref):
    err = np.abs(out - ref)
    assert err.max() <= 2e-2 and err.mean() / np.abs(ref).mean() <= 1e-2, (err.max(), err.mean())


@pytest.mark.parametrize("mode", ["reference", "page", "page4", "host"])
def test_polar_cache_replays_reference_and_matches_oracle(monkeypatch, mode):
    set_env(monkeypatch, mode)
    g = np.load(os.path.join(GOLDEN, "schedule.npz"))
    L, bs, H, sink, local, interval, prefill, steps, max_new = (int(x) for x in g["params"])
    cache = make_cache(g)
    keys = [from_u16(g["keys0"]), from_u16(g["keys1"])]         # [bs, H, T, D]
    vals = from_u16(g["values"])
    for l in range(L):
        kl = keys[l][:, :, :prefill].transpose(1, 2).contiguous()
        vl = vals[:, :, :prefill].transpose(1, 2).contiguous()
        kk, vv = cache.prefill_update_kv_cache(None, kl, vl, l, 0)
        assert kk.shape[1] == prefill
    gen = torch.Generator(device=DEV).manual_seed(3)
    checked = 0
    for t in range(steps):
        pos = prefill + t
        for l in range(L):
            cache.decode_update_kv_cache(keys[l][:, :, pos:pos + 1].transpose(1, 2).contiguous(),
                                         vals[:, :, pos:pos + 1].transpose(1, 2).contiguous(), l)
            if t in (0, 23, 24, 50, 99) and l == 1:
                q = torch.randn(bs, 1, 4 * H, 128, generator=gen, device=DEV).to(torch.bfloat16)
                out = cache.compute(q, l)
                torch.cuda.synchronize()
                total = cache.current_seq_len[l]
                kl = to_u16(keys[l][:, :, :total])
                vl = to_u16(vals[:, :, :total])
                if mode in ("reference", "host"):
                    ref, _ = oracle_reference_compute(cache, l, q, kl, vl, cache.final_topk)
                    close(O.bf16_to_f32(to_u16(out)).reshape(ref.shape), ref)
                elif mode == "page":
                    # the reference's own chain with page knobs: final_topk = nk * 16 keeps
                    # every token of every selected chunk
                    nk = cache.sched.plan[1]
                    ref, _ = oracle_reference_compute(cache, l, q, kl, vl, nk * 16)
                    close(O.bf16_to_f32(to_u16(out)).reshape(ref.shape), ref)
                else:
                    R = bs * H
                    n_chunks, nk, _, _ = cache.sched.plan
                    near_start = sink + n_chunks * 16
                    raw = np.concatenate([kl[:, :, :sink], kl[:, :, near_start:total]], axis=2).reshape(R, -1, 128)
                    rawv = np.concatenate([vl[:, :, :sink], vl[:, :, near_start:total]], axis=2).reshape(R, -1, 128)
                    ro, _, _ = O.page_decode(
                        to_u16(q).reshape(R, 4, 128), to_u16(cache.chunk_min[l]).reshape(R, -1, 128),
                        to_u16(cache.chunk_max[l]).reshape(R, -1, 128),
                        cache.chunk_valid[l].cpu().numpy().astype(np.uint8).reshape(R, -1),
                        cache.kivi_packed[l].cpu().numpy().reshape(R, -1, 16, 16),
                        cache.vcodes_t[l].cpu().numpy().reshape(R, -1, 128, 2),
                        to_u16(cache.vmeta[l]).reshape(R, -1, 2, 4, 16), np.ascontiguousarray(raw),
                        np.ascontiguousarray(rawv), n_chunks, nk, raw.shape[1], 1 / np.sqrt(128))
                    close(O.bf16_to_f32(to_u16(out)).reshape(R, 4, 128), O.bf16_to_f32(ro))
                checked += 1
    assert checked == 5
    # final chunk metadata == the reference's (bit-exact), every layer
    n_valid = cache.sched.actual_retrieval // 16
    for l in range(L):
        assert (to_u16(cache.chunk_min[l])[:, :, :n_valid] == g["chunk_min"][l][:, :, :n_valid]).all()
        assert (to_u16(cache.chunk_max[l])[:, :, :n_valid] == g["chunk_max"][l][:, :, :n_valid]).all()
        assert (to_u16(cache.chunk_centroid[l])[:, :, :n_valid] == g["centroid"][l][:, :, :n_valid]).all()
        assert (cache.kivi_packed[l].cpu().numpy()[:, :, :n_valid] == g["packed"][l][:, :, :n_valid]).all()
        assert (cache.chunk_valid[l].cpu().numpy()[:, :, :n_valid]).all()
    assert cache.context == prefill + steps
    assert cache.cpu_valid_end == [cache.sched.actual_retrieval] * L


def test_polar_cache_full_attention_branch(monkeypatch):
    """Below the retrieval threshold compute() attends every stored token."""
    set_env(monkeypatch, "reference")
    g = np.load(os.path.join(GOLDEN, "schedule.npz"))
    cache = make_cache(g, final_topk=100)   # sink + local + 2F > total -> full attention
    L, bs, H = 2, 2, 2
    keys = from_u16(g["keys0"])
    vals = from_u16(g["values"])
    cache.prefill_update_kv_cache(None, keys[:, :, :107].transpose(1, 2).contiguous(),
                                  vals[:, :, :107].transpose(1, 2).contiguous(), 0, 0)
    q = torch.randn(bs, 1, 4 * H, 128, device=DEV).to(torch.bfloat16)
    out = cache.compute(q, 0)
    qf = O.bf16_to_f32(to_u16(q)).reshape(bs, 4 * H, 128)
    Kf = O.bf16_to_f32(to_u16(keys[:, :, :107]))
    Vf = O.bf16_to_f32(to_u16(vals[:, :, :107]))
    for b in range(bs):
        for h in range(H):
            ro, _ = O.attn_dense(qf[b, h * 4:(h + 1) * 4], Kf[b, h], Vf[b, h], 1 / np.sqrt(128))
            close(O.bf16_to_f32(to_u16(out[b, 0, h * 4:(h + 1) * 4])), ro)


def test_host_retrieval_tier_equals_hbm_cache(monkeypatch):
    """The offload tier (retrieval rows in host-pinned memory, gathered over
    the host link) selects the same rows and returns the same output as the
    HBM-resident cache, step for step across flushes; the host zone holds
    exactly the retrieval rows."""
    g = np.load(os.path.join(GOLDEN, "schedule.npz"))
    L, bs, H, sink, local, interval, prefill, steps, max_new = (int(x) for x in g["params"])
    caches = {}
    for mode in ("reference", "host"):
        set_env(monkeypatch, mode)
        caches[mode] = make_cache(g)
    hb, ho = caches["reference"], caches["host"]
    assert ho.host_tier and not hb.host_tier and ho.keys[0].is_pinned()
    keys = [from_u16(g["keys0"]), from_u16(g["keys1"])]
    vals = from_u16(g["values"])
    for c in (hb, ho):
        for l in range(L):
            c.prefill_update_kv_cache(None, keys[l][:, :, :prefill].transpose(1, 2).contiguous(),
                                      vals[:, :, :prefill].transpose(1, 2).contiguous(), l, 0)
    gen = torch.Generator(device=DEV).manual_seed(8)
    for t in range(steps):
        pos = prefill + t
        for l in range(L):
            for c in (hb, ho):
                c.decode_update_kv_cache(keys[l][:, :, pos:pos + 1].transpose(1, 2).contiguous(),
                                         vals[:, :, pos:pos + 1].transpose(1, 2).contiguous(), l)
            if t % 7 == 0:
                q = torch.randn(bs, 1, 4 * H, 128, generator=gen, device=DEV).to(torch.bfloat16)
                a, b = hb.compute(q, l), ho.compute(q, l)
                torch.cuda.synchronize()
                n_chunks, nk, _, skipped = ho.sched.plan
                min_total = max(ho.FULL_ATTENTION_THRESHOLD, sink + local + 2 * ho.final_topk)
                if ho.current_seq_len[l] >= min_total and n_chunks > 0:  # the retrieval branch ran
                    n = min(ho.final_topk, nk * 16) + skipped
                    assert torch.equal(hb._scratch[hb.device]["final"][:, :, :n],
                                       ho._scratch[ho.device]["final"][:, :, :n])
                assert torch.equal(a, b), (t, l)
    assert int(ho._scratch[ho.device]["status"].item()) == 0
    r = ho.sched.actual_retrieval
    for l in range(L):
        assert torch.equal(ho.keys[l][:, :, sink:sink + r], keys[l][:, :, sink:sink + r].cpu())
        assert torch.equal(ho.values[l][:, :, sink:sink + r], vals[:, :, sink:sink + r].cpu())
        for name in ("chunk_min", "chunk_max", "chunk_centroid", "kivi_packed"):
            assert torch.equal(getattr(hb, name)[l], getattr(ho, name)[l])


def test_host_retrieval_full_attention_branch(monkeypatch):
    """Below the retrieval threshold the offload tier gathers every host row
    and attends all stored tokens."""
    set_env(monkeypatch, "host")
    g = np.load(os.path.join(GOLDEN, "schedule.npz"))
    cache = make_cache(g, final_topk=100)
    bs, H = 2, 2
    keys = from_u16(g["keys0"])
    vals = from_u16(g["values"])
    cache.prefill_update_kv_cache(None, keys[:, :, :107].transpose(1, 2).contiguous(),
                                  vals[:, :, :107].transpose(1, 2).contiguous(), 0, 0)
    assert cache.win_base[0] > cache.sink_size  # some rows live only on the host
    q = torch.randn(bs, 1, 4 * H, 128, device=DEV).to(torch.bfloat16)
    out = cache.compute(q, 0)
    qf = O.bf16_to_f32(to_u16(q)).reshape(bs, 4 * H, 128)
    Kf = O.bf16_to_f32(to_u16(keys[:, :, :107]))
    Vf = O.bf16_to_f32(to_u16(vals[:, :, :107]))
    for b in range(bs):
        for h in range(H):
            ro, _ = O.attn_dense(qf[b, h * 4:(h + 1) * 4], Kf[b, h], Vf[b, h], 1 / np.sqrt(128))
            close(O.bf16_to_f32(to_u16(out[b, 0, h * 4:(h + 1) * 4])), ro)
