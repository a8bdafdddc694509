"""Generate golden fixtures from the reference's own PyTorch implementation.

Run in a container where the reference snapshot is mounted (CPU torch is
enough):

    python tests/golden/make_golden.py --ref <path of the reference checkout>

It imports the ZoomKV runtime's pure-PyTorch functions, drives them on small
seeded inputs and stores inputs + outputs as .npz files next to this script.
The fixtures are committed; the tests only read them (the reference is not
needed at test time).  bf16 tensors are stored as uint16 bit patterns.

Functions pinned (paths relative to runtime/zoomkv_urania_runtime_20261011/):
  * polar_cache._compute_and_store_chunk_minmax / _kivi_pack_chunks
    (cache_hub/polar_cache_quest_density_single_layer_kivi.py:2025-2157,
    :1965-2020) driven through a stub object, several calls with carry
  * quant_pack.pack_kcache_4bit / unpack_kcache_4bit (cache_hub/kivi/quant_pack.py)
  * qk_dot.dequant_kcache_4bit / partial_chunk_kivi_qk_ref (cache_hub/kivi/qk_dot.py)
  * QuestPytorch.quest_chunk_score (cache_hub/quest/quest_ops.py:22-31)
  * polar_cache._partial_chunk_density_scores_torch (:2246-2262)
  * lse_merge_torch (cache_hub/lse_merge/lse_merge.py:79-119)
  * candidate-budget arithmetic _quest_aligned_candidate_tokens /
    _quest_candidate_ratio / _refresh_quest_chunk_cache (:1798-1925)
  * the offload-bookkeeping state machine: _prefill_lockstep_batch,
    decode_update_kv_cache, _update_polar_index, get_region_indices
    (:880-1004, :1516-1583, :1379-1512, :1173-1259) driven step by step
  * ParisKV (cache_hub/polar_cache.py): batch_encode (:1130-1198),
    _count_cluster_keys (:1203-1226), _encode_query_blocks (:1108-1127) and
    the bucket ordering of get_cache_cnt_fused (:1688-1728), with the sign
    codebook read from turboquant/codebooks/*.json
  * update_cache_cnt_overall_ref / generate_test_input
    (cache_hub/collision_fused/collision_test.py:17-121)
  * python_rabitq_scores / make_inputs (cache_hub/rerank/test_rerank_topk.py:27-111)
  * ParisKV's prefill / decode_update / flush state machine
    (cache_hub/polar_cache.py:523-657, 837-853, 919-1065) driven step by step
"""
from __future__ import annotations

import argparse
import functools
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
RUNTIME = "runtime/zoomkv_urania_runtime_20261011"


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16).copy()


def synth_keys(gen: torch.Generator, shape, outliers=4, scale=10.0) -> torch.Tensor:
    """K ~ N(0,1) with `outliers` random channels per head scaled x10 (bf16)."""
    k = torch.randn(shape, generator=gen, dtype=torch.float32)
    heads, dim = shape[1], shape[-1]
    for h in range(heads):
        ch = torch.randperm(dim, generator=gen)[:outliers]
        k[:, h, ..., ch] *= scale
    return k.to(torch.bfloat16)


def make_stub(zmod, bs, kv, n_max, chunk=16, dim=128, layers=1):
    pc = zmod.polar_cache
    s = types.SimpleNamespace()
    s._use_quest_chunk_coarse = True
    s.quest_chunk_size = chunk
    s._kivi_bits = 4
    s._chunk_n_max = n_max
    s._chunk_carry_count = [0] * layers
    s._chunk_valid_end = [0] * layers
    s._chunk_carry_keys = [torch.zeros(bs, kv, chunk - 1, dim, dtype=torch.bfloat16) for _ in range(layers)]
    s._chunk_merge_buffer = [torch.zeros(bs, kv, chunk, dim, dtype=torch.bfloat16) for _ in range(layers)]
    s._chunk_key_min_gpu = [torch.zeros(bs, kv, n_max, dim, dtype=torch.bfloat16) for _ in range(layers)]
    s._chunk_key_max_gpu = [torch.zeros(bs, kv, n_max, dim, dtype=torch.bfloat16) for _ in range(layers)]
    s._chunk_key_centroid_gpu = [torch.zeros(bs, kv, n_max, dim, dtype=torch.bfloat16) for _ in range(layers)]
    s._chunk_valid_mask_gpu = [torch.zeros(bs, kv, n_max, dtype=torch.bool) for _ in range(layers)]
    s.key_kivi_packed_gpu = [torch.zeros(bs, kv, n_max, dim // 8, chunk, dtype=torch.int32) for _ in range(layers)]
    s._kivi_pack_chunks = functools.partial(pc._kivi_pack_chunks, s)
    s._compute_and_store_chunk_minmax = functools.partial(pc._compute_and_store_chunk_minmax, s)
    return s


def gen_encode(zmod, out):
    """Prefill of 75 retrieval tokens, then updates of 30, 7, 40 tokens
    (exercises aligned chunks, carry append, carry merge, tail carry)."""
    g = torch.Generator().manual_seed(1234)
    bs, kv, dim, chunk = 2, 2, 128, 16
    seg = [75, 30, 7, 40]
    total = sum(seg)
    keys = synth_keys(g, (bs, kv, total, dim))
    n_max = (total + chunk - 1) // chunk + 1
    s = make_stub(zmod, bs, kv, n_max)
    start = 0
    carries = []
    for n in seg:
        s._compute_and_store_chunk_minmax(0, keys[:, :, start:start + n, :].contiguous(), abs_token_start=start)
        start += n
        carries.append(s._chunk_carry_count[0])
    np.savez_compressed(
        os.path.join(out, "encode_carry.npz"),
        keys=bf16_bits(keys), segments=np.array(seg), carries=np.array(carries),
        chunk_min=bf16_bits(s._chunk_key_min_gpu[0]), chunk_max=bf16_bits(s._chunk_key_max_gpu[0]),
        centroid=bf16_bits(s._chunk_key_centroid_gpu[0]),
        valid=s._chunk_valid_mask_gpu[0].numpy().astype(np.uint8),
        packed=s.key_kivi_packed_gpu[0].numpy(), valid_end=np.array(s._chunk_valid_end[0]),
        carry_keys=bf16_bits(s._chunk_carry_keys[0]), n_max=np.array(n_max))


def gen_pack(out):
    from cache_hub.kivi.quant_pack import pack_kcache_4bit, unpack_kcache_4bit
    g = torch.Generator().manual_seed(7)
    bs, kv, T, dim, chunk = 1, 2, 64, 128, 16
    keys = synth_keys(g, (bs, kv, T, dim))
    kc = keys.view(bs, kv, T // chunk, chunk, dim)
    mn, mx = kc.amin(dim=3), kc.amax(dim=3)
    # a flat channel (max == min) exercises the 1e-8 divisor clamp
    keys2 = keys.clone()
    keys2[:, :, :chunk, 5] = 0.75
    mn2, mx2 = keys2.view(bs, kv, T // chunk, chunk, dim).amin(3), keys2.view(bs, kv, T // chunk, chunk, dim).amax(3)
    packed, scale = pack_kcache_4bit(keys2, mn2, mx2, chunk)
    approx = unpack_kcache_4bit(packed, mn2, mx2, chunk)
    np.savez_compressed(
        os.path.join(out, "kivi_pack.npz"),
        keys=bf16_bits(keys2), chunk_min=bf16_bits(mn2), chunk_max=bf16_bits(mx2),
        packed=packed.numpy(), scale=bf16_bits(scale), approx=bf16_bits(approx))
    del mn, mx


def gen_kivi_qk(out):
    from cache_hub.kivi.qk_dot import dequant_kcache_4bit, partial_chunk_kivi_qk_ref
    from cache_hub.kivi.quant_pack import pack_kcache_4bit
    g = torch.Generator().manual_seed(99)
    bs, kv, n_chunks, chunk, dim, nk = 2, 2, 24, 16, 128, 10
    keys = synth_keys(g, (bs, kv, n_chunks * chunk, dim))
    kc = keys.view(bs, kv, n_chunks, chunk, dim)
    mn, mx = kc.amin(dim=3).contiguous(), kc.amax(dim=3).contiguous()
    packed_tm, _ = pack_kcache_4bit(keys, mn, mx, chunk)              # [bs,kv,T,16]
    packed_cm = packed_tm.view(bs, kv, n_chunks, chunk, dim // 8).transpose(-1, -2).contiguous()
    raw_q = torch.randn(bs, kv, dim, generator=g).to(torch.bfloat16)
    chunk_ids = torch.stack([torch.randperm(n_chunks, generator=g)[:nk] for _ in range(bs * kv)]).view(bs, kv, nk)
    dense = torch.rand(bs, kv, nk, generator=g) < 0.4
    kch = dequant_kcache_4bit(packed_cm, mn, mx, chunk_ids, chunk)
    sc, ix = partial_chunk_kivi_qk_ref(chunk_ids, dense, packed_cm, mn, mx, raw_q,
                                       group_size=chunk, dense_topk=16, sparse_topk=8)
    np.savez_compressed(
        os.path.join(out, "kivi_qk.npz"),
        keys=bf16_bits(keys), chunk_min=bf16_bits(mn), chunk_max=bf16_bits(mx), packed=packed_cm.numpy(),
        raw_q=bf16_bits(raw_q), chunk_ids=chunk_ids.numpy(), dense=dense.numpy().astype(np.uint8),
        dequant=bf16_bits(kch), ref_scores=sc.numpy(), ref_idx=ix.numpy())


def gen_quest_density(zmod, out):
    from cache_hub.quest.quest_ops import QuestPytorch
    g = torch.Generator().manual_seed(5)
    bs, kv, n_max, n_chunks, dim, chunk = 2, 2, 40, 37, 128, 16
    keys = synth_keys(g, (bs, kv, n_max * chunk, dim))
    kc = keys.view(bs, kv, n_max, chunk, dim)
    mn, mx = kc.amin(3).contiguous(), kc.amax(3).contiguous()
    cent = kc.mean(3).contiguous()
    valid = torch.ones(bs, kv, n_max, dtype=torch.bool)
    valid[:, :, 3] = False
    q = torch.randn(bs, kv, 4, dim, generator=g).to(torch.bfloat16)
    raw_q = q.mean(dim=2)
    scores = torch.empty(bs, kv, n_chunks, dtype=torch.float32)
    QuestPytorch().quest_chunk_score(raw_q, mn, mx, scores, n_chunks, valid)
    ids = torch.stack([torch.randperm(n_chunks, generator=g)[:12] for _ in range(bs * kv)]).view(bs, kv, 12)
    ids[0, 0, 0] = -1                     # invalid ids -> -1e30
    ids[1, 1, 2] = n_max + 3
    dens = torch.empty(bs, kv, 12)
    zmod.polar_cache._partial_chunk_density_scores_torch(ids, cent, raw_q, dens)
    np.savez_compressed(
        os.path.join(out, "quest_density.npz"),
        q=bf16_bits(q), raw_q=bf16_bits(raw_q), chunk_min=bf16_bits(mn), chunk_max=bf16_bits(mx),
        centroid=bf16_bits(cent), valid=valid.numpy().astype(np.uint8), n_chunks=np.array(n_chunks),
        quest_scores=scores.numpy(), density_ids=ids.numpy(), density=dens.numpy())


def gen_lse(out):
    from cache_hub.lse_merge.lse_merge import lse_merge_torch
    g = torch.Generator().manual_seed(3)
    bs, heads, dim = 3, 32, 128
    a = torch.randn(bs, 1, heads, dim, generator=g).to(torch.bfloat16)
    b = torch.randn(bs, 1, heads, dim, generator=g).to(torch.bfloat16)
    la = torch.randn(bs, heads, 1, generator=g) * 3
    lb = torch.randn(bs, heads, 1, generator=g) * 3
    m = lse_merge_torch(a, la, b, lb)
    np.savez_compressed(os.path.join(out, "lse_merge.npz"), a=bf16_bits(a), b=bf16_bits(b),
                        la=la.numpy(), lb=lb.numpy(), merged=bf16_bits(m))


def gen_host_logic(zmod, out):
    """Candidate budget / nk / n_dense / skipped tail under the production
    ZoomKV knobs (run/eval_math_aime.py:212-236) and under a forced budget."""
    pc = zmod.polar_cache
    rows = []
    for force in (None, 2048, 1024):
        s = types.SimpleNamespace(
            quest_chunk_size=16, quest_coarse_candidate_ratio=0.4, _dynamic_cand_enabled=True,
            _dynamic_cand_thresholds=[5000, 10001], _dynamic_cand_ratios=[0.7, 0.5, 0.4],
            _force_cand_tokens=force, cds_dense_ratio=0.3)
        s._quest_candidate_ratio = functools.partial(pc._quest_candidate_ratio, s)
        for kv_len in [0, 1, 15, 16, 17, 100, 1000, 4095, 4999, 5000, 5001, 10000, 10001, 10002,
                       20000, 32640, 32768, 65536, 131072]:
            tgt = pc._quest_aligned_candidate_tokens(s, kv_len)
            n_chunks = kv_len // 16
            nk = max(1, min(n_chunks, tgt // 16)) if kv_len >= 16 else 0
            n_dense = max(1, int(nk * 0.3)) if nk else 0
            rows.append(dict(force=force, kv_len=kv_len, cand_tokens=tgt, n_chunks=n_chunks, nk=nk,
                             n_dense=n_dense, skipped=kv_len - n_chunks * 16))
    with open(os.path.join(out, "host_logic.json"), "w") as f:
        json.dump(rows, f, indent=0)


class _Ev:
    def record(self, *a):
        pass

    def wait(self, *a):
        pass

    def synchronize(self):
        pass


def gen_schedule(zmod, out):
    """Drive the reference's own prefill / decode_update / flush / region code
    (offload bookkeeping) on CPU tensors through a stub, for 2 layers, batch 2,
    2 KV heads: record per-step state and the final chunk metadata."""
    pc = zmod.polar_cache
    L, bs, H, D = 2, 2, 2, 128
    sink, local, interval = 4, 32, 24
    prefill, steps, max_new = 107, 100, 120
    g = torch.Generator().manual_seed(2024)
    total_tokens = prefill + steps
    keys = synth_keys(g, (bs, H, total_tokens, D))            # [bs, H, T, D] per layer 0
    keys1 = synth_keys(g, (bs, H, total_tokens, D))
    vals = torch.randn(bs, H, total_tokens, D, generator=g).to(torch.bfloat16)
    layer_keys = [keys, keys1]
    s = make_stub(zmod, bs, H, (prefill + max_new + 15) // 16, layers=L)
    s.layer_num, s.batch_size, s.kv_head, s.head_dim, s.dtype = L, bs, H, D, torch.bfloat16
    s.sink_size, s.local_size, s.steady_size = sink, local, sink + local
    s.dynamic_update_interval = interval
    s.max_new_length = max_new
    s.input_length = prefill
    s.valid_start = [0, 0]
    s.enable_offload = True
    s.gpu_kv_capacity = sink + local + interval
    s.cpu_kv_capacity = prefill + max_new - sink - local
    s.unified_keys_gpu = [torch.zeros(bs, H, s.gpu_kv_capacity, D, dtype=torch.bfloat16) for _ in range(L)]
    s.unified_values_gpu = [torch.zeros(bs, H, s.gpu_kv_capacity, D, dtype=torch.bfloat16) for _ in range(L)]
    s.unified_keys_cpu = [torch.zeros(bs, H, s.cpu_kv_capacity, D, dtype=torch.bfloat16) for _ in range(L)]
    s.unified_values_cpu = [torch.zeros(bs, H, s.cpu_kv_capacity, D, dtype=torch.bfloat16) for _ in range(L)]
    s._offload_keys_buffer = [torch.zeros(bs, H, interval, D, dtype=torch.bfloat16) for _ in range(L)]
    s._offload_values_buffer = [torch.zeros(bs, H, interval, D, dtype=torch.bfloat16) for _ in range(L)]
    s.cpu_valid_end = [0] * L
    s._inflight_offload_buffers = [None] * L
    s._layer_offload_inflight = [False] * L
    s._main_events = [_Ev() for _ in range(L)]
    s._copy_events = [_Ev() for _ in range(L)]
    s._copy_stream = None
    s._actual_retrieval_length = None
    s.current_seq_len = [0] * L
    s.context = 0
    s._decode_step_counter = 0
    s._cached_region_total_len = -1
    s._cached_region_info = None
    s._arange_buffer = torch.arange(prefill + max_new)
    s._debug_flush = False
    s.device = torch.device("cpu")
    s.final_topk = 100
    s.MAX_SKIPPED_INDICES = 512
    s._chunk_skipped_indices_gpu = [torch.zeros(bs, H, 512, dtype=torch.int64) for _ in range(L)]
    s._chunk_skipped_count = [0] * L
    s._quest_scores_buffer = torch.empty(bs * H * s._chunk_n_max)
    s.cds_dense_ratio = 0.3
    s.quest_coarse_candidate_ratio = 0.4
    s._dynamic_cand_enabled = True
    s._dynamic_cand_thresholds, s._dynamic_cand_ratios = [5000, 10001], [0.7, 0.5, 0.4]
    s._force_cand_tokens = None
    s._topk_keys_buffer = None
    for name in ("_refresh_quest_chunk_cache", "_refresh_live_skipped_indices", "_quest_aligned_candidate_tokens",
                 "_quest_candidate_ratio", "_compute_local_start", "get_region_indices", "_update_polar_index",
                 "decode_update_kv_cache", "_sync_layer_offload", "_prefill_lockstep_batch"):
        setattr(s, name, functools.partial(getattr(pc, name), s))
    s._sync_offload_copies = lambda: None
    # prefill: pre-set the retrieval length so the stub never allocates pinned host buffers
    retrieval = max(sink, prefill - local) - sink
    s._actual_retrieval_length = retrieval
    s._refresh_quest_chunk_cache(retrieval)
    for l in range(L):
        k4 = layer_keys[l][:, :, :prefill].transpose(1, 2).contiguous()   # [bs, T, H, D]
        v4 = vals[:, :, :prefill].transpose(1, 2).contiguous()
        s._prefill_lockstep_batch(k4, v4, l)
    trace = []
    for t in range(steps):
        pos = prefill + t
        for l in range(L):
            k1 = layer_keys[l][:, :, pos:pos + 1].transpose(1, 2).contiguous()
            v1 = vals[:, :, pos:pos + 1].transpose(1, 2).contiguous()
            s.decode_update_kv_cache(k1, v1, l)
            reg = s.get_region_indices(l)
            trace.append(dict(step=t, layer=l, total_len=int(reg["total_len"]),
                              retrieval_length=int(reg["retrieval_length"]), local_len=int(reg["local_len"]),
                              cpu_valid_end=int(s.cpu_valid_end[l]), actual=int(s._actual_retrieval_length),
                              nk=int(s._cached_quest_nk), n_chunks=int(s._cached_quest_n_chunks),
                              skipped=int(s._chunk_skipped_count[l]), carry=int(s._chunk_carry_count[l])))
    np.savez_compressed(
        os.path.join(out, "schedule.npz"),
        keys0=bf16_bits(keys), keys1=bf16_bits(keys1), values=bf16_bits(vals),
        chunk_min=np.stack([bf16_bits(s._chunk_key_min_gpu[l]) for l in range(L)]),
        chunk_max=np.stack([bf16_bits(s._chunk_key_max_gpu[l]) for l in range(L)]),
        centroid=np.stack([bf16_bits(s._chunk_key_centroid_gpu[l]) for l in range(L)]),
        packed=np.stack([s.key_kivi_packed_gpu[l].numpy() for l in range(L)]),
        valid=np.stack([s._chunk_valid_mask_gpu[l].numpy().astype(np.uint8) for l in range(L)]),
        skipped_idx=np.stack([s._chunk_skipped_indices_gpu[l].numpy() for l in range(L)]),
        params=np.array([L, bs, H, sink, local, interval, prefill, steps, max_new]))
    with open(os.path.join(out, "schedule_trace.json"), "w") as f:
        json.dump(trace, f)


def rabitq_stub(pmod, signs):
    """The fields of ParisKV's polar_cache that batch_encode and
    _encode_query_blocks read (cache_hub/polar_cache.py:262-273, :428)."""
    st = types.SimpleNamespace()
    st.quantizer = types.SimpleNamespace(B=16, m=8, srht_diagonal_signs=[signs])
    st.polar_B, st.polar_m, st.polar_K_omega = 16, 8, 256
    st._hadamard_scale = 1.0 / np.sqrt(128)
    st._mag_thresholds = torch.tensor([0.0843, 0.1698, 0.2578, 0.3499, 0.4487, 0.5585, 0.6901], dtype=torch.bfloat16)
    st._mag_centers = torch.tensor([0.0420, 0.1266, 0.2130, 0.3025, 0.3973, 0.5001, 0.6169, 0.7633],
                                   dtype=torch.bfloat16)
    st._bitpack_shifts = (1 << torch.arange(8, dtype=torch.uint8))
    st._pack_4bit_codes = types.MethodType(pmod.polar_cache._pack_4bit_codes, st)
    return st


def gen_rabitq(pmod, ref_root, out):
    """ParisKV encode + query + collision ordering (config-2 shapes, reduced N)."""
    pc = pmod.polar_cache
    torch.manual_seed(42)  # the reference seeds the SRHT signs with 42 (:81-90; CPU generator here)
    signs = torch.randint(0, 2, (128,), dtype=torch.bfloat16) * 2 - 1
    st = rabitq_stub(pmod, signs)
    g = torch.Generator().manual_seed(7)
    bs, H, N, G = 2, 2, 1024, 4
    spread = torch.exp(torch.randn(bs, H, N, 1, generator=g) * 0.5)   # norm spread
    keys = (torch.randn(bs, H, N, 128, generator=g) * spread).to(torch.bfloat16)
    codebook, weight, packed = pc.batch_encode(st, keys)
    hist = pc._count_cluster_keys(st, codebook, "cpu")
    q = torch.randn(bs, 1, H * G, 128, generator=g).to(torch.bfloat16)
    q_avg = q[:, 0].view(bs, H, G, 128).mean(dim=2)
    q_blocks, q_norm = pc._encode_query_blocks(st, q_avg)
    with open(os.path.join(ref_root, RUNTIME, "turboquant/codebooks/codebook_d128_m8_Kr1_Kw256_rabitq_sign.json")) as f:
        signs_cb = torch.tensor(json.load(f)["angular_signs"], dtype=torch.int8)
    V_T = torch.where(signs_cb >= 0, 1, -1).to(torch.bfloat16).T.contiguous()       # [8, 256]
    scores = torch.matmul(q_blocks, V_T)                                             # [bs,H,16,256] bf16
    sorted_ids = scores.argsort(dim=-1, descending=True, stable=True)                # ties -> lower id
    sys.path.insert(0, os.path.join(ref_root, RUNTIME, "cache_hub/collision_fused"))
    import collision_test as ct  # noqa: E402  (imports only torch / triton at module level)
    coll = 0.25
    tiers = [0.05, 0.15, 0.30, 0.50, 0.75, 1.0]
    targets = [int(np.ceil(N * coll * r)) for r in tiers]
    cnt = ct.update_cache_cnt_overall_ref(sorted_ids, hist, codebook.to(torch.int32), tiers, N, coll)
    np.savez_compressed(
        os.path.join(out, "rabitq_encode.npz"), keys=bf16_bits(keys), signs=bf16_bits(signs),
        codes=codebook.permute(0, 1, 3, 2).contiguous().numpy(), weight=bf16_bits(weight.permute(0, 1, 3, 2)),
        packed=packed.permute(0, 1, 3, 2, 4).contiguous().numpy(), hist=hist.numpy(), q=bf16_bits(q),
        q_mean=bf16_bits(q_avg), q_blocks=bf16_bits(q_blocks), q_norm=bf16_bits(q_norm),
        bucket_scores=bf16_bits(scores), sorted_ids=sorted_ids.numpy().astype(np.int16),
        targets=np.array(targets, np.int64), cnt=cnt.numpy())
    # the collision reference's own generator (random orders / counts), seed 42
    sid, ckc, cb, tr, kv_len, cr = ct.generate_test_input(bs=1, kv_heads=8, B=16, num_clusters=256, kv_len=1024,
                                                          collision_ratio=0.2)
    cnt2 = ct.update_cache_cnt_overall_ref(sid, ckc, cb, tr, kv_len, cr)
    np.savez_compressed(
        os.path.join(out, "collision_ref.npz"), sorted_ids=sid.numpy().astype(np.int16), hist=ckc.numpy(),
        codes=cb.numpy().astype(np.uint8), targets=np.array([int(np.ceil(kv_len * r * cr)) for r in tr], np.int64),
        cnt=cnt2.numpy())


def gen_pariskv_schedule(pmod, out):
    """Drive ParisKV's own prefill / decode_update / _update_polar_index /
    get_region_indices (cache_hub/polar_cache.py:523-657, 837-853, 919-1065)
    on CPU tensors through a stub: 2 layers, batch 2, 2 KV heads; record the
    per-step state and the final retrieval codes and bucket counts."""
    pc = pmod.polar_cache
    L, bs, H, D = 2, 2, 2, 128
    sink, local, interval = 4, 40, 24
    prefill, steps, max_new = 150, 100, 120
    g = torch.Generator().manual_seed(77)
    T = prefill + steps
    layer_keys = [(torch.randn(bs, H, T, D, generator=g) * 1.5).to(torch.bfloat16) for _ in range(L)]
    vals = torch.randn(bs, H, T, D, generator=g).to(torch.bfloat16)
    torch.manual_seed(42)
    signs = torch.randint(0, 2, (128,), dtype=torch.bfloat16) * 2 - 1
    s = rabitq_stub(pmod, signs)
    cap = prefill + max_new
    s.layer_num, s.batch_size, s.kv_head, s.head_dim, s.dtype = L, bs, H, D, torch.bfloat16
    s.sink_size, s.local_size, s.steady_size = sink, local, sink + local
    s.dynamic_update_interval = interval
    s.input_length, s.max_new_length = prefill, max_new
    s.valid_start = [0, 0]
    s.enable_offload = True
    s.gpu_kv_capacity = sink + local + interval
    s.unified_keys_gpu = [torch.zeros(bs, H, s.gpu_kv_capacity, D, dtype=torch.bfloat16) for _ in range(L)]
    s.unified_values_gpu = [torch.zeros(bs, H, s.gpu_kv_capacity, D, dtype=torch.bfloat16) for _ in range(L)]
    s.unified_keys_cpu = [torch.zeros(bs, H, cap, D, dtype=torch.bfloat16) for _ in range(L)]
    s.unified_values_cpu = [torch.zeros(bs, H, cap, D, dtype=torch.bfloat16) for _ in range(L)]
    s._offload_keys_buffer = [torch.zeros(bs, H, interval, D, dtype=torch.bfloat16) for _ in range(L)]
    s._offload_values_buffer = [torch.zeros(bs, H, interval, D, dtype=torch.bfloat16) for _ in range(L)]
    s.codebook_gpu = [torch.zeros(bs, H, 16, cap, dtype=torch.uint8) for _ in range(L)]
    s.key_block_weight_gpu = [torch.zeros(bs, H, 16, cap, dtype=torch.bfloat16) for _ in range(L)]
    s.key_4bit_packed_gpu = [torch.zeros(bs, H, 16, cap, 4, dtype=torch.uint8) for _ in range(L)]
    s.cluster_key_counts_gpu = [torch.zeros(bs, H, 16, 256, dtype=torch.int32) for _ in range(L)]
    s.cpu_valid_end = [0] * L
    s._inflight_offload_buffers = [None] * L
    s._layer_offload_inflight = [False] * L
    s._main_events = [_Ev() for _ in range(L)]
    s._copy_events = [_Ev() for _ in range(L)]
    s._copy_stream = None
    s.current_seq_len = [0] * L
    s.context = 0
    s._decode_step_counter = 0
    s.final_topk = 100
    s.device = torch.device("cpu")
    s._actual_retrieval_length = max(sink, prefill - local) - sink   # skips the pinned-buffer allocation
    for name in ("batch_encode", "_count_cluster_keys", "_compute_local_start", "get_region_indices",
                 "_update_polar_index", "decode_update_kv_cache", "_sync_layer_offload", "_prefill_lockstep_batch"):
        setattr(s, name, functools.partial(getattr(pc, name), s))
    s._sync_offload_copies = lambda: None
    for l in range(L):
        s._prefill_lockstep_batch(layer_keys[l][:, :, :prefill].transpose(1, 2).contiguous(),
                                  vals[:, :, :prefill].transpose(1, 2).contiguous(), l)
    trace = []
    for t in range(steps):
        pos = prefill + t
        for l in range(L):
            s.decode_update_kv_cache(layer_keys[l][:, :, pos:pos + 1].transpose(1, 2).contiguous(),
                                     vals[:, :, pos:pos + 1].transpose(1, 2).contiguous(), l)
            reg = s.get_region_indices(l)
            trace.append([t, l, int(reg["total_len"]), int(reg["retrieval_length"]), int(reg["local_len"]),
                          int(s.cpu_valid_end[l]), int(s._actual_retrieval_length)])
    n = s._actual_retrieval_length
    np.savez_compressed(
        os.path.join(out, "pariskv_schedule.npz"),
        keys=np.stack([bf16_bits(k) for k in layer_keys]), values=bf16_bits(vals), signs=bf16_bits(signs),
        trace=np.array(trace, np.int64), params=np.array([L, bs, H, sink, local, interval, prefill, steps, max_new]),
        codes=np.stack([s.codebook_gpu[l][:, :, :, sink:sink + n].permute(0, 1, 3, 2).contiguous().numpy()
                        for l in range(L)]),
        weight=np.stack([bf16_bits(s.key_block_weight_gpu[l][:, :, :, sink:sink + n].permute(0, 1, 3, 2))
                         for l in range(L)]),
        packed=np.stack([s.key_4bit_packed_gpu[l][:, :, :, sink:sink + n].permute(0, 1, 3, 2, 4).contiguous().numpy()
                         for l in range(L)]),
        hist=np.stack([s.cluster_key_counts_gpu[l].numpy() for l in range(L)]))


def gen_rerank4(ref_root, out):
    """Sequential-bf16 RaBitQ rerank scores from the reference's own test."""
    sys.path.insert(0, os.path.join(ref_root, RUNTIME, "cache_hub/rerank"))
    import test_rerank_topk as tr  # noqa: E402
    cases = {}
    for i, (seed, kv_len, cand) in enumerate([(42, 256, 64), (77, 1024, 256), (999, 512, 512)]):
        ci, k4, kw, qb, qn, mc = tr.make_inputs(1, 2, 16, 8, kv_len, cand, "cpu", seed=seed)
        sc = tr.python_rabitq_scores(ci, k4, kw, qb, qn, mc, 16, 8)
        cases.update({f"c{i}_cand": ci.numpy(), f"c{i}_packed": k4.permute(0, 1, 3, 2, 4).contiguous().numpy(),
                      f"c{i}_weight": bf16_bits(kw.permute(0, 1, 3, 2)), f"c{i}_q_blocks": bf16_bits(qb),
                      f"c{i}_q_norm": bf16_bits(qn), f"c{i}_scores": bf16_bits(sc)})
    cases["centers"] = bf16_bits(mc)
    np.savez_compressed(os.path.join(out, "rerank4.npz"), **cases)


def main():
    ap = argparse.ArgumentParser()
    # the reference checkout: ZKV_REFERENCE_ROOT, else a sibling directory of
    # the repository named "reference"
    repo = os.path.dirname(os.path.dirname(HERE))
    ap.add_argument("--ref", default=os.environ.get("ZKV_REFERENCE_ROOT") or
                    os.path.join(os.path.dirname(repo), "reference"))
    ap.add_argument("--out", default=HERE)
    a = ap.parse_args()
    sys.path.insert(0, os.path.join(a.ref, RUNTIME))
    torch.set_num_threads(1)
    import cache_hub.polar_cache_quest_density_single_layer_kivi as zmod
    gen_encode(zmod, a.out)
    gen_pack(a.out)
    gen_kivi_qk(a.out)
    gen_quest_density(zmod, a.out)
    gen_lse(a.out)
    gen_host_logic(zmod, a.out)
    gen_schedule(zmod, a.out)
    import cache_hub.polar_cache as pmod
    gen_rabitq(pmod, a.ref, a.out)
    gen_pariskv_schedule(pmod, a.out)
    gen_rerank4(a.ref, a.out)
    print("golden fixtures written to", a.out)


if __name__ == "__main__":
    main()
