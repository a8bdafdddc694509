"""Drop-in ParisKV `polar_cache` (RaBitQ / polar-ANN retrieval) on the
libzkv sm_100a kernels.

Load it the way the reference's decode loop loads a cache backend
(model_hub/qwen.py:336-350):

    POLAR_CACHE_MODULE=zoomkv_revision_b200.pariskv_cache

It restates `cache_hub/polar_cache.py` (referred to as REF below; paths
relative to runtime/zoomkv_urania_runtime_20261011/):

  * same constructor keywords (REF:135-190), methods
    prefill_update_kv_cache / sync / decode_update_kv_cache / compute /
    get_region_indices and the `context` attribute;
  * same zones and flush schedule: sink | retrieval (encoded, offloaded in
    the reference) | local + update buffer; layer 0 flushes once the near
    zone holds local + interval tokens, encoding the oldest tokens into the
    retrieval index (REF:1044-1065, 919-1042, 837-857);
  * the retrieval step of `compute` (REF:1230-1415, 1528-1832): GQA-mean
    query, SRHT blocks, 6-tier collision counts from the bucket order of
    q . V (get_cache_cnt_fused), top `ceil(N * candidate_ratio)` candidates,
    4-bit RaBitQ rerank to `final_topk`, attention over sink + selected +
    local tokens, with the adaptive ratios of `_get_adaptive_ratios`
    (REF:1457-1525) and its POLAR_* overrides.

B200 layout: one absolute-position K/V buffer per layer in HBM (no host
offload; `cpu_valid_end` keeps its bookkeeping meaning) and the retrieval
codes token-major ([rows, cap, 16]) so the candidate gather reads 64 + 32
contiguous bytes per key.  Selections break ties by the lower index; the
reference's torch.topk / radix top-k leave ties unspecified.
"""
from __future__ import annotations

import json
import math
import os
import types

import torch

from . import ops

# collision tiers: fraction of the collision budget per tier (REF:1707-1712)
_TIERS = (0.05, 0.15, 0.30, 0.50, 0.75, 1.0)


def _adaptive_ratios(retrieval_len: int):
    """(candidate_ratio, collision_ratio) by retrieval length, with the
    reference's environment overrides (REF:1321-1330, 1457-1525)."""
    e = os.environ
    fixed = e.get("POLAR_FIXED_CANDIDATE_RATIO", "")
    if fixed:
        return float(fixed), float(fixed)
    dyn = e.get("POLAR_ADAPTIVE_DYNAMIC_CAND_RATIOS", "").strip()
    if dyn:
        ratios = [float(x) for x in dyn.split(",") if x.strip()]
        th = [int(x) for x in e.get("POLAR_ADAPTIVE_DYNAMIC_CAND_THRESHOLDS", "5000,10000").split(",") if x.strip()]
        if len(ratios) != len(th) + 1:
            raise ValueError("POLAR_ADAPTIVE_DYNAMIC_CAND_RATIOS must have exactly one more value than "
                             "POLAR_ADAPTIVE_DYNAMIC_CAND_THRESHOLDS")
        idx = 0
        while idx < len(th) and retrieval_len >= th[idx]:
            idx += 1
        cand = coll = ratios[idx]
        coll_env = e.get("POLAR_ADAPTIVE_DYNAMIC_COLL_RATIOS", "").strip()
        if coll_env:
            coll_r = [float(x) for x in coll_env.split(",") if x.strip()]
            if len(coll_r) != len(ratios):
                raise ValueError("POLAR_ADAPTIVE_DYNAMIC_COLL_RATIOS must match POLAR_ADAPTIVE_DYNAMIC_CAND_RATIOS length")
            coll = coll_r[idx]
    elif retrieval_len < 5000:
        cand, coll = 0.5, 0.5
    elif retrieval_len < 10000:
        cand, coll = 0.25, 0.3
    elif retrieval_len < 30000:
        cand, coll = 0.2, 0.25
    else:
        cand, coll = 0.12, 0.2
    if e.get("POLAR_ADAPTIVE_FORCE_CANDIDATE_RATIO") is not None:
        cand = float(e["POLAR_ADAPTIVE_FORCE_CANDIDATE_RATIO"])
    if e.get("POLAR_ADAPTIVE_FORCE_COLLISION_RATIO") is not None:
        coll = float(e["POLAR_ADAPTIVE_FORCE_COLLISION_RATIO"])
    return cand, coll


def srht_signs(device) -> torch.Tensor:
    """The SRHT diagonal of the reference quantizer: seed 42, randint(0, 2) on
    `device`, as +-1 bf16, leaving the caller's RNG state untouched (REF:79-90)."""
    cpu_state = torch.get_rng_state()
    cuda_state = torch.cuda.get_rng_state(device) if torch.device(device).type == "cuda" else None
    torch.manual_seed(42)
    try:
        s = torch.randint(0, 2, (128,), device=device, dtype=torch.bfloat16) * 2 - 1
    finally:
        torch.set_rng_state(cpu_state)
        if cuda_state is not None:
            torch.cuda.set_rng_state(cuda_state, device)
    return s


def _check_codebook(path: str) -> None:
    """The kernels use the 256 LSB-first sign patterns of 8 dims as the bucket
    codebook; a codebook file, when present, must be exactly that."""
    if not path or not os.path.exists(path):
        return
    with open(path) as f:
        cb = json.load(f)
    cfg = cb.get("config", {})
    if (cfg.get("d"), cfg.get("m"), cfg.get("K_omega")) != (128, 8, 256):
        raise ValueError(f"codebook {path}: this build implements d=128, m=8, K_omega=256")
    signs = cb.get("angular_signs") or cb.get("angular_centers")
    for k, row in enumerate(signs):
        if sum((1 << j) for j, v in enumerate(row) if v >= 0) != k:
            raise ValueError(f"codebook {path}: entry {k} is not the LSB-first sign pattern of {k}")


class polar_cache:
    """ParisKV RaBitQ retrieval cache (see module docstring)."""

    def __init__(self, valid_start, layer_num: int, batch_size: int, max_length: int, num_key_value_heads: int,
                 num_heads: int, head_dim: int, dtype: torch.dtype, layer_mapping: dict, max_new_length: int,
                 sink_size: int, local_size: int, core: int = 0, nprobe: int = 0, cache_unit_size: int = 0,
                 cache_cluster_num: int = 0, num_gpus: int = 1, model_size: int = 0, codebook_path: str = "",
                 collision_ratio: float = 0.3, candidate_ratio: float = 0.05, final_topk: int = 100,
                 dynamic_update_interval: int = 512, full_attention_threshold: int = 2000, enable_offload: bool = True,
                 **ablation_flags) -> None:
        del core, nprobe, cache_unit_size, cache_cluster_num, ablation_flags
        if head_dim != 128:
            raise ValueError(f"head_dim={head_dim}: the kernels implement head_dim 128")
        if dtype != torch.bfloat16:
            raise ValueError(f"dtype={dtype}: the cache stores bf16")
        _check_codebook(codebook_path)
        self.layer_num, self.batch_size, self.max_length = layer_num, batch_size, max_length
        self.kv_head, self.num_heads, self.head_dim, self.dtype = num_key_value_heads, num_heads, head_dim, dtype
        self.layer_mapping, self.num_gpus, self.model_size = layer_mapping, num_gpus, model_size
        self.valid_start = valid_start
        self.sink_size, self.local_size = sink_size, local_size
        self.steady_size = sink_size + local_size
        self.dynamic_update_interval = dynamic_update_interval if dynamic_update_interval is not None else local_size
        self.group_size = num_heads // num_key_value_heads
        self.max_new_length = max_new_length
        self.input_length = max_length - max_new_length
        self.FULL_ATTENTION_THRESHOLD = full_attention_threshold
        self.collision_ratio, self.candidate_ratio, self.final_topk = collision_ratio, candidate_ratio, final_topk
        self.enable_offload = enable_offload
        self.current_seq_len = [0] * layer_num
        self.cpu_valid_end = [0] * layer_num
        self._actual_retrieval_length = None
        self._decode_step_counter = 0
        self.context = 0
        devs = [torch.device(layer_mapping[str(l)]) if isinstance(layer_mapping, dict) and str(l) in layer_mapping
                else torch.device("cuda", torch.cuda.current_device()) for l in range(layer_num)]
        self._layer_dev = devs
        self.device = devs[0]
        self.quantizer = types.SimpleNamespace(srht_diagonal_signs=[srht_signs(self.device)], B=16, m=8)
        bs, H, D, cap = batch_size, num_key_value_heads, head_dim, max_length
        self.keys, self.values, self.layouts = [], [], []
        for l in range(layer_num):
            d = devs[l]
            self.keys.append(torch.zeros(bs, H, cap, D, dtype=torch.bfloat16, device=d))
            self.values.append(torch.zeros(bs, H, cap, D, dtype=torch.bfloat16, device=d))
            self.layouts.append(ops.RqLayout.alloc(bs * H, cap, d))
        self._centers = {d: torch.tensor(ops.MAG_CENTERS, dtype=torch.bfloat16, device=d) for d in set(devs)}
        self._status = {d: torch.zeros(1, dtype=torch.int32, device=d) for d in set(devs)}
        self._last_topk_indices = None

    # ------------------------------------------------------------------ helpers
    def _signs(self, dev):
        s = self.quantizer.srht_diagonal_signs[0]
        return s if s.device == dev else s.to(dev)

    def _encode(self, l: int, tok_lo: int, tok_hi: int) -> None:
        """Retrieval codes of tokens [tok_lo, tok_hi) (absolute) of layer l,
        added to the bucket histogram (batch_encode + _count_cluster_keys)."""
        if tok_hi <= tok_lo:
            return
        k = self.keys[l][:, :, tok_lo:tok_hi]   # [bs, H, n, 128] view of the absolute buffer
        ops.rq_encode(k, self._signs(k.device), self.layouts[l], tok_start=tok_lo)

    def get_region_indices(self, layer_idx, device=None):
        """REF:837-853: zones from the committed retrieval boundary."""
        device = self._layer_dev[layer_idx] if device is None else device
        total = self.current_seq_len[layer_idx]
        retrieval = self.cpu_valid_end[layer_idx]
        sink_end = min(self.sink_size, total)
        local_start = min(total, self.sink_size + retrieval)
        return {"sink_indices": torch.arange(sink_end, device=device, dtype=torch.long),
                "local_indices": torch.arange(local_start, total, device=device, dtype=torch.long),
                "retrieval_start": self.sink_size, "retrieval_length": retrieval, "total_len": total,
                "local_len": total - local_start}

    def _compute_local_start(self, layer_idx=0):
        return max(self.sink_size, self.current_seq_len[layer_idx] - self.local_size)

    # ------------------------------------------------------------------ prefill / decode
    def prefill_update_kv_cache(self, query_states, key_states, value_states, layer_idx, batch_idx):
        """REF:503-657 (lockstep batch): k/v [bs, T, H, D]."""
        del query_states
        bsz = key_states.shape[0]
        vs = int(self.valid_start[0]) if hasattr(self.valid_start, "__len__") else int(self.valid_start)
        if bsz != self.batch_size:
            raise NotImplementedError("this build implements the lockstep prefill (bsz == batch_size)")
        if hasattr(self.valid_start, "__len__") and any(int(v) != vs for v in list(self.valid_start)[:bsz]):
            raise ValueError("lockstep prefill requires the same valid_start across the batch")
        if bsz > 1 and batch_idx != 0:
            return key_states[:, vs:], value_states[:, vs:]
        l = layer_idx
        seq_len = key_states.shape[1]
        n = seq_len - vs
        self.keys[l][:, :, :n].copy_(key_states[:, vs:].transpose(1, 2))
        self.values[l][:, :, :n].copy_(value_states[:, vs:].transpose(1, 2))
        retrieval_start = self.sink_size
        retrieval_end = max(retrieval_start, n - self.local_size)
        retrieval = retrieval_end - retrieval_start
        if self._actual_retrieval_length is None:
            self._actual_retrieval_length = retrieval
        self.current_seq_len[l] = n
        if retrieval > 0:
            self._encode(l, retrieval_start, retrieval_end)
            self.cpu_valid_end[l] = retrieval
        if l == self.layer_num - 1:
            self.context += n
        return key_states[:, vs:], value_states[:, vs:]

    def sync(self, layer_idx, batch_idx):
        """REF:2375-2379: nothing is in flight on a side stream in this build."""
        return None

    def _update_polar_index(self) -> None:
        """REF:919-1042: encode the oldest near-zone tokens into the index."""
        new_end = self._compute_local_start(0)
        old_end = self._actual_retrieval_length + self.sink_size
        num = new_end - old_end
        assert num > 0, f"flush of {num} tokens"
        self._actual_retrieval_length = new_end - self.sink_size
        for l in range(self.layer_num):
            self._encode(l, old_end, new_end)
            self.cpu_valid_end[l] += num
        self.steady_size = self.sink_size + self.local_size

    def decode_update_kv_cache(self, key_states, value_states, layer_idx):
        """REF:1044-1065: flush a full buffer (layer 0), then append one token."""
        current = self.current_seq_len[layer_idx]
        if layer_idx == 0 and self._actual_retrieval_length is not None:
            near = current - min(self.sink_size, current) - self.cpu_valid_end[0]
            if near >= self.local_size + self.dynamic_update_interval:
                assert all(c == current for c in self.current_seq_len)
                self._update_polar_index()
        if current >= self.max_length:
            raise RuntimeError(f"cache full ({self.max_length} tokens)")
        self.keys[layer_idx][:, :, current].copy_(key_states[:, 0])
        self.values[layer_idx][:, :, current].copy_(value_states[:, 0])
        self.current_seq_len[layer_idx] = current + 1
        if layer_idx == 0:
            self._decode_step_counter += 1
        if layer_idx == self.layer_num - 1:
            self.context += 1
        return None, None

    # ------------------------------------------------------------------ decode attention
    def compute(self, queries, layer_idx):
        """REF:1230-1415: queries [bs, 1, num_heads, 128] -> same shape."""
        l = layer_idx
        dev = self._layer_dev[l]
        total = self.current_seq_len[l]
        valid = self.cpu_valid_end[l]
        q = queries if queries.is_contiguous() else queries.contiguous()
        status = self._status[dev]
        min_total = max(self.FULL_ATTENTION_THRESHOLD, self.sink_size + self.local_size + self.final_topk * 2)
        if total < min_total or valid <= 0:
            return ops.attn_rows(q, self.keys[l], self.values[l], seg0=(0, total), status=status)
        cand_ratio, coll_ratio = _adaptive_ratios(valid)
        C = max(1, int(math.ceil(valid * cand_ratio)))
        C = min(C, valid)
        qe = ops.rq_query(q, self._signs(dev), self.group_size)
        lay = self.layouts[l].tokens(self.sink_size)
        cand = ops.collision_topk(qe["q_blocks"], lay, valid, ops.tier_targets(valid, coll_ratio, _TIERS), C)
        F = min(self.final_topk, C)
        _, final = ops.partial_rerank_cuda(cand, lay, qe["q_blocks"], qe["q_norm"], self._centers[dev], final_topk=F)
        self._last_topk_indices = final
        local_start = min(total, self.sink_size + valid)
        bs = self.batch_size
        return ops.attn_rows(q, self.keys[l], self.values[l], seg0=(0, min(self.sink_size, total)),
                             sel=final.view(bs, self.kv_head, F), sel_offset=self.sink_size,
                             seg1=(local_start, total), status=status)
