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

B200 layout: one absolute-position K/V buffer per layer in HBM by default
(`cpu_valid_end` keeps its bookkeeping meaning); with ZKV_HOST_RETRIEVAL=1
the raw retrieval rows live in host-pinned memory, as the reference keeps
them, and the final rows are gathered over the host link (zkv_h2d_gather_kv)
into an HBM window before attention.  The retrieval
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
        # offload tier (env ZKV_HOST_RETRIEVAL=1, with enable_offload): the raw
        # retrieval rows live in host-pinned memory (`keys` / `values`,
        # absolute positions); HBM keeps the codes and one window per layer
        # [sink | staging | near], the near part from the end of the
        # retrieval zone on (encoding is per token, so that is also the local
        # start).  compute() gathers the final rows into the staging rows.
        self.host_tier = os.environ.get("ZKV_HOST_RETRIEVAL", "0") in ("1", "true", "True", "yes", "on")
        if self.host_tier and not enable_offload:
            raise ValueError("ZKV_HOST_RETRIEVAL=1 needs enable_offload=True (the offload zone bookkeeping)")
        min_total = max(full_attention_threshold, sink_size + local_size + final_topk * 2)
        self._stage = min(cap, max(final_topk, min_total))
        self._near_cap = local_size + self.dynamic_update_interval + 8
        self.win_k, self.win_v, self.win_base = [], [], [sink_size] * layer_num
        self.keys, self.values, self.layouts = [], [], []
        for l in range(layer_num):
            d = devs[l]
            if self.host_tier:
                self.keys.append(torch.zeros(bs, H, cap, D, dtype=torch.bfloat16, pin_memory=True))
                self.values.append(torch.zeros(bs, H, cap, D, dtype=torch.bfloat16, pin_memory=True))
                W = sink_size + self._stage + self._near_cap
                self.win_k.append(torch.zeros(bs, H, W, D, dtype=torch.bfloat16, device=d))
                self.win_v.append(torch.zeros(bs, H, W, D, dtype=torch.bfloat16, device=d))
            else:
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

    def _encode(self, l: int, tok_lo: int, tok_hi: int, src=None) -> None:
        """Retrieval codes of tokens [tok_lo, tok_hi) (absolute) of layer l,
        added to the bucket histogram (batch_encode + _count_cluster_keys).
        src: the keys of exactly those tokens when they are not read from the
        HBM cache (offload tier)."""
        if tok_hi <= tok_lo:
            return
        k = self.keys[l][:, :, tok_lo:tok_hi] if src is None else src   # [bs, H, n, 128]
        ops.rq_encode(k, self._signs(k.device), self.layouts[l], tok_start=tok_lo)

    def _win_slot(self, l: int, pos: int) -> int:
        """Window row of absolute position pos (offload tier)."""
        s = self.sink_size
        if pos < s:
            return pos
        j = pos - self.win_base[l]
        if j < 0 or j >= self._near_cap:
            raise RuntimeError(f"position {pos} is outside the near window of layer {l}")
        return s + self._stage + j

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
        kk, vv = key_states[:, vs:].transpose(1, 2), value_states[:, vs:].transpose(1, 2)
        retrieval_start = self.sink_size
        retrieval_end = max(retrieval_start, n - self.local_size)
        retrieval = retrieval_end - retrieval_start
        if self.host_tier:
            s = self.sink_size
            ns = min(s, n)
            self.win_k[l][:, :, :ns].copy_(kk[:, :, :ns])
            self.win_v[l][:, :, :ns].copy_(vv[:, :, :ns])
            if retrieval > 0:
                self.keys[l][:, :, s:retrieval_end].copy_(kk[:, :, s:retrieval_end])
                self.values[l][:, :, s:retrieval_end].copy_(vv[:, :, s:retrieval_end])
            base = max(s, retrieval_end)
            m = max(0, n - base)
            if m > self._near_cap:
                raise RuntimeError(f"prefill leaves {m} near tokens; the window holds {self._near_cap}")
            off = s + self._stage
            self.win_k[l][:, :, off:off + m].copy_(kk[:, :, base:base + m])
            self.win_v[l][:, :, off:off + m].copy_(vv[:, :, base:base + m])
            self.win_base[l] = base
        else:
            self.keys[l][:, :, :n].copy_(kk)
            self.values[l][:, :, :n].copy_(vv)
        if self._actual_retrieval_length is None:
            self._actual_retrieval_length = retrieval
        self.current_seq_len[l] = n
        if retrieval > 0:
            self._encode(l, retrieval_start, retrieval_end,
                         src=kk[:, :, retrieval_start:retrieval_end].contiguous() if self.host_tier else None)
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
            if self.host_tier:
                # the window starts at old_end: encode from it, move the rows to
                # the host zone, slide the window to new_end
                off, total = self.sink_size + self._stage, self.current_seq_len[l]
                wk, wv = self.win_k[l], self.win_v[l]
                self._encode(l, old_end, new_end, src=wk[:, :, off:off + num])
                self.keys[l][:, :, old_end:new_end].copy_(wk[:, :, off:off + num])
                self.values[l][:, :, old_end:new_end].copy_(wv[:, :, off:off + num])
                m = total - new_end
                if m > 0:
                    wk[:, :, off:off + m].copy_(wk[:, :, off + num:off + num + m].clone())
                    wv[:, :, off:off + m].copy_(wv[:, :, off + num:off + num + m].clone())
                self.win_base[l] = new_end
            else:
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
        if self.host_tier:
            w = self._win_slot(layer_idx, current)
            self.win_k[layer_idx][:, :, w].copy_(key_states[:, 0])
            self.win_v[layer_idx][:, :, w].copy_(value_states[:, 0])
        else:
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
            if self.host_tier:
                s, base = self.sink_size, self.win_base[l]
                n_h = max(0, base - s) if total > s else 0
                if n_h > self._stage:
                    raise RuntimeError(f"full attention over {n_h} host rows exceeds the {self._stage} staging rows")
                if n_h > 0:
                    ar = torch.arange(n_h, dtype=torch.int64, device=dev).expand(self.batch_size, self.kv_head, n_h)
                    ops.h2d_gather_rows(self.keys[l], self.values[l], ar, self.win_k[l], self.win_v[l], src_offset=s,
                                        dst_offset=s, status=status)
                off = s + self._stage
                return ops.attn_rows(q, self.win_k[l], self.win_v[l], seg0=(0, min(total, s) + n_h),
                                     seg1=(off, off + max(0, total - base)), status=status)
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
        if self.host_tier:  # the F final rows come over the host link into the staging rows
            s, base = self.sink_size, self.win_base[l]
            ops.h2d_gather_rows(self.keys[l], self.values[l], final.view(bs, self.kv_head, F), self.win_k[l],
                                self.win_v[l], src_offset=s, dst_offset=s, status=status)
            off = s + self._stage
            return ops.attn_rows(q, self.win_k[l], self.win_v[l], seg0=(0, s + F),
                                 seg1=(off + local_start - base, off + total - base), status=status)
        return ops.attn_rows(q, self.keys[l], self.values[l], seg0=(0, min(self.sink_size, total)),
                             sel=final.view(bs, self.kv_head, F), sel_offset=self.sink_size,
                             seg1=(local_start, total), status=status)
