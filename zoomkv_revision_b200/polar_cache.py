"""Drop-in ZoomKV `polar_cache`: HBM-resident KV cache + sparse decode attention
on the libzkv sm_100a kernels.

Load it the way the reference's decode loop loads its cache backend
(model_hub/qwen.py:336-350 imports `POLAR_CACHE_MODULE` and instantiates
`polar_cache(**kwargs)`):

    POLAR_CACHE_MODULE=zoomkv_revision_b200.polar_cache

It restates `cache_hub/polar_cache_quest_density_single_layer_kivi.py`
(referred to as REF below; paths relative to
runtime/zoomkv_urania_runtime_20261011/):

  * same constructor keywords (REF:106-139), same methods
    prefill_update_kv_cache / sync / decode_update_kv_cache / compute /
    get_region_indices and the `context` attribute;
  * same zones (sink | retrieval | near = local + update buffer), same flush
    schedule (layer 0 flushes once the near zone holds local + interval
    tokens, REF:1527-1540, 1379-1512), same carry / skipped-tail semantics
    (REF:2025-2157, 1895-1925), same candidate budget (REF:1798-1880) and the
    same POLAR_* environment knobs;
  * `compute` runs the production retrieval pipeline (REF:1589-1775,
    2688-2779): Quest chunk scores -> top-nk chunks -> CDS density classify
    -> KIVI stage-2 per-chunk top-k -> global top-k + skipped tail ->
    attention over sink + selected + near tokens.

B200 layout: every layer keeps ONE absolute-position K/V buffer in HBM
(180 GB makes the reference's CPU-pinned retrieval zone unnecessary), so a
flush only encodes the newly completed chunks in place -- no D2H copy and no
local-window slide; the reference's offload bookkeeping (`cpu_valid_end`)
is kept so zone boundaries are identical.  The `enable_offload` keyword is
accepted and selects that bookkeeping.

Offload tier (env ZKV_HOST_RETRIEVAL=1, reference attention mode, with
enable_offload=True): for contexts beyond HBM the raw rows of the retrieval
zone live in host-pinned memory (`keys` / `values`, absolute positions),
as in the reference (REF:519-611).  HBM keeps one window per layer
(`win_k` / `win_v`): [sink | staging | near], the near part holding every
token from the first unencoded chunk on.  A flush copies the rows that join
the retrieval zone to the host, encodes the completed chunks from the
window and slides it (REF:1379-1512); compute() gathers the selected rows
from the host into the staging rows (zkv_h2d_gather_kv, the replacement of
trans_h2d.cu) and attends [sink + staged] and the near rows of the window.
The chunk metadata and KIVI codes stay in HBM.

Attention modes (env ZKV_ATTENTION_MODE):
  "reference" (default)  the production chain: Quest -> CDS -> KIVI stage 2
                         -> top final_topk tokens, attention over the raw bf16
                         rows of the selected tokens, as the reference does;
  "page"                 the reference's page mode (dense_topk = sparse_topk =
                         16, final_topk = the page budget): Quest top-nk
                         chunks, attention over their raw bf16 rows + sink +
                         near rows: zkv_page_decode_raw, four launches per
                         layer chained by programmatic dependent launch;
  "page4"                a lossy variant of page mode: the selected pages are
                         read as 4-bit KIVI keys and 4-bit values (group 32),
                         dequantised in registers (zkv_page_decode).

Chunk size: this build implements the production chunk of 16 tokens
(POLAR_QUEST_CHUNK=16, run/eval_math_aime.py:216); any other value raises.
"""
from __future__ import annotations

import math
import os
from typing import Optional

import torch

from . import ops

CHUNK = 16
_TRUE = ("1", "true", "True", "yes", "on")


# --------------------------------------------------------------------------- configuration
def env_config(final_topk: int = 100) -> dict:
    """The POLAR_* knobs the reference reads in __init__ (REF:186-430), with the
    reference's defaults.  ZoomKV production values are set by
    run/eval_math_aime.py:212-236 (apply_zoomkv_env)."""
    e = os.environ
    chunk = int(e.get("POLAR_QUEST_CHUNK", str(CHUNK)))
    cfg = dict(
        chunk=chunk,
        cand_ratio=float(e.get("POLAR_QUEST_CAND_RATIO", "0.05")),
        dynamic=e.get("POLAR_QUEST_DYNAMIC_CAND_RATIO", "0") not in ("0", "false", "False", ""),
        thresholds=[5000, 10000],
        ratios=[0.7, 0.5, 0.4],
        force_cand_tokens=int(e["POLAR_FORCE_CAND_TOKENS"]) if e.get("POLAR_FORCE_CAND_TOKENS") else None,
        dense_ratio=float(e.get("POLAR_CDS_DENSE_RATIO", "0.1")),
        dense_topk=int(e.get("POLAR_CDS_DENSE_TOPK", "16")),
        sparse_topk=int(e.get("POLAR_CDS_SPARSE_TOPK", "8")),
        max_skipped=int(e.get("POLAR_MAX_SKIPPED_INDICES", "512")),
        kivi_bits=int(e.get("POLAR_KIVI_BITS", "4")),
        stage1=e.get("POLAR_QUEST_STAGE1", "1") not in ("0", "false", "False", ""),
        attention_mode=e.get("ZKV_ATTENTION_MODE", "reference").strip().lower(),
        host_retrieval=e.get("ZKV_HOST_RETRIEVAL", "0") in _TRUE,
        # hierarchical Quest knobs of the separate-kernel cache (its :210-237);
        # off here, as in the single-layer cache this drop-in mirrors
        hierarchical=e.get("POLAR_QUEST_HIERARCHICAL", "0") not in ("0", "false", "False", ""),
        large_chunk=int(e.get("POLAR_QUEST_LARGE_CHUNK", "256")),
        large_ratio=float(e.get("POLAR_QUEST_LARGE_RATIO", "0.3")),
        small_ratio=float(e.get("POLAR_QUEST_SMALL_RATIO", "0.3")),
    )
    if cfg["dynamic"]:
        try:
            th = [int(x) for x in e.get("POLAR_QUEST_DYNAMIC_CAND_THRESHOLDS", "5000,10000").split(",") if x.strip()]
            ra = [float(x) for x in e.get("POLAR_QUEST_DYNAMIC_CAND_RATIOS", "0.7,0.5,0.4").split(",") if x.strip()]
            if len(ra) != len(th) + 1:
                raise ValueError("need len(ratios) == len(thresholds) + 1")
            cfg["thresholds"], cfg["ratios"] = th, ra
        except ValueError:
            # REF:220-234: invalid dynamic config falls back to the fixed ratio
            cfg["dynamic"] = False
    if cfg["chunk"] != CHUNK:
        raise ValueError(f"POLAR_QUEST_CHUNK={cfg['chunk']}: this build implements chunk 16 only")
    if cfg["kivi_bits"] != 4:
        raise ValueError(f"POLAR_KIVI_BITS={cfg['kivi_bits']}: this build implements 4-bit KIVI only")
    if cfg["attention_mode"] not in ("reference", "page", "page4"):
        raise ValueError(f"ZKV_ATTENTION_MODE must be 'reference', 'page' or 'page4'; got {cfg['attention_mode']!r}")
    if cfg["hierarchical"]:
        if cfg["large_chunk"] % cfg["chunk"] or not 1 <= cfg["large_chunk"] // cfg["chunk"] <= 16:
            raise ValueError(f"POLAR_QUEST_LARGE_CHUNK={cfg['large_chunk']}: must be 16..256 in multiples of 16")
        if cfg["attention_mode"] != "page":
            raise ValueError("POLAR_QUEST_HIERARCHICAL=1 serves ZKV_ATTENTION_MODE=page")
    return cfg


def hier_plan(n_chunks: int, factor: int, large_ratio: float, small_ratio: float):
    """(n_large, nk_large, nk_small) of the hierarchical branch of
    _refresh_quest_chunk_cache (separate-kernel cache :1462-1468)."""
    n_large = n_chunks // factor
    if n_large <= 0:
        return 0, 0, 0
    nk_large = min(max(1, int(math.ceil(n_large * large_ratio))), n_large)
    nk_sub = nk_large * factor
    nk_small = min(max(1, int(math.ceil(nk_sub * small_ratio))), nk_sub)
    return n_large, nk_large, nk_small


# --------------------------------------------------------------------------- host logic (CPU-testable)
def quest_candidate_ratio(kv_len: int, cfg: dict) -> float:
    """REF:1818-1825 (_quest_candidate_ratio)."""
    if not cfg["dynamic"]:
        return cfg["cand_ratio"]
    for threshold, ratio in zip(cfg["thresholds"], cfg["ratios"]):
        if kv_len < threshold:
            return ratio
    return cfg["ratios"][-1]


def quest_aligned_candidate_tokens(kv_len: int, cfg: dict) -> int:
    """REF:1798-1815: ceil_to_chunk(ceil(ratio*kv_len)) (or the forced budget),
    clipped to the chunk-aligned retrieval length."""
    c = cfg["chunk"]
    if kv_len <= 0:
        return 0
    if kv_len < c:
        return kv_len
    cap = (kv_len // c) * c
    target = cfg["force_cand_tokens"] if cfg["force_cand_tokens"] is not None else \
        math.ceil(kv_len * quest_candidate_ratio(kv_len, cfg))
    target_aligned = max(c, ((target + c - 1) // c) * c)
    return min(cap, target_aligned)


def quest_chunk_plan(kv_len: int, cfg: dict):
    """(n_chunks, nk, n_dense, skipped) of _refresh_quest_chunk_cache /
    _refresh_live_skipped_indices (REF:1830-1880, 1895-1916)."""
    c = cfg["chunk"]
    kv_len = max(0, int(kv_len))
    n_chunks = kv_len // c
    skipped = kv_len - n_chunks * c
    if skipped > cfg["max_skipped"]:
        raise RuntimeError(f"[chunk_minmax] live skipped indices overflow: kv_len={kv_len}, "
                           f"skipped={skipped} > MAX={cfg['max_skipped']}")
    if kv_len < c:
        return 0, 0, 0, skipped
    nk = max(1, min(n_chunks, quest_aligned_candidate_tokens(kv_len, cfg) // c))
    n_dense = max(1, int(nk * cfg["dense_ratio"]))
    return n_chunks, nk, n_dense, skipped


def compute_local_start(total_len: int, input_length: int, sink: int, local: int, interval: int) -> int:
    """REF:1262-1277 (_compute_local_start): start of the local window by the
    update-buffer arithmetic; the flush encodes up to here."""
    steady = sink + local
    if input_length >= steady:
        update = max(0, total_len - input_length) % interval
    elif total_len >= steady:
        update = (total_len - steady) % interval
    else:
        update = 0
    local_end = max(total_len - update, sink)
    return max(sink, local_end - local)


def region(total_len: int, cpu_len: Optional[int], input_length: int, sink: int, local: int, interval: int):
    """(retrieval_length, local_start, local_len) of get_region_indices
    (REF:1173-1259).  cpu_len = cpu_valid_end in offload bookkeeping, None
    for the all-GPU arithmetic."""
    if cpu_len is not None and cpu_len >= 0:
        retrieval_length = cpu_len
        local_start = sink + retrieval_length
        local_len = max(0, total_len - local_start)
    else:
        local_start = compute_local_start(total_len, input_length, sink, local, interval)
        retrieval_length = max(0, local_start - sink)
        local_len = total_len - local_start if local_start < total_len else 0
    return retrieval_length, local_start, local_len


def flush_due(current_len: int, sink: int, cpu_valid_end0: int, local: int, interval: int) -> bool:
    """REF:1527-1540: layer 0 flushes when the near zone holds local + interval."""
    near_len = current_len - min(sink, current_len) - cpu_valid_end0
    return near_len >= local + interval


class CacheSchedule:
    """Token bookkeeping of the cache, free of tensors (CPU-testable): zone
    lengths per layer, the offload boundary `cpu_valid_end`, the encoded
    retrieval length and the flush schedule, exactly as the reference keeps
    them (REF:880-1004 prefill zones, REF:1516-1583 decode append,
    REF:1379-1512 flush, REF:1830-1925 refresh)."""

    def __init__(self, layer_num, sink, local, interval, input_length, cfg, offload=True):
        self.layer_num, self.sink, self.local, self.interval = layer_num, sink, local, interval
        self.input_length, self.cfg, self.offload = input_length, cfg, offload
        self.current_seq_len = [0] * layer_num
        self.cpu_valid_end = [0] * layer_num if offload else None
        self.actual_retrieval = None
        self.plan = (0, 0, 0, 0)
        self.decode_steps = 0

    def prefill(self, layer, seq_len, valid_start):
        """Zones of a prefill of seq_len tokens with left padding valid_start.
        Returns (n_stored, retrieval_length, (enc_lo, enc_hi)) -- the encoded
        chunk-aligned retrieval range in zone coordinates."""
        n = seq_len - valid_start
        retrieval_length = max(0, (seq_len - self.local) - (valid_start + self.sink))
        if self.actual_retrieval is None:
            self.actual_retrieval = retrieval_length
            self.plan = quest_chunk_plan(retrieval_length, self.cfg)
        if self.cpu_valid_end is not None:
            self.cpu_valid_end[layer] = retrieval_length
        self.current_seq_len[layer] = n
        return n, retrieval_length, (0, (retrieval_length // CHUNK) * CHUNK)

    def flush_due(self, layer) -> bool:
        return self.cpu_valid_end is not None and layer == 0 and flush_due(
            self.current_seq_len[layer], self.sink, int(self.cpu_valid_end[0]), self.local, self.interval)

    def flush(self):
        """Extend the retrieval zone to the local start.  Returns
        (enc_lo, enc_hi, num_new): the chunk-aligned zone range to encode."""
        if any(n != self.current_seq_len[0] for n in self.current_seq_len):
            raise RuntimeError(f"cache flush requires all layer lengths to match: {self.current_seq_len}")
        new_end = compute_local_start(self.current_seq_len[0], self.input_length, self.sink, self.local,
                                      self.interval)
        old_end = self.actual_retrieval + self.sink
        num_new = new_end - old_end
        if num_new <= 0:
            raise AssertionError(f"num_new_tokens={num_new} <= 0")
        old_r, new_r = self.actual_retrieval, new_end - self.sink
        self.actual_retrieval = new_r
        self.plan = quest_chunk_plan(new_r, self.cfg)
        if self.cpu_valid_end is not None:
            self.cpu_valid_end = [int(c) + num_new for c in self.cpu_valid_end]
        return (old_r // CHUNK) * CHUNK, (new_r // CHUNK) * CHUNK, num_new

    def append(self, layer) -> int:
        """Position of this layer's new token; commits the step at the last layer."""
        pos = self.current_seq_len[layer]
        self.current_seq_len[layer] = pos + 1
        if layer == self.layer_num - 1:
            if any(n != self.current_seq_len[0] for n in self.current_seq_len):
                raise RuntimeError(f"decode step layer lengths diverged before cache commit: "
                                   f"{self.current_seq_len}")
            self.decode_steps += 1
        return pos

    def region(self, layer):
        cpu_len = int(self.cpu_valid_end[layer]) if self.cpu_valid_end is not None else None
        return region(self.current_seq_len[layer], cpu_len, self.input_length, self.sink, self.local, self.interval)


def offload_window(sink: int, local: int, interval: int, final_topk: int, max_skipped: int, threshold: int,
                   cap: int):
    """(stage, near_cap) of the offload tier's HBM window [sink | stage |
    near]: stage rows hold the gathered selection (final_topk + skipped) or,
    below the retrieval threshold, every host row; the near part holds every
    token from the first unencoded chunk on -- at most local + interval
    tokens of near zone plus a chunk's skipped tail plus the appended token."""
    min_total = max(threshold, sink + local + final_topk * 2)
    stage = min(cap, max(final_topk + max_skipped, min_total))
    return stage, local + interval + 2 * CHUNK


# --------------------------------------------------------------------------- the cache
class polar_cache:
    """ZoomKV sparse decode-attention cache (see module docstring)."""

    def __init__(self, valid_start, layer_num: int, batch_size: int, max_length: int, num_key_value_heads: int,
                 num_heads: int, head_dim: int, dtype: torch.dtype, layer_mapping: dict, max_new_length: int,
                 sink_size: int, local_size: int, core: int = 0, nprobe: int = 0, cache_unit_size: int = 0,
                 cache_cluster_num: int = 0, num_gpus: int = 1, model_size: int = 0, codebook_path: str = "",
                 collision_ratio: float = 0.3, candidate_ratio: float = 0.05, final_topk: int = 100,
                 dynamic_update_interval: int = 512, full_attention_threshold: int = 2000,
                 enable_offload: bool = True, debug_offload_coords: bool = False, enable_rerank: bool = False,
                 enable_recall: bool = False, enable_alpha_correction: bool = False,
                 enable_rerank_error_ablation: bool = False, enable_coarse_recall_ablation: bool = False,
                 enable_rerank_recall_ablation: bool = False, adaptive_topk_enabled: bool = False,
                 adaptive_topk_threshold: float = 0.9, adaptive_topk_min_k: int = 100,
                 adaptive_topk_max_k: int = 400) -> None:
        del core, nprobe, cache_unit_size, cache_cluster_num, codebook_path, collision_ratio  # unused (REF:183-185)
        del debug_offload_coords, enable_rerank, enable_recall, enable_alpha_correction
        del enable_rerank_error_ablation, enable_coarse_recall_ablation, enable_rerank_recall_ablation
        del adaptive_topk_enabled, adaptive_topk_threshold, adaptive_topk_min_k, adaptive_topk_max_k
        if head_dim != 128:
            raise ValueError(f"head_dim={head_dim}: the kernels implement head_dim 128")
        if dtype != torch.bfloat16:
            raise ValueError(f"dtype={dtype}: the cache stores bf16")
        if num_heads % num_key_value_heads:
            raise ValueError("num_heads must be a multiple of num_key_value_heads")
        self.layer_num = layer_num
        self.batch_size = batch_size
        self.max_length = max_length
        self.kv_head = num_key_value_heads
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.layer_mapping = layer_mapping
        self.num_gpus = num_gpus
        self.model_size = model_size
        self.valid_start = valid_start
        self.sink_size = sink_size
        self.local_size = local_size
        self.steady_size = sink_size + local_size
        self.dynamic_update_interval = dynamic_update_interval if dynamic_update_interval is not None else local_size
        self.group_size = num_heads // num_key_value_heads
        self.max_new_length = max_new_length
        self.input_length = max_length - max_new_length
        self.FULL_ATTENTION_THRESHOLD = full_attention_threshold
        self.final_topk = final_topk
        self.candidate_ratio = candidate_ratio
        self.enable_offload = enable_offload
        self.cfg = env_config(final_topk)
        self.quest_chunk_size = self.cfg["chunk"]
        self.MAX_SKIPPED_INDICES = self.cfg["max_skipped"]
        self.attention_mode = self.cfg["attention_mode"]
        self.host_tier = self.cfg["host_retrieval"]
        if self.host_tier and not enable_offload:
            raise ValueError("ZKV_HOST_RETRIEVAL=1 needs enable_offload=True (the offload zone bookkeeping)")
        if self.host_tier and self.attention_mode != "reference":
            raise ValueError("the host-pinned retrieval zone serves ZKV_ATTENTION_MODE=reference; the page modes "
                             "read their pages from HBM")
        self.sched = CacheSchedule(layer_num, sink_size, local_size, self.dynamic_update_interval, self.input_length,
                                   self.cfg, offload=enable_offload)
        self.context = 0

        self.unified_kv_capacity = self.input_length + max_new_length
        self.cap = self.unified_kv_capacity
        self._n_max = (self.cap + CHUNK - 1) // CHUNK
        devs = list(layer_mapping.values()) if layer_mapping else []
        self._layer_dev = [torch.device(layer_mapping.get(str(l), layer_mapping.get(l, devs[0]))) if devs
                           else torch.device("cuda", torch.cuda.current_device()) for l in range(layer_num)]
        self.device = self._layer_dev[0]
        bs, H, D, nm = batch_size, num_key_value_heads, head_dim, self._n_max
        self.keys, self.values = [], []
        self.win_k, self.win_v, self.win_base = [], [], [sink_size] * layer_num
        # offload-tier window: staging rows for the gathered selection (or,
        # below the retrieval threshold, every host row) + the near rows
        self._stage, self._near_cap = offload_window(sink_size, local_size, self.dynamic_update_interval, final_topk,
                                                     self.MAX_SKIPPED_INDICES, full_attention_threshold, self.cap)
        self.chunk_min, self.chunk_max, self.chunk_centroid, self.chunk_valid, self.kivi_packed = [], [], [], [], []
        self.vcodes_t, self.vmeta, self.kscale = [], [], []
        for l in range(layer_num):
            d = dict(device=self._layer_dev[l])
            if self.host_tier:
                self.keys.append(torch.zeros(bs, H, self.cap, D, dtype=torch.bfloat16, pin_memory=True))
                self.values.append(torch.zeros(bs, H, self.cap, D, dtype=torch.bfloat16, pin_memory=True))
                W = sink_size + self._stage + self._near_cap
                self.win_k.append(torch.zeros(bs, H, W, D, dtype=torch.bfloat16, **d))
                self.win_v.append(torch.zeros(bs, H, W, D, dtype=torch.bfloat16, **d))
            else:
                self.keys.append(torch.zeros(bs, H, self.cap, D, dtype=torch.bfloat16, **d))
                self.values.append(torch.zeros(bs, H, self.cap, D, dtype=torch.bfloat16, **d))
            self.chunk_min.append(torch.zeros(bs, H, nm, D, dtype=torch.bfloat16, **d))
            self.chunk_max.append(torch.zeros(bs, H, nm, D, dtype=torch.bfloat16, **d))
            self.chunk_centroid.append(torch.zeros(bs, H, nm, D, dtype=torch.bfloat16, **d))
            self.chunk_valid.append(torch.zeros(bs, H, nm, dtype=torch.bool, **d))
            self.kivi_packed.append(torch.zeros(bs, H, nm, 16, 16, dtype=torch.int32, **d))
            if self.attention_mode == "page4":
                self.vcodes_t.append(torch.zeros(bs, H, nm, D, 2, dtype=torch.int32, **d))
                self.vmeta.append(torch.zeros(bs, H, nm, 2, 4, 16, dtype=torch.bfloat16, **d))
                self.kscale.append(torch.zeros(bs, H, nm, D, dtype=torch.bfloat16, **d))
        # per-device scratch for the decode pipeline (preallocated: no
        # allocation on the decode path)
        self._scratch = {}
        for dev in dict.fromkeys(self._layer_dev):
            d = dict(device=dev)
            F = final_topk
            self._scratch[dev] = dict(
                # intermediates of the one-call retrieval chain, sized for the
                # largest plan (n_chunks = nk = n_dense = n_max)
                workspace=torch.empty(ops.reference_select_ws_bytes(bs * H, nm, nm, nm), dtype=torch.uint8, **d),
                final=torch.empty(bs, H, F + self.MAX_SKIPPED_INDICES, dtype=torch.int64, **d),
                skipped=torch.zeros(bs, H, self.MAX_SKIPPED_INDICES, dtype=torch.int64, **d),
                status=torch.zeros(1, dtype=torch.int32, **d),
                arange=torch.arange(self.cap, dtype=torch.int64, **d),
            )
        self._page_layers = [None] * layer_num
        self._raw_layers = [None] * layer_num
        # hierarchical Quest: per-large-chunk bounding boxes (separate-kernel cache :1762-1798)
        self.hq_factor = self.cfg["large_chunk"] // CHUNK if self.cfg["hierarchical"] else 0
        self.large_min, self.large_max, self.large_valid, self._large_layers = [], [], [], [None] * layer_num
        if self.hq_factor:
            nml = (nm + self.hq_factor - 1) // self.hq_factor
            for l in range(layer_num):
                d = dict(device=self._layer_dev[l])
                self.large_min.append(torch.zeros(bs, H, nml, D, dtype=torch.bfloat16, **d))
                self.large_max.append(torch.zeros(bs, H, nml, D, dtype=torch.bfloat16, **d))
                self.large_valid.append(torch.zeros(bs, H, nml, dtype=torch.uint8, **d))

    # ------------------------------------------------------------------ state (reference attribute names)
    @property
    def current_seq_len(self):
        return self.sched.current_seq_len

    @property
    def cpu_valid_end(self):
        return self.sched.cpu_valid_end

    @property
    def _actual_retrieval_length(self):
        return self.sched.actual_retrieval

    @property
    def _decode_step_counter(self):
        return self.sched.decode_steps

    # ------------------------------------------------------------------ helpers
    def _refresh_skipped(self) -> None:
        """Write the live skipped tail [16 n_chunks, kv_len) (REF:1895-1925)."""
        n_chunks, _, _, skipped = self.sched.plan
        kv_len = self.sched.actual_retrieval or 0
        if skipped > 0:
            for sc in self._scratch.values():
                sc["skipped"][:, :, :skipped].copy_(
                    torch.arange(n_chunks * CHUNK, kv_len, dtype=torch.int64, device=sc["skipped"].device))

    def _encode_range(self, l: int, rows: slice, tok_lo: int, tok_hi: int, src_k=None) -> None:
        """Encode the retrieval-zone tokens [tok_lo, tok_hi) (zone coordinates,
        both multiples of 16) of layer l: chunk min/max/mean + KIVI codes
        (+ 4-bit values in page4 mode).  src_k: the keys of exactly those
        tokens when they are not read from the HBM cache (offload tier)."""
        if tok_hi <= tok_lo:
            return
        s = self.sink_size
        k = self.keys[l][rows, :, s + tok_lo:s + tok_hi] if src_k is None else src_k
        ops.kivi_encode_chunks(k, self.chunk_min[l][rows], self.chunk_max[l][rows], self.chunk_centroid[l][rows],
                               self.chunk_valid[l][rows], self.kivi_packed[l][rows], tok_lo // CHUNK,
                               kscale=self.kscale[l][rows] if self.attention_mode == "page4" else None)
        if self.attention_mode == "page4":
            v = self.values[l][rows, :, s + tok_lo:s + tok_hi]
            ops.vquant_encode(v, self.vcodes_t[l][rows], self.vmeta[l][rows], tok_lo)
        if self.hq_factor:  # the large chunks the new chunks touch (:1762-1798)
            f, c_lo, c_hi = self.hq_factor, tok_lo // CHUNK, tok_hi // CHUNK
            ops.quest_large_minmax(self.chunk_min[l][rows], self.chunk_max[l][rows], c_hi, f,
                                   self.large_min[l][rows], self.large_max[l][rows], self.large_valid[l][rows],
                                   g_lo=c_lo // f, g_hi=min((c_hi + f - 1) // f, self.large_min[l].shape[2]))

    def _rows(self, batch_idx=None) -> slice:
        return slice(0, self.batch_size) if batch_idx is None else slice(batch_idx, batch_idx + 1)

    # ------------------------------------------------------------------ prefill
    def prefill_update_kv_cache(self, query_states, key_states, value_states, layer_idx, batch_idx):
        """REF:863-877: bsz == 1 -> one sample at batch_idx, bsz > 1 -> the
        whole batch in lockstep (only on batch_idx == 0).  Returns the keys /
        values without the left padding."""
        del query_states
        bsz = key_states.shape[0]
        vs_list = self.valid_start if isinstance(self.valid_start, (list, tuple)) else None
        if bsz == 1:
            vs = int(vs_list[batch_idx]) if vs_list is not None else int(self.valid_start)
            rows = self._rows(batch_idx)
        else:
            vs = int(vs_list[0]) if vs_list is not None else int(self.valid_start)
            if vs_list is not None and any(int(v) != vs for v in vs_list[:bsz]):
                raise AssertionError("lockstep multi-batch prefill requires the same valid_start across the batch")
            if batch_idx != 0:
                return key_states[:, vs:], value_states[:, vs:]
            if bsz != self.batch_size:
                raise AssertionError(f"bsz({bsz}) must equal cache batch_size({self.batch_size}) for lockstep mode.")
            rows = self._rows(None)
        seq_len = key_states.shape[1]
        if seq_len > self.input_length:
            raise AssertionError("prefill longer than the cache's input length")
        n = seq_len - vs
        if n > self.cap:
            raise RuntimeError(f"prefill of {n} tokens exceeds the cache capacity {self.cap}")
        kk = key_states[:, vs:seq_len].transpose(1, 2).to(torch.bfloat16)
        vv = value_states[:, vs:seq_len].transpose(1, 2).to(torch.bfloat16)
        if not self.host_tier:
            self.keys[layer_idx][rows, :, :n].copy_(kk)
            self.values[layer_idx][rows, :, :n].copy_(vv)
        first = self.sched.actual_retrieval is None
        _, r_len, (lo, hi) = self.sched.prefill(layer_idx, seq_len, vs)
        if first:
            self._refresh_skipped()
        if self.host_tier:
            self._prefill_host(layer_idx, rows, kk, vv, n, r_len, hi)
            s = self.sink_size
            self._encode_range(layer_idx, rows, lo, hi, src_k=kk[:, :, s + lo:s + hi])
        else:
            self._encode_range(layer_idx, rows, lo, hi)
        last_call = (layer_idx == self.layer_num - 1) and (bsz > 1 or batch_idx + bsz == self.batch_size)
        if last_call:
            self.context += n
        return key_states[:, vs:], value_states[:, vs:]

    def _prefill_host(self, l, rows, kk, vv, n, r_len, enc_hi):
        """Offload tier: sink rows to the window, retrieval rows to the host
        zone, and every token from the first unencoded chunk on to the near
        part of the window."""
        s = self.sink_size
        ns = min(s, n)
        self.win_k[l][rows, :, :ns].copy_(kk[:, :, :ns])
        self.win_v[l][rows, :, :ns].copy_(vv[:, :, :ns])
        if r_len > 0:
            self.keys[l][rows, :, s:s + r_len].copy_(kk[:, :, s:s + r_len])
            self.values[l][rows, :, s:s + r_len].copy_(vv[:, :, s:s + r_len])
        base = s + enc_hi
        m = max(0, n - base)
        if m > self._near_cap:
            raise RuntimeError(f"prefill leaves {m} unencoded tokens; the near window holds {self._near_cap}")
        off = s + self._stage
        self.win_k[l][rows, :, off:off + m].copy_(kk[:, :, base:base + m])
        self.win_v[l][rows, :, off:off + m].copy_(vv[:, :, base:base + m])
        self.win_base[l] = base

    def _win_slot(self, l: int, pos: int) -> int:
        """Window row of absolute position pos (offload tier)."""
        s = self.sink_size
        if pos < s:
            return pos
        j = pos - self.win_base[l]
        if j < 0 or j >= self._near_cap:
            raise RuntimeError(f"position {pos} is outside the near window of layer {l} "
                               f"(base {self.win_base[l]}, capacity {self._near_cap})")
        return s + self._stage + j

    def sync(self, layer_idx, batch_idx):
        """REF:2789-2793: nothing to wait for (no host copies)."""
        del layer_idx, batch_idx

    # ------------------------------------------------------------------ decode append + flush
    def decode_update_kv_cache(self, key_states, value_states, layer_idx):
        """REF:1516-1583: flush at layer 0 when the near zone is full, then
        append this layer's token."""
        if self.sched.flush_due(layer_idx):
            self._update_polar_index()
        pos = self.sched.current_seq_len[layer_idx]
        if pos >= self.cap:
            raise RuntimeError(f"KV write is outside the cache: layer={layer_idx}, current={pos}, "
                               f"capacity={self.cap}")
        if self.host_tier:
            w = self._win_slot(layer_idx, pos)
            self.win_k[layer_idx][:, :, w].copy_(key_states[:, 0])
            self.win_v[layer_idx][:, :, w].copy_(value_states[:, 0])
        else:
            self.keys[layer_idx][:, :, pos].copy_(key_states[:, 0])
            self.values[layer_idx][:, :, pos].copy_(value_states[:, 0])
        self.sched.append(layer_idx)
        if layer_idx == self.layer_num - 1:
            self.context += 1
        return None, None

    def _update_polar_index(self) -> None:
        """REF:1379-1512: extend the retrieval zone to the local start and
        encode the chunks the new tokens complete.  The live carry of the
        previous flush is read from the same buffer, so every chunk matches
        the reference's carry-merged chunk byte for byte."""
        old_r = self.sched.actual_retrieval
        lo, hi, _ = self.sched.flush()
        self._refresh_skipped()
        if not self.host_tier:
            for l in range(self.layer_num):
                self._encode_range(l, self._rows(None), lo, hi)
            return
        s, new_r = self.sink_size, self.sched.actual_retrieval
        off = s + self._stage
        for l in range(self.layer_num):
            base, total = self.win_base[l], self.current_seq_len[l]
            wk, wv = self.win_k[l], self.win_v[l]
            # rows that joined the retrieval zone -> host zone (the D2H offload)
            a, b = s + old_r - base, s + new_r - base
            self.keys[l][:, :, s + old_r:s + new_r].copy_(wk[:, :, off + a:off + b])
            self.values[l][:, :, s + old_r:s + new_r].copy_(wv[:, :, off + a:off + b])
            # the completed chunks start at the window base (s + lo == base)
            self._encode_range(l, self._rows(None), lo, hi, src_k=wk[:, :, off:off + hi - lo])
            # slide: the window now starts at the first unencoded token
            nb = s + hi
            m = total - nb
            if nb > base and m > 0:
                wk[:, :, off:off + m].copy_(wk[:, :, off + nb - base:off + nb - base + m].clone())
                wv[:, :, off:off + m].copy_(wv[:, :, off + nb - base:off + nb - base + m].clone())
            self.win_base[l] = nb

    # ------------------------------------------------------------------ regions
    def get_region_indices(self, layer_idx, device=None):
        """REF:1173-1259 (index tensors are views of a preallocated arange)."""
        del device
        total = self.current_seq_len[layer_idx]
        r_len, local_start, local_len = self.sched.region(layer_idx)
        ar = self._scratch[self._layer_dev[layer_idx]]["arange"]
        return {"sink_indices": ar[:self.sink_size],
                "local_indices": ar[local_start:total] if local_len > 0 else ar[:0],
                "retrieval_start": self.sink_size, "retrieval_length": r_len, "total_len": total,
                "local_len": local_len}

    # ------------------------------------------------------------------ decode attention
    def compute(self, queries, layer_idx):
        """REF:1589-1775: queries [bs, 1, num_heads, 128] -> [bs, 1, num_heads, 128]."""
        l = layer_idx
        dev = self._layer_dev[l]
        sc = self._scratch[dev]
        total = self.current_seq_len[l]
        s = self.sink_size
        cpu_len = int(self.cpu_valid_end[l]) if self.cpu_valid_end is not None else None
        r_len, local_start, _ = self.sched.region(l)
        encoded = self.sched.actual_retrieval or 0
        valid_length = cpu_len if cpu_len is not None else min(r_len, encoded)
        min_total = max(self.FULL_ATTENTION_THRESHOLD, s + self.local_size + self.final_topk * 2)
        q = queries if queries.is_contiguous() else queries.contiguous()
        if total < min_total or valid_length <= 0 or not self.cfg["stage1"]:
            # full attention over every stored token (REF:1631-1646, 1280-1334)
            if self.host_tier:
                return self._full_attention_host(q, l, total, sc)
            return ops.attn_rows(q, self.keys[l], self.values[l], seg0=(0, total), status=sc["status"])
        n_chunks, nk, n_dense, skipped = self.sched.plan
        n_valid_chunks = valid_length // CHUNK
        if self.attention_mode == "page":
            return self._compute_page_raw(q, l, n_chunks, nk, total)
        if self.attention_mode == "page4":
            return self._compute_page(q, l, n_chunks, nk, valid_length, total)
        torch.cuda.nvtx.range_push("stage1_stage2_select")
        k = min(self.final_topk, nk * CHUNK)
        final = sc["final"]
        ops.reference_select(q, self.chunk_min[l], self.chunk_max[l], self.chunk_centroid[l], self.chunk_valid[l],
                             self.kivi_packed[l], n_chunks, n_valid_chunks, nk, n_dense,
                             max(1, min(self.cfg["dense_topk"], CHUNK)), max(1, min(self.cfg["sparse_topk"], CHUNK)),
                             k, sc["skipped"][:, :, :skipped], final, sc["workspace"])
        torch.cuda.nvtx.range_pop()
        if self.host_tier:
            # REF:1710-1750: the selected rows come over the host link into
            # the staging rows; attention reads [sink + staged] and the near
            # rows of the window
            torch.cuda.nvtx.range_push("h2d_gather_kv")
            n = k + skipped
            ops.h2d_gather_rows(self.keys[l], self.values[l], final, self.win_k[l], self.win_v[l], n_sel=n,
                                src_offset=s, dst_offset=s, status=sc["status"])
            torch.cuda.nvtx.range_pop()
            torch.cuda.nvtx.range_push("compute_attention")
            off, base = s + self._stage, self.win_base[l]
            out = ops.attn_rows(q, self.win_k[l], self.win_v[l], seg0=(0, s + n),
                                seg1=(off + local_start - base, off + total - base), status=sc["status"])
            torch.cuda.nvtx.range_pop()
            return out
        torch.cuda.nvtx.range_push("compute_attention")
        # sink + selected retrieval tokens + near zone [local_start, total)
        # (REF:1752-1761: the all-GPU gather uses the same three segments)
        out = ops.attn_rows(q, self.keys[l], self.values[l], seg0=(0, s), sel=final[:, :, :k + skipped],
                            sel_offset=s, seg1=(local_start, total), status=sc["status"])
        torch.cuda.nvtx.range_pop()
        return out

    def _full_attention_host(self, q, l, total, sc):
        """Offload tier below the retrieval threshold: every host row
        [sink, window base) is gathered into the staging rows, then attention
        covers sink + staged + the near rows."""
        s, base = self.sink_size, self.win_base[l]
        n_h = max(0, base - s) if total > s else 0
        if n_h > self._stage:
            raise RuntimeError(f"full attention over {n_h} host rows exceeds the {self._stage} staging rows")
        if n_h > 0:
            ar = self._scratch[self._layer_dev[l]]["arange"][:n_h].expand(self.batch_size, self.kv_head, n_h)
            ops.h2d_gather_rows(self.keys[l], self.values[l], ar, self.win_k[l], self.win_v[l], src_offset=s,
                                dst_offset=s, status=sc["status"])
        off = s + self._stage
        return ops.attn_rows(q, self.win_k[l], self.win_v[l], seg0=(0, min(total, s) + n_h),
                             seg1=(off, off + max(0, total - base)), status=sc["status"])

    def _compute_page_raw(self, q, l, n_chunks, nk, total):
        """The reference's page mode: Quest top-nk of the encoded chunks, then
        attention over their raw rows, the sink rows and every row from the
        first unencoded token on (the skipped tail and the near zone)
        (REF:1589-1775 with dense_topk = sparse_topk = 16 and final_topk =
        nk * 16)."""
        if self._raw_layers[l] is None:
            self._raw_layers[l] = ops.RawLayer(self.chunk_min[l], self.chunk_max[l], self.chunk_valid[l],
                                               self.keys[l], self.values[l], page_base=self.sink_size)
        s = self.sink_size
        status = self._scratch[self._layer_dev[l]]["status"]
        if self.hq_factor:
            # hierarchical pick (separate-kernel cache :1852-1940): every token
            # of the nk_small picked chunks is attended (the reference's result
            # when final_topk >= 16 * nk_small); chunks past the last whole large
            # chunk are its live skipped tokens and are attended with the near rows
            f = self.hq_factor
            n_large, nk_large, nk_small = hier_plan(n_chunks, f, self.cfg["large_ratio"], self.cfg["small_ratio"])
            if n_large > 0:
                if self._large_layers[l] is None:
                    self._large_layers[l] = ops.LargeLayer(self.large_min[l], self.large_max[l], self.large_valid[l])
                near_start = s + n_large * f * CHUNK
                return ops.page_decode_raw_hier(q, self._raw_layers[l], self._large_layers[l], n_chunks, f, nk_large,
                                                nk_small, total - near_start, n_sink=s, near_start=near_start,
                                                status=status)
            # no whole large chunk yet: every retrieval token is a live skipped one
            return ops.page_decode_raw(q, self._raw_layers[l], 0, 0, total - s, n_sink=s, near_start=s,
                                       status=status)
        near_start = s + n_chunks * CHUNK
        return ops.page_decode_raw(q, self._raw_layers[l], n_chunks, nk, total - near_start, n_sink=s,
                                   near_start=near_start, status=status)

    def _compute_page(self, q, l, n_chunks, nk, valid_length, total):
        """Page4 (lossy) decode over the encoded chunks' 4-bit pages; the carry
        tail and the near zone are attended as raw rows."""
        if self._page_layers[l] is None:
            self._page_layers[l] = ops.PageLayer(self.chunk_min[l], self.chunk_max[l], self.chunk_valid[l],
                                                 self.kivi_packed[l], self.vcodes_t[l], self.vmeta[l], self.keys[l],
                                                 self.values[l], self.kscale[l])
        s = self.sink_size
        near_start = s + n_chunks * CHUNK
        return ops.page_decode(q, self._page_layers[l], n_chunks, nk, total - near_start, n_sink=s,
                               near_start=near_start, status=self._scratch[self._layer_dev[l]]["status"])
