"""Tensor-level operators over the libzkv C ABI.

The functions keep the reference's operator names and argument meaning
(paths relative to runtime/zoomkv_urania_runtime_20261011/ of the reference):

=====================================  ==============================================
this module                            reference operator
=====================================  ==============================================
quest_chunk_score                      cache_hub/quest/quest_chunk_score.cu (pybind)
float_topk / float_topk_3d             cache_hub/topk/float_topk_ops.py:63-106
radix_topk_3d                          cache_hub/topk/__init__.py (radix_topk_3d)
partial_chunk_density_scores_cuda      cache_hub/rerank/rerank.py:612-633
dense_mask_from_topk_cuda              cache_hub/rerank/rerank.py:587-609
partial_chunk_kivi_qk_dense_sparse_cuda cache_hub/kivi/kivi_qk_dot_ops.py:29-67
float_topk_gather_concat_3d            cache_hub/topk/float_topk_gather_concat_ops.py:77-125
lse_merge_cuda                         cache_hub/lse_merge/lse_merge.py:122-144
kivi_encode_chunks                     polar_cache._compute_and_store_chunk_minmax +
                                       _kivi_pack_chunks (aligned chunks)
attn_rows                              h2d_gather_kv + torch.cat + flash_attn_with_kvcache
h2d_gather_kv / h2d_gather_kv_packed   cache_hub/gather_trans/trans_h2d.py:65-161 (offload tier)
page_decode_raw                        polar_cache.compute in page mode (REF:1589-1775): Quest top-nk
                                       chunks, attention over their raw rows + sink + near (one launch)
page_decode                            (fused page mode over 4-bit KIVI K/V pages, lossy; no counterpart)
reference_select                       polar_cache.compute retrieval chain (REF:1589-1775) as one call
vquant_encode                          (per-token 4-bit values; no counterpart)
RqLayout / rq_encode / batch_encode    cache_hub/polar_cache.py batch_encode (:1130-1198)
                                       + _count_cluster_keys (:1203-1226)
rq_query                               cache_hub/polar_cache.py _encode_query_blocks (:1108-1127)
get_cache_cnt_fused                    cache_hub/polar_cache.py:1688-1728 (collision.cu)
collision_topk                         get_cache_cnt_fused + _coarse_filter_truncate (:1730-1747)
partial_rerank_cuda                    cache_hub/rerank/rerank.py:352-400 (+ topk/gather :1750-1832)
coarse_2bit_score_cuda                 cache_hub/rerank/rerank.py:636-690
rq_popcount_topk                       (1-bit x 4-bit popcount rerank + exact IP; no counterpart)
=====================================  ==============================================

Errors follow the reference: wrong dtype -> TypeError, wrong shape / range ->
ValueError / RuntimeError, and a non-zero C status -> RuntimeError.  There
is no CPU path: every op requires CUDA tensors and the compiled library.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import check, lib

__all__ = [
    "quest_chunk_score", "float_topk", "float_topk_3d", "radix_topk_3d", "partial_chunk_density_scores_cuda",
    "dense_mask_from_topk_cuda", "partial_chunk_kivi_qk_dense_sparse_cuda", "float_topk_gather_concat_3d",
    "lse_merge_cuda", "lse_merge_n", "kivi_encode_chunks", "vquant_encode", "attn_rows", "page_decode",
    "h2d_gather_kv", "h2d_gather_kv_packed", "h2d_gather_rows", "page_decode_scored",
    "PageLayer", "page_attend", "RawLayer", "page_decode_raw", "page_decode_raw_ws_bytes", "gqa_mean", "reference_select", "reference_select_ws_bytes", "RqLayout", "rq_encode", "batch_encode", "rq_query", "get_cache_cnt_fused", "collision_topk",
    "partial_rerank_cuda", "coarse_2bit_score_cuda", "rq_popcount_topk", "MAG_CENTERS", "MAG_THRESHOLDS",
]


_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(t: torch.Tensor) -> int:
    """The current CUDA stream of t's device (its raw handle)."""
    if _RAW_STREAM is not None and t.device.index is not None:
        return _RAW_STREAM(t.device.index)
    return torch.cuda.current_stream(t.device).cuda_stream


def _cuda(*ts):
    for name, t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor")


def _dtype(name, t, dt):
    if t.dtype != dt:
        raise TypeError(f"{name} must be {dt}; got {t.dtype}")


def _contig(name, t):
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _p(t):
    return None if t is None else t.data_ptr()


# ----------------------------------------------------------------- Quest stage-1
def quest_chunk_score(raw_q, chunk_min, chunk_max, scores_out, n_chunks, chunk_valid=None):
    """scores_out[b,h,c] = sum_d max(q*max, q*min) for c < n_chunks (in place).

    raw_q [bs,kv,128] bf16; chunk_min/max [bs,kv,n_max,128] bf16 (or views
    of a chunk range of such buffers); scores_out: n_chunks*bs*kv fp32
    elements laid out [bs,kv,n_chunks]; chunk_valid [bs,kv,n_max] bool or None.
    """
    _cuda(("raw_q", raw_q), ("chunk_min", chunk_min), ("chunk_max", chunk_max), ("scores", scores_out),
          ("valid", chunk_valid))
    _dtype("raw_q", raw_q, torch.bfloat16)
    _contig("raw_q", raw_q)
    for n, t in (("chunk_min", chunk_min), ("chunk_max", chunk_max)):
        _dtype(n, t, torch.bfloat16)
        if t.stride(3) != 1 or t.stride(2) != 128 or t.stride(0) != t.shape[1] * t.stride(1):
            raise ValueError(f"{n} must be a chunk range of a contiguous [bs, kv, n_max, 128] buffer")
    _dtype("scores_out", scores_out, torch.float32)
    _contig("scores_out", scores_out)
    if raw_q.shape[-1] != 128:
        raise ValueError("quest_chunk_score: only head_dim==128 is supported")
    bs, kv = raw_q.shape[0], raw_q.shape[1]
    n_max = chunk_min.stride(1) // 128
    n_chunks = int(n_chunks)
    if n_chunks > chunk_min.shape[2]:
        raise ValueError("n_chunks must <= chunk_n_max")
    if scores_out.numel() < bs * kv * n_chunks:
        raise ValueError("scores_out too small")
    if chunk_valid is not None:
        _dtype("chunk_valid", chunk_valid, torch.bool)
        if chunk_valid.stride(2) != 1 or chunk_valid.stride(1) != n_max:
            raise ValueError("chunk_valid must match chunk_min's layout")
    check(lib().zkv_quest_score(_p(raw_q), _p(chunk_min), _p(chunk_max), _p(chunk_valid), _p(scores_out), bs * kv,
                                n_chunks, n_max, _stream(raw_q)), "zkv_quest_score")


def quest_chunk_score_gqa(q, chunk_min, chunk_max, scores_out, n_chunks, chunk_valid=None):
    """quest_chunk_score with the GQA mean folded into the kernel: q
    [bs, 1, kv*G, 128] bf16 (the decode query) instead of raw_q."""
    _cuda(("q", q), ("chunk_min", chunk_min), ("chunk_max", chunk_max), ("scores", scores_out),
          ("valid", chunk_valid))
    _dtype("q", q, torch.bfloat16)
    _contig("q", q)
    for n, t in (("chunk_min", chunk_min), ("chunk_max", chunk_max)):
        _dtype(n, t, torch.bfloat16)
        if t.stride(3) != 1 or t.stride(2) != 128 or t.stride(0) != t.shape[1] * t.stride(1):
            raise ValueError(f"{n} must be a chunk range of a contiguous [bs, kv, n_max, 128] buffer")
    _dtype("scores_out", scores_out, torch.float32)
    _contig("scores_out", scores_out)
    bs, kv = chunk_min.shape[0], chunk_min.shape[1]
    G = q.shape[2] // kv
    n_max = chunk_min.stride(1) // 128
    n_chunks = int(n_chunks)
    if n_chunks > chunk_min.shape[2] or scores_out.numel() < bs * kv * n_chunks:
        raise ValueError("n_chunks / scores_out size")
    if chunk_valid is not None:
        _dtype("chunk_valid", chunk_valid, torch.bool)
    check(lib().zkv_quest_score_gqa(_p(q), G, _p(chunk_min), _p(chunk_max), _p(chunk_valid), _p(scores_out), bs * kv,
                                    n_chunks, n_max, _stream(q)), "zkv_quest_score_gqa")


# ----------------------------------------------------------------- top-k
def float_topk(scores: torch.Tensor, k: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """Top-k indices [B, k] int64 of fp32 [B, L] (ties -> lowest index, ascending)."""
    _cuda(("scores", scores))
    if scores.dim() != 2:
        raise ValueError("scores must be 2D [B, L]")
    if k <= 0:
        raise ValueError(f"k must be positive, got {k}")
    if k > scores.shape[1]:
        raise ValueError(f"k={k} cannot exceed L={scores.shape[1]}")
    s = scores if scores.dtype == torch.float32 else scores.float()
    if s.stride(1) != 1:
        s = s.contiguous()
    B, L = s.shape
    if out is None:
        out = torch.empty(B, k, dtype=torch.int64, device=s.device)
    check(lib().zkv_topk_f32(_p(s), B, L, s.stride(0), int(k), _p(out), _stream(s)), "zkv_topk_f32")
    return out


def float_topk_3d(scores: torch.Tensor, k: int, out: torch.Tensor | None = None) -> torch.Tensor:
    if scores.dim() != 3:
        raise ValueError("scores must be 3D [bs, kv_heads, n_chunks]")
    bs, kv, L = scores.shape
    if k > L:
        raise ValueError(f"k={k} cannot exceed n_chunks={L}")
    s = scores.reshape(bs * kv, L)
    o = float_topk(s, k, None if out is None else out.view(bs * kv, k))
    return o.view(bs, kv, k)


def radix_topk_3d(vals: torch.Tensor, k: int) -> torch.Tensor:
    """Top-k indices of int32 [bs, kv, L] (ties -> lowest index, ascending)."""
    _cuda(("vals", vals))
    _dtype("vals", vals, torch.int32)
    bs, kv, L = vals.shape
    v = vals.reshape(bs * kv, L)
    if v.stride(1) != 1:
        v = v.contiguous()
    out = torch.empty(bs * kv, k, dtype=torch.int64, device=vals.device)
    check(lib().zkv_topk_i32(_p(v), bs * kv, L, v.stride(0), int(k), _p(out), _stream(vals)), "zkv_topk_i32")
    return out.view(bs, kv, k)


# ----------------------------------------------------------------- CDS
def partial_chunk_density_scores_cuda(chunk_ids, chunk_centroids, raw_q, out_scores, kernel=None):
    """out_scores[b,h,j] = centroid[b,h,chunk_ids[b,h,j]] . raw_q[b,h] (fp32; -1e30 if invalid)."""
    del kernel
    _cuda(("chunk_ids", chunk_ids), ("centroids", chunk_centroids), ("raw_q", raw_q), ("out", out_scores))
    if out_scores.dtype != torch.float32:
        raise TypeError(f"out_scores must be float32, got {out_scores.dtype}")
    if chunk_centroids.dtype != torch.bfloat16:
        chunk_centroids = chunk_centroids.to(torch.bfloat16)
    if raw_q.dtype != torch.bfloat16:
        raw_q = raw_q.to(torch.bfloat16)
    ids = chunk_ids if chunk_ids.dtype == torch.int64 else chunk_ids.long()
    ids, cent, q = ids.contiguous(), chunk_centroids.contiguous(), raw_q.contiguous()
    _contig("out_scores", out_scores)
    bs, kv, nk = ids.shape
    n_max = cent.shape[2]
    check(lib().zkv_chunk_density(_p(ids), _p(cent), _p(q), _p(out_scores), bs * kv, nk, n_max, n_max,
                                  _stream(ids)), "zkv_chunk_density")


def dense_mask_from_topk_cuda(positions, mask, kernel=None):
    """mask.fill_(False); mask.scatter_(2, positions, True) in one launch."""
    del kernel
    _cuda(("positions", positions), ("mask", mask))
    _dtype("positions", positions, torch.int64)
    _dtype("mask", mask, torch.bool)
    pos = positions.contiguous()
    _contig("mask", mask)
    bs, kv, nk = mask.shape
    check(lib().zkv_mask_from_topk(_p(pos), _p(mask), bs * kv, pos.shape[2], nk, _stream(mask)),
          "zkv_mask_from_topk")


# ----------------------------------------------------------------- KIVI stage-2
def partial_chunk_kivi_qk_dense_sparse_cuda(chunk_ids, dense_mask, packed_K, chunk_min, chunk_max, raw_q,
                                            dense_topk, sparse_topk, group_size, out_scores, out_indices,
                                            kernel=None):
    """KIVI dequant . raw_q per selected chunk + per-chunk top dense/sparse (in place).

    packed_K [bs,kv,n_chunks,16,16] int32 chunk-major (may be a chunk-axis
    slice of a larger buffer); chunk_min/max [bs,kv,n_max,128] bf16.
    """
    del kernel
    if chunk_ids.dtype != torch.int64:
        chunk_ids = chunk_ids.to(torch.int64)
    if dense_mask.dtype != torch.bool:
        dense_mask = dense_mask.bool()
    if packed_K.dtype != torch.int32:
        raise TypeError(f"packed_K must be int32; got {packed_K.dtype}")
    for name, t in (("chunk_min", chunk_min), ("chunk_max", chunk_max), ("raw_q", raw_q)):
        if t.dtype != torch.bfloat16:
            raise TypeError(f"{name} must be bfloat16; got {t.dtype}")
    if out_scores.dtype != torch.float32:
        raise TypeError(f"out_scores must be float32; got {out_scores.dtype}")
    if out_indices.dtype != torch.int64:
        raise TypeError(f"out_indices must be int64; got {out_indices.dtype}")
    if group_size != 16:
        raise ValueError(f"group_size must be 16 on this build; got {group_size}")
    _cuda(("chunk_ids", chunk_ids), ("packed_K", packed_K), ("out_scores", out_scores))
    if packed_K.dim() != 5 or packed_K.shape[3] != 16 or packed_K.shape[4] != 16:
        raise ValueError(f"packed_K must be chunk-major [bs, kv, n_chunks, 16, 16]; got {tuple(packed_K.shape)}")
    bs, kv, n_pk = packed_K.shape[:3]
    if packed_K.stride(4) != 1 or packed_K.stride(3) != 16 or packed_K.stride(2) != 256 or \
            packed_K.stride(0) != kv * packed_K.stride(1):
        raise ValueError("packed_K must be a chunk-axis slice of a contiguous buffer")
    pk_ld = packed_K.stride(1) // 256
    if chunk_min.shape[-1] != 128:
        raise ValueError("kivi cuda kernel: only head_dim=128 supported")
    ids, dm = chunk_ids.contiguous(), dense_mask.contiguous()
    cmin, cmax, q = chunk_min.contiguous(), chunk_max.contiguous(), raw_q.contiguous()
    nk = ids.shape[2]
    _contig("out_scores", out_scores)
    _contig("out_indices", out_indices)
    if out_scores.shape[2] < nk * 16 or out_indices.shape[2] < nk * 16:
        raise ValueError("out_scores/out_indices too small")
    check(lib().zkv_kivi_qk(_p(ids), _p(dm), _p(packed_K), n_pk, pk_ld, _p(cmin), _p(cmax), cmin.shape[2], _p(q),
                            bs * kv, nk, int(dense_topk), int(sparse_topk), _p(out_scores), _p(out_indices),
                            out_scores.shape[2], _stream(ids)), "zkv_kivi_qk")


def float_topk_gather_concat_3d(scores, lut, skipped, out, k):
    """out[:,:,:k] = lut[top_k(scores)]; out[:,:,k:k+sk] = skipped.  Returns out."""
    _cuda(("scores", scores), ("lut", lut), ("skipped", skipped), ("out", out))
    _dtype("scores", scores, torch.float32)
    _dtype("lut", lut, torch.int64)
    _dtype("skipped", skipped, torch.int64)
    _dtype("out", out, torch.int64)
    if scores.shape != lut.shape:
        raise ValueError(f"scores/lut shape mismatch: {scores.shape} vs {lut.shape}")
    bs, kv, L = scores.shape
    sk = skipped.shape[2]
    if not (0 < k <= L):
        raise ValueError(f"k={k} out of range [1, {L}]")
    if out.shape[2] < k + sk:
        raise ValueError(f"out last dim={out.shape[2]} must be >= k+sk={k + sk}")
    _contig("out", out)
    s, lu = scores.contiguous(), lut.contiguous()
    if sk > 0 and (skipped.stride(2) != 1 or skipped.stride(0) != kv * skipped.stride(1)):
        skipped = skipped.contiguous()
    sk_ld = skipped.stride(1) if sk > 0 else 0
    check(lib().zkv_topk_gather_concat(_p(s), _p(lu), _p(skipped) if sk > 0 else None, sk_ld, _p(out), bs * kv, L,
                                       int(k), sk, out.shape[2], _stream(s)), "zkv_topk_gather_concat")
    return out


# ----------------------------------------------------------------- one-call retrieval chain
def reference_select_ws_bytes(rows: int, n_chunks: int, nk: int, n_dense: int) -> int:
    return int(lib().zkv_reference_select_ws_bytes(rows, n_chunks, nk, n_dense))


def reference_select(q, chunk_min, chunk_max, centroid, chunk_valid, packed, n_chunks: int, n_valid_chunks: int,
                     nk: int, n_dense: int, dense_topk: int, sparse_topk: int, k: int, skipped, final_out, workspace,
                     raw_q_out=None):
    """The reference-mode retrieval chain of one layer in one C call:
    q [bs, 1, H*G, 128] bf16; chunk tensors [bs, H, n_max, ...]; skipped
    [bs, H, >= sk] int64 (sk = skipped.shape[2]); final_out [bs, H, >= k+sk]
    int64; workspace uint8 CUDA tensor of >= reference_select_ws_bytes(...)."""
    bs, H, n_max = chunk_min.shape[:3]
    rows = bs * H
    G = q.shape[-2] // H
    for name, t in (("q", q), ("chunk_min", chunk_min), ("chunk_max", chunk_max), ("centroid", centroid)):
        _dtype(name, t, torch.bfloat16)
        _contig(name, t)
    _dtype("packed", packed, torch.int32)
    _contig("packed", packed)
    _dtype("final_out", final_out, torch.int64)
    _contig("final_out", final_out)
    _dtype("workspace", workspace, torch.uint8)
    sk = skipped.shape[2] if skipped is not None else 0
    sk_ld = 0
    if sk > 0:
        _dtype("skipped", skipped, torch.int64)
        if skipped.stride(2) != 1 or skipped.stride(0) != H * skipped.stride(1):
            skipped = skipped.contiguous()
        sk_ld = skipped.stride(1)
    valid = None
    if chunk_valid is not None:
        valid = chunk_valid if chunk_valid.dtype == torch.uint8 else chunk_valid.view(torch.uint8)
    layer = _lib.ZkvRefLayer(_p(chunk_min), _p(chunk_max), _p(centroid), _p(valid), _p(packed))
    check(lib().zkv_reference_select(_p(q), G, ctypes.byref(layer), rows, n_max, n_chunks, n_valid_chunks, nk,
                                     n_dense, dense_topk, sparse_topk, k, _p(skipped) if sk > 0 else None, sk_ld, sk,
                                     _p(final_out), final_out.shape[-1], _p(raw_q_out), _p(workspace),
                                     workspace.numel(), _stream(q)), "zkv_reference_select")
    return final_out


# ----------------------------------------------------------------- merge
def lse_merge_cuda(attn_out_a, lse_a, attn_out_b, lse_b):
    """Merge two attention partials ([bs,1,heads,dim] + lse [bs,heads,1])."""
    if not attn_out_a.is_cuda:
        raise ValueError("attn_out_a must be a CUDA tensor")
    if attn_out_a.shape != attn_out_b.shape:
        raise ValueError(f"attn outputs must have identical shape, got {attn_out_a.shape} and {attn_out_b.shape}")
    bs, _, heads, dim = attn_out_a.shape
    a = attn_out_a.to(torch.bfloat16).contiguous()
    b = attn_out_b.to(torch.bfloat16).contiguous()
    la = lse_a.to(torch.float32).reshape(bs, heads).contiguous()
    lb = lse_b.to(torch.float32).reshape(bs, heads).contiguous()
    out = torch.empty_like(a)
    check(lib().zkv_lse_merge(_p(a), _p(la), _p(b), _p(lb), _p(out), None, bs * heads, dim, _stream(a)),
          "zkv_lse_merge")
    return out.to(attn_out_a.dtype)


def lse_merge_n(parts: torch.Tensor, lses: torch.Tensor, out: torch.Tensor, lse_out: torch.Tensor | None = None):
    """parts [n, rows, dim] fp32, lses [n, rows] -> out [rows, dim] bf16 (+ lse_out [rows])."""
    _dtype("parts", parts, torch.float32)
    _dtype("lses", lses, torch.float32)
    n, rows, dim = parts.shape
    check(lib().zkv_lse_merge_n(_p(parts.contiguous()), _p(lses.contiguous()), n, rows, dim, _p(out), _p(lse_out),
                                _stream(parts)), "zkv_lse_merge_n")
    return out


# ----------------------------------------------------------------- encode
def kivi_encode_chunks(keys, chunk_min, chunk_max, chunk_centroid, chunk_valid, packed, chunk_start: int,
                       kscale=None):
    """Write metadata + KIVI codes of the aligned chunks of `keys` [bs,kv,T,128]
    (T % 16 == 0; token stride 128) at chunk indices chunk_start.. of the
    [bs,kv,n_max,...] buffers (+ the KIVI scales when kscale is given)."""
    _dtype("keys", keys, torch.bfloat16)
    bs, kv, T, D = keys.shape
    if D != 128 or T % 16:
        raise ValueError(f"keys must be [bs,kv,16*n,128]; got {tuple(keys.shape)}")
    if keys.stride(3) != 1 or keys.stride(2) != 128 or keys.stride(0) != kv * keys.stride(1):
        keys = keys.contiguous()
    n_max = chunk_min.shape[2]
    for n, t in (("chunk_min", chunk_min), ("chunk_max", chunk_max), ("packed", packed)):
        _contig(n, t)
    check(lib().zkv_kivi_encode(_p(keys), keys.stride(1), bs * kv, T // 16, int(chunk_start), n_max, _p(chunk_min),
                                _p(chunk_max), _p(chunk_centroid), _p(chunk_valid), _p(packed), _p(kscale),
                                _stream(keys)),
          "zkv_kivi_encode")


def vquant_encode(values, vcodes_t, vmeta, tok_start: int):
    """Per-token 4-bit values of `values` [bs,kv,T,128] into the page buffers
    vcodes_t [bs,kv,n_pages,128,2] int32 / vmeta [bs,kv,n_pages,2,4,16] bf16."""
    _dtype("values", values, torch.bfloat16)
    bs, kv, T, D = values.shape
    if values.stride(3) != 1 or values.stride(2) != 128 or values.stride(0) != kv * values.stride(1):
        values = values.contiguous()
    n_pages = vcodes_t.shape[2]
    check(lib().zkv_vquant_encode(_p(values), values.stride(1), bs * kv, T, int(tok_start), n_pages, _p(vcodes_t),
                                  _p(vmeta), _stream(values)), "zkv_vquant_encode")


# ----------------------------------------------------------------- attention
def attn_rows(q, keys, values, *, seg0=(0, 0), sel=None, sel_offset=0, seg1=(0, 0), scale=None, out=None, lse=None,
              split=0, status=None):
    """Decode attention of q [bs,1,H*G,128] over the raw rows of keys/values
    [bs,H,cap,128] at [seg0) U sel[b,h,:]+sel_offset U [seg1) -> out [bs,1,H*G,128]."""
    _dtype("q", q, torch.bfloat16)
    bs, H, cap, D = keys.shape
    G = q.shape[2] // H
    qc = q.contiguous()
    if keys.stride(3) != 1 or keys.stride(2) != 128 or keys.stride(0) != H * keys.stride(1):
        raise ValueError("keys must be [bs,H,cap,128] with contiguous rows")
    if values.stride() != keys.stride():
        raise ValueError("keys and values must share a layout")
    if out is None:
        out = torch.empty(bs, 1, H * G, D, dtype=torch.bfloat16, device=q.device)
    n_sel, sel_ld, sp = 0, 0, None
    if sel is not None and sel.shape[-1] > 0:
        if sel.stride(2) != 1 or sel.stride(0) != H * sel.stride(1):
            sel = sel.contiguous()
        n_sel, sel_ld, sp = sel.shape[2], sel.stride(1), _p(sel)
    scale = (1.0 / D ** 0.5) if scale is None else float(scale)
    check(lib().zkv_attn_rows(_p(qc), _p(keys), _p(values), keys.stride(1), bs * H, G, int(seg0[0]), int(seg0[1]),
                              sp, n_sel, sel_ld, int(sel_offset), int(seg1[0]), int(seg1[1]), scale, _p(out),
                              _p(lse), int(split), _p(status), _stream(q)), "zkv_attn_rows")
    return out


# ----------------------------------------------------------------- offload tier (host-pinned rows)
def _require(cond, msg):
    if not cond:
        raise AssertionError(msg)


def _pinned_src(src_k, src_v):
    _require(src_k.shape == src_v.shape, "src_k_caches and src_v_caches must have the same shape")
    _require(src_k.dim() == 4 and src_k.shape[-1] == 128, "src caches must be [bs, heads, kv_len, 128]")
    _require(not src_k.is_cuda and not src_v.is_cuda, "src caches must be CPU tensors")
    _require(src_k.is_pinned() and src_v.is_pinned(), "src caches must be host-pinned (pin_memory=True)")
    _require(src_k.dtype == torch.bfloat16 and src_v.dtype == torch.bfloat16, "src caches must be bfloat16")
    _require(src_k.is_contiguous() and src_v.is_contiguous(), "src caches must be contiguous")


def h2d_gather_kv(src_k_caches, src_v_caches, selected_indices, dst_k_caches, dst_v_caches, status=None):
    """dst[b,h,j] = src[b,h,selected_indices[b,h,j]] for j < topk, K and V.

    Reference: cache_hub/gather_trans/trans_h2d.py:65-105 (same checks, as
    AssertionError).  src_* host-pinned [bs,heads,kv_len,128] bf16;
    selected_indices CUDA [bs,heads,topk] int64; dst_* CUDA
    [bs,heads,max_topk >= topk,128] bf16; rows j >= topk are not written.
    An index outside [0, kv_len) is skipped and reported through `status`
    (int32 CUDA word, ZKV_ERR_RANGE) when one is given."""
    _pinned_src(src_k_caches, src_v_caches)
    bs, heads, kv_len, dim = src_k_caches.shape
    _require(selected_indices.dim() == 3 and tuple(selected_indices.shape[:2]) == (bs, heads),
             "selected_indices must be [bs, heads, topk]")
    topk = selected_indices.shape[2]
    _require(dst_k_caches.shape == dst_v_caches.shape, "dst_k_caches and dst_v_caches must have the same shape")
    _require(dst_k_caches.dim() == 4 and tuple(dst_k_caches.shape[:2]) == (bs, heads) and dst_k_caches.shape[3] == dim,
             "dst caches must be [bs, heads, max_topk, 128]")
    _require(dst_k_caches.shape[-2] >= topk, "dst caches hold fewer rows than topk")
    _require(dst_k_caches.is_cuda and dst_v_caches.is_cuda and selected_indices.is_cuda,
             "dst caches and selected_indices must be CUDA tensors")
    _require(dst_k_caches.dtype == torch.bfloat16 and dst_v_caches.dtype == torch.bfloat16,
             "dst caches must be bfloat16")
    _require(selected_indices.dtype == torch.int64, "selected_indices must be int64")
    _require(dst_k_caches.is_contiguous() and dst_v_caches.is_contiguous() and selected_indices.is_contiguous(),
             "dst caches and selected_indices must be contiguous")
    check(lib().zkv_h2d_gather_kv(_p(src_k_caches), _p(src_v_caches), bs * heads, kv_len, _p(selected_indices), topk,
                                  topk, 0, _p(dst_k_caches), _p(dst_v_caches), dst_k_caches.shape[2], 0, _p(status),
                                  _stream(dst_k_caches)), "zkv_h2d_gather_kv")


def h2d_gather_kv_packed(src_k_caches, src_v_caches, dst_k_packed, dst_v_packed, indices_packed, cu_seqlens_topk,
                         cu_seqlens_k, sl_end: int, global_k: int, status=None):
    """Variable-K gather into a flash-attention varlen packed buffer.

    Reference: cache_hub/gather_trans/trans_h2d.py:108-161.  For every
    vh = b*heads + h, rows [cu_seqlens_k[vh] + sl_end, cu_seqlens_k[vh+1]) of
    dst_*_packed [total_k,128] receive src[b,h,indices_packed[cu_seqlens_topk
    [vh] + slot]] for slot < min(global_k, segment length); the first sl_end
    rows of every segment are left as they are."""
    _pinned_src(src_k_caches, src_v_caches)
    bs, heads, kv_len, dim = src_k_caches.shape
    V = bs * heads
    _require(dst_k_packed.is_cuda and dst_v_packed.is_cuda, "dst_*_packed must be CUDA tensors")
    _require(indices_packed.is_cuda and cu_seqlens_topk.is_cuda and cu_seqlens_k.is_cuda,
             "indices and cu_seqlens must be CUDA tensors")
    _require(dst_k_packed.dtype == torch.bfloat16 and dst_v_packed.dtype == torch.bfloat16,
             "dst_*_packed must be bfloat16")
    _require(indices_packed.dtype == torch.int64, "indices_packed must be int64")
    _require(cu_seqlens_topk.dtype == torch.int32 and cu_seqlens_k.dtype == torch.int32, "cu_seqlens must be int32")
    _require(dst_k_packed.is_contiguous() and dst_v_packed.is_contiguous(), "dst_*_packed must be contiguous")
    _require(dst_k_packed.dim() == 2 and dst_k_packed.shape[1] == dim, "dst_*_packed must be [total_k, 128]")
    _require(dst_v_packed.shape == dst_k_packed.shape, "dst_k_packed and dst_v_packed must have the same shape")
    _require(cu_seqlens_topk.shape[0] == V + 1 and cu_seqlens_k.shape[0] == V + 1, "cu_seqlens must be [V + 1]")
    _require(indices_packed.dim() == 1, "indices_packed must be 1-D")
    _require(indices_packed.is_contiguous() and cu_seqlens_topk.is_contiguous() and cu_seqlens_k.is_contiguous(),
             "indices and cu_seqlens must be contiguous")
    check(lib().zkv_h2d_gather_kv_packed(_p(src_k_caches), _p(src_v_caches), V, kv_len, _p(indices_packed),
                                         _p(cu_seqlens_topk), _p(cu_seqlens_k), int(sl_end), int(global_k),
                                         _p(dst_k_packed), _p(dst_v_packed), dst_k_packed.shape[0], _p(status),
                                         _stream(dst_k_packed)), "zkv_h2d_gather_kv_packed")


def h2d_gather_rows(src_k, src_v, sel, dst_k, dst_v, *, n_sel=None, src_offset=0, dst_offset=0, status=None):
    """Offload-tier gather with offsets: dst[b,h,dst_offset+j] =
    src[b,h,sel[b,h,j]+src_offset] for j < n_sel.  src_* host-pinned
    [bs,H,cap,128]; dst_* CUDA [bs,H,dst_len,128] (row-contiguous, any
    leading strides equal); sel CUDA [bs,H,>=n_sel] int64 with unit last
    stride."""
    bs, H, cap, _ = src_k.shape
    n = sel.shape[2] if n_sel is None else int(n_sel)
    if dst_k.stride(3) != 1 or dst_k.stride(2) != 128 or dst_k.stride(0) != H * dst_k.stride(1):
        raise ValueError("dst_k must be [bs,H,len,128] with contiguous rows")
    if dst_v.stride() != dst_k.stride():
        raise ValueError("dst_k and dst_v must share a layout")
    if sel.stride(2) != 1 or sel.stride(0) != H * sel.stride(1):
        raise ValueError("sel must be [bs,H,n] with unit last stride")
    check(lib().zkv_h2d_gather_kv(_p(src_k), _p(src_v), bs * H, cap, _p(sel), sel.stride(1), n, int(src_offset),
                                  _p(dst_k), _p(dst_v), dst_k.stride(1) // 128, int(dst_offset), _p(status),
                                  _stream(dst_k)), "zkv_h2d_gather_kv")


class PageLayer:
    """Tensors of one layer of the page-mode cache ([bs, H, ...] each)."""

    def __init__(self, chunk_min, chunk_max, valid, kcodes, vcodes_t, vmeta, near_k, near_v, kscale):
        self.tensors = (chunk_min, chunk_max, valid, kcodes, vcodes_t, vmeta, near_k, near_v, kscale)
        self.struct = _lib.ZkvPageLayer(
            _p(chunk_min), _p(chunk_max), _p(valid), _p(kcodes), _p(vcodes_t), _p(vmeta), _p(near_k), _p(near_v),
            near_k.shape[2], _p(kscale))


_SPLIT_WS: dict = {}
_SM_COUNT: dict = {}


def _sm_count(dev) -> int:
    i = dev.index if dev.index is not None else torch.cuda.current_device()
    if i not in _SM_COUNT:
        _SM_COUNT[i] = torch.cuda.get_device_properties(i).multi_processor_count
    return _SM_COUNT[i]


def page_decode_split_ws_bytes(rows: int, n_c: int) -> int:
    return int(lib().zkv_page_decode_split_ws_bytes(int(rows), int(n_c)))


def page_decode_plan(rows: int, n_c: int, nk: int, cluster: int = 0, split=None, device=None) -> dict:
    """How page_decode runs a layer: {'split': bool, 'parts': clusters per
    row, 'launches': kernels per call} (the rule zkv_page_decode_split and
    page_decode apply)."""
    dev = torch.device("cuda") if device is None else torch.device(device)
    cs = cluster if cluster in (1, 2, 4, 8) else 8
    two_level = cs > 1 and n_c > 2048 and nk < n_c
    if split is None:
        split = two_level and 2 * rows * cs <= _sm_count(dev)
    if not (split and two_level):
        return {"split": False, "parts": 1, "launches": 1}
    parts = max(1, min(4, (2 * _sm_count(dev)) // (rows * cs)))
    return {"split": True, "parts": parts, "launches": 3 if parts > 1 else 2}


def page_decode(q, layer: PageLayer, n_c: int, nk: int, n_near: int, *, n_sink: int = 0, near_start: int = 0,
                scale=None, out=None, lse=None, sel_out=None, status=None, cluster=0, split=None, workspace=None):
    """Fused page-mode decode: q [bs,1,H*G,128] -> out [bs,1,H*G,128].

    Raw rows attended besides the selected pages: [0, n_sink) and
    [near_start, near_start + n_near) of the layer's near buffers.

    split: None picks the long-context form (zkv_page_decode_split: Quest
    scores on every SM, then the fused select + attention) when the rows'
    clusters fill at most half of the SMs and n_c > 2048; True / False force
    it on / off (same selection; the split form may spread a row's pages over
    several clusters and merge their (out, lse), so the output can differ from
    the fused form by fp32 rounding).  workspace: optional uint8 device
    tensor for the split form (default: one cached buffer per device, so
    concurrent calls on different streams should pass their own)."""
    cmin = layer.tensors[0]
    bs, H, n_max, D = cmin.shape
    G = q.shape[2] // H
    qc = q.contiguous()
    if out is None:
        out = torch.empty(bs, 1, H * G, D, dtype=torch.bfloat16, device=q.device)
    scale = (1.0 / D ** 0.5) if scale is None else float(scale)
    rows = bs * H
    if split is None:
        cs = cluster if cluster in (1, 2, 4, 8) else 8
        split = cs > 1 and n_c > 2048 and nk < n_c and 2 * rows * cs <= _sm_count(q.device)
    if split:
        need = page_decode_split_ws_bytes(rows, n_c)
        if workspace is None:
            key = q.device.index if q.device.index is not None else torch.cuda.current_device()
            ws = _SPLIT_WS.get(key)
            if ws is None or ws.numel() < need:
                ws = torch.empty(max(need, 1), dtype=torch.uint8, device=q.device)
                _SPLIT_WS[key] = ws
            workspace = ws
        check(lib().zkv_page_decode_split(_p(qc), ctypes.byref(layer.struct), rows, G, n_max, int(n_c), int(nk),
                                          int(n_sink), int(near_start), int(n_near), scale, _p(out), _p(lse),
                                          _p(sel_out), _p(status), int(cluster), _p(workspace),
                                          int(workspace.numel()), _stream(q)), "zkv_page_decode_split")
        return out
    check(lib().zkv_page_decode(_p(qc), ctypes.byref(layer.struct), rows, G, n_max, int(n_c), int(nk), int(n_sink),
                                int(near_start), int(n_near), scale, _p(out), _p(lse), _p(sel_out), _p(status),
                                int(cluster), _stream(q)), "zkv_page_decode")
    return out


def page_attend(q, layer: PageLayer, sel, sel_lo: int, sel_hi: int, *, n_sink: int = 0, near_start: int = 0,
                n_near: int = 0, scale=None, out=None, out_f32=None, lse=None, status=None, cluster=0):
    """Attention over externally selected pages (sequence split): sel
    [bs, H, n_sel] global page ids; this layer buffer holds pages
    [sel_lo, sel_hi).  Returns out_f32 [bs, H*G, 128] fp32 when given, else
    bf16 out [bs, 1, H*G, 128]; lse [bs, H*G] fp32 (natural log) if given."""
    cmin = layer.tensors[0]
    bs, H, _, D = cmin.shape
    n_max = cmin.stride(1) // D   # row stride in pages (views of a chunk range keep the full stride)
    G = q.shape[2] // H
    _dtype("sel", sel, torch.int64)
    _contig("sel", sel)
    qc = q.contiguous()
    if out is None and out_f32 is None:
        out = torch.empty(bs, 1, H * G, D, dtype=torch.bfloat16, device=q.device)
    scale = (1.0 / D ** 0.5) if scale is None else float(scale)
    check(lib().zkv_page_attend(_p(qc), ctypes.byref(layer.struct), bs * H, G, n_max, _p(sel), sel.shape[-1],
                                int(sel_lo), int(sel_hi), int(n_sink), int(near_start), int(n_near), scale, _p(out),
                                _p(out_f32), _p(lse), _p(status), int(cluster), _stream(q)), "zkv_page_attend")
    return out_f32 if out_f32 is not None else out


def page_decode_scored(q, layer: PageLayer, scores, n_c: int, nk: int, own_lo: int, own_hi: int, parts: int,
                       out_f32, lse, *, n_sink: int = 0, near_start: int = 0, n_near: int = 0, scale=None,
                       sel_out=None, status=None, cluster=0):
    """Select + attend step of the sequence split: top nk of the score row
    scores [bs, H, >= n_c] fp32 (global chunk ids), attention over the
    selected pages in [own_lo, own_hi) that this layer buffer holds (page
    id - own_lo) plus the raw rows, over `parts` clusters per row.  Writes
    out_f32 [parts, bs*H*G, 128] and lse [parts, bs*H*G] partials."""
    cmin = layer.tensors[0]
    bs, H, _, D = cmin.shape
    n_max = cmin.stride(1) // D
    G = q.shape[2] // H
    _dtype("scores", scores, torch.float32)
    if scores.stride(-1) != 1 or scores.stride(0) != H * scores.stride(1):
        raise ValueError("scores must be [bs, H, n] with unit last stride")
    qc = q.contiguous()
    scale = (1.0 / D ** 0.5) if scale is None else float(scale)
    check(lib().zkv_page_decode_scored(_p(qc), ctypes.byref(layer.struct), bs * H, G, n_max, _p(scores),
                                       scores.stride(1), int(n_c), int(nk), int(own_lo), int(own_hi), int(n_sink),
                                       int(near_start), int(n_near), scale, int(parts), _p(out_f32), _p(lse),
                                       _p(sel_out), _p(status), int(cluster), _stream(q)), "zkv_page_decode_scored")
    return out_f32


class RawLayer:
    """One layer of the raw-page cache: Quest metadata chunk_min / chunk_max
    [bs, H, n_max, 128] bf16 (+ valid [bs, H, n_max] or None) and the raw
    keys / values [bs, H, cap, 128] bf16 at absolute token positions; chunk c
    covers tokens page_base + 16 c .. + 15 (page_base = the sink size)."""

    def __init__(self, chunk_min, chunk_max, valid, keys, values, page_base: int = 0):
        for n, t in (("chunk_min", chunk_min), ("chunk_max", chunk_max), ("keys", keys), ("values", values)):
            _dtype(n, t, torch.bfloat16)
            _cuda((n, t))
        for n, t in (("chunk_min", chunk_min), ("chunk_max", chunk_max)):
            _contig(n, t)
        for n, t in (("keys", keys), ("values", values)):
            if t.dim() != 4 or t.shape[3] != 128 or t.stride(3) != 1 or t.stride(2) != 128 or \
                    t.stride(0) != t.shape[1] * t.stride(1):
                raise ValueError(f"{n} must be [bs, H, cap, 128] with rows of 128 contiguous elements")
        if keys.shape != values.shape or keys.stride() != values.stride():
            raise ValueError("keys and values must have the same shape and strides")
        if valid is not None:
            _contig("valid", valid)
        self.tensors = (chunk_min, chunk_max, valid, keys, values)
        self.page_base = int(page_base)
        self.struct = _lib.ZkvRawLayer(_p(chunk_min), _p(chunk_max), _p(valid), _p(keys), _p(values),
                                       keys.stride(1), self.page_base)


_RAW_WS: dict = {}
_RAW_NEED: dict = {}


def page_decode_raw_ws_bytes(rows: int, n_c: int, nk: int, n_sink: int, n_near: int) -> int:
    return int(lib().zkv_page_decode_raw_ws_bytes(int(rows), int(n_c), int(nk), int(n_sink), int(n_near)))


def page_decode_raw(q, layer: RawLayer, n_c: int, nk: int, n_near: int, *, n_sink: int = 0, near_start: int = 0,
                    scale=None, out=None, lse=None, sel_out=None, status=None, workspace=None):
    """Page mode over raw rows: q [bs,1,H*G,128] -> out [bs,1,H*G,128] bf16.

    Quest scores of chunks [0, n_c), top nk chunks, then attention over the
    selected chunks' raw rows, the sink rows [0, n_sink) and the near rows
    [near_start, near_start + n_near) of layer.keys / layer.values.
    workspace: optional uint8 device tensor of at least
    page_decode_raw_ws_bytes(...) bytes, scratch only (default: one cached
    buffer per device, so calls on concurrent streams should pass their
    own)."""
    cmin = layer.tensors[0]
    bs, H, n_max, D = cmin.shape
    _dtype("q", q, torch.bfloat16)
    G = q.shape[2] // H
    qc = q.contiguous()
    if out is None:
        out = torch.empty(bs, 1, H * G, D, dtype=torch.bfloat16, device=q.device)
    scale = (1.0 / D ** 0.5) if scale is None else float(scale)
    rows = bs * H
    if workspace is None:
        shape = (rows, int(n_c), int(nk), int(n_sink), int(n_near))
        need = _RAW_NEED.get(shape)
        if need is None:
            need = _RAW_NEED[shape] = page_decode_raw_ws_bytes(*shape)
        key = q.device.index if q.device.index is not None else torch.cuda.current_device()
        ws = _RAW_WS.get(key)
        if ws is None or ws.numel() < need:
            ws = torch.empty(max(need, 1 << 20), dtype=torch.uint8, device=q.device)
            _RAW_WS[key] = ws
        workspace = ws
    check(lib().zkv_page_decode_raw(_p(qc), ctypes.byref(layer.struct), rows, G, n_max, int(n_c), int(nk),
                                    int(n_sink), int(near_start), int(n_near), scale, _p(out), _p(lse),
                                    _p(sel_out), _p(status), _p(workspace), int(workspace.numel()), _stream(q)),
          "zkv_page_decode_raw")
    return out


def raw_split_range(n_c: int, world: int, rank: int):
    """(lo, hi): the global pages [lo, hi) rank holds in the raw sequence
    split (per = ceil(n_c / world) rounded up to 16 pages)."""
    lo, hi = ctypes.c_int(), ctypes.c_int()
    check(lib().zkv_raw_split_range(int(n_c), int(world), int(rank), ctypes.byref(lo), ctypes.byref(hi)),
          "zkv_raw_split_range")
    return lo.value, hi.value


def page_decode_raw_split(q, layer: RawLayer, split, n_c: int, nk: int, n_near: int, *, n_sink: int = 0,
                          near_start: int = 0, scale=None, out=None, lse=None, sel_out=None, status=None,
                          workspace=None):
    """One rank's share of page_decode_raw under the sequence split:
    q [bs,1,H*G,128] (the same on every rank) -> out [bs,1,H*G,128] bf16,
    the same on every rank.  layer holds this rank's pages
    raw_split_range(n_c, world, rank) as its local pages (rank 0 also the
    sink / near rows); n_c and nk count the whole row's pages.  split: an
    object with .struct (a ZkvRawSplit over the group's exchange buffers),
    .rank and .world (seqsplit.RawSplitGroup).  sel_out [bs*H, nk] int64:
    the whole selection (global ids).  workspace: uint8 device tensor of at
    least zkv_page_decode_raw_split_ws_bytes(...) (default: one cached
    buffer per device)."""
    cmin = layer.tensors[0]
    bs, H, n_max, D = cmin.shape
    _dtype("q", q, torch.bfloat16)
    G = q.shape[2] // H
    qc = q.contiguous()
    if out is None:
        out = torch.empty(bs, 1, H * G, D, dtype=torch.bfloat16, device=q.device)
    scale = (1.0 / D ** 0.5) if scale is None else float(scale)
    rows = bs * H
    if workspace is None:
        shape = ("split", rows, int(n_c), split.world, split.rank, int(nk), int(n_sink), int(n_near))
        need = _RAW_NEED.get(shape)
        if need is None:
            need = _RAW_NEED[shape] = int(lib().zkv_page_decode_raw_split_ws_bytes(*shape[1:]))
        key = ("split", q.device.index if q.device.index is not None else torch.cuda.current_device())
        ws = _RAW_WS.get(key)
        if ws is None or ws.numel() < need:
            ws = torch.empty(max(need, 1 << 20), dtype=torch.uint8, device=q.device)
            _RAW_WS[key] = ws
        workspace = ws
    check(lib().zkv_page_decode_raw_split(_p(qc), ctypes.byref(layer.struct), ctypes.byref(split.struct), rows, G,
                                          n_max, int(n_c), int(nk), int(n_sink), int(near_start), int(n_near),
                                          scale, _p(out), _p(lse), _p(sel_out), _p(status), _p(workspace),
                                          int(workspace.numel()), _stream(q)),
          "zkv_page_decode_raw_split")
    return out


class LargeLayer:
    """Hierarchical Quest metadata of one layer: large_min / large_max
    [bs, H, n_max_large, 128] bf16 and large_valid [bs, H, n_max_large]
    (bool or uint8), the per-large-chunk bounding boxes of
    polar_cache_kivi_quest_density_seperate_kernel.py:1762-1798."""

    def __init__(self, large_min, large_max, large_valid):
        for n, t in (("large_min", large_min), ("large_max", large_max), ("large_valid", large_valid)):
            _cuda((n, t))
            _contig(n, t)
        _dtype("large_min", large_min, torch.bfloat16)
        _dtype("large_max", large_max, torch.bfloat16)
        if large_min.shape != large_max.shape or tuple(large_valid.shape) != tuple(large_min.shape[:3]):
            raise ValueError("large_min / large_max [bs, H, n_max_large, 128] and large_valid [bs, H, n_max_large]")
        self.tensors = (large_min, large_max, large_valid)
        self.struct = _lib.ZkvQuestLarge(_p(large_min), _p(large_max), _p(large_valid), large_min.shape[2])


def quest_large_minmax(chunk_min, chunk_max, valid_end: int, factor: int, large_min, large_max, large_valid,
                       g_lo: int = 0, g_hi=None):
    """_update_large_chunk_minmax (polar_cache_kivi_quest_density_seperate_
    kernel.py:1762-1798) for groups [g_lo, g_hi) in place: group g covers
    chunks [g*factor, min(g*factor + factor, valid_end))."""
    bs, H, n_max, D = chunk_min.shape
    nml = large_min.shape[2]
    g_hi = nml if g_hi is None else int(g_hi)
    for n, t in (("chunk_min", chunk_min), ("chunk_max", chunk_max)):
        _contig(n, t)
    check(lib().zkv_quest_large_minmax(_p(chunk_min), _p(chunk_max), bs * H, n_max, int(valid_end), int(factor),
                                       int(g_lo), g_hi, _p(large_min), _p(large_max), _p(large_valid), nml,
                                       _stream(chunk_min)), "zkv_quest_large_minmax")


def page_decode_raw_hier(q, layer: RawLayer, large: LargeLayer, n_c: int, factor: int, nk_large: int, nk_small: int,
                         n_near: int, *, n_sink: int = 0, near_start: int = 0, scale=None, out=None, lse=None,
                         sel_out=None, status=None, workspace=None):
    """page_decode_raw with the hierarchical Quest pick: Quest over the
    n_c // factor large chunks, their top nk_large, the sub-chunk scores of
    those, the top nk_small sub-chunks mapped back to chunk ids, attention
    over those pages' raw rows + sink + near rows."""
    cmin = layer.tensors[0]
    bs, H, n_max, D = cmin.shape
    _dtype("q", q, torch.bfloat16)
    G = q.shape[2] // H
    qc = q.contiguous()
    if out is None:
        out = torch.empty(bs, 1, H * G, D, dtype=torch.bfloat16, device=q.device)
    scale = (1.0 / D ** 0.5) if scale is None else float(scale)
    rows = bs * H
    if workspace is None:
        shape = ("hier", rows, int(n_c), int(factor), int(nk_large), int(nk_small), int(n_sink), int(n_near))
        need = _RAW_NEED.get(shape)
        if need is None:
            need = _RAW_NEED[shape] = int(lib().zkv_page_decode_raw_hier_ws_bytes(*shape[1:]))
        key = q.device.index if q.device.index is not None else torch.cuda.current_device()
        ws = _RAW_WS.get(key)
        if ws is None or ws.numel() < need:
            ws = torch.empty(max(need, 1 << 20), dtype=torch.uint8, device=q.device)
            _RAW_WS[key] = ws
        workspace = ws
    check(lib().zkv_page_decode_raw_hier(_p(qc), ctypes.byref(layer.struct), ctypes.byref(large.struct), rows, G,
                                         n_max, int(n_c), int(factor), int(nk_large), int(nk_small), int(n_sink),
                                         int(near_start), int(n_near), scale, _p(out), _p(lse), _p(sel_out),
                                         _p(status), _p(workspace), int(workspace.numel()), _stream(q)),
          "zkv_page_decode_raw_hier")
    return out


# ----------------------------------------------------------------- decode-loop caller
def rmsnorm(x, w, eps: float, out=None):
    """Row-wise RMSNorm of x [..., dim] bf16 with weight w [dim] (fp32 inside)."""
    _dtype("x", x, torch.bfloat16)
    _contig("x", x)
    out = torch.empty_like(x) if out is None else out
    check(lib().zkv_rmsnorm(_p(x), _p(w), _p(out), x.numel() // x.shape[-1], x.shape[-1], float(eps), _stream(x)),
          "zkv_rmsnorm")
    return out


def qk_norm_rope(qkv, q_norm, k_norm, cos, sin, pos, hq: int, hkv: int, eps: float, q, k, v):
    """qkv [rows, (hq + 2 hkv) * 128] -> q / k (per-head RMSNorm + rotate-half
    RoPE at position pos[0], a device int64) and v, into the given buffers."""
    _contig("qkv", qkv)
    rows = qkv.numel() // ((hq + 2 * hkv) * 128)
    check(lib().zkv_qk_norm_rope(_p(qkv), _p(q_norm), _p(k_norm), _p(cos), _p(sin), _p(pos), rows, hq, hkv,
                                 float(eps), _p(q), _p(k), _p(v), _stream(qkv)), "zkv_qk_norm_rope")


def silu_mul(gu, out):
    """out [rows, ffn] = silu(gu[:, :ffn]) * gu[:, ffn:] (bf16, fp32 inside)."""
    _contig("gu", gu)
    ffn = gu.shape[-1] // 2
    check(lib().zkv_silu_mul(_p(gu), _p(out), gu.numel() // gu.shape[-1], ffn, _stream(gu)), "zkv_silu_mul")
    return out


def gqa_mean(q, heads: int, out=None):
    """raw_q [bs, H, 128] bf16 = GQA mean of q [bs, 1, H*G, 128] (fp32 sum in
    head order / G, as the fused kernels compute it)."""
    _dtype("q", q, torch.bfloat16)
    qc = q.contiguous()
    bs = qc.shape[0]
    G = qc.shape[-2] // heads
    if out is None:
        out = torch.empty(bs, heads, 128, dtype=torch.bfloat16, device=q.device)
    check(lib().zkv_gqa_mean(_p(qc), bs * heads, G, _p(out), _stream(q)), "zkv_gqa_mean")
    return out


# ----------------------------------------------------------------- ParisKV / RaBitQ
# Magnitude thresholds / reconstruction centres (cache_hub/polar_cache.py:267-270)
MAG_THRESHOLDS = (0.0843, 0.1698, 0.2578, 0.3499, 0.4487, 0.5585, 0.6901)
MAG_CENTERS = (0.0420, 0.1266, 0.2130, 0.3025, 0.3973, 0.5001, 0.6169, 0.7633)


def _row_stride(name, t, lead=2):
    """Stride that flattens the leading `lead` dims of t into rows."""
    if lead == 2 and t.dim() >= 2 and t.shape[0] > 1 and t.stride(0) != t.shape[1] * t.stride(1):
        raise ValueError(f"{name}: batch and head dims must flatten into rows")
    return t.stride(lead - 1)


class RqLayout:
    """Per-key ParisKV codes of one layer (device tensors) + the C struct.

    Token-major (this build, `alloc`): codes [rows, cap, 16] u8, packed
    [rows, cap, 16] int32 (one word = one block's 8 nibbles), weight
    [rows, cap, 16] bf16, factor [rows, cap] f32, hist [rows, 16, 256] i32.
    Block-major (the reference's tensors, `from_reference`): codebook
    [bs, H, 16, len] u8, key_4bit [bs, H, 16, len, 4] u8, key_block_weight
    [bs, H, 16, len] bf16 (views sliced along len are accepted)."""

    def __init__(self, codes, packed, weight, factor, hist, strides):
        self.codes, self.packed, self.weight, self.factor, self.hist = codes, packed, weight, factor, hist
        self._strides = strides
        (cr, cb, ct), (pr, pb, pt), (wr, wb, wt), fr = strides
        self._s = _lib.ZkvRqLayout(
            _p(codes), cr, cb, ct, _p(packed), pr, pb, pt, _p(weight), wr, wb, wt, _p(factor), fr, _p(hist))

    def tokens(self, lo: int) -> "RqLayout":
        """The same layout with token 0 at token `lo` (token-major buffers of
        `alloc`): kernels then index keys relative to `lo`."""
        (cr, cb, ct), (pr, pb, pt), (wr, wb, wt), fr = self._strides
        if not (cb == 1 and ct == 16 and pb == 1 and pt == 16):
            raise ValueError("tokens(): token-major layouts only")
        v = RqLayout(self.codes[:, lo:], self.packed[:, lo:], self.weight[:, lo:],
                     None if self.factor is None else self.factor[:, lo:], self.hist, self._strides)
        return v

    @classmethod
    def alloc(cls, rows: int, cap: int, device) -> "RqLayout":
        z = dict(device=device)
        codes = torch.zeros(rows, cap, 16, dtype=torch.uint8, **z)
        packed = torch.zeros(rows, cap, 16, dtype=torch.int32, **z)
        weight = torch.zeros(rows, cap, 16, dtype=torch.bfloat16, **z)
        factor = torch.zeros(rows, cap, dtype=torch.float32, **z)
        hist = torch.zeros(rows, 16, 256, dtype=torch.int32, **z)
        return cls(codes, packed, weight, factor, hist,
                   ((cap * 16, 1, 16), (cap * 16, 1, 16), (cap * 16, 1, 16), cap))

    @classmethod
    def from_reference(cls, codebook, key_4bit=None, key_block_weight=None, cluster_key_counts=None) -> "RqLayout":
        _cuda(("codebook", codebook), ("key_4bit", key_4bit), ("key_block_weight", key_block_weight),
              ("cluster_key_counts", cluster_key_counts))
        _dtype("codebook", codebook, torch.uint8)
        cs = (_row_stride("codebook", codebook), codebook.stride(2), codebook.stride(3))
        ps = ws = (0, 0, 0)
        if key_4bit is not None:
            _dtype("key_4bit", key_4bit, torch.uint8)
            if key_4bit.shape[-1] != 4 or key_4bit.stride(-1) != 1 or key_4bit.data_ptr() % 4:
                raise ValueError("key_4bit must be [bs, H, 16, len, 4] with 4-byte aligned contiguous blocks")
            ps = tuple(x // 4 for x in (_row_stride("key_4bit", key_4bit), key_4bit.stride(2), key_4bit.stride(3)))
        if key_block_weight is not None:
            _dtype("key_block_weight", key_block_weight, torch.bfloat16)
            ws = (_row_stride("key_block_weight", key_block_weight), key_block_weight.stride(2),
                  key_block_weight.stride(3))
        hist = None
        if cluster_key_counts is not None:
            _dtype("cluster_key_counts", cluster_key_counts, torch.int32)
            _contig("cluster_key_counts", cluster_key_counts)
            hist = cluster_key_counts
        return cls(codebook, key_4bit, key_block_weight, None, hist, (cs, ps, ws, 0))

    @property
    def struct(self):
        return ctypes.byref(self._s)


def rq_encode(keys, signs, lay: RqLayout, tok_start: int = 0):
    """Encode keys [rows, T, 128] (or [bs, H, T, 128]) bf16 into `lay` at
    tokens [tok_start, tok_start + T) and add them to lay.hist."""
    _cuda(("keys", keys), ("signs", signs))
    _dtype("keys", keys, torch.bfloat16)
    _dtype("signs", signs, torch.bfloat16)
    if keys.stride(-1) != 1 or keys.shape[-1] != 128:
        raise ValueError("keys must be [..., T, 128] with a contiguous last dim")
    if keys.dim() == 4:
        ld, rows, T = _row_stride("keys", keys), keys.shape[0] * keys.shape[1], keys.shape[2]
        if keys.stride(2) != 128:
            raise ValueError("keys tokens must be contiguous rows of 128")
    else:
        ld, rows, T = keys.stride(0), keys.shape[0], keys.shape[1]
    check(lib().zkv_rq_encode(_p(keys), ld, rows, T, tok_start, _p(signs.contiguous()), lay.struct, _stream(keys)),
          "zkv_rq_encode")


def batch_encode(Y, signs):
    """Reference-layout form of ParisKV batch_encode: Y [bs, H, len, 128] bf16
    -> (codebook [bs,H,16,len] u8, block_weight [bs,H,16,len] bf16,
    packed_4bit [bs,H,16,len,4] u8, cluster_key_counts [bs,H,16,256] i32)."""
    bs, H, T, _ = Y.shape
    z = dict(device=Y.device)
    codebook = torch.empty(bs, H, 16, T, dtype=torch.uint8, **z)
    weight = torch.empty(bs, H, 16, T, dtype=torch.bfloat16, **z)
    packed = torch.empty(bs, H, 16, T, 4, dtype=torch.uint8, **z)
    counts = torch.zeros(bs, H, 16, 256, dtype=torch.int32, **z)
    lay = RqLayout.from_reference(codebook, packed, weight, counts)
    rq_encode(Y, signs, lay)
    return codebook, weight, packed, counts


def rq_query(q, signs, group: int = 4, *, planes: bool = False):
    """q [bs, 1, H*G, 128] or [rows, G, 128] bf16 -> dict(q_blocks [rows,128],
    q_norm [rows], q_mean [rows,128] bf16; planes [rows,4,16] u8 and qparams
    [rows,4] f32 when planes=True)."""
    _cuda(("q", q), ("signs", signs))
    _dtype("q", q, torch.bfloat16)
    q = q.contiguous()
    rows = q.numel() // (group * 128)
    dev = q.device
    out = dict(q_blocks=torch.empty(rows, 128, dtype=torch.bfloat16, device=dev),
               q_norm=torch.empty(rows, dtype=torch.bfloat16, device=dev),
               q_mean=torch.empty(rows, 128, dtype=torch.bfloat16, device=dev))
    pl = qp = None
    if planes:
        pl = out["planes"] = torch.empty(rows, 4, 16, dtype=torch.uint8, device=dev)
        qp = out["qparams"] = torch.empty(rows, 4, dtype=torch.float32, device=dev)
    check(lib().zkv_rq_query(_p(q), rows, group, _p(signs.contiguous()), _p(out["q_blocks"]), _p(out["q_norm"]),
                             _p(out["q_mean"]), _p(pl), _p(qp), _stream(q)), "zkv_rq_query")
    return out


_TIER_RATIOS = (0.05, 0.15, 0.30, 0.50, 0.75, 1.0)


def tier_targets(kv_len: int, collision_ratio: float, tier_ratios=_TIER_RATIOS):
    """ceil(kv_len * collision_ratio * r) per tier (polar_cache.py:1711-1712)."""
    import math
    return [int(math.ceil(kv_len * collision_ratio * r)) for r in tier_ratios]


def _targets_tensor(targets):
    t = torch.tensor(list(targets), dtype=torch.int64)
    return t, t.numel()


def get_cache_cnt_fused(q_blocks, lay: RqLayout, kv_len: int, targets, out=None):
    """cache_cnt [rows, kv_len] int32 (update_cache_cnt with the bucket order
    computed from q_blocks)."""
    rows = q_blocks.numel() // 128
    if out is None:
        out = torch.empty(rows, kv_len, dtype=torch.int32, device=q_blocks.device)
    t, nt = _targets_tensor(targets)
    check(lib().zkv_collision_topk(_p(q_blocks.contiguous()), lay.struct, rows, kv_len, t.data_ptr(), nt, 0, None,
                                   _p(out), _stream(q_blocks)), "zkv_collision_topk")
    return out


def collision_topk(q_blocks, lay: RqLayout, kv_len: int, targets, C: int, idx_out=None, cnt_out=None):
    """Top-C keys by collision count (ties to the lower index), ascending
    index order: [rows, C] int64."""
    rows = q_blocks.numel() // 128
    if idx_out is None:
        idx_out = torch.empty(rows, C, dtype=torch.int64, device=q_blocks.device)
    t, nt = _targets_tensor(targets)
    check(lib().zkv_collision_topk(_p(q_blocks.contiguous()), lay.struct, rows, kv_len, t.data_ptr(), nt, C,
                                   _p(idx_out), _p(cnt_out), _stream(q_blocks)), "zkv_collision_topk")
    return idx_out


def partial_rerank_cuda(coarse_indices, lay: RqLayout, q_blocks, q_norm, mag_centers=None, final_topk: int = 0,
                        scores_out=None, final_out=None):
    """4-bit RaBitQ scores [rows, C] bf16 of coarse_indices [rows, C] (the
    reference's partial_rerank_cuda); with final_topk > 0 also the top-F key
    ids [rows, F] (ties to the lower candidate position, ascending order)."""
    _cuda(("coarse_indices", coarse_indices), ("q_blocks", q_blocks), ("q_norm", q_norm))
    _dtype("coarse_indices", coarse_indices, torch.int64)
    ci = coarse_indices.contiguous()
    C = ci.shape[-1]
    rows = ci.numel() // C
    dev = ci.device
    if mag_centers is None:
        mag_centers = torch.tensor(MAG_CENTERS, dtype=torch.bfloat16, device=dev)
    if scores_out is None:
        scores_out = torch.empty(rows, C, dtype=torch.bfloat16, device=dev)
    if final_topk > 0 and final_out is None:
        final_out = torch.empty(rows, final_topk, dtype=torch.int64, device=dev)
    check(lib().zkv_rq_rerank4(_p(ci), C, lay.struct, _p(q_blocks.contiguous()), _p(q_norm.contiguous()),
                               _p(mag_centers.contiguous()), rows, _p(scores_out), final_topk,
                               _p(final_out) if final_topk > 0 else None, _stream(ci)), "zkv_rq_rerank4")
    return (scores_out, final_out) if final_topk > 0 else scores_out


def coarse_2bit_score_cuda(lay: RqLayout, q_signs, q_mags, kv_len: int, out=None):
    """int32 [rows, kv_len] 2-bit-plane popcount scores (coarse_2bit_score.cu)."""
    rows = q_signs.numel() // 16
    if out is None:
        out = torch.empty(rows, kv_len, dtype=torch.int32, device=q_signs.device)
    check(lib().zkv_coarse2bit(lay.struct, _p(q_signs.contiguous()), _p(q_mags.contiguous()), rows, kv_len, _p(out),
                               _stream(q_signs)), "zkv_coarse2bit")
    return out


def rq_popcount_topk(cand, lay: RqLayout, planes, qparams, K: int, *, C: int | None = None, keys=None,
                     q_mean=None, est_out=None):
    """Popcount-estimate rerank: keep the K best of cand [rows, C] (None = keys
    0..C-1), return (sel [rows, K] int64 ascending, est [rows, C] f32 or None,
    ip [rows, K] f32 exact <k, q_mean> or None)."""
    rows = planes.shape[0]
    dev = planes.device
    if cand is not None:
        cand = cand.contiguous()
        C = cand.shape[-1]
    sel = torch.empty(rows, K, dtype=torch.int64, device=dev)
    ip = None
    ld = 0
    if keys is not None:
        ip = torch.empty(rows, K, dtype=torch.float32, device=dev)
        ld = keys.stride(0) if keys.dim() == 3 else _row_stride("keys", keys)
    check(lib().zkv_rq_popcount_topk(_p(cand), C, lay.struct, _p(planes), _p(qparams), rows, K, _p(sel), _p(est_out),
                                     _p(keys), ld, _p(q_mean), _p(ip), _stream(planes)), "zkv_rq_popcount_topk")
    return sel, est_out, ip
