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
page_decode                            (fused page-mode decode; no single counterpart)
vquant_encode                          (per-token 4-bit values; no counterpart)
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
    "PageLayer",
]


def _stream(t: torch.Tensor) -> int:
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

    raw_q [bs,kv,128] bf16; chunk_min/max [bs,kv,n_max,128] bf16;
    scores_out: n_chunks*bs*kv fp32 elements laid out [bs,kv,n_chunks];
    chunk_valid [bs,kv,n_max] bool or None.
    """
    _cuda(("raw_q", raw_q), ("chunk_min", chunk_min), ("chunk_max", chunk_max), ("scores", scores_out),
          ("valid", chunk_valid))
    for n, t in (("raw_q", raw_q), ("chunk_min", chunk_min), ("chunk_max", chunk_max)):
        _dtype(n, t, torch.bfloat16)
        _contig(n, t)
    _dtype("scores_out", scores_out, torch.float32)
    _contig("scores_out", scores_out)
    if raw_q.shape[-1] != 128:
        raise ValueError("quest_chunk_score: only head_dim==128 is supported")
    bs, kv = raw_q.shape[0], raw_q.shape[1]
    n_max = chunk_min.shape[2]
    n_chunks = int(n_chunks)
    if n_chunks > n_max:
        raise ValueError("n_chunks must <= chunk_n_max")
    if scores_out.numel() < bs * kv * n_chunks:
        raise ValueError("scores_out too small")
    if chunk_valid is not None:
        _dtype("chunk_valid", chunk_valid, torch.bool)
        _contig("chunk_valid", chunk_valid)
    check(lib().zkv_quest_score(_p(raw_q), _p(chunk_min), _p(chunk_max), _p(chunk_valid), _p(scores_out), bs * kv,
                                n_chunks, n_max, _stream(raw_q)), "zkv_quest_score")


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
def kivi_encode_chunks(keys, chunk_min, chunk_max, chunk_centroid, chunk_valid, packed, chunk_start: int):
    """Write metadata + KIVI codes of the aligned chunks of `keys` [bs,kv,T,128]
    (T % 16 == 0; token stride 128) at chunk indices chunk_start.. of the
    [bs,kv,n_max,...] buffers."""
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
                                _p(chunk_max), _p(chunk_centroid), _p(chunk_valid), _p(packed), _stream(keys)),
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


class PageLayer:
    """Tensors of one layer of the page-mode cache ([bs, H, ...] each)."""

    def __init__(self, chunk_min, chunk_max, valid, kcodes, vcodes_t, vmeta, near_k, near_v):
        self.tensors = (chunk_min, chunk_max, valid, kcodes, vcodes_t, vmeta, near_k, near_v)
        self.struct = _lib.ZkvPageLayer(
            _p(chunk_min), _p(chunk_max), _p(valid), _p(kcodes), _p(vcodes_t), _p(vmeta), _p(near_k), _p(near_v),
            near_k.shape[2])


def page_decode(q, layer: PageLayer, n_c: int, nk: int, n_near: int, *, n_sink: int = 0, near_start: int = 0,
                scale=None, out=None, lse=None, sel_out=None, status=None, cluster=0):
    """Fused page-mode decode: q [bs,1,H*G,128] -> out [bs,1,H*G,128].

    Raw rows attended besides the selected pages: [0, n_sink) and
    [near_start, near_start + n_near) of the layer's near buffers."""
    cmin = layer.tensors[0]
    bs, H, n_max, D = cmin.shape
    G = q.shape[2] // H
    qc = q.contiguous()
    if out is None:
        out = torch.empty(bs, 1, H * G, D, dtype=torch.bfloat16, device=q.device)
    scale = (1.0 / D ** 0.5) if scale is None else float(scale)
    check(lib().zkv_page_decode(_p(qc), ctypes.byref(layer.struct), bs * H, G, n_max, int(n_c), int(nk), int(n_sink),
                                int(near_start), int(n_near), scale, _p(out), _p(lse), _p(sel_out), _p(status),
                                int(cluster), _stream(q)), "zkv_page_decode")
    return out
