"""ctypes front-end of the C oracle (oracle/zkv_oracle.c) plus numpy helpers.

TEST INFRASTRUCTURE ONLY: this module is the checker used by tests/, by
__graft_entry__.smoke() and by bench.py's CPU-baseline legs.  It never runs
on the product path.  Each wrapper names the reference function it restates
(paths relative to runtime/zoomkv_urania_runtime_20261011/).

bf16 arrays are numpy uint16 bit patterns throughout.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libzkv_oracle.so")

__all__ = [
    "build_oracle", "lib", "bf16_to_f32", "f32_to_bf16", "kivi_encode_chunks", "vquant_tokens",
    "quest_score", "topk_f32", "topk_i32", "chunk_density", "mask_from_topk", "kivi_qk",
    "topk_gather_concat", "attn_dense", "page_decode", "lse_merge", "kivi_dequant_chunk",
    "vdequant_tokens", "page_layout_values", "kivi_scale", "rq_mag_tables", "rq_encode", "rq_query", "collision_weights",
    "collision_count", "update_cache_cnt_sorted", "rerank4", "coarse2bit", "rq_query_4bit", "popcount_est",
    "exact_ip", "h2d_gather", "h2d_gather_packed", "page_decode_raw", "large_minmax", "sub_chunk_score",
    "map_back", "hier_select", "hier_plan",
]


def build_oracle(force: bool = False) -> str:
    srcs = [os.path.join(HERE, f) for f in ("zkv_oracle.c", "zkv_oracle_rabitq.c", "zkv_oracle.h")]
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < max(map(os.path.getmtime, srcs)):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_LIB = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            build_oracle()
        _LIB = ctypes.CDLL(LIB_PATH)
    return _LIB


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


# ----------------------------------------------------------------- bf16 utils
def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(f: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(f, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


# ----------------------------------------------------------------- encode
def kivi_encode_chunks(keys: np.ndarray, chunk: int = 16):
    """keys [..., n_chunks*chunk, D] bf16 -> (min, max, centroid [..., n_chunks, D],
    packed [..., n_chunks, D/8, chunk] int32).  Restates
    _compute_and_store_chunk_minmax + _kivi_pack_chunks for aligned chunks."""
    L = lib()
    keys = np.ascontiguousarray(keys, dtype=np.uint16)
    *lead, T, D = keys.shape
    nc = T // chunk
    flat = np.ascontiguousarray(keys.reshape(-1, T, D)[:, :nc * chunk])
    R = flat.shape[0]
    mn = np.empty((R, nc, D), np.uint16)
    mx = np.empty_like(mn)
    ce = np.empty_like(mn)
    pk = np.empty((R, nc, D // 8, chunk), np.int32)
    L.orc_kivi_encode_rows(_p(flat), R, nc * chunk, D, chunk, _p(mn), _p(mx), _p(ce), _p(pk))
    shp = tuple(lead)
    return (mn.reshape(shp + (nc, D)), mx.reshape(shp + (nc, D)), ce.reshape(shp + (nc, D)),
            pk.reshape(shp + (nc, D // 8, chunk)))


def vquant_tokens(v: np.ndarray, group: int = 32):
    """v [..., D] bf16 -> (codes [..., D/8] int32, meta [..., D/group, 2] bf16)."""
    L = lib()
    v = np.ascontiguousarray(v, dtype=np.uint16)
    D = v.shape[-1]
    flat = v.reshape(-1, D)
    codes = np.empty((flat.shape[0], D // 8), np.int32)
    meta = np.empty((flat.shape[0], D // group, 2), np.uint16)
    L.orc_vquant_rows(_p(flat), ctypes.c_int64(flat.shape[0]), D, group, _p(codes), _p(meta))
    return codes.reshape(v.shape[:-1] + (D // 8,)), meta.reshape(v.shape[:-1] + (D // group, 2))


def kivi_scale(mn: np.ndarray, mx: np.ndarray) -> np.ndarray:
    """KIVI key scale bf16(bf16(mx - mn) / 15) per chunk and dim (quant_pack.py:64)."""
    return _scale_ladder(mn, mx)


def _scale_ladder(mn: np.ndarray, mx: np.ndarray) -> np.ndarray:
    diff = f32_to_bf16(bf16_to_f32(mx) - bf16_to_f32(mn))
    return f32_to_bf16(bf16_to_f32(diff) / np.float32(15.0))


def _dequant_ladder(codes: np.ndarray, scale: np.ndarray, zero: np.ndarray) -> np.ndarray:
    prod = f32_to_bf16(codes.astype(np.float32) * bf16_to_f32(scale))
    return f32_to_bf16(bf16_to_f32(prod) + bf16_to_f32(zero))


def kivi_dequant_chunk(packed: np.ndarray, mn: np.ndarray, mx: np.ndarray) -> np.ndarray:
    """packed [..., D/8, chunk] + per-chunk mn/mx [..., D] -> keys [..., chunk, D] bf16
    (dequant_kcache_4bit, cache_hub/kivi/qk_dot.py:253-305)."""
    npk, chunk = packed.shape[-2:]
    w = packed.astype(np.uint32).swapaxes(-1, -2)                       # [..., chunk, D/8]
    codes = (w[..., None] >> (4 * np.arange(8, dtype=np.uint32))) & 15  # [..., chunk, D/8, 8]
    codes = codes.reshape(w.shape[:-1] + (npk * 8,))
    scale = _scale_ladder(mn, mx)[..., None, :]
    return _dequant_ladder(codes, scale, mn[..., None, :])


def vdequant_tokens(codes: np.ndarray, meta: np.ndarray) -> np.ndarray:
    """codes [..., D/8] int32 + meta [..., D/32, 2] -> values [..., D] bf16."""
    w = codes.astype(np.uint32)
    c = ((w[..., None] >> (4 * np.arange(8, dtype=np.uint32))) & 15).reshape(w.shape[:-1] + (w.shape[-1] * 8,))
    grp = c.shape[-1] // meta.shape[-2]
    scale = np.repeat(meta[..., 0], grp, axis=-1)
    zero = np.repeat(meta[..., 1], grp, axis=-1)
    return _dequant_ladder(c, scale, zero)


# ----------------------------------------------------------------- scoring / top-k
def quest_score(raw_q, mn, mx, valid=None, n_chunks=None):
    """raw_q [R,128], mn/mx [R,n_max,128] bf16 -> scores [R,n_chunks] fp32."""
    L = lib()
    raw_q = np.ascontiguousarray(raw_q, np.uint16).reshape(-1, 128)
    R = raw_q.shape[0]
    mn = np.ascontiguousarray(mn, np.uint16).reshape(R, -1, 128)
    mx = np.ascontiguousarray(mx, np.uint16).reshape(R, -1, 128)
    n_max = mn.shape[1]
    n_chunks = n_max if n_chunks is None else int(n_chunks)
    v = None if valid is None else np.ascontiguousarray(valid, np.uint8).reshape(R, n_max)
    out = np.empty((R, n_chunks), np.float32)
    L.orc_quest_score(_p(raw_q), _p(mn), _p(mx), _p(v), _p(out), R, n_chunks, n_max)
    return out


def topk_f32(scores: np.ndarray, k: int) -> np.ndarray:
    L = lib()
    s = np.ascontiguousarray(scores, np.float32)
    R, n = s.reshape(-1, s.shape[-1]).shape
    out = np.empty((R, k), np.int64)
    L.orc_topk_f32(_p(s), R, n, ctypes.c_int64(n), k, _p(out))
    return out.reshape(s.shape[:-1] + (k,))


# ----------------------------------------------------------------- hierarchical Quest
def hier_plan(n_chunks: int, factor: int, large_ratio: float = 0.3, small_ratio: float = 0.3):
    """(n_large, nk_large, nk_small) of _refresh_quest_chunk_cache's
    hierarchical branch (polar_cache_kivi_quest_density_seperate_kernel.py:
    1462-1468)."""
    import math
    n_large = n_chunks // factor
    if n_large <= 0:
        return 0, 0, 0
    nk_large = min(max(1, int(math.ceil(n_large * large_ratio))), n_large)
    nk_sub = nk_large * factor
    nk_small = min(max(1, int(math.ceil(nk_sub * small_ratio))), nk_sub)
    return n_large, nk_large, nk_small


def large_minmax(mn, mx, valid_end: int, factor: int, n_max_large: int | None = None):
    """_update_large_chunk_minmax (:1762-1798) over every group ->
    (large_min, large_max, large_valid)."""
    L = lib()
    mn = np.ascontiguousarray(mn, np.uint16)
    mx = np.ascontiguousarray(mx, np.uint16)
    lead, n_max = mn.shape[:-2], mn.shape[-2]
    R = int(np.prod(lead)) if lead else 1
    nml = (n_max + factor - 1) // factor if n_max_large is None else int(n_max_large)
    lmn = np.empty((R, nml, 128), np.uint16)
    lmx = np.empty((R, nml, 128), np.uint16)
    lv = np.empty((R, nml), np.uint8)
    L.orc_large_minmax.argtypes = [ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int] * 5 + [ctypes.c_void_p] * 3
    L.orc_large_minmax(_p(mn), _p(mx), R, n_max, int(valid_end), int(factor), nml, _p(lmn), _p(lmx), _p(lv))
    return lmn.reshape(lead + (nml, 128)), lmx.reshape(lead + (nml, 128)), lv.reshape(lead + (nml,))


def sub_chunk_score(raw_q, mn, mx, large_idx, factor: int):
    """quest_sub_chunk_score (quest/quest_chunk_score.cu:263-360)."""
    L = lib()
    q = np.ascontiguousarray(raw_q, np.uint16).reshape(-1, 128)
    R = q.shape[0]
    mn = np.ascontiguousarray(mn, np.uint16).reshape(R, -1, 128)
    mx = np.ascontiguousarray(mx, np.uint16).reshape(R, -1, 128)
    li = np.ascontiguousarray(large_idx, np.int64).reshape(R, -1)
    out = np.empty((R, li.shape[1] * factor), np.float32)
    L.orc_sub_chunk_score.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 4 + [ctypes.c_void_p]
    L.orc_sub_chunk_score(_p(q), _p(mn), _p(mx), _p(li), R, mn.shape[1], li.shape[1], int(factor), _p(out))
    return out


def map_back(large_idx, sub_pos, factor: int, n_chunks: int):
    """quest_map_back (quest/quest_chunk_score.cu:363-416)."""
    L = lib()
    li = np.ascontiguousarray(large_idx, np.int64)
    sp = np.ascontiguousarray(sub_pos, np.int64)
    R = int(np.prod(li.shape[:-1])) if li.ndim > 1 else 1
    out = np.empty(sp.shape, np.int64)
    L.orc_map_back.argtypes = [ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int] * 5 + [ctypes.c_void_p]
    L.orc_map_back(_p(li), _p(sp), R, li.shape[-1], sp.shape[-1], int(factor), int(n_chunks), _p(out))
    return out


def hier_select(raw_q, mn, mx, lmn, lmx, lvalid, n_chunks: int, factor: int, nk_large: int, nk_small: int):
    """_quest_pick_coarse_indices_hierarchical (:1852-1940) -> (chunk ids
    [R, nk_small], large ids [R, nk_large], sub scores [R, nk_large*factor])."""
    L = lib()
    q = np.ascontiguousarray(raw_q, np.uint16).reshape(-1, 128)
    R = q.shape[0]
    mn = np.ascontiguousarray(mn, np.uint16).reshape(R, -1, 128)
    mx = np.ascontiguousarray(mx, np.uint16).reshape(R, -1, 128)
    lmn = np.ascontiguousarray(lmn, np.uint16).reshape(R, -1, 128)
    lmx = np.ascontiguousarray(lmx, np.uint16).reshape(R, -1, 128)
    lv = None if lvalid is None else np.ascontiguousarray(lvalid, np.uint8).reshape(R, -1)
    out = np.empty((R, nk_small), np.int64)
    li = np.empty((R, nk_large), np.int64)
    sub = np.empty((R, nk_large * factor), np.float32)
    L.orc_hier_select.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] + [ctypes.c_void_p] * 3 + \
        [ctypes.c_int] * 6 + [ctypes.c_void_p] * 3
    L.orc_hier_select(_p(q), _p(mn), _p(mx), mn.shape[1], _p(lmn), _p(lmx), _p(lv), lmn.shape[1], R, int(n_chunks),
                      int(factor), int(nk_large), int(nk_small), _p(out), _p(li), _p(sub))
    return out, li, sub


def topk_i32(vals: np.ndarray, k: int) -> np.ndarray:
    L = lib()
    s = np.ascontiguousarray(vals, np.int32)
    R, n = s.reshape(-1, s.shape[-1]).shape
    out = np.empty((R, k), np.int64)
    L.orc_topk_i32(_p(s), R, n, ctypes.c_int64(n), k, _p(out))
    return out.reshape(s.shape[:-1] + (k,))


def chunk_density(chunk_ids, centroid, raw_q, n_chunks=None):
    L = lib()
    ids = np.ascontiguousarray(chunk_ids, np.int64)
    R, nk = ids.reshape(-1, ids.shape[-1]).shape
    cent = np.ascontiguousarray(centroid, np.uint16).reshape(R, -1, 128)
    n_max = cent.shape[1]
    q = np.ascontiguousarray(raw_q, np.uint16).reshape(R, 128)
    out = np.empty((R, nk), np.float32)
    L.orc_chunk_density(_p(ids), _p(cent), _p(q), _p(out), R, nk,
                        n_max if n_chunks is None else int(n_chunks), n_max)
    return out.reshape(ids.shape)


def mask_from_topk(positions, nk):
    L = lib()
    p = np.ascontiguousarray(positions, np.int64)
    R, nd = p.reshape(-1, p.shape[-1]).shape
    m = np.empty((R, nk), np.uint8)
    L.orc_mask_from_topk(_p(p), _p(m), R, nd, nk)
    return m.reshape(p.shape[:-1] + (nk,))


def kivi_qk(chunk_ids, dense, packed, mn, mx, raw_q, dense_topk, sparse_topk, chunk=16):
    L = lib()
    ids = np.ascontiguousarray(chunk_ids, np.int64)
    R, nk = ids.reshape(-1, ids.shape[-1]).shape
    dm = np.ascontiguousarray(dense, np.uint8).reshape(R, nk)
    pk = np.ascontiguousarray(packed, np.int32).reshape(R, -1, 16, chunk)
    mn = np.ascontiguousarray(mn, np.uint16).reshape(R, -1, 128)
    mx = np.ascontiguousarray(mx, np.uint16).reshape(R, -1, 128)
    q = np.ascontiguousarray(raw_q, np.uint16).reshape(R, 128)
    sc = np.empty((R, nk * chunk), np.float32)
    ix = np.empty((R, nk * chunk), np.int64)
    L.orc_kivi_qk(_p(ids), _p(dm), _p(pk), pk.shape[1], _p(mn), _p(mx), mn.shape[1], _p(q), R, nk,
                  chunk, dense_topk, sparse_topk, _p(sc), _p(ix))
    return sc.reshape(ids.shape[:-1] + (nk * chunk,)), ix.reshape(ids.shape[:-1] + (nk * chunk,))


def topk_gather_concat(scores, lut, skipped, k):
    L = lib()
    s = np.ascontiguousarray(scores, np.float32)
    R, n = s.reshape(-1, s.shape[-1]).shape
    lu = np.ascontiguousarray(lut, np.int64).reshape(R, n)
    sk = np.ascontiguousarray(skipped, np.int64).reshape(R, -1)
    out = np.empty((R, k + sk.shape[1]), np.int64)
    L.orc_topk_gather_concat(_p(s), _p(lu), _p(sk), _p(out), R, n, k, sk.shape[1],
                             ctypes.c_int64(out.shape[1]))
    return out.reshape(s.shape[:-1] + (out.shape[1],))


def attn_dense(q: np.ndarray, K: np.ndarray, V: np.ndarray, scale: float):
    """q [G,D] fp32, K/V [n,D] fp32 -> (out [G,D] fp32, lse [G]) in fp64."""
    L = lib()
    q = np.ascontiguousarray(q, np.float32)
    K = np.ascontiguousarray(K, np.float32)
    V = np.ascontiguousarray(V, np.float32)
    G, D = q.shape
    out = np.empty((G, D), np.float32)
    lse = np.empty((G,), np.float32)
    L.orc_attn_dense(_p(q), _p(K), _p(V), K.shape[0], G, D, ctypes.c_float(scale), _p(out), _p(lse))
    return out, lse


def page_decode(q, mn, mx, valid, kcodes, vcodes, vmeta, nearK, nearV, n_c, nk, n_near,
                scale, threads=1):
    """Rows = flattened (batch, kv_head).  See zkv_oracle.h:orc_page_decode."""
    L = lib()
    q = np.ascontiguousarray(q, np.uint16)
    R, G, D = q.shape
    arrs = [np.ascontiguousarray(a) for a in (mn, mx, kcodes, vcodes, vmeta, nearK, nearV)]
    mn, mx, kcodes, vcodes, vmeta, nearK, nearV = arrs
    n_max = mn.shape[1]
    near_ld = nearK.shape[1]
    v = None if valid is None else np.ascontiguousarray(valid, np.uint8)
    out = np.empty((R, G, D), np.uint16)
    lse = np.empty((R, G), np.float32)
    sel = np.empty((R, nk), np.int64)
    L.orc_page_decode(_p(q), _p(mn), _p(mx), _p(v), _p(kcodes), _p(vcodes), _p(vmeta), _p(nearK),
                      _p(nearV), R, G, n_max, n_c, nk, near_ld, n_near, ctypes.c_float(scale),
                      _p(out), _p(lse), _p(sel), int(threads))
    return out, lse, sel


def page_decode_raw(q, mn, mx, valid, keys, values, n_c, nk, *, page_base=0, n_sink=0, near_start=0, n_near=0,
                    scale=1.0 / np.sqrt(128), threads=1):
    """Page mode over raw rows (see zkv_oracle.h:orc_page_decode_raw).
    q [R,G,128] bf16; mn/mx [R,n_max,128]; keys/values [R,cap,128] bf16
    (absolute token positions).  Returns (out [R,G,128] bf16, lse [R,G],
    sel [R,nk])."""
    L = lib()
    q = np.ascontiguousarray(q, np.uint16)
    R, G, D = q.shape
    mn = np.ascontiguousarray(mn, np.uint16).reshape(R, -1, D)
    mx = np.ascontiguousarray(mx, np.uint16).reshape(R, -1, D)
    keys = np.ascontiguousarray(keys, np.uint16).reshape(R, -1, D)
    values = np.ascontiguousarray(values, np.uint16).reshape(R, -1, D)
    n_max, cap = mn.shape[1], keys.shape[1]
    v = None if valid is None else np.ascontiguousarray(valid, np.uint8).reshape(R, n_max)
    nsel = nk if n_c > 0 else 0
    out = np.empty((R, G, D), np.uint16)
    lse = np.empty((R, G), np.float32)
    sel = np.empty((R, max(nsel, 1)), np.int64)
    L.orc_page_decode_raw(_p(q), _p(mn), _p(mx), _p(v), _p(keys), _p(values), ctypes.c_int64(cap),
                          ctypes.c_int64(page_base), R, G, n_max, int(n_c), int(nk), int(n_sink), int(near_start),
                          int(n_near), ctypes.c_float(scale), _p(out), _p(lse), _p(sel), int(threads))
    return out, lse, sel[:, :nsel]


def lse_merge(a, la, b, lb):
    L = lib()
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    R, dim = a.reshape(-1, a.shape[-1]).shape
    la = np.ascontiguousarray(la, np.float32).reshape(R)
    lb = np.ascontiguousarray(lb, np.float32).reshape(R)
    out = np.empty((R, dim), np.float32)
    lo = np.empty((R,), np.float32)
    L.orc_lse_merge(_p(a), _p(la), _p(b), _p(lb), _p(out), _p(lo), R, dim)
    return out.reshape(a.shape), lo


# ----------------------------------------------------------------- layouts
def page_layout_values(codes: np.ndarray, meta: np.ndarray):
    """Per-token value codes [R, T, D/8] + meta [R, T, D/32, 2] (T % 16 == 0)
    -> page layout vcodes_t [R, T/16, D, 2] int32 and vmeta [R, T/16, 2, D/32, 16]
    (the layout zkv_vquant_encode writes and the page-mode attention reads)."""
    R, T, W = codes.shape
    D = W * 8
    w = codes.astype(np.uint32)
    c = ((w[..., None] >> (4 * np.arange(8, dtype=np.uint32))) & 15).reshape(R, T, D)
    P = T // 16
    c = c.reshape(R, P, 16, D)
    sh = (4 * np.arange(8, dtype=np.uint32))[:, None]
    w0 = (c[:, :, :8, :].astype(np.uint32) << sh).sum(axis=2, dtype=np.uint64).astype(np.uint32)
    w1 = (c[:, :, 8:, :].astype(np.uint32) << sh).sum(axis=2, dtype=np.uint64).astype(np.uint32)
    vcodes_t = np.stack([w0, w1], axis=-1).view(np.int32)
    m = meta.reshape(R, P, 16, D // 32, 2)
    vmeta = np.ascontiguousarray(m.transpose(0, 1, 4, 3, 2))
    return np.ascontiguousarray(vcodes_t), vmeta


# ----------------------------------------------------------------- ParisKV / RaBitQ
# Token-major layouts: codes [R, cap, 16] u8, packed [R, cap, 64] u8,
# weight [R, cap, 16] bf16, factor [R, cap] f32, hist [R, 16, 256] i32.
def rq_mag_tables():
    thr = np.empty(7, np.uint16)
    cen = np.empty(8, np.uint16)
    lib().orc_rq_mag_tables(_p(thr), _p(cen))
    return thr, cen


def rq_encode(keys: np.ndarray, signs: np.ndarray):
    """keys [R, T, 128] bf16 -> codes, packed, weight, factor, hist
    (ParisKV batch_encode + _count_cluster_keys)."""
    keys = np.ascontiguousarray(keys, dtype=np.uint16)
    R, T, D = keys.shape
    codes = np.zeros((R, T, 16), np.uint8)
    packed = np.zeros((R, T, 64), np.uint8)
    weight = np.zeros((R, T, 16), np.uint16)
    factor = np.zeros((R, T), np.float32)
    hist = np.zeros((R, 16, 256), np.int32)
    L = lib()
    L.orc_rq_encode_rows.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                     ctypes.c_int64] + [ctypes.c_void_p] * 6
    L.orc_rq_encode_rows(_p(keys), T * D, R, T, 0, T, _p(np.ascontiguousarray(signs, np.uint16)), _p(codes),
                         _p(packed), _p(weight), _p(factor), _p(hist))
    return codes, packed, weight, factor, hist


def rq_query(q: np.ndarray, signs: np.ndarray):
    """q [R, G, 128] bf16 -> (q_blocks [R, 128] bf16, q_norm [R] bf16, q_mean [R, 128] bf16)."""
    q = np.ascontiguousarray(q, dtype=np.uint16)
    R, G, D = q.shape
    qb = np.empty((R, D), np.uint16)
    qn = np.empty(R, np.uint16)
    qm = np.empty((R, D), np.uint16)
    L = lib()
    L.orc_rq_query.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int] + [ctypes.c_void_p] * 4
    L.orc_rq_query(_p(q), R, G, _p(np.ascontiguousarray(signs, np.uint16)), _p(qb), _p(qn), _p(qm))
    return qb, qn, qm


def collision_weights(q_blocks: np.ndarray, hist: np.ndarray, targets) -> np.ndarray:
    """-> table [R, 16, 256] u8 of per-bucket tier hits."""
    q_blocks = np.ascontiguousarray(q_blocks, np.uint16).reshape(-1, 128)
    R = q_blocks.shape[0]
    t = np.ascontiguousarray(targets, np.int64)
    table = np.empty((R, 16, 256), np.uint8)
    L = lib()
    L.orc_collision_weights.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                        ctypes.c_void_p]
    L.orc_collision_weights(_p(q_blocks), _p(np.ascontiguousarray(hist, np.int32)), R, _p(t), len(t), _p(table))
    return table


def collision_count(table: np.ndarray, codes: np.ndarray, kv_len: int | None = None) -> np.ndarray:
    codes = np.ascontiguousarray(codes, np.uint8)
    R, cap, _ = codes.shape
    kv_len = cap if kv_len is None else kv_len
    cnt = np.empty((R, kv_len), np.int32)
    L = lib()
    L.orc_collision_count.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_void_p]
    L.orc_collision_count(_p(np.ascontiguousarray(table, np.uint8)), _p(codes), cap, R, kv_len, _p(cnt))
    return cnt


def update_cache_cnt_sorted(sorted_ids, hist, codes_bm, targets) -> np.ndarray:
    """update_cache_cnt_overall_ref with given sorted ids; codes block-major [R, B, kv_len]."""
    sorted_ids = np.ascontiguousarray(sorted_ids, np.int64)
    R, B, K = sorted_ids.shape
    codes_bm = np.ascontiguousarray(codes_bm, np.int32)
    kv_len = codes_bm.shape[-1]
    t = np.ascontiguousarray(targets, np.int64)
    cnt = np.empty((R, kv_len), np.int32)
    L = lib()
    L.orc_update_cache_cnt_sorted.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 4 + [ctypes.c_void_p,
                                                                                          ctypes.c_int, ctypes.c_void_p]
    L.orc_update_cache_cnt_sorted(_p(sorted_ids), _p(np.ascontiguousarray(hist, np.int32)), _p(codes_bm), R, B, K,
                                  kv_len, _p(t), len(t), _p(cnt))
    return cnt


def rerank4(cand, packed, weight, q_blocks, q_norm, cen8=None) -> np.ndarray:
    """Sequential-bf16 4-bit RaBitQ scores [R, C] bf16 of candidate keys."""
    cand = np.ascontiguousarray(cand, np.int64)
    R, C = cand.shape
    packed = np.ascontiguousarray(packed, np.uint8)
    cap = packed.shape[1]
    if cen8 is None:
        cen8 = rq_mag_tables()[1]
    out = np.empty((R, C), np.uint16)
    L = lib()
    L.orc_rerank4.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64] + \
        [ctypes.c_void_p] * 3 + [ctypes.c_int, ctypes.c_void_p]
    L.orc_rerank4(_p(cand), C, _p(packed), _p(np.ascontiguousarray(weight, np.uint16)), cap,
                  _p(np.ascontiguousarray(q_blocks, np.uint16)), _p(np.ascontiguousarray(q_norm, np.uint16)),
                  _p(np.ascontiguousarray(cen8, np.uint16)), R, _p(out))
    return out


def coarse2bit(packed, q_signs, q_mags, kv_len: int | None = None) -> np.ndarray:
    packed = np.ascontiguousarray(packed, np.uint8)
    R, cap, _ = packed.shape
    kv_len = cap if kv_len is None else kv_len
    out = np.empty((R, kv_len), np.int32)
    L = lib()
    L.orc_coarse2bit.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                 ctypes.c_int, ctypes.c_void_p]
    L.orc_coarse2bit(_p(packed), cap, _p(np.ascontiguousarray(q_signs, np.uint8)),
                     _p(np.ascontiguousarray(q_mags, np.uint8)), R, kv_len, _p(out))
    return out


def rq_query_4bit(q_blocks, q_norm):
    q_blocks = np.ascontiguousarray(q_blocks, np.uint16).reshape(-1, 128)
    R = q_blocks.shape[0]
    planes = np.empty((R, 4, 16), np.uint8)
    qp = np.empty((R, 4), np.float32)
    L = lib()
    L.orc_rq_query_4bit.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    L.orc_rq_query_4bit(_p(q_blocks), _p(np.ascontiguousarray(q_norm, np.uint16)), R, _p(planes), _p(qp))
    return planes, qp


def popcount_est(cand, codes, factor, planes, qparams):
    """-> (est [R, C] f32, ints [R, C, 2] i32 = (I, P)); cand None = all keys."""
    codes = np.ascontiguousarray(codes, np.uint8)
    R, cap, _ = codes.shape
    if cand is not None:
        cand = np.ascontiguousarray(cand, np.int64)
        C = cand.shape[1]
    else:
        C = cap
    est = np.empty((R, C), np.float32)
    ints = np.empty((R, C, 2), np.int32)
    L = lib()
    L.orc_popcount_est.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    L.orc_popcount_est(_p(cand), C, _p(codes), _p(np.ascontiguousarray(factor, np.float32)), cap,
                       _p(np.ascontiguousarray(planes, np.uint8)), _p(np.ascontiguousarray(qparams, np.float32)), R,
                       _p(est), _p(ints))
    return est, ints


def exact_ip(idx, keys, q) -> np.ndarray:
    """idx [R, n] -> fp32 <keys[r, idx], q[r]> (lane-tree order); keys [R, T, 128] bf16."""
    idx = np.ascontiguousarray(idx, np.int64)
    keys = np.ascontiguousarray(keys, np.uint16)
    R, n = idx.shape
    out = np.empty((R, n), np.float32)
    L = lib()
    L.orc_exact_ip.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                               ctypes.c_int, ctypes.c_void_p]
    L.orc_exact_ip(_p(idx), n, _p(keys), keys.shape[1] * 128, _p(np.ascontiguousarray(q, np.uint16)), R, _p(out))
    return out


def h2d_gather(src: np.ndarray, idx: np.ndarray, dst: np.ndarray) -> np.ndarray:
    """Dense offload gather, cache_hub/gather_trans/trans_h2d.cu:83-140:
    dst[b, h, j] = src[b, h, idx[b, h, j]] for j < topk; rows j >= topk of
    dst keep their contents.  src [bs,H,L,128], idx [bs,H,topk], dst
    [bs,H,>=topk,128] (any element type; a row copy)."""
    out = dst.copy()
    bs, H, topk = idx.shape
    for b in range(bs):
        for h in range(H):
            out[b, h, :topk] = src[b, h, idx[b, h]]
    return out


def h2d_gather_packed(src: np.ndarray, idx: np.ndarray, cu_topk: np.ndarray, cu_k: np.ndarray, sl_end: int,
                      global_k: int, dst: np.ndarray) -> np.ndarray:
    """Varlen offload gather, trans_h2d.cu:228-283: for vh = b*H + h and
    slot < min(global_k, cu_topk[vh+1] - cu_topk[vh]):
    dst[cu_k[vh] + sl_end + slot] = src[b, h, idx[cu_topk[vh] + slot]]."""
    out = dst.copy()
    bs, H = src.shape[:2]
    for vh in range(bs * H):
        st, n = int(cu_topk[vh]), int(cu_topk[vh + 1] - cu_topk[vh])
        n = min(n, int(global_k))
        if n <= 0:
            continue
        d0 = int(cu_k[vh]) + sl_end
        out[d0:d0 + n] = src[vh // H, vh % H, idx[st:st + n]]
    return out
