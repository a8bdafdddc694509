"""ctypes binding of libzkv.so (the C ABI declared in include/zkv.h).

The library is loaded from the package directory.  There is no fallback: if
the shared object is missing, cannot be loaded, or a call returns a non-zero
status, a RuntimeError is raised.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libzkv.so")

ZKV_OK = 0
ZKV_ERR_TIMEOUT = 6
ZKV_ERR_RANGE = 7

_c_void_p = ctypes.c_void_p
_i32 = ctypes.c_int
_i64 = ctypes.c_int64
_f32 = ctypes.c_float


class ZkvPageLayer(ctypes.Structure):
    """Mirror of `zkv_page_layer` (include/zkv.h)."""
    _fields_ = [
        ("chunk_min", _c_void_p), ("chunk_max", _c_void_p), ("valid", _c_void_p),
        ("kcodes", _c_void_p), ("vcodes_t", _c_void_p), ("vmeta", _c_void_p),
        ("near_k", _c_void_p), ("near_v", _c_void_p), ("near_ld", _i64), ("kscale", _c_void_p),
    ]


class ZkvRawLayer(ctypes.Structure):
    """Mirror of `zkv_raw_layer` (include/zkv.h)."""
    _fields_ = [
        ("chunk_min", _c_void_p), ("chunk_max", _c_void_p), ("valid", _c_void_p),
        ("keys", _c_void_p), ("values", _c_void_p), ("kv_ld_row", _i64), ("page_base", _i64),
    ]


class ZkvRawSplit(ctypes.Structure):
    """Mirror of `zkv_raw_split` (include/zkv.h)."""
    _fields_ = [("peer_base", ctypes.POINTER(_c_void_p)), ("bytes", ctypes.c_size_t), ("rank", _i32),
                ("world", _i32)]


class ZkvQuestLarge(ctypes.Structure):
    """Mirror of `zkv_quest_large` (include/zkv.h)."""
    _fields_ = [("large_min", _c_void_p), ("large_max", _c_void_p), ("large_valid", _c_void_p),
                ("n_max_large", _i32)]


class ZkvRqLayout(ctypes.Structure):
    """Mirror of `zkv_rq_layout` (include/zkv.h)."""
    _fields_ = [
        ("codes", _c_void_p), ("codes_row", _i64), ("codes_blk", _i64), ("codes_tok", _i64),
        ("packed", _c_void_p), ("packed_row", _i64), ("packed_blk", _i64), ("packed_tok", _i64),
        ("weight", _c_void_p), ("weight_row", _i64), ("weight_blk", _i64), ("weight_tok", _i64),
        ("factor", _c_void_p), ("factor_row", _i64), ("hist", _c_void_p),
    ]


class ZkvRefLayer(ctypes.Structure):
    """Mirror of `zkv_ref_layer` (include/zkv.h)."""
    _fields_ = [("chunk_min", _c_void_p), ("chunk_max", _c_void_p), ("centroid", _c_void_p), ("valid", _c_void_p),
                ("packed", _c_void_p)]


class ZkvPeerSeg(ctypes.Structure):
    """Mirror of `zkv_peer_seg` (include/zkv.h)."""
    _fields_ = [("src", _c_void_p), ("src_ld_bytes", _i64), ("dst_off_bytes", _i64), ("dst_ld_bytes", _i64),
                ("row_bytes", _i64), ("rows", _i32), ("pad", _i32)]


_RQ = ctypes.POINTER(ZkvRqLayout)

# name -> argtypes (restype is int status unless noted)
_SIGNATURES = {
    "zkv_kivi_encode": [_c_void_p, _i64, _i32, _i32, _i32, _i32, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                        _c_void_p, _c_void_p, _c_void_p],
    "zkv_vquant_encode": [_c_void_p, _i64, _i32, _i32, _i32, _i32, _c_void_p, _c_void_p, _c_void_p],
    "zkv_quest_score": [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32, _c_void_p],
    "zkv_quest_score_gqa": [_c_void_p, _i32, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32, _c_void_p],
    "zkv_topk_f32": [_c_void_p, _i32, _i32, _i64, _i32, _c_void_p, _c_void_p],
    "zkv_topk_i32": [_c_void_p, _i32, _i32, _i64, _i32, _c_void_p, _c_void_p],
    "zkv_chunk_density": [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32, _i32, _c_void_p],
    "zkv_mask_from_topk": [_c_void_p, _c_void_p, _i32, _i32, _i32, _c_void_p],
    "zkv_kivi_qk": [_c_void_p, _c_void_p, _c_void_p, _i32, _i32, _c_void_p, _c_void_p, _i32, _c_void_p, _i32, _i32, _i32,
                    _i32, _c_void_p, _c_void_p, _i64, _c_void_p],
    "zkv_topk_gather_concat": [_c_void_p, _c_void_p, _c_void_p, _i64, _c_void_p, _i32, _i32, _i32, _i32, _i64, _c_void_p],
    "zkv_page_decode_scored": [_c_void_p, ctypes.POINTER(ZkvPageLayer), _i32, _i32, _i32, _c_void_p, _i64, _i32,
                               _i32, _i64, _i64, _i32, _i32, _i32, _f32, _i32, _c_void_p, _c_void_p, _c_void_p,
                               _c_void_p, _i32, _c_void_p],
    "zkv_peer_handle_bytes": [],
    "zkv_peer_alloc": [ctypes.c_size_t, ctypes.POINTER(_c_void_p), _c_void_p],
    "zkv_peer_open": [_c_void_p, ctypes.POINTER(_c_void_p)],
    "zkv_peer_close": [_c_void_p],
    "zkv_peer_free": [_c_void_p],
    "zkv_peer_put": [ctypes.POINTER(ZkvPeerSeg), _i32, ctypes.POINTER(_c_void_p), _i64, _i32, _i32, _c_void_p,
                     _c_void_p, _i32, _c_void_p],
    "zkv_peer_exchange": [ctypes.POINTER(ZkvPeerSeg), _i32, ctypes.POINTER(_c_void_p), _i64, _i32, _i32, _c_void_p,
                          _c_void_p, _i32, _c_void_p, _c_void_p],
    "zkv_peer_wait": [_c_void_p, _c_void_p, _i32, _c_void_p, _c_void_p],
    "zkv_peer_set_wait_ms": [_i32],
    "zkv_h2d_gather_kv": [_c_void_p, _c_void_p, _i32, _i64, _c_void_p, _i64, _i32, _i64, _c_void_p, _c_void_p, _i64,
                          _i64, _c_void_p, _c_void_p],
    "zkv_h2d_gather_kv_packed": [_c_void_p, _c_void_p, _i32, _i64, _c_void_p, _c_void_p, _c_void_p, _i32, _i32,
                                 _c_void_p, _c_void_p, _i64, _c_void_p, _c_void_p],
    "zkv_attn_rows": [_c_void_p, _c_void_p, _c_void_p, _i64, _i32, _i32, _i32, _i32, _c_void_p, _i32, _i64, _i64,
                      _i32, _i32, _f32, _c_void_p, _c_void_p, _i32, _c_void_p, _c_void_p],
    "zkv_page_decode": [_c_void_p, ctypes.POINTER(ZkvPageLayer), _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _f32,
                        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _c_void_p],
    "zkv_page_decode_split_ws_bytes": [_i32, _i32],
    "zkv_page_decode_split": [_c_void_p, ctypes.POINTER(ZkvPageLayer), _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
                              _f32, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _c_void_p, ctypes.c_size_t,
                              _c_void_p],
    "zkv_page_decode_raw_ws_bytes": [_i32, _i32, _i32, _i32, _i32],
    "zkv_page_decode_raw": [_c_void_p, ctypes.POINTER(ZkvRawLayer), _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
                            _f32, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, ctypes.c_size_t, _c_void_p],
    "zkv_rmsnorm": [_c_void_p, _c_void_p, _c_void_p, _i32, _i32, ctypes.c_float, _c_void_p],
    "zkv_qk_norm_rope": [_c_void_p] * 6 + [_i32, _i32, _i32, ctypes.c_float] + [_c_void_p] * 4,
    "zkv_silu_mul": [_c_void_p, _c_void_p, _i32, _i32, _c_void_p],
    "zkv_quest_large_minmax": [_c_void_p, _c_void_p, _i32, _i32, _i32, _i32, _i32, _i32, _c_void_p, _c_void_p,
                               _c_void_p, _i32, _c_void_p],
    "zkv_page_decode_raw_hier_ws_bytes": [_i32] * 7,
    "zkv_page_decode_raw_hier": [_c_void_p, ctypes.POINTER(ZkvRawLayer), ctypes.POINTER(ZkvQuestLarge)] +
                                [_i32] * 10 + [ctypes.c_float, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                               ctypes.c_size_t, _c_void_p],
    "zkv_raw_split_range": [_i32, _i32, _i32, ctypes.POINTER(_i32), ctypes.POINTER(_i32)],
    "zkv_raw_split_buffer_bytes": [_i32] * 4,
    "zkv_page_decode_raw_split_ws_bytes": [_i32] * 7,
    "zkv_page_decode_raw_split": [_c_void_p, ctypes.POINTER(ZkvRawLayer), ctypes.POINTER(ZkvRawSplit)] +
                                 [_i32] * 8 + [ctypes.c_float, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                               _c_void_p, ctypes.c_size_t, _c_void_p],
    "zkv_lse_merge": [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _c_void_p],
    "zkv_lse_merge_n": [_c_void_p, _c_void_p, _i32, _i32, _i32, _c_void_p, _c_void_p, _c_void_p],
    "zkv_rq_encode": [_c_void_p, _i64, _i32, _i32, _i32, _c_void_p, _RQ, _c_void_p],
    "zkv_rq_query": [_c_void_p, _i32, _i32] + [_c_void_p] * 7,
    "zkv_collision_topk": [_c_void_p, _RQ, _i32, _i32, _c_void_p, _i32, _i32, _c_void_p, _c_void_p, _c_void_p],
    "zkv_rq_rerank4": [_c_void_p, _i32, _RQ, _c_void_p, _c_void_p, _c_void_p, _i32, _c_void_p, _i32, _c_void_p,
                       _c_void_p],
    "zkv_coarse2bit": [_RQ, _c_void_p, _c_void_p, _i32, _i32, _c_void_p, _c_void_p],
    "zkv_rq_popcount_topk": [_c_void_p, _i32, _RQ, _c_void_p, _c_void_p, _i32, _i32, _c_void_p, _c_void_p, _c_void_p,
                             _i64, _c_void_p, _c_void_p, _c_void_p],
    "zkv_reference_select_ws_bytes": [_i32, _i32, _i32, _i32],
    "zkv_reference_select": [_c_void_p, _i32, ctypes.POINTER(ZkvRefLayer)] + [_i32] * 9 +
                            [_c_void_p, _i64, _i32, _c_void_p, _i64, _c_void_p, _c_void_p, ctypes.c_size_t, _c_void_p],
    "zkv_reference_select_noalloc": [_c_void_p, _i32, ctypes.POINTER(ZkvRefLayer)] + [_i32] * 9 +
                                    [_c_void_p, _i64, _i32, _c_void_p, _i64, _c_void_p, _c_void_p],
    "zkv_gqa_mean": [_c_void_p, _i32, _i32, _c_void_p, _c_void_p],
    "zkv_page_attend": [_c_void_p, ctypes.POINTER(ZkvPageLayer), _i32, _i32, _i32, _c_void_p, _i32, _i64, _i64, _i32,
                        _i32, _i32, _f32, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _c_void_p],
    "zkv_version": [],
    "zkv_status_string": [_i32],
}

_RESTYPES = {"zkv_status_string": ctypes.c_char_p, "zkv_reference_select_ws_bytes": ctypes.c_size_t,
             "zkv_page_decode_split_ws_bytes": ctypes.c_size_t, "zkv_page_decode_raw_ws_bytes": ctypes.c_size_t,
             "zkv_page_decode_raw_hier_ws_bytes": ctypes.c_size_t, "zkv_raw_split_buffer_bytes": ctypes.c_size_t,
             "zkv_page_decode_raw_split_ws_bytes": ctypes.c_size_t}

_lock = threading.Lock()
_lib = None


def exported_symbols() -> list[str]:
    return sorted(_SIGNATURES)


def lib() -> ctypes.CDLL:
    """Load libzkv.so (raises if absent -- the CUDA path has no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"libzkv.so not found at {LIB_PATH}; build it with "
                    "`python -m zoomkv_revision_b200.build` (no CPU fallback exists)")
            h = ctypes.CDLL(LIB_PATH)
            for name, argt in _SIGNATURES.items():
                fn = getattr(h, name)
                fn.argtypes = argt
                fn.restype = _RESTYPES.get(name, ctypes.c_int)
            _lib = h
    return _lib


def check(status: int, what: str) -> None:
    if status != ZKV_OK:
        msg = lib().zkv_status_string(int(status)).decode()
        raise RuntimeError(f"{what} failed: status {status} ({msg})")
