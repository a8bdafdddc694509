"""Seeded synthetic decode workloads with the shapes of the benchmark configs.

The reference's evaluation data (MATH-500 / AIME-2025 prompts and Qwen3
weights) is not available, so keys/values/queries are drawn the way the
benchmark configs describe them:

  * q ~ N(0, 1) bf16, V ~ N(0, 1) bf16;
  * K ~ N(0, 1) with 4 random channels per KV head scaled x10 (outliers),
    rotated with rotate-half RoPE at their token positions
    (model_hub/qwen.py:550-598 formula, theta a parameter), then bf16.

`build_page_cache` lays the keys/values out exactly as the page-mode cache
does (Quest metadata + KIVI codes + 4-bit values + bf16 near window) using the
library's own encode kernels.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops

HEAD_DIM = 128
CHUNK = 16


def rope_rotate_half(x: torch.Tensor, pos: torch.Tensor, theta: float = 1.0e6) -> torch.Tensor:
    """x [..., T, D] fp32, pos [T] -> rotate-half RoPE (cos/sin over D/2 freqs)."""
    d = x.shape[-1]
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, device=x.device, dtype=torch.float32) / d))
    ang = pos.to(torch.float32)[:, None] * inv[None, :]
    cos = torch.cat([ang.cos(), ang.cos()], dim=-1)
    sin = torch.cat([ang.sin(), ang.sin()], dim=-1)
    x1, x2 = x[..., : d // 2], x[..., d // 2:]
    rot = torch.cat([-x2, x1], dim=-1)
    return x * cos + rot * sin


def outlier_channels(gen: torch.Generator, heads: int, device, outliers: int = 4) -> torch.Tensor:
    """[heads, outliers] channel ids scaled x10 (fixed per head for a sequence)."""
    return torch.stack([torch.randperm(HEAD_DIM, generator=gen, device=device)[:outliers] for _ in range(heads)])


def synth_keys(gen: torch.Generator, bs: int, heads: int, T: int, device, pos0: int = 0,
               channels: torch.Tensor | None = None, theta: float = 1.0e6) -> torch.Tensor:
    if channels is None:
        channels = outlier_channels(gen, heads, device)
    k = torch.randn(bs, heads, T, HEAD_DIM, generator=gen, device=device, dtype=torch.float32)
    for h in range(heads):
        k[:, h, :, channels[h]] *= 10.0
    pos = torch.arange(pos0, pos0 + T, device=device)
    return rope_rotate_half(k, pos, theta).to(torch.bfloat16)


def synth_values(gen: torch.Generator, bs: int, heads: int, T: int, device) -> torch.Tensor:
    return torch.randn(bs, heads, T, HEAD_DIM, generator=gen, device=device, dtype=torch.float32).to(torch.bfloat16)


def synth_query(gen: torch.Generator, bs: int, q_heads: int, device) -> torch.Tensor:
    return torch.randn(bs, 1, q_heads, HEAD_DIM, generator=gen, device=device, dtype=torch.float32).to(torch.bfloat16)


@dataclass
class PageCache:
    """One layer of the page-mode cache (all [bs, H, ...])."""
    chunk_min: torch.Tensor   # [bs,H,n_max,128] bf16
    chunk_max: torch.Tensor
    centroid: torch.Tensor
    valid: torch.Tensor       # [bs,H,n_max] bool
    kcodes: torch.Tensor      # [bs,H,n_max,16,16] int32
    vcodes_t: torch.Tensor    # [bs,H,n_max,128,2] int32
    vmeta: torch.Tensor       # [bs,H,n_max,2,4,16] bf16
    kscale: torch.Tensor      # [bs,H,n_max,128] bf16 KIVI key scales
    near_k: torch.Tensor      # [bs,H,near_cap,128] bf16
    near_v: torch.Tensor
    n_c: int
    n_near: int

    def layer(self) -> ops.PageLayer:
        return ops.PageLayer(self.chunk_min, self.chunk_max, self.valid, self.kcodes, self.vcodes_t, self.vmeta,
                             self.near_k, self.near_v, self.kscale)

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.chunk_min, self.chunk_max, self.kcodes, self.vcodes_t,
                                                           self.vmeta, self.near_k, self.near_v))


def alloc_page_cache(bs: int, heads: int, n_max: int, near_cap: int, device) -> PageCache:
    z = dict(device=device)
    return PageCache(
        chunk_min=torch.zeros(bs, heads, n_max, HEAD_DIM, dtype=torch.bfloat16, **z),
        chunk_max=torch.zeros(bs, heads, n_max, HEAD_DIM, dtype=torch.bfloat16, **z),
        centroid=torch.zeros(bs, heads, n_max, HEAD_DIM, dtype=torch.bfloat16, **z),
        valid=torch.zeros(bs, heads, n_max, dtype=torch.bool, **z),
        kcodes=torch.zeros(bs, heads, n_max, 16, 16, dtype=torch.int32, **z),
        vcodes_t=torch.zeros(bs, heads, n_max, HEAD_DIM, 2, dtype=torch.int32, **z),
        vmeta=torch.zeros(bs, heads, n_max, 2, 4, 16, dtype=torch.bfloat16, **z),
        kscale=torch.zeros(bs, heads, n_max, HEAD_DIM, dtype=torch.bfloat16, **z),
        near_k=torch.zeros(bs, heads, near_cap, HEAD_DIM, dtype=torch.bfloat16, **z),
        near_v=torch.zeros(bs, heads, near_cap, HEAD_DIM, dtype=torch.bfloat16, **z),
        n_c=0, n_near=0)


def build_page_cache(seed: int, bs: int, heads: int, n_retrieval: int, n_near: int, device,
                     keep_raw: bool = False, slab: int = 4096):
    """Fill a page cache with synthetic tokens [0, n_retrieval) (pages) and
    [n_retrieval, n_retrieval + n_near) (near window).  Returns (cache, raw)
    where raw = (K, V) bf16 [bs,H,T,128] when keep_raw, else None."""
    assert n_retrieval % CHUNK == 0
    gen = torch.Generator(device=device).manual_seed(seed)
    chans = outlier_channels(gen, heads, device)
    n_c = n_retrieval // CHUNK
    pc = alloc_page_cache(bs, heads, max(n_c, 1), max(n_near, 1), device)
    raw_k, raw_v = [], []
    # same outlier channels for the whole sequence of a head
    for t0 in range(0, n_retrieval, slab):
        t1 = min(n_retrieval, t0 + slab)
        g2 = torch.Generator(device=device).manual_seed(seed * 1000003 + t0)
        k = synth_keys(g2, bs, heads, t1 - t0, device, pos0=t0, channels=chans)
        v = synth_values(g2, bs, heads, t1 - t0, device)
        ops.kivi_encode_chunks(k, pc.chunk_min, pc.chunk_max, pc.centroid, pc.valid, pc.kcodes, t0 // CHUNK,
                               kscale=pc.kscale)
        ops.vquant_encode(v, pc.vcodes_t, pc.vmeta, t0)
        if keep_raw:
            raw_k.append(k)
            raw_v.append(v)
    if n_near:
        k = synth_keys(gen, bs, heads, n_near, device, pos0=n_retrieval, channels=chans)
        v = synth_values(gen, bs, heads, n_near, device)
        pc.near_k[:, :, :n_near].copy_(k)
        pc.near_v[:, :, :n_near].copy_(v)
        if keep_raw:
            raw_k.append(k)
            raw_v.append(v)
    pc.n_c, pc.n_near = n_c, n_near
    raw = (torch.cat(raw_k, dim=2), torch.cat(raw_v, dim=2)) if keep_raw else None
    return pc, raw


@dataclass
class RawCache:
    """One layer of the raw-page cache: Quest metadata over the retrieval zone
    and the raw K/V rows at absolute positions [sink | retrieval | near]."""
    chunk_min: torch.Tensor   # [bs,H,n_c,128] bf16
    chunk_max: torch.Tensor
    valid: torch.Tensor       # [bs,H,n_c] bool
    keys: torch.Tensor        # [bs,H,cap,128] bf16
    values: torch.Tensor
    n_sink: int
    n_c: int
    near_start: int
    n_near: int

    def layer(self) -> ops.RawLayer:
        return ops.RawLayer(self.chunk_min, self.chunk_max, self.valid, self.keys, self.values, self.n_sink)


def build_raw_cache(seed: int, bs: int, heads: int, n_retrieval: int, n_near: int, device, n_sink: int = 0,
                    slab: int = 4096) -> RawCache:
    """Synthetic tokens laid out as the reference's unified cache: sink rows
    [0, n_sink), retrieval rows [n_sink, n_sink + n_retrieval) (16-token
    chunks with Quest min/max from the library's encode kernel) and near rows
    after them.  Keys: N(0,1), 4 outlier channels x10 per head, RoPE at the
    token position; values N(0,1)."""
    assert n_retrieval % CHUNK == 0
    gen = torch.Generator(device=device).manual_seed(seed)
    chans = outlier_channels(gen, heads, device)
    n_c = n_retrieval // CHUNK
    cap = max(1, n_sink + n_retrieval + n_near)
    keys = torch.empty(bs, heads, cap, HEAD_DIM, dtype=torch.bfloat16, device=device)
    values = torch.empty_like(keys)
    cmin = torch.zeros(bs, heads, max(n_c, 1), HEAD_DIM, dtype=torch.bfloat16, device=device)
    cmax = torch.zeros_like(cmin)
    valid = torch.zeros(bs, heads, max(n_c, 1), dtype=torch.bool, device=device)
    packed = torch.empty(bs, heads, max(n_c, 1), 16, 16, dtype=torch.int32, device=device)
    for t0 in range(0, cap, slab):
        t1 = min(cap, t0 + slab)
        g2 = torch.Generator(device=device).manual_seed(seed * 1000003 + t0)
        keys[:, :, t0:t1] = synth_keys(g2, bs, heads, t1 - t0, device, pos0=t0, channels=chans)
        values[:, :, t0:t1] = synth_values(g2, bs, heads, t1 - t0, device)
    if n_c:
        ops.kivi_encode_chunks(keys[:, :, n_sink:n_sink + n_retrieval], cmin, cmax, None, valid, packed, 0)
    del packed
    return RawCache(cmin, cmax, valid, keys, values, n_sink, n_c, n_sink + n_retrieval, n_near)


def raw_algorithmic_bytes(rows: int, n_c: int, nk: int, n_raw: int, G: int = 4) -> int:
    """Compulsory HBM bytes of one raw page-mode launch: Quest min/max of all
    chunks (512 B each) + the selected pages' raw K and V rows (16 x 512 B)
    + the sink / near raw rows (512 B each) + q in / out (bf16)."""
    per_row = n_c * 512 + nk * 16 * 512 + n_raw * 512 + 2 * G * HEAD_DIM * 2
    return rows * per_row


def page_algorithmic_bytes(rows: int, n_c: int, nk: int, n_near: int, G: int = 4) -> int:
    """Compulsory HBM bytes of one page-mode decode launch: Quest min/max of
    all chunks + selected pages (K codes 1 KiB, V codes 1 KiB, V scale/zero
    256 B, min/max rows 512 B re-read for dequant) + near rows (512 B/token)
    + q in / out (bf16)."""
    per_row = n_c * 512 + nk * (1024 + 1024 + 256 + 512) + n_near * 512 + 2 * G * HEAD_DIM * 2
    return rows * per_row
