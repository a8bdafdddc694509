"""Sequence-split page-mode decode over one process per GPU (long contexts).

The retrieval pages of a layer are split into contiguous ranges, one per
rank (rank r owns pages [r*per, min(n_c, (r+1)*per)), per = ceil(n_c/world));
rank 0 also holds the sink and near rows.  One decode step per layer:

  1. every rank scores its own pages (Quest upper bounds, fp32);
  2. all-gather of the per-rank score rows (per*4 bytes per KV head) --
     every rank then holds the whole score row, padded with -inf;
  3. every rank runs the same deterministic top-nk (ties to the lower page
     id), so the selection equals the single-GPU selection exactly;
  4. every rank attends over the selected pages it owns (+ rank 0 the raw
     rows), producing a normalised fp32 partial and its log-sum-exp;
  5. all-gather of the partials, then a local log-sum-exp merge.

The collectives are plain NCCL all-gathers (no data-path collective inside
a kernel).  The compute steps go through a backend object; the product
backend is `CudaBackend` (libzkv kernels, no CPU path).  Reference: the
sequence split replaces the single-device gather of polar_cache.compute
(cache_hub/polar_cache_quest_density_single_layer_kivi.py:1589-1775) for
contexts beyond one device; the merge is lse_merge (lse_merge/lse_merge.py).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import ops


def _all_gather(out, inp, group=None):
    """out[r] = inp of rank r (NCCL: one all_gather_into_tensor; other
    backends: the list form into views of out)."""
    if inp.is_cuda:
        dist.all_gather_into_tensor(out, inp, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), inp, group=group)


def split_range(n_c: int, world: int, rank: int):
    """(lo, hi, per): the pages rank owns and the per-rank stride."""
    per = max(1, math.ceil(n_c / world))
    lo = min(n_c, rank * per)
    return lo, min(n_c, lo + per), per


class CudaBackend:
    """libzkv kernels for the compute steps of the split decode."""

    def raw_q(self, q, heads):
        return ops.gqa_mean(q, heads)

    def local_scores(self, raw_q, layer: ops.PageLayer, n_loc: int, local, out):
        """Scores of this rank's n_loc pages into out[..., :n_loc] (the
        kernel writes [rows][n_loc] densely into `local`)."""
        if n_loc > 0:
            bs, H = out.shape[:2]
            cmin, cmax, valid = layer.tensors[0], layer.tensors[1], layer.tensors[2]
            ops.quest_chunk_score(raw_q, cmin, cmax, local, n_loc, valid)
            out[:, :, :n_loc].copy_(local[:bs * H * n_loc].view(bs, H, n_loc))
        return out

    def global_topk(self, scores, nk: int, out):
        return ops.float_topk_3d(scores, nk, out=out)

    def attend(self, q, layer, sel, lo, hi, n_sink, near_start, n_near, out_f32, lse, status):
        return ops.page_attend(q, layer, sel, lo, hi, n_sink=n_sink, near_start=near_start, n_near=n_near,
                               out_f32=out_f32, lse=lse, status=status)

    def merge(self, parts, lses, out):
        return ops.lse_merge_n(parts, lses, out)


@dataclass
class SplitBuffers:
    """Preallocated per-step buffers of one rank (no allocation per step)."""
    local: torch.Tensor       # [bs*H*per] fp32 staging of the local scores
    scores: torch.Tensor      # [bs, H, per] fp32, tail -inf
    gathered: torch.Tensor    # [world, bs, H, per]
    row: torch.Tensor         # [bs, H, world*per]
    sel: torch.Tensor         # [bs, H, nk] int64
    part: torch.Tensor        # [bs, H*G, 128] fp32
    lse: torch.Tensor         # [bs, H*G] fp32
    parts: torch.Tensor       # [world, bs*H*G, 128]
    lses: torch.Tensor        # [world, bs*H*G]
    out: torch.Tensor         # [bs, 1, H*G, 128] bf16
    status: torch.Tensor      # [1] int32

    @classmethod
    def alloc(cls, bs, H, G, per, nk, world, device):
        z = dict(device=device)
        f32 = dict(dtype=torch.float32, **z)
        return cls(local=torch.empty(bs * H * per, **f32),
                   scores=torch.full((bs, H, per), -math.inf, **f32),
                   gathered=torch.empty(world, bs, H, per, **f32),
                   row=torch.empty(bs, H, world * per, **f32),
                   sel=torch.empty(bs, H, nk, dtype=torch.int64, **z),
                   part=torch.empty(bs, H * G, 128, **f32),
                   lse=torch.empty(bs, H * G, **f32),
                   parts=torch.empty(world, bs * H * G, 128, **f32),
                   lses=torch.empty(world, bs * H * G, **f32),
                   out=torch.empty(bs, 1, H * G, 128, dtype=torch.bfloat16, **z),
                   status=torch.zeros(1, dtype=torch.int32, **z))


def decode_step(q, layer: ops.PageLayer, n_c: int, nk: int, bufs: SplitBuffers, *, rank: int, world: int,
                group=None, n_sink: int = 0, near_start: int = 0, n_near: int = 0, backend=None):
    """One split decode step of one layer on this rank.  `layer` holds this
    rank's pages as its pages 0.. (views of a chunk range are fine).
    Returns the merged output [bs, 1, H*G, 128] bf16 (same on every rank)
    and the selected global page ids [bs, H, nk]."""
    be = backend or CudaBackend()
    bs, H = layer.tensors[0].shape[:2]
    lo, hi, per = split_range(n_c, world, rank)
    raw_q = be.raw_q(q, H)
    be.local_scores(raw_q, layer, hi - lo, bufs.local, bufs.scores)
    if world > 1:
        _all_gather(bufs.gathered, bufs.scores, group)
        bufs.row.copy_(bufs.gathered.permute(1, 2, 0, 3).reshape(bs, H, world * per))
    else:
        bufs.row.copy_(bufs.scores)
    be.global_topk(bufs.row, nk, bufs.sel)
    own_raw = rank == 0
    be.attend(q, layer, bufs.sel, lo, hi, n_sink if own_raw else 0, near_start, n_near if own_raw else 0,
              bufs.part, bufs.lse, bufs.status)
    if world > 1:
        _all_gather(bufs.parts, bufs.part.reshape(-1, 128), group)
        _all_gather(bufs.lses, bufs.lse.reshape(-1), group)
    else:
        bufs.parts[0].copy_(bufs.part.reshape(-1, 128))
        bufs.lses[0].copy_(bufs.lse.reshape(-1))
    be.merge(bufs.parts, bufs.lses, bufs.out.view(-1, 128))
    return bufs.out, bufs.sel


def local_layer(layer: ops.PageLayer, lo: int, hi: int) -> ops.PageLayer:
    """View of pages [lo, hi) of a full layer as a rank-local layer."""
    t = layer.tensors
    cut = [x[:, :, lo:max(hi, lo + 1)] for x in t[:6]]
    return ops.PageLayer(*cut, t[6], t[7], t[8][:, :, lo:max(hi, lo + 1)])
