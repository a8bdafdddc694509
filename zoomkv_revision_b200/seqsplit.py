"""Sequence-split page-mode decode over one process per GPU (long contexts).

Raw-row page mode: `RawSplitGroup` (zkv_page_decode_raw_split) -- the
exchanges live inside the decode's own four kernels (scores and partials as
tagged-word peer stores over NVLink with bounded waits); see its docstring.

4-bit page mode: the retrieval pages of a layer are split into contiguous ranges, one per
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

Two transports carry the exchanges of steps 2 and 5:

  * `decode_step_p2p` (the product on NVLink): every rank writes its slice
    straight into every peer's buffer with stores over NVLink and raises a
    flag there, and the same launch then waits on its own flags with a
    bounded poll (zkv_peer_exchange).  The buffers are shared once through
    CUDA IPC (`PeerGroup`).  A layer is 5 launches -- scores, exchange,
    select + attend, exchange, merge -- none of them a collective, and the
    step can be captured in a CUDA graph (the epochs live on the device);
  * `decode_step` with NCCL all-gathers (any backend torch.distributed
    offers; also the CPU/gloo form the host-logic tests run).

The compute steps go through a backend object; the product backend is
`CudaBackend` (libzkv kernels, no CPU path).  Reference: the
sequence split replaces the single-device gather of polar_cache.compute
(cache_hub/polar_cache_quest_density_single_layer_kivi.py:1589-1775) for
contexts beyond one device; the merge is lse_merge (lse_merge/lse_merge.py).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist

import ctypes

from . import _lib, ops


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


# --------------------------------------------------------------------------- peer-memory transport
class _CudaArray:
    """A raw device pointer exposed as a CUDA array (torch.as_tensor wraps it
    without a copy; the owner keeps the allocation alive)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 2, "strides": None}


def _view(ptr: int, shape, dtype, device):
    typestr = {torch.float32: "<f4", torch.int32: "<i4"}[dtype]
    return torch.as_tensor(_CudaArray(ptr, shape, typestr), device=device)


_FLAGS_A, _FLAGS_B, _EPOCH, _DONE, _HEADER = 0, 32, 64, 68, 256


def _share_buffer(nbytes: int, world: int, rank: int, group=None):
    """Allocate this rank's zeroed exchange buffer (zkv_peer_alloc), send its
    IPC handle to every rank (all_gather_object on `group`) and map every
    peer's buffer (zkv_peer_open).  Returns (own base, the mappings this
    process opened, a ctypes array of every rank's base in rank order)."""
    L = _lib.lib()
    ptr = ctypes.c_void_p()
    handle = (ctypes.c_char * L.zkv_peer_handle_bytes())()
    _lib.check(L.zkv_peer_alloc(int(nbytes), ctypes.byref(ptr), handle), "zkv_peer_alloc")
    handles = [None] * world
    if world > 1:
        dist.all_gather_object(handles, bytes(handle), group=group)
    bases, opened = [], []
    for r in range(world):
        if r == rank:
            bases.append(ptr.value)
            continue
        p = ctypes.c_void_p()
        _lib.check(L.zkv_peer_open(handles[r], ctypes.byref(p)), "zkv_peer_open")
        opened.append(p.value)
        bases.append(p.value)
    return ptr.value, opened, (ctypes.c_void_p * world)(*bases)


def peer_layout(rows: int, G: int, per: int, world: int, P: int) -> dict:
    """Byte offsets of the shared buffer (the same on every rank): header,
    score row [rows][world*per] fp32, partial outputs [world*P][rows*G][128]
    fp32, partial lse [world*P][rows*G] fp32; every region 256-byte aligned."""
    a256 = lambda x: (x + 255) // 256 * 256
    off_row = _HEADER
    off_parts = off_row + a256(rows * world * per * 4)
    off_lses = off_parts + a256(world * P * rows * G * 128 * 4)
    return {"row": off_row, "parts": off_parts, "lses": off_lses, "total": off_lses + a256(world * P * rows * G * 4)}


class PeerGroup:
    """One IPC-shared buffer per rank for the split decode's exchanges.

    Byte layout (every rank the same): a 256-byte header (flags of the
    score exchange at 0, flags of the partial exchange at 32 -- one uint32
    per rank --, the device epoch at 64, the put kernel's CTA counter at
    68), then
      row    [rows][world*per] fp32  score row; rank r writes columns
                                     [r*per, r*per + n_loc_r), the rest -inf
      parts  [world*P][rows*G][128] fp32, lses [world*P][rows*G] fp32:
             rank r's P per-cluster partials at slots r*P .. r*P + P - 1.
    Rank-local staging (scores, selection, partials, output) is ordinary
    torch memory.  Handles travel once through torch.distributed
    (all_gather_object on `group`)."""

    def __init__(self, bs, H, G, n_c, nk, world, rank, device, group=None):
        self.bs, self.H, self.G, self.nk, self.world, self.rank = bs, H, G, nk, world, rank
        self.device = torch.device(device)
        self.lo, self.hi, self.per = split_range(n_c, world, rank)
        self.n_c, self.n_loc = n_c, self.hi - self.lo
        rows = bs * H
        self.rows = rows
        # clusters per row of the select + attend kernel (as the split form:
        # about two CTA waves' worth of clusters)
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.P = P = max(1, min(4, (2 * sms) // (rows * 8)))
        lay = peer_layout(rows, G, self.per, world, P)
        self.off_row, self.off_parts, self.off_lses, total = lay["row"], lay["parts"], lay["lses"], lay["total"]
        self.base, self._opened, self.peer_base = _share_buffer(total, world, rank, group)
        dev = self.device
        self.row = _view(self.base + self.off_row, (bs, H, world * self.per), torch.float32, dev)
        self.parts = _view(self.base + self.off_parts, (world * P, rows * G, 128), torch.float32, dev)
        self.lses = _view(self.base + self.off_lses, (world * P, rows * G), torch.float32, dev)
        self.row.fill_(-math.inf)
        self.flags_a = self.base + _FLAGS_A
        self.flags_b = self.base + _FLAGS_B
        self.epoch = self.base + _EPOCH
        self.done = self.base + _DONE
        f32 = dict(dtype=torch.float32, device=dev)
        self.local = torch.empty(max(1, rows * self.n_loc), **f32)
        self.sel = torch.empty(bs, H, nk, dtype=torch.int64, device=dev)
        self.part = torch.empty(P, rows * G, 128, **f32)
        self.lse = torch.empty(P, rows * G, **f32)
        self.out = torch.empty(bs, 1, H * G, 128, dtype=torch.bfloat16, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        S = _lib.ZkvPeerSeg
        self._seg_scores = (S * 1)(S(self.local.data_ptr(), self.n_loc * 4, self.off_row + rank * self.per * 4,
                                     world * self.per * 4, self.n_loc * 4, rows if self.n_loc > 0 else 0, 0))
        pb, lb = P * rows * G * 128 * 4, P * rows * G * 4
        self._seg_parts = (S * 2)(S(self.part.data_ptr(), pb, self.off_parts + rank * pb, pb, pb, 1, 0),
                                  S(self.lse.data_ptr(), lb, self.off_lses + rank * lb, lb, lb, 1, 0))
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier(group=group)  # every mapping is open before the first put
        self._group = group

    def _put(self, segs, n_seg, flag_off, stream):
        _lib.check(_lib.lib().zkv_peer_put(segs, n_seg, self.peer_base, flag_off, self.rank, self.world,
                                           self.epoch, self.done, 0, stream), "zkv_peer_put")

    def _exchange(self, segs, n_seg, flag_off, stream):
        _lib.check(_lib.lib().zkv_peer_exchange(segs, n_seg, self.peer_base, flag_off, self.rank, self.world,
                                                self.epoch, self.done, 0, self.status.data_ptr(), stream),
                   "zkv_peer_exchange")

    def _wait(self, flags, stream):
        _lib.check(_lib.lib().zkv_peer_wait(flags, self.epoch, self.world, self.status.data_ptr(), stream),
                   "zkv_peer_wait")

    def check(self):
        """Raise if a peer wait of this group gave up (a rank did not arrive
        within the wait limit, zkv_peer_set_wait_ms).  Reads the status word,
        so it synchronises with the group's stream work.  After a timeout the
        ranks' epochs disagree: close this group and build a new one."""
        st = int(self.status.item())
        if st != 0:
            raise RuntimeError(f"peer exchange failed: status {st} ({_lib.lib().zkv_status_string(st).decode()}); "
                               "the peer group must be rebuilt")

    def close(self):
        """Unmap the peers and free the own buffer (after a barrier, so no
        peer still writes into it)."""
        if self.base is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self._group)
        L = _lib.lib()
        for p in self._opened:
            L.zkv_peer_close(ctypes.c_void_p(p))
        self._opened = []
        self.row = self.parts = self.lses = None
        L.zkv_peer_free(ctypes.c_void_p(self.base))
        self.base = None


def decode_step_p2p(q, layer: ops.PageLayer, pg: PeerGroup, *, n_sink: int = 0, near_start: int = 0,
                    n_near: int = 0, check: bool = True):
    """decode_step over peer memory: score own pages -> put scores into every
    peer's score row -> wait -> select + attend the own selected pages in one
    kernel (zkv_page_decode_scored, P clusters per row) -> put the P partial
    (out, lse) into every peer -> wait -> LSE merge of all world*P partials.
    Returns the merged output [bs, 1, H*G, 128] bf16 (same on every rank)
    and the selected global page ids [bs, H, nk].

    check: raise (PeerGroup.check) when a peer wait of this step gave up
    instead of returning a merge of stale partials; it synchronises the
    stream once per step, and is skipped while the stream is being captured
    into a CUDA graph (check the group after replaying the graph)."""
    stream = torch.cuda.current_stream(q.device).cuda_stream
    if pg.n_loc > 0:
        cmin, cmax, valid = layer.tensors[0], layer.tensors[1], layer.tensors[2]
        ops.quest_chunk_score_gqa(q, cmin, cmax, pg.local, pg.n_loc, valid)
    pg._exchange(pg._seg_scores, 1, _FLAGS_A, stream)
    own_raw = pg.rank == 0
    ops.page_decode_scored(q, layer, pg.row, pg.world * pg.per, pg.nk, pg.lo, pg.hi, pg.P, pg.part, pg.lse,
                           n_sink=n_sink if own_raw else 0, near_start=near_start, n_near=n_near if own_raw else 0,
                           sel_out=pg.sel, status=pg.status)
    pg._exchange(pg._seg_parts, 2, _FLAGS_B, stream)
    ops.lse_merge_n(pg.parts, pg.lses, pg.out.view(-1, 128))
    if check and not torch.cuda.is_current_stream_capturing():
        pg.check()
    return pg.out, pg.sel


# --------------------------------------------------------------------------- raw-row split
class RawSplitGroup:
    """Sequence split of the raw-row page decode (ops.page_decode_raw) over
    `world` ranks, one process per GPU, with the exchanges fused into the
    decode's own kernels (zkv_page_decode_raw_split):

      * the score kernel stores each rank's Quest scores straight into every
        rank's score row (peer stores over NVLink) as 64-bit words {score,
        epoch of the call}, so no fence or flag is needed;
      * every rank's select kernel waits (bounded) until every word of its
        row carries the call's epoch and picks the top nk of the whole row --
        the same kernel and keys as on one GPU, so the selection is the
        single-GPU selection exactly;
      * each rank attends the selected pages it holds (rank 0 also the sink
        and near rows), and the merge kernel stores each (row, head)'s
        partial into every rank as tagged words, waits for all of them and
        combines them in rank order: every rank ends with the same output.

    Four launches per layer, as on one GPU; no collective and no separate
    exchange launch.  Rank r holds the pages ops.raw_split_range(n_c, world,
    r).  The exchange buffer (zkv_raw_split_buffer_bytes) is allocated
    zeroed and shared once through CUDA IPC; its epochs live on the device,
    so a captured CUDA graph replays correctly as long as every rank replays
    the same calls.  One group serves any number of layers called in
    sequence (the partial exchange of one call orders it before the next
    call's score stores)."""

    def __init__(self, rows: int, G: int, n_c: int, world: int, rank: int, device, group=None):
        self.rows, self.G, self.n_c, self.world, self.rank = rows, G, n_c, world, rank
        self.device = torch.device(device)
        self.lo, self.hi = ops.raw_split_range(n_c, world, rank)
        self.n_loc = self.hi - self.lo
        L = _lib.lib()
        nbytes = int(L.zkv_raw_split_buffer_bytes(rows, G, n_c, world))
        if nbytes == 0:
            raise ValueError("invalid raw split shape")
        self.base, self._opened, self.peer_base = _share_buffer(nbytes, world, rank, group)
        self.nbytes = nbytes
        self.struct = _lib.ZkvRawSplit(ctypes.cast(self.peer_base, ctypes.POINTER(ctypes.c_void_p)), nbytes, rank,
                                       world)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)
        if world > 1:
            dist.barrier(group=group)  # every mapping is open before the first store
        self._group = group

    def decode(self, q, layer: ops.RawLayer, nk: int, n_near: int, **kw):
        """ops.page_decode_raw_split over this group's buffers (status word:
        the group's unless given)."""
        kw.setdefault("status", self.status)
        bs, H = layer.tensors[0].shape[:2]
        if bs * H != self.rows or q.shape[2] != self.rows // bs * self.G:
            raise ValueError(f"this group was built for {self.rows} rows of G = {self.G}; got {bs * H} rows of "
                             f"G = {q.shape[2] // H}")
        return ops.page_decode_raw_split(q, layer, self, self.n_c, nk, n_near, **kw)

    def check(self):
        """Raise if a wait of this group gave up (a rank did not arrive within
        the wait limit, zkv_peer_set_wait_ms); reads the status word, so it
        synchronises.  After a timeout the ranks' epochs disagree: close this
        group and build a new one."""
        st = int(self.status.item())
        if st != 0:
            raise RuntimeError(f"raw split exchange failed: status {st} "
                               f"({_lib.lib().zkv_status_string(st).decode()}); the group must be rebuilt")

    def close(self):
        """Unmap the peers and free the own buffer (after a barrier, so no
        peer still writes into it)."""
        if self.base is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self._group)
        L = _lib.lib()
        for p in self._opened:
            L.zkv_peer_close(ctypes.c_void_p(p))
        self._opened = []
        L.zkv_peer_free(ctypes.c_void_p(self.base))
        self.base = None


def local_raw_layer(rc, lo: int, hi: int, rank: int):
    """This rank's share of a full raw cache (workload.RawCache) as a
    RawLayer: pages [lo, hi) as local pages 0.. (their Quest metadata and
    raw rows copied out), and on rank 0 the sink rows in front and the near
    rows behind them.  Returns (layer, near_start) for the rank's call."""
    bs, H, _, D = rc.keys.shape
    ns, nn = (rc.n_sink, rc.n_near) if rank == 0 else (0, 0)
    n_loc = hi - lo
    base = ns
    near_start = base + 16 * n_loc
    cap = max(1, near_start + nn)
    keys = torch.zeros(bs, H, cap, D, dtype=rc.keys.dtype, device=rc.keys.device)
    values = torch.zeros_like(keys)
    t0 = rc.n_sink + 16 * lo
    keys[:, :, base:near_start] = rc.keys[:, :, t0:t0 + 16 * n_loc]
    values[:, :, base:near_start] = rc.values[:, :, t0:t0 + 16 * n_loc]
    if ns:
        keys[:, :, :ns] = rc.keys[:, :, :ns]
        values[:, :, :ns] = rc.values[:, :, :ns]
    if nn:
        keys[:, :, near_start:near_start + nn] = rc.keys[:, :, rc.near_start:rc.near_start + nn]
        values[:, :, near_start:near_start + nn] = rc.values[:, :, rc.near_start:rc.near_start + nn]
    cmin = rc.chunk_min[:, :, lo:hi].contiguous()
    cmax = rc.chunk_max[:, :, lo:hi].contiguous()
    valid = rc.valid[:, :, lo:hi].contiguous()
    return ops.RawLayer(cmin, cmax, valid, keys, values, base), near_start


def set_peer_wait_ms(ms: int) -> None:
    """Time limit of the peer waits for launches enqueued from now on."""
    _lib.check(_lib.lib().zkv_peer_set_wait_ms(int(ms)), "zkv_peer_set_wait_ms")
