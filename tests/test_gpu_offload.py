"""GPU: the offload-tier gather (zkv_h2d_gather_kv / _packed) copies the
selected K/V rows from host-pinned memory bit for bit, as the oracle's
restatement of cache_hub/gather_trans/trans_h2d.cu does, on the cases of the
reference's own checks (trans_h2d.py:168-259 and
test_trans_h2d_packed_pathological.py: production-scale segments over seeds
0, 1, 2, 7, 42; every segment of length 1; mixed lengths; batch 2; empty
segments; the sink+local rows of every packed segment left untouched)."""
import numpy as np
import pytest
import torch

import oracle as O
from conftest import to_u16
from zoomkv_revision_b200 import _lib, ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _pinned_kv(bs, H, L, seed):
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(bs, H, L, 128, generator=g).to(torch.bfloat16).pin_memory()
    v = torch.randn(bs, H, L, 128, generator=g).to(torch.bfloat16).pin_memory()
    return k, v


@pytest.mark.parametrize("bs,H,L,topk", [(2, 8, 32 * 1024, 100), (1, 8, 4096, 1), (3, 2, 777, 300)])
def test_dense_gather_bit_exact(bs, H, L, topk):
    """The reference's own check (trans_h2d.py:168-204): dst pre-zeroed with
    max_topk = 0.2 kv_len rows, random indices (duplicates allowed)."""
    k, v = _pinned_kv(bs, H, L, seed=topk)
    g = torch.Generator().manual_seed(5)
    idx = torch.randint(0, L, (bs, H, topk), generator=g, dtype=torch.int64)
    max_topk = max(topk, int(L * 0.2))
    dk = torch.zeros(bs, H, max_topk, 128, dtype=torch.bfloat16, device=DEV)
    dv = torch.zeros_like(dk)
    ops.h2d_gather_kv(k, v, idx.to(DEV), dk, dv)
    torch.cuda.synchronize()
    z = np.zeros((bs, H, max_topk, 128), np.uint16)
    assert np.array_equal(to_u16(dk), O.h2d_gather(to_u16(k), idx.numpy(), z))
    assert np.array_equal(to_u16(dv), O.h2d_gather(to_u16(v), idx.numpy(), z))


def _packed_case(bs, H, L, sl_end, ks, seed):
    k, v = _pinned_kv(bs, H, L, seed)
    V = bs * H
    ak = torch.tensor(ks, dtype=torch.int32)
    cu_topk = torch.zeros(V + 1, dtype=torch.int32)
    torch.cumsum(ak, 0, out=cu_topk[1:])
    cu_k = torch.zeros(V + 1, dtype=torch.int32)
    torch.cumsum(ak + sl_end, 0, out=cu_k[1:])
    g = torch.Generator().manual_seed(seed)
    idx = torch.cat([torch.randint(0, L, (int(n),), generator=g, dtype=torch.int64) for n in ks])
    total_k = int(cu_k[-1])
    sentinel = torch.full((total_k, 128), 7.5, dtype=torch.bfloat16)
    dk, dv = sentinel.to(DEV), sentinel.to(DEV)
    global_k = int(ak.max())
    ops.h2d_gather_kv_packed(k, v, dk, dv, idx.to(DEV), cu_topk.to(DEV), cu_k.to(DEV), sl_end, global_k)
    torch.cuda.synchronize()
    s16 = to_u16(sentinel)
    for src, dst in ((k, dk), (v, dv)):
        ref = O.h2d_gather_packed(to_u16(src), idx.numpy(), cu_topk.numpy(), cu_k.numpy(), sl_end, global_k, s16)
        got = to_u16(dst)
        assert np.array_equal(got, ref)
        for vh in range(V):  # the sink+local rows of every segment keep the sentinel
            c0 = int(cu_k[vh])
            assert np.array_equal(got[c0:c0 + sl_end], s16[c0:c0 + sl_end])


@pytest.mark.parametrize("seed", [0, 1, 2, 7, 42])
def test_packed_production_scale(seed):
    gg = torch.Generator().manual_seed(seed)
    ks = torch.randint(50, 801, (8,), generator=gg, dtype=torch.int32).tolist()
    _packed_case(1, 8, 16384, 320, ks, seed)


@pytest.mark.parametrize("name,bs,L,ks,seed", [
    ("k1_all", 1, 8192, [1] * 8, 11),
    ("mixed", 1, 16384, [1, 50, 100, 200, 400, 600, 800, 50], 99),
    ("bs2", 2, 16384, None, 123),
    ("zero_k", 1, 8192, [0, 50, 0, 200, 0, 100, 0, 50], 314),
])
def test_packed_pathological(name, bs, L, ks, seed):
    if ks is None:
        g = torch.Generator().manual_seed(seed)
        ks = torch.randint(100, 601, (bs * 8,), generator=g, dtype=torch.int32).tolist()
    _packed_case(bs, 8, L, 320, ks, seed)


def test_gather_with_offsets_into_a_window():
    """The cache's form: zone-relative indices (src offset) written after the
    sink rows of a window buffer (dst offset), first n of a wider index row."""
    bs, H, L, s, n = 2, 4, 3000, 7, 50
    k, v = _pinned_kv(bs, H, L, seed=3)
    sel = torch.randint(0, L - s, (bs, H, n + 9), generator=torch.Generator().manual_seed(1))
    win_k = torch.zeros(bs, H, s + n + 20, 128, dtype=torch.bfloat16, device=DEV)
    win_v = torch.zeros_like(win_k)
    ops.h2d_gather_rows(k, v, sel.to(DEV), win_k, win_v, n_sel=n, src_offset=s, dst_offset=s)
    torch.cuda.synchronize()
    ref = np.zeros((bs, H, s + n + 20, 128), np.uint16)
    for b in range(bs):
        for h in range(H):
            ref[b, h, s:s + n] = to_u16(k)[b, h, sel[b, h, :n].numpy() + s]
    assert np.array_equal(to_u16(win_k), ref)


def test_out_of_range_index_is_skipped_and_reported():
    bs, H, L, topk = 1, 2, 1000, 8
    k, v = _pinned_kv(bs, H, L, seed=4)
    idx = torch.arange(topk, dtype=torch.int64).repeat(bs, H, 1)
    idx[0, 1, 3] = L + 5
    idx[0, 0, 6] = -1
    dk = torch.zeros(bs, H, topk, 128, dtype=torch.bfloat16, device=DEV)
    dv = torch.zeros_like(dk)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.h2d_gather_kv(k, v, idx.to(DEV), dk, dv, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == _lib.ZKV_ERR_RANGE
    got, src = to_u16(dk), to_u16(k)
    for h in range(H):
        for j in range(topk):
            bad = (h, j) in ((1, 3), (0, 6))
            assert np.array_equal(got[0, h, j], np.zeros(128, np.uint16) if bad else src[0, h, j])


def test_argument_checks():
    k, v = _pinned_kv(1, 2, 64, seed=6)
    idx = torch.zeros(1, 2, 4, dtype=torch.int64, device=DEV)
    dk = torch.zeros(1, 2, 4, 128, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(AssertionError):  # pageable source (the reference asserts is_pinned)
        ops.h2d_gather_kv(k.clone(), v.clone(), idx, dk, dk.clone())
    with pytest.raises(AssertionError):  # fewer destination rows than topk
        ops.h2d_gather_kv(k, v, torch.zeros(1, 2, 5, dtype=torch.int64, device=DEV), dk, dk.clone())
    # through the C ABI, a pageable source is refused before any launch
    pageable = torch.zeros(2 * 64 * 128, dtype=torch.bfloat16)
    rc = _lib.lib().zkv_h2d_gather_kv(pageable.data_ptr(), pageable.data_ptr(), 2, 64, idx.data_ptr(), 4, 4, 0,
                                      dk.data_ptr(), dk.data_ptr(), 4, 0, None, None)
    assert rc == 1  # ZKV_ERR_ARG
