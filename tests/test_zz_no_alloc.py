"""GPU: zkv_reference_select_noalloc (library-owned scratch, no allocation)
called through the C ABI equals zkv_reference_select with a caller
workspace, on two calls in a row; sizes beyond its buffer are rejected."""
import ctypes

import pytest
import torch

from zoomkv_revision_b200 import _lib
from zoomkv_revision_b200 import workload as W

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _layer(pc):
    return _lib.ZkvRefLayer(pc.chunk_min.data_ptr(), pc.chunk_max.data_ptr(), pc.centroid.data_ptr(),
                            pc.valid.data_ptr(), pc.kcodes.data_ptr())


def _args(pc, q, nk, n_dense, k, skipped, final):
    bs, H, n_max = pc.chunk_min.shape[:3]
    sk = skipped.shape[-1]
    return [q.data_ptr(), 4, ctypes.byref(_layer(pc)), bs * H, n_max, pc.n_c, pc.n_c, nk, n_dense, 8, 8, k,
            skipped.data_ptr() if sk else None, sk, sk, final.data_ptr(), final.shape[-1], None]


def test_noalloc_matches_workspace_entry_two_calls():
    torch.cuda.set_device(DEV)
    lib = _lib.lib()
    stream = torch.cuda.current_stream(DEV).cuda_stream
    cases = [(2, 4, 16 * 400, 160, 48, 100, 9), (4, 2, 16 * 900, 360, 108, 250, 0)]
    for seed, (bs, H, n_ret, nk, n_dense, F, sk) in enumerate(cases):
        pc, _ = W.build_page_cache(40 + seed, bs, H, n_ret, 16, DEV)
        q = W.synth_query(torch.Generator(device=DEV).manual_seed(seed), bs, H * 4, DEV)
        skipped = torch.arange(5000, 5000 + sk, dtype=torch.int64, device=DEV).repeat(bs, H, 1).contiguous()
        out_a = torch.full((bs, H, F + sk), -1, dtype=torch.int64, device=DEV)
        out_b = torch.full((bs, H, F + sk), -2, dtype=torch.int64, device=DEV)
        rows = bs * H
        need = lib.zkv_reference_select_ws_bytes(rows, pc.n_c, nk, n_dense)
        assert 0 < need <= (16 << 20)
        ws = torch.empty(need, dtype=torch.uint8, device=DEV)
        a = _args(pc, q, nk, n_dense, F, skipped, out_a)
        st = lib.zkv_reference_select(*a[:-1], None, ws.data_ptr(), need, stream)
        assert st == 0, lib.zkv_status_string(st)
        b = _args(pc, q, nk, n_dense, F, skipped, out_b)
        st = lib.zkv_reference_select_noalloc(*b[:-1], None, stream)
        assert st == 0, lib.zkv_status_string(st)
        torch.cuda.synchronize()
        assert torch.equal(out_a, out_b), f"call {seed}"
        assert int(out_b.min()) >= 0


def test_noalloc_rejects_sizes_beyond_buffer():
    torch.cuda.set_device(DEV)
    lib = _lib.lib()
    rows, n_c, nk, n_dense = 64, 2048, 2048, 2048
    assert lib.zkv_reference_select_ws_bytes(rows, n_c, nk, n_dense) > (16 << 20)
    t = torch.zeros(16, dtype=torch.int64, device=DEV)   # valid pointers; nothing is launched
    layer = _lib.ZkvRefLayer(t.data_ptr(), t.data_ptr(), t.data_ptr(), None, t.data_ptr())
    st = lib.zkv_reference_select_noalloc(t.data_ptr(), 4, ctypes.byref(layer), rows, n_c, n_c, n_c, nk, n_dense, 8,
                                          8, 100, None, 0, 0, t.data_ptr(), 100, None,
                                          torch.cuda.current_stream(DEV).cuda_stream)
    assert st == 3, lib.zkv_status_string(st)
    assert b"limit" in lib.zkv_status_string(st)
