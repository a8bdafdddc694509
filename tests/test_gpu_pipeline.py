"""GPU: the one-call reference-mode retrieval chain (zkv_reference_select)
equals the single-op chain and the oracle, bit for bit."""
import numpy as np
import pytest
import torch

import oracle as O
from conftest import to_u16
from zoomkv_revision_b200 import ops
from zoomkv_revision_b200 import workload as W

pytestmark = pytest.mark.gpu
DEV = "cuda"


def make_layer(seed, bs, H, n_ret):
    pc, raw = W.build_page_cache(seed, bs, H, n_ret, 16, torch.device(DEV), keep_raw=True)
    q = W.synth_query(torch.Generator(device=DEV).manual_seed(seed + 1), bs, H * 4, torch.device(DEV))
    return pc, q


@pytest.mark.parametrize("bs,H,n_ret,nk,n_dense,dt,st,F,sk", [
    (2, 2, 16 * 300, 120, 36, 8, 8, 100, 7),
    (1, 4, 16 * 64, 64, 64, 16, 16, 1024, 0),
    (3, 1, 16 * 500, 40, 1, 16, 4, 17, 15),
])
def test_reference_select_equals_op_chain(bs, H, n_ret, nk, n_dense, dt, st, F, sk):
    pc, q = make_layer(bs * 100 + nk, bs, H, n_ret)
    n_c = pc.n_c
    n_valid = n_c - 3  # a partly encoded tail: ids >= n_valid score -1e30 in stage 2
    rows = bs * H
    skipped = torch.arange(1000, 1000 + sk, dtype=torch.int64, device=DEV).repeat(bs, H, 1)
    k = min(F, nk * 16)
    ws = torch.empty(ops.reference_select_ws_bytes(rows, n_c, nk, n_dense), dtype=torch.uint8, device=DEV)
    final = torch.full((bs, H, k + sk + 5), -7, dtype=torch.int64, device=DEV)
    raw_q = torch.empty(rows, 128, dtype=torch.bfloat16, device=DEV)
    ops.reference_select(q, pc.chunk_min, pc.chunk_max, pc.centroid, pc.valid, pc.kcodes, n_c, n_valid, nk, n_dense,
                         dt, st, k, skipped, final, ws, raw_q_out=raw_q)
    # the same chain through the single-op entry points
    qf = O.bf16_to_f32(to_u16(q)).reshape(rows, 4, 128)
    acc = np.zeros((rows, 128), np.float32)
    for g in range(4):
        acc = (acc + qf[:, g]).astype(np.float32)   # head order, fp32
    assert np.array_equal(to_u16(raw_q), O.f32_to_bf16(acc / np.float32(4)))
    rq = raw_q.view(bs, H, 128)
    scores = torch.empty(bs, H, n_c, dtype=torch.float32, device=DEV)
    ops.quest_chunk_score(rq, pc.chunk_min, pc.chunk_max, scores, n_c, pc.valid)
    ids = ops.float_topk_3d(scores, nk)
    dens = torch.empty(bs, H, nk, dtype=torch.float32, device=DEV)
    ops.partial_chunk_density_scores_cuda(ids, pc.centroid, rq, dens)
    pos = ops.float_topk_3d(dens, n_dense)
    mask = torch.empty(bs, H, nk, dtype=torch.bool, device=DEV)
    ops.dense_mask_from_topk_cuda(pos, mask)
    ksc = torch.empty(bs, H, nk * 16, dtype=torch.float32, device=DEV)
    kix = torch.empty(bs, H, nk * 16, dtype=torch.int64, device=DEV)
    ops.partial_chunk_kivi_qk_dense_sparse_cuda(ids, mask, pc.kcodes[:, :, :n_valid], pc.chunk_min, pc.chunk_max, rq,
                                                dt, st, 16, ksc, kix)
    ref = torch.empty(bs, H, k + sk, dtype=torch.int64, device=DEV)
    ops.float_topk_gather_concat_3d(ksc, kix, skipped, ref, k)
    torch.cuda.synchronize()
    assert torch.equal(final[:, :, :k + sk], ref)
    assert torch.all(final[:, :, k + sk:] == -7)
    # and the oracle
    R = rows
    mn, mx = to_u16(pc.chunk_min).reshape(R, -1, 128), to_u16(pc.chunk_max).reshape(R, -1, 128)
    oq = to_u16(raw_q)
    osc = O.quest_score(oq, mn, mx, pc.valid.cpu().numpy().astype(np.uint8).reshape(R, -1), n_c)
    oids = O.topk_f32(osc, nk)
    odens = O.chunk_density(oids, to_u16(pc.centroid).reshape(R, -1, 128), oq)
    omask = O.mask_from_topk(O.topk_f32(odens, n_dense), nk)
    pk = pc.kcodes.cpu().numpy().reshape(R, -1, 16, 16)
    oks, okx = O.kivi_qk(oids, omask, np.ascontiguousarray(pk[:, :n_valid]), mn, mx, oq, dt, st)
    ofinal = O.topk_gather_concat(oks, okx, skipped.cpu().numpy().reshape(R, sk), k)
    assert np.array_equal(final[:, :, :k + sk].cpu().numpy().reshape(R, -1), ofinal)


def test_reference_select_rejects_short_workspace():
    pc, q = make_layer(5, 1, 2, 16 * 64)
    need = ops.reference_select_ws_bytes(2, pc.n_c, 32, 8)
    ws = torch.empty(need - 256, dtype=torch.uint8, device=DEV)
    final = torch.empty(1, 2, 64, dtype=torch.int64, device=DEV)
    with pytest.raises(RuntimeError, match="status 3"):
        ops.reference_select(q, pc.chunk_min, pc.chunk_max, pc.centroid, pc.valid, pc.kcodes, pc.n_c, pc.n_c, 32, 8,
                             8, 8, 64, None, final, ws)
