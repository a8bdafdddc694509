"""GPU parity of the ParisKV / RaBitQ kernels (through the C ABI via ops)
against the reference fixtures and the CPU oracle; bit-exact throughout
(integer counts, codes, index sets; bf16/fp32 in the restated order)."""
import numpy as np
import pytest
import torch

import oracle as O
from conftest import from_u16, golden, to_u16
from zoomkv_revision_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _enc_fixture():
    g = golden("rabitq_encode.npz")
    bs, H, N, D = g["keys"].shape
    return g, bs, H, N, D


@pytest.mark.parametrize("layout", ["token", "reference"])
def test_encode_matches_reference(layout):
    g, bs, H, N, D = _enc_fixture()
    R = bs * H
    keys = from_u16(g["keys"]).to(DEV)
    signs = from_u16(g["signs"]).to(DEV)
    if layout == "token":
        lay = ops.RqLayout.alloc(R, N, DEV)
        ops.rq_encode(keys, signs, lay)
        torch.cuda.synchronize()
        codes, packed, weight = lay.codes.cpu().numpy(), lay.packed.cpu().view(torch.uint8).numpy(), to_u16(lay.weight)
        hist = lay.hist.cpu().numpy()
        fac = lay.factor.cpu().numpy()
        _, _, _, ofac, _ = O.rq_encode(g["keys"].reshape(R, N, D), g["signs"])
        assert np.array_equal(fac, ofac)
    else:
        cb, w, p4, cnt = ops.batch_encode(keys, signs)
        torch.cuda.synchronize()
        codes = cb.permute(0, 1, 3, 2).cpu().numpy()
        packed = p4.permute(0, 1, 3, 2, 4).cpu().numpy()
        weight = to_u16(w.permute(0, 1, 3, 2))
        hist = cnt.cpu().numpy()
    assert np.array_equal(codes.reshape(R, N, 16), g["codes"].reshape(R, N, 16))
    assert np.array_equal(packed.reshape(R, N, 64), g["packed"].reshape(R, N, 64))
    assert np.array_equal(weight.reshape(R, N, 16), g["weight"].reshape(R, N, 16))
    assert np.array_equal(hist.reshape(R, 16, 256), g["hist"].reshape(R, 16, 256))


def test_encode_appends_in_place():
    """Two encode calls at different token offsets == one call (flush path)."""
    g, bs, H, N, D = _enc_fixture()
    R = bs * H
    keys = from_u16(g["keys"]).to(DEV).reshape(R, N, D)
    signs = from_u16(g["signs"]).to(DEV)
    lay = ops.RqLayout.alloc(R, N, DEV)
    ops.rq_encode(keys[:, :333], signs, lay, tok_start=0)
    ops.rq_encode(keys[:, 333:], signs, lay, tok_start=333)
    torch.cuda.synchronize()
    assert np.array_equal(lay.codes.cpu().numpy(), g["codes"].reshape(R, N, 16))
    assert np.array_equal(lay.hist.cpu().numpy(), g["hist"].reshape(R, 16, 256))


def test_query_matches_reference():
    g, bs, H, N, D = _enc_fixture()
    R = bs * H
    q = from_u16(g["q"]).to(DEV)
    out = ops.rq_query(q, from_u16(g["signs"]).to(DEV), 4, planes=True)
    torch.cuda.synchronize()
    assert np.array_equal(to_u16(out["q_mean"]), g["q_mean"].reshape(R, D))
    assert np.array_equal(to_u16(out["q_blocks"]), g["q_blocks"].reshape(R, D))
    assert np.array_equal(to_u16(out["q_norm"]), g["q_norm"].reshape(R))
    pl, qp = O.rq_query_4bit(g["q_blocks"].reshape(R, D), g["q_norm"].reshape(R))
    assert np.array_equal(out["planes"].cpu().numpy(), pl)
    assert np.array_equal(out["qparams"].cpu().numpy(), qp)


@pytest.mark.parametrize("layout", ["token", "reference"])
def test_collision_counts_match_reference(layout):
    g, bs, H, N, D = _enc_fixture()
    R = bs * H
    qb = from_u16(g["q_blocks"]).to(DEV).reshape(R, D)
    hist = torch.from_numpy(g["hist"].reshape(R, 16, 256)).to(DEV)
    if layout == "token":
        lay = ops.RqLayout.alloc(R, N, DEV)
        lay.codes.copy_(torch.from_numpy(g["codes"].reshape(R, N, 16)))
        lay.hist.copy_(hist)
    else:
        cb = torch.from_numpy(np.ascontiguousarray(g["codes"].transpose(0, 1, 3, 2))).to(DEV)
        lay = ops.RqLayout.from_reference(cb, cluster_key_counts=hist.reshape(bs, H, 16, 256).contiguous())
    cnt = ops.get_cache_cnt_fused(qb, lay, N, g["targets"])
    torch.cuda.synchronize()
    assert np.array_equal(cnt.cpu().numpy(), g["cnt"].reshape(R, N))


def _check_selection(idx, cnt, C):
    """Top-C by count, ties to the lowest index, ascending order."""
    R = cnt.shape[0]
    ref = O.topk_i32(cnt, C)
    assert np.array_equal(idx, ref)
    for r in range(R):
        assert np.all(np.diff(idx[r]) > 0)


@pytest.mark.parametrize("N,C,R", [(1000, 100, 3), (8192, 1, 2), (20000, 20000, 2), (65536, 4096, 4),
                                   (70001, 7001, 2)])
def test_collision_topk_vs_oracle(N, C, R):
    rng = np.random.default_rng(N + C)
    keys = O.f32_to_bf16(rng.standard_normal((R, N, 128)).astype(np.float32))
    q = O.f32_to_bf16(rng.standard_normal((R, 4, 128)).astype(np.float32))
    signs = O.f32_to_bf16(np.where(rng.random(128) < 0.5, -1.0, 1.0).astype(np.float32))
    lay = ops.RqLayout.alloc(R, N, DEV)
    ops.rq_encode(from_u16(keys).to(DEV), from_u16(signs).to(DEV), lay)
    qo = ops.rq_query(from_u16(q).to(DEV), from_u16(signs).to(DEV), 4)
    targets = ops.tier_targets(N, 0.2)
    cnt = torch.empty(R, N, dtype=torch.int32, device=DEV)
    idx = ops.collision_topk(qo["q_blocks"], lay, N, targets, C, cnt_out=cnt)
    torch.cuda.synchronize()
    table = O.collision_weights(to_u16(qo["q_blocks"]), lay.hist.cpu().numpy(), targets)
    ocnt = O.collision_count(table, lay.codes.cpu().numpy())
    assert np.array_equal(cnt.cpu().numpy(), ocnt)
    _check_selection(idx.cpu().numpy(), ocnt, C)


def test_collision_topk_heavy_ties():
    """All keys share one code -> every count equal -> lowest indices win."""
    R, N, C = 2, 30000, 777
    lay = ops.RqLayout.alloc(R, N, DEV)
    lay.codes.fill_(37)
    lay.hist[:, :, 37] = N
    qb = torch.randn(R, 128, device=DEV).to(torch.bfloat16)
    idx = ops.collision_topk(qb, lay, N, ops.tier_targets(N, 0.3), C)
    torch.cuda.synchronize()
    assert np.array_equal(idx.cpu().numpy(), np.tile(np.arange(C), (R, 1)))


def test_rerank4_matches_reference_scores():
    g = golden("rerank4.npz")
    cen = from_u16(g["centers"]).to(DEV)
    for i in range(3):
        cand = torch.from_numpy(g[f"c{i}_cand"]).to(DEV)                          # [1, H, C]
        p4 = torch.from_numpy(np.ascontiguousarray(g[f"c{i}_packed"].transpose(0, 1, 3, 2, 4))).to(DEV)
        w = from_u16(np.ascontiguousarray(g[f"c{i}_weight"].transpose(0, 1, 3, 2))).to(DEV)
        lay = ops.RqLayout.from_reference(torch.zeros(1, 2, 16, p4.shape[3], dtype=torch.uint8, device=DEV), p4, w)
        H, C = cand.shape[1], cand.shape[2]
        F = max(1, C // 4)
        sc, fin = ops.partial_rerank_cuda(cand.reshape(H, C), lay, from_u16(g[f"c{i}_q_blocks"]).to(DEV).reshape(H, 128),
                                          from_u16(g[f"c{i}_q_norm"]).to(DEV).reshape(H), cen, final_topk=F)
        torch.cuda.synchronize()
        # the production kernel's scores (bf16 fused multiply-adds), measured
        # from the reference's own build: tests/golden/ref_cuda.npz
        ref = golden("ref_cuda.npz")[f"rerank_c{i}"].reshape(H, C)
        assert np.array_equal(to_u16(sc), ref), i
        sel = O.topk_f32(O.bf16_to_f32(ref) + np.float32(0.0), F)
        assert np.array_equal(fin.cpu().numpy(), np.take_along_axis(g[f"c{i}_cand"].reshape(H, C), sel, 1)), i


@pytest.mark.parametrize("N,C,F", [(5000, 1500, 100), (8000, 5000, 300)])
def test_rerank4_token_layout_vs_oracle(N, C, F):
    """Cluster-split scoring; rank 0 selects with the small-n select up to
    4096 candidates and the general select beyond."""
    rng = np.random.default_rng(11)
    R = 3
    keys = O.f32_to_bf16((rng.standard_normal((R, N, 128)) * rng.uniform(0.2, 3, (R, N, 1))).astype(np.float32))
    signs = O.f32_to_bf16(np.where(rng.random(128) < 0.5, -1.0, 1.0).astype(np.float32))
    q = O.f32_to_bf16(rng.standard_normal((R, 4, 128)).astype(np.float32))
    codes, packed, weight, factor, hist = O.rq_encode(keys, signs)
    qb, qn, qm = O.rq_query(q, signs)
    cand = np.sort(np.stack([rng.permutation(N)[:C] for _ in range(R)]), axis=1).astype(np.int64)
    lay = ops.RqLayout.alloc(R, N, DEV)
    lay.packed.copy_(torch.from_numpy(packed.view(np.int32).reshape(R, N, 16)))
    lay.weight.copy_(from_u16(weight))
    sc, fin = ops.partial_rerank_cuda(torch.from_numpy(cand).to(DEV), lay, from_u16(qb).to(DEV), from_u16(qn).to(DEV),
                                      final_topk=F)
    torch.cuda.synchronize()
    osc = O.rerank4(cand, packed, weight, qb, qn)
    assert np.array_equal(to_u16(sc), osc)
    sel = O.topk_f32(O.bf16_to_f32(osc) + np.float32(0.0), F)
    assert np.array_equal(fin.cpu().numpy(), np.take_along_axis(cand, sel, 1))


@pytest.mark.parametrize("layout", ["token", "reference"])
def test_coarse2bit_vs_oracle(layout):
    rng = np.random.default_rng(4)
    R, N = 4, 3001
    packed = rng.integers(0, 256, (R, N, 64), dtype=np.uint8)
    qs = rng.integers(0, 256, (R, 16), dtype=np.uint8)
    qm = rng.integers(0, 256, (R, 16), dtype=np.uint8)
    if layout == "token":
        lay = ops.RqLayout.alloc(R, N, DEV)
        lay.packed.copy_(torch.from_numpy(packed.view(np.int32).reshape(R, N, 16)))
    else:
        p4 = torch.from_numpy(np.ascontiguousarray(packed.reshape(1, R, N, 16, 4).transpose(0, 1, 3, 2, 4))).to(DEV)
        lay = ops.RqLayout.from_reference(torch.zeros(1, R, 16, N, dtype=torch.uint8, device=DEV), p4)
    out = ops.coarse_2bit_score_cuda(lay, torch.from_numpy(qs).to(DEV), torch.from_numpy(qm).to(DEV), N)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), O.coarse2bit(packed, qs, qm))


@pytest.mark.parametrize("N,C,K", [(4096, None, 1024), (20000, 4096, 1024), (3000, 700, 700), (8000, 6000, 1000)])
def test_popcount_topk_vs_oracle(N, C, K):
    rng = np.random.default_rng(N + K)
    R = 3
    keys = O.f32_to_bf16((rng.standard_normal((R, N, 128)) * rng.uniform(0.2, 3, (R, N, 1))).astype(np.float32))
    signs = O.f32_to_bf16(np.where(rng.random(128) < 0.5, -1.0, 1.0).astype(np.float32))
    q = O.f32_to_bf16(rng.standard_normal((R, 4, 128)).astype(np.float32))
    codes, packed, weight, factor, hist = O.rq_encode(keys, signs)
    qb, qn, qm = O.rq_query(q, signs)
    planes, qp = O.rq_query_4bit(qb, qn)
    lay = ops.RqLayout.alloc(R, N, DEV)
    lay.codes.copy_(torch.from_numpy(codes))
    lay.factor.copy_(torch.from_numpy(factor))
    cand = None if C is None else np.sort(np.stack([rng.permutation(N)[:C] for _ in range(R)]), axis=1)
    Cn = N if C is None else C
    est = torch.empty(R, Cn, dtype=torch.float32, device=DEV)
    kd = from_u16(keys).to(DEV)
    sel, _, ip = ops.rq_popcount_topk(None if cand is None else torch.from_numpy(cand).to(DEV), lay,
                                      torch.from_numpy(planes).to(DEV), torch.from_numpy(qp).to(DEV), K, C=Cn,
                                      keys=kd, q_mean=from_u16(qm).to(DEV), est_out=est)
    torch.cuda.synchronize()
    oest, _ = O.popcount_est(cand, codes, factor, planes, qp)
    assert np.array_equal(est.cpu().numpy(), oest)
    if K < Cn:
        pos = O.topk_f32(oest + np.float32(0.0), K)
    else:
        pos = np.tile(np.arange(Cn), (R, 1))
    osel = pos if cand is None else np.take_along_axis(cand, pos, 1)
    assert np.array_equal(sel.cpu().numpy(), osel)
    assert np.array_equal(ip.cpu().numpy(), O.exact_ip(osel, keys, qm))


def test_config2_pipeline_properties():
    """Config-2 shape per row (65536 keys, 4096 candidates, 1024 kept) on 8
    rows: the selection invariants hold at full size."""
    R, N, C, K = 8, 65536, 4096, 1024
    g = torch.Generator(device=DEV).manual_seed(2)
    keys = (torch.randn(R, N, 128, generator=g, device=DEV) *
            torch.exp(torch.randn(R, N, 1, generator=g, device=DEV) * 0.5)).to(torch.bfloat16)
    q = torch.randn(R, 4, 128, generator=g, device=DEV).to(torch.bfloat16)
    signs = (torch.randint(0, 2, (128,), generator=g, device=DEV) * 2 - 1).to(torch.bfloat16)
    lay = ops.RqLayout.alloc(R, N, DEV)
    ops.rq_encode(keys, signs, lay)
    qo = ops.rq_query(q, signs, 4, planes=True)
    cnt = torch.empty(R, N, dtype=torch.int32, device=DEV)
    cand = ops.collision_topk(qo["q_blocks"], lay, N, ops.tier_targets(N, 0.2), C, cnt_out=cnt)
    sel, _, ip = ops.rq_popcount_topk(cand, lay, qo["planes"], qo["qparams"], K, keys=keys, q_mean=qo["q_mean"])
    torch.cuda.synchronize()
    cnt, cand, sel = cnt.cpu().numpy(), cand.cpu().numpy(), sel.cpu().numpy()
    assert int(lay.hist.sum()) == R * 16 * N
    for r in range(R):
        c = cnt[r]
        chosen = np.zeros(N, bool)
        chosen[cand[r]] = True
        assert chosen.sum() == C and np.all(np.diff(cand[r]) > 0)
        thr = c[chosen].min()
        assert c[~chosen].max() <= thr
        tie_in, tie_out = np.where(chosen & (c == thr))[0], np.where(~chosen & (c == thr))[0]
        assert tie_out.size == 0 or tie_in.max() < tie_out.min()
        assert np.all(np.isin(sel[r], cand[r])) and np.all(np.diff(sel[r]) > 0)
    ex = torch.einsum("rkd,rd->rk", keys.float()[torch.arange(R)[:, None], torch.from_numpy(sel).to(DEV)],
                      qo["q_mean"].float())
    assert torch.allclose(ex, ip, rtol=1e-4, atol=1e-3)
