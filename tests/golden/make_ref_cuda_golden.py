"""Golden fixtures from the reference's own CUDA kernels (run on a B200).

The modules are the reference's production kernels, built from its sources
by oracle/build_ref.py into oracle/_ref/.  This script feeds them seeded
inputs (some taken from the committed PyTorch-reference fixtures of this
directory) and writes inputs + outputs to one .npz, which is committed as
tests/golden/ref_cuda.npz.  The oracle and the library's kernels are then
checked against the production CUDA semantics, not only against the
reference's PyTorch fallbacks:

  quest      quest_chunk_score (quest_chunk_score.cu:106-154), fp32 scores
  kivi_qk    partial_chunk_kivi_qk_dense_sparse (kivi_qk_dot.cu:325-460)
  density    partial_chunk_density_scores + mask_from_topk
             (rerank_topk.cu:626-690, :956-999)
  topk       float_topk_3d (float_topk.cu:280-346): index sets
  collision  update_cache_cnt (collision.cu:446-463), int32 counts
  rerank     partial_rerank_scores (rerank.cu:230-299), bf16 scores
  coarse2bit coarse_2bit_score (coarse_2bit_score.cu:161-230), int32 scores
  hier       hierarchical Quest as _quest_pick_coarse_indices_hierarchical
             (polar_cache_kivi_quest_density_seperate_kernel.py:1852-1940)
             calls it: quest_chunk_score over the large chunks, float_topk_3d,
             quest_sub_chunk_score, float_topk_3d, quest_map_back
             (quest_chunk_score.cu:263-416) -> tests/golden/ref_cuda_hier.npz

    python tests/golden/make_ref_cuda_golden.py OUT.npz     # needs a GPU
    python tests/golden/make_ref_cuda_golden.py --hier OUT.npz
"""
from __future__ import annotations

import importlib.machinery
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle as O  # noqa: E402


def load_ref(name: str):
    path = os.path.join(ROOT, "oracle", "_ref", name, name + ".so")
    loader = importlib.machinery.ExtensionFileLoader(name, path)
    spec = importlib.util.spec_from_file_location(name, path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


def t_bf16(a: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(dev)


def u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def keys_bf16(rng, shape, outliers=4):
    k = rng.standard_normal(shape, dtype=np.float32)
    for idx in np.ndindex(*shape[:-2]):
        k[idx][:, rng.choice(shape[-1], outliers, replace=False)] *= 10.0
    return O.f32_to_bf16(k)


def gen_quest(dev, out):
    m = load_ref("ref_quest")
    rng = np.random.default_rng(101)
    bs, kv, n_max, n_c = 2, 4, 300, 290
    keys = keys_bf16(rng, (bs * kv, n_max * 16, 128))
    mn, mx, _, _ = O.kivi_encode_chunks(keys)
    mn = mn.reshape(bs, kv, n_max, 128)
    mx = mx.reshape(bs, kv, n_max, 128)
    q = O.f32_to_bf16(rng.standard_normal((bs, kv, 128), dtype=np.float32))
    valid = (rng.random((bs, kv, n_max)) > 0.05)
    for with_valid in (False, True):
        sc = torch.empty(bs, kv, n_c, dtype=torch.float32, device=dev)
        m.quest_chunk_score(t_bf16(q, dev), t_bf16(mn, dev), t_bf16(mx, dev), sc, n_c,
                            torch.from_numpy(valid).to(dev) if with_valid else None)
        torch.cuda.synchronize()
        out[f"quest_scores_v{int(with_valid)}"] = sc.cpu().numpy()
    out.update(quest_q=q, quest_min=mn, quest_max=mx, quest_valid=valid.astype(np.uint8),
               quest_n_chunks=np.int64(n_c))


def gen_kivi_qk(dev, out):
    m = load_ref("ref_kivi_qk")
    d = np.load(os.path.join(HERE, "kivi_qk.npz"))
    ids = torch.from_numpy(d["chunk_ids"]).to(dev)
    dense = torch.from_numpy(d["dense"].astype(bool)).to(dev)
    packed = torch.from_numpy(d["packed"]).to(dev)
    mn, mx, q = (t_bf16(d[k], dev) for k in ("chunk_min", "chunk_max", "raw_q"))
    bs, kv, nk = d["chunk_ids"].shape
    for dt, st in ((16, 16), (16, 8), (8, 8), (8, 4)):
        sc = torch.empty(bs, kv, nk * 16, dtype=torch.float32, device=dev)
        ix = torch.empty(bs, kv, nk * 16, dtype=torch.int64, device=dev)
        m.partial_chunk_kivi_qk_dense_sparse(ids, dense, packed, mn, mx, q, dt, st, 16, sc, ix)
        torch.cuda.synchronize()
        out[f"kivi_scores_{dt}_{st}"] = sc.cpu().numpy()
        out[f"kivi_idx_{dt}_{st}"] = ix.cpu().numpy()


def gen_density(dev, out):
    m = load_ref("ref_rerank_topk")
    d = np.load(os.path.join(HERE, "quest_density.npz"))
    ids = torch.from_numpy(d["density_ids"]).to(dev)
    cent, q = t_bf16(d["centroid"], dev), t_bf16(d["raw_q"], dev)
    dens = torch.empty(ids.shape, dtype=torch.float32, device=dev)
    m.partial_chunk_density_scores(ids, cent, q, dens)
    rng = np.random.default_rng(7)
    nk, nd = ids.shape[-1], 5
    pos = np.stack([rng.permutation(nk)[:nd] for _ in range(ids.shape[0] * ids.shape[1])]).reshape(
        ids.shape[0], ids.shape[1], nd).astype(np.int64)
    mask = torch.ones(ids.shape, dtype=torch.bool, device=dev)
    m.mask_from_topk(torch.from_numpy(pos).to(dev), mask)
    torch.cuda.synchronize()
    out.update(density=dens.cpu().numpy(), mask_pos=pos, mask=mask.cpu().numpy().astype(np.uint8))


def gen_topk(dev, out):
    m = load_ref("ref_float_topk")
    rng = np.random.default_rng(13)
    bs, kv, L, k = 2, 4, 2040, 128
    s = rng.standard_normal((bs, kv, L)).astype(np.float32)
    s[0] = np.round(s[0] * 4) / 4          # heavy ties
    s[1, :, ::7] = -np.inf
    idx = m.float_topk_3d(torch.from_numpy(s).to(dev), k)
    torch.cuda.synchronize()
    out.update(topk_scores=s, topk_k=np.int64(k), topk_idx=idx.cpu().numpy().astype(np.int64))


def gen_collision(dev, out):
    m = load_ref("ref_collision")
    d = np.load(os.path.join(HERE, "collision_ref.npz"))
    sorted_ids = torch.from_numpy(d["sorted_ids"].astype(np.int64)).to(dev)
    hist = torch.from_numpy(d["hist"].astype(np.int32)).to(dev)
    codes = torch.from_numpy(d["codes"]).to(dev)
    bs, kv, _, L = d["codes"].shape
    cnt = torch.zeros(bs, kv, L, dtype=torch.int32, device=dev)
    m.update_cache_cnt(sorted_ids, hist, codes, [int(x) for x in d["targets"]], cnt)
    torch.cuda.synchronize()
    out["collision_cnt"] = cnt.cpu().numpy()


def gen_rerank(dev, out):
    m = load_ref("ref_rerank")
    d = np.load(os.path.join(HERE, "rerank4.npz"))
    cen = t_bf16(d["centers"], dev)
    for c in ("c0", "c1", "c2"):
        cand = torch.from_numpy(d[f"{c}_cand"]).to(dev)
        packed = np.ascontiguousarray(d[f"{c}_packed"].transpose(0, 1, 3, 2, 4))  # [bs,kv,B,L,4]
        weight = np.ascontiguousarray(d[f"{c}_weight"].transpose(0, 1, 3, 2))     # [bs,kv,B,L]
        sc = torch.empty(cand.shape, dtype=torch.bfloat16, device=dev)
        m.partial_rerank_scores(cand, torch.from_numpy(packed).to(dev), t_bf16(weight, dev),
                                t_bf16(d[f"{c}_q_blocks"], dev), t_bf16(d[f"{c}_q_norm"], dev), cen, 16, 8, sc)
        torch.cuda.synchronize()
        out[f"rerank_{c}"] = u16(sc)


def gen_coarse2bit(dev, out):
    m = load_ref("ref_coarse2bit")
    rng = np.random.default_rng(29)
    bs, kv, B, L = 2, 2, 16, 1024
    packed = rng.integers(0, 256, (bs, kv, B, L, 4), dtype=np.uint8)
    qs = rng.integers(0, 256, (bs, kv, B), dtype=np.uint8)
    qm = rng.integers(0, 256, (bs, kv, B), dtype=np.uint8)
    sc = torch.empty(bs, kv, L, dtype=torch.int32, device=dev)
    m.coarse_2bit_score(torch.from_numpy(packed).to(dev), torch.from_numpy(qs).to(dev),
                        torch.from_numpy(qm).to(dev), B, 8, sc)
    torch.cuda.synchronize()
    out.update(c2_packed=packed, c2_qs=qs, c2_qm=qm, c2_scores=sc.cpu().numpy())


def gen_hier(dev, out):
    mq = load_ref("ref_quest")
    mt = load_ref("ref_float_topk")
    rng = np.random.default_rng(211)
    bs, kv, n_max, n_c, factor = 2, 4, 2048, 2040, 16
    keys = keys_bf16(rng, (bs * kv, n_max * 16, 128))
    mn, mx, _, _ = O.kivi_encode_chunks(keys)
    mn = mn.reshape(bs * kv, n_max, 128)
    mx = mx.reshape(bs * kv, n_max, 128)
    nml = n_max // factor
    lmn, lmx, lv = O.large_minmax(mn, mx, n_c, factor, nml)
    lv[1, 5] = 0
    n_large, nk_large, nk_small = O.hier_plan(n_c, factor)
    q = O.f32_to_bf16(rng.standard_normal((bs, kv, 128), dtype=np.float32))
    shp = (bs, kv)
    ls = torch.empty(bs, kv, n_large, dtype=torch.float32, device=dev)
    mq.quest_chunk_score(t_bf16(q, dev), t_bf16(lmn.reshape(shp + (nml, 128)), dev),
                         t_bf16(lmx.reshape(shp + (nml, 128)), dev), ls, n_large,
                         torch.from_numpy(lv.reshape(shp + (nml,)).astype(bool)).to(dev))
    li = mt.float_topk_3d(ls, nk_large).clamp(min=0, max=n_large - 1).contiguous()
    sub = torch.empty(bs, kv, nk_large * factor, dtype=torch.float32, device=dev)
    mq.quest_sub_chunk_score(t_bf16(q, dev), t_bf16(mn.reshape(shp + (n_max, 128)), dev),
                             t_bf16(mx.reshape(shp + (n_max, 128)), dev), li, sub, nk_large, factor)
    pos = mt.float_topk_3d(sub, nk_small).contiguous()
    idx = torch.empty(bs, kv, nk_small, dtype=torch.int64, device=dev)
    mq.quest_map_back(li, pos, idx, factor, n_c)
    torch.cuda.synchronize()
    out.update(hier_q=q, hier_min=mn.reshape(shp + (n_max, 128)), hier_max=mx.reshape(shp + (n_max, 128)),
               hier_lmin=lmn.reshape(shp + (nml, 128)), hier_lmax=lmx.reshape(shp + (nml, 128)),
               hier_lvalid=lv.reshape(shp + (nml,)), hier_n_c=np.int64(n_c), hier_factor=np.int64(factor),
               hier_nk_large=np.int64(nk_large), hier_nk_small=np.int64(nk_small),
               hier_large_scores=ls.cpu().numpy(), hier_large_idx=li.cpu().numpy(), hier_sub_scores=sub.cpu().numpy(),
               hier_sub_pos=pos.cpu().numpy(), hier_chunk_idx=idx.cpu().numpy())


def main(path, gens=None):
    dev = torch.device("cuda", 0)
    out = {}
    for fn in gens or (gen_quest, gen_kivi_qk, gen_density, gen_topk, gen_collision, gen_rerank, gen_coarse2bit):
        fn(dev, out)
        print(fn.__name__, "ok", flush=True)
    np.savez_compressed(path, **out)
    print("wrote", path, sorted(out))


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "--hier":
        main(sys.argv[2] if len(sys.argv) > 2 else os.path.join(HERE, "ref_cuda_hier.npz"), [gen_hier])
    else:
        main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "ref_cuda.npz"))
