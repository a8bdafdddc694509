"""Golden fixture for hierarchical Quest from the reference's PyTorch path.

Run where the reference checkout is available (CPU torch is enough):

    python tests/golden/make_hier_golden.py --ref <path of the reference checkout>

The separate-kernel ZoomKV cache (runtime/zoomkv_urania_runtime_20261011/
cache_hub/polar_cache_kivi_quest_density_seperate_kernel.py) picks Quest
chunks in two levels.  This script drives its own methods on a stub object:

  * _update_large_chunk_minmax (:1762-1798), in two calls (chunks [0, 200)
    then [200, 290)) so that the touched-group logic runs;
  * _quest_pick_coarse_indices_hierarchical (:1852-1940) with the module's
    PyTorch Quest kernel (cache_hub/quest/quest_ops.py QuestPytorch:
    quest_chunk_score, quest_sub_chunk_score, quest_map_back) and torch.topk
    standing in for the CUDA float_topk_3d (the stub's _topk_3d).

Outputs: tests/golden/hier_quest.npz (inputs, large min/max/valid, the
stage-1 scores, the selected large chunks, the sub-chunk scores and the final
chunk ids).  bf16 tensors are stored as uint16 bit patterns.
"""
from __future__ import annotations

import argparse
import math
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
RUNTIME = "runtime/zoomkv_urania_runtime_20261011"
sys.path.insert(0, HERE)

from make_golden import bf16_bits, synth_keys  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True)
    ap.add_argument("--out", default=os.path.join(HERE, "hier_quest.npz"))
    a = ap.parse_args()
    sys.path.insert(0, os.path.join(a.ref, RUNTIME))
    torch.set_num_threads(1)
    import cache_hub.polar_cache_kivi_quest_density_seperate_kernel as m
    from cache_hub.quest.quest_ops import QuestPytorch

    g = torch.Generator().manual_seed(17)
    bs, kv, n_max, n_chunks, factor, dim = 2, 2, 300, 290, 16, 128
    n_max_large = (n_max + factor - 1) // factor
    keys = synth_keys(g, (bs, kv, n_max * 16, dim))
    kc = keys.view(bs, kv, n_max, 16, dim)
    mn, mx = kc.amin(3).contiguous(), kc.amax(3).contiguous()

    s = types.SimpleNamespace()
    s._hq_factor = factor
    s._chunk_n_max_large = n_max_large
    s._chunk_key_min_gpu = [mn]
    s._chunk_key_max_gpu = [mx]
    s._chunk_valid_end = [200]
    s._chunk_key_min_gpu_large = [torch.zeros(bs, kv, n_max_large, dim, dtype=torch.bfloat16)]
    s._chunk_key_max_gpu_large = [torch.zeros(bs, kv, n_max_large, dim, dtype=torch.bfloat16)]
    s._chunk_valid_mask_gpu_large = [torch.zeros(bs, kv, n_max_large, dtype=torch.bool)]
    s._chunk_valid_end_large = [0]
    upd = m.polar_cache._update_large_chunk_minmax
    upd(s, 0, 0, 200, slice(None))
    s._chunk_valid_end = [n_chunks]
    upd(s, 0, 200, n_chunks, slice(None))

    n_large = n_chunks // factor
    nk_large = min(max(1, int(math.ceil(n_large * 0.3))), n_large)
    nk_small = min(max(1, int(math.ceil(nk_large * factor * 0.3))), nk_large * factor)
    s._cached_quest_n_chunks = n_chunks
    s._cached_hq_n_large = n_large
    s._cached_hq_nk_large = nk_large
    s._cached_hq_nk_small = nk_small
    s._cached_hq_scores_large_view = torch.empty(bs, kv, n_large)
    s._cached_hq_scores_sub_view = torch.empty(bs, kv, nk_large * factor)
    s._cached_hq_large_min_views = [s._chunk_key_min_gpu_large[0]]
    s._cached_hq_large_max_views = [s._chunk_key_max_gpu_large[0]]
    s._cached_hq_large_valid_views = [s._chunk_valid_mask_gpu_large[0]]
    s._cached_chunk_min_views = [mn]
    s._cached_chunk_max_views = [mx]
    s._cached_hq_chunk_idx = torch.empty(bs, kv, nk_small, dtype=torch.int64)
    s._quest_kernel = QuestPytorch()
    picks = []

    def topk(scores, k):
        idx = torch.topk(scores, k, dim=-1).indices
        picks.append(idx.clone())
        return idx

    s._topk_3d = topk
    q = torch.randn(bs, kv, 4, dim, generator=g).to(torch.bfloat16)
    raw_q = q.mean(dim=2)
    chunk_idx, nk = m.polar_cache._quest_pick_coarse_indices_hierarchical(s, raw_q=raw_q, layer_idx=0)
    assert nk == nk_small
    np.savez_compressed(
        a.out, raw_q=bf16_bits(raw_q), chunk_min=bf16_bits(mn), chunk_max=bf16_bits(mx),
        n_chunks=np.int64(n_chunks), factor=np.int64(factor), nk_large=np.int64(nk_large),
        nk_small=np.int64(nk_small), large_min=bf16_bits(s._chunk_key_min_gpu_large[0]),
        large_max=bf16_bits(s._chunk_key_max_gpu_large[0]),
        large_valid=s._chunk_valid_mask_gpu_large[0].numpy().astype(np.uint8),
        large_scores=s._cached_hq_scores_large_view.numpy(), large_idx=picks[0].numpy(),
        sub_scores=s._cached_hq_scores_sub_view.numpy(), sub_pos=picks[1].numpy(),
        chunk_idx=chunk_idx.numpy())
    print("wrote", a.out, "n_large", n_large, "nk_large", nk_large, "nk_small", nk_small)


if __name__ == "__main__":
    main()
