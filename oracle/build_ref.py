"""Build the reference's own CUDA kernels for sm_100a into oracle/_ref/.

TEST INFRASTRUCTURE ONLY.  These modules are the reference's production
kernels (plain CUDA torch extensions), compiled from the reference tree where
its sources lie, with the compile flags the reference's own loaders pass
(cache_hub/quest/quest_ops.py:101-107 adds --use_fast_math for the Quest
kernel; cache_hub/rerank/rerank.py:311-316 uses -O3 -std=c++20 for the rest)
plus the sm_100a target.  They only generate golden fixtures
(tests/golden/make_ref_cuda_golden.py, run on a B200); nothing in the
package loads them, and GPU tests read the committed fixtures, not these.

    ZKV_REFERENCE_ROOT=<reference checkout> python oracle/build_ref.py

The outputs stay out of git (oracle/_ref/ is ignored) but travel with the
repository snapshot to the GPU box.
"""
from __future__ import annotations

import multiprocessing as mp
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
RUNTIME = os.path.join("runtime", "zoomkv_urania_runtime_20261011", "cache_hub")

# module name -> (source path under the runtime's cache_hub, extra nvcc flags)
MODULES = {
    "ref_quest": ("quest/quest_chunk_score.cu", ["-O3", "--use_fast_math", "-std=c++20"]),
    "ref_kivi_qk": ("kivi/kivi_qk_dot.cu", ["-O3", "-std=c++20"]),
    "ref_rerank_topk": ("rerank/rerank_topk.cu", ["-O3", "-std=c++20"]),
    "ref_float_topk": ("topk/float_topk.cu", ["-O3", "-std=c++20"]),
    "ref_collision": ("collision_fused/collision.cu", ["-O3", "-std=c++20"]),
    "ref_rerank": ("rerank/rerank.cu", ["-O3", "-std=c++20"]),
    "ref_coarse2bit": ("rerank/coarse_2bit_score.cu", ["-O3", "-std=c++20"]),
    "ref_hier_quest": ("quest/fused_hierarchical_quest.cu", ["-O3", "--use_fast_math", "-std=c++20"]),
}


def _build(args):
    name, src, flags = args
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    from torch.utils.cpp_extension import load
    bdir = os.path.join(OUT, name)
    os.makedirs(bdir, exist_ok=True)
    load(name=name, sources=[src], build_directory=bdir, extra_cuda_cflags=flags, verbose=False)
    return name


def build(root: str, names=None, jobs: int = 8) -> list[str]:
    base = os.path.join(root, RUNTIME)
    todo = []
    for name, (rel, flags) in MODULES.items():
        if names and name not in names:
            continue
        src = os.path.join(base, rel)
        if not os.path.exists(src):
            raise FileNotFoundError(src)
        todo.append((name, src, flags))
    with mp.get_context("spawn").Pool(min(jobs, len(todo))) as pool:
        return pool.map(_build, todo)


def module_path(name: str) -> str:
    return os.path.join(OUT, name, name + ".so")


if __name__ == "__main__":
    root = os.environ.get("ZKV_REFERENCE_ROOT")
    if not root or not os.path.isdir(root):
        sys.exit("set ZKV_REFERENCE_ROOT to the reference checkout")
    print(build(root, sys.argv[1:] or None))
