"""The lossy 4-bit page mode (`page4`) against the raw-row page mode.

Both modes select the same Quest top-nk pages of the same cache; `page`
attends the selected pages' raw bf16 rows (the reference's page mode,
within 2e-2 / 1e-2 of an fp64 softmax, tests/test_gpu_raw.py), `page4` reads
them as 4-bit KIVI keys and 4-bit values (group 32).  The difference between
the two is the error the 4-bit pages add; it is reported, and it is outside
the north-star tolerance by design, which is why `page4` is never the
default.  Inputs follow the benchmark configs: keys N(0,1) with 4 outlier
channels x10, values N(0,1)."""
import numpy as np
import pytest
import torch

from zoomkv_revision_b200 import polar_cache as P
from zoomkv_revision_b200 import workload as W

pytestmark = pytest.mark.gpu
DEV = "cuda"


def build(monkeypatch, mode, bs, H, ctx, budget, seed):
    env = {"ZKV_ATTENTION_MODE": mode, "POLAR_QUEST_CHUNK": "16", "POLAR_FORCE_CAND_TOKENS": str(budget),
           "POLAR_CDS_DENSE_TOPK": "16", "POLAR_CDS_SPARSE_TOPK": "16", "ZKV_HOST_RETRIEVAL": "0"}
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    c = P.polar_cache(valid_start=[0] * bs, layer_num=1, batch_size=bs, max_length=ctx + 16, num_key_value_heads=H,
                      num_heads=4 * H, head_dim=128, dtype=torch.bfloat16, layer_mapping={"0": DEV},
                      max_new_length=16, sink_size=0, local_size=128, final_topk=budget, dynamic_update_interval=128,
                      full_attention_threshold=0, enable_offload=True)
    g = torch.Generator(device=DEV).manual_seed(seed)
    kk = torch.randn(bs, ctx, H, 128, generator=g, device=DEV)
    kk[..., :4] *= 10.0
    vv = torch.randn(bs, ctx, H, 128, generator=g, device=DEV)
    c.prefill_update_kv_cache(None, kk.to(torch.bfloat16), vv.to(torch.bfloat16), 0, 0)
    return c


@pytest.mark.parametrize("name,bs,H,ctx,budget", [("config0", 1, 8, 4096, 1024), ("config1-layer", 8, 8, 32768, 2048)])
def test_page4_error_against_raw_pages(monkeypatch, capsys, name, bs, H, ctx, budget):
    raw = build(monkeypatch, "page", bs, H, ctx, budget, 3)
    p4 = build(monkeypatch, "page4", bs, H, ctx, budget, 3)
    assert raw.sched.plan == p4.sched.plan
    q = W.synth_query(torch.Generator(device=DEV).manual_seed(9), bs, 4 * H, DEV)
    a = raw.compute(q, 0).float()
    b = p4.compute(q, 0).float()
    torch.cuda.synchronize()
    err = (b - a).abs()
    mean_rel = err.mean().item() / max(a.abs().mean().item(), 1e-12)
    with capsys.disabled():
        print(f"\n{name}: page4 (4-bit K and V pages) vs raw-row pages, {raw.sched.plan[1]} of "
              f"{raw.sched.plan[0]} pages: max-abs {err.max().item():.3e}, mean-rel {mean_rel:.3e}")
    assert np.isfinite(err.max().item())
