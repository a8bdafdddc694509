"""The decode-loop caller (zoomkv_revision_b200/decode_loop.py) on a small
Qwen3-shaped model: CUDA-graph replay equals the eager loop bit for bit, and
the loop's logits follow a plain PyTorch forward that attends every stored
token with SDPA (teacher-forced on the loop's own tokens), so the cache
wiring (RoPE positions, K/V append, GQA) is checked end to end."""
import pytest
import torch
import torch.nn.functional as F

from zoomkv_revision_b200 import decode_loop as DL
from zoomkv_revision_b200 import polar_cache as P

pytestmark = pytest.mark.gpu
DEV = "cuda"
SMALL = DL.Shape(hidden=256, layers=2, heads=2, kv_heads=1, head_dim=128, ffn=512, vocab=1000)


def make_cache(monkeypatch, mode, B, prompt, max_new, threshold):
    env = {"ZKV_ATTENTION_MODE": mode, "POLAR_QUEST_CHUNK": "16", "POLAR_FORCE_CAND_TOKENS": "64",
           "POLAR_CDS_DENSE_TOPK": "16", "POLAR_CDS_SPARSE_TOPK": "16", "ZKV_HOST_RETRIEVAL": "0"}
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    s = SMALL
    return P.polar_cache(valid_start=[0] * B, layer_num=s.layers, batch_size=B, max_length=prompt + max_new,
                         num_key_value_heads=s.kv_heads, num_heads=s.heads, head_dim=s.head_dim,
                         dtype=torch.bfloat16, layer_mapping={str(l): DEV for l in range(s.layers)},
                         max_new_length=max_new, sink_size=4, local_size=16, final_topk=64,
                         dynamic_update_interval=16, full_attention_threshold=threshold, enable_offload=True)


def run(monkeypatch, mode, graphs, steps, B=2, prompt=48, threshold=0, temperature=0.6, seed=42):
    w = DL.Weights(SMALL, DEV, seed=1, std=0.05)
    cache = make_cache(monkeypatch, mode, B, prompt, steps + 16, threshold)
    loop = DL.DecodeLoop(SMALL, w, cache, B, prompt + steps + 16, DEV, use_graphs=graphs, temperature=temperature,
                         seed=seed)
    ids = torch.randint(0, SMALL.vocab, (B, prompt), generator=torch.Generator().manual_seed(7)).to(DEV)
    tok = loop.prefill(ids)
    toks, logits = [tok], []
    for _ in range(steps):
        tok = loop.step(tok)
        toks.append(tok)
        logits.append(loop.logits.clone())
    torch.cuda.synchronize()
    return ids, torch.stack(toks, 1), logits, loop


@pytest.mark.parametrize("mode", ["page", "reference"])
def test_graphs_equal_eager(monkeypatch, mode):
    _, t1, l1, _ = run(monkeypatch, mode, True, 40)
    _, t2, l2, _ = run(monkeypatch, mode, False, 40)
    assert torch.equal(t1, t2)
    for a, b in zip(l1, l2):
        assert torch.equal(a, b)


def test_loop_follows_dense_pytorch_forward(monkeypatch):
    """Full attention everywhere (threshold above the context): the loop's
    logits against a PyTorch forward over every stored token."""
    steps = 24
    ids, toks, logits, loop = run(monkeypatch, "page", False, steps, threshold=10 ** 6, temperature=0.0)
    s, w = SMALL, loop.w
    seq = torch.cat([ids, toks[:, :steps]], 1)             # the tokens the loop consumed
    B, T = seq.shape
    x = F.embedding(seq, w.embed)
    cos, sin = loop.cos[:T], loop.sin[:T]
    for L in w.layers:
        q, k, v = loop._qkv(x, L, cos, sin)
        o = F.scaled_dot_product_attention(q.transpose(1, 2).float(), k.transpose(1, 2).float(),
                                           v.transpose(1, 2).float(), is_causal=True,
                                           enable_gqa=True).to(torch.bfloat16)
        x = loop._post_attn(x, o.transpose(1, 2), L)
    ref = loop._lm(x)                                       # [B, T, vocab]
    for i in range(steps):
        got, want = logits[i], ref[:, ids.shape[1] + i]
        scale = want.abs().max().item()
        assert (got - want).abs().max().item() <= 0.05 * scale, i


def test_fused_elementwise_kernels_match_torch():
    """zkv_rmsnorm, zkv_qk_norm_rope and zkv_silu_mul against the PyTorch
    forms used in prefill (one bf16 rounding apart at most)."""
    from zoomkv_revision_b200 import ops
    g = torch.Generator(device=DEV).manual_seed(0)
    B, s = 5, DL.Shape(hidden=512, heads=4, kv_heads=2, ffn=384)
    x = torch.randn(B, s.hidden, generator=g, device=DEV).to(torch.bfloat16)
    wn = (1 + 0.1 * torch.randn(s.hidden, generator=g, device=DEV)).to(torch.bfloat16)
    got = ops.rmsnorm(x, wn, 1e-6)
    want = DL.rmsnorm(x, wn, 1e-6)
    assert ((got.float() - want.float()).abs() <= 2 ** -7 * want.float().abs() + 1e-3).all()
    D = 128
    qkv = torch.randn(B, (s.heads + 2 * s.kv_heads) * D, generator=g, device=DEV).to(torch.bfloat16)
    qw = (1 + 0.1 * torch.randn(D, generator=g, device=DEV)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(D, generator=g, device=DEV)).to(torch.bfloat16)
    cos, sin = DL.rope_tables(s, 64, DEV)
    pos = torch.tensor([37], device=DEV)
    q = torch.empty(B, s.heads, D, dtype=torch.bfloat16, device=DEV)
    k = torch.empty(B, s.kv_heads, D, dtype=torch.bfloat16, device=DEV)
    v = torch.empty_like(k)
    ops.qk_norm_rope(qkv, qw, kw, cos, sin, pos, s.heads, s.kv_heads, 1e-6, q, k, v)
    qq, kk, vv = qkv.split([s.heads * D, s.kv_heads * D, s.kv_heads * D], -1)
    rq = DL.apply_rope(DL.rmsnorm(qq.reshape(B, 1, s.heads, D), qw, 1e-6), cos[37:38], sin[37:38])[:, 0]
    rk = DL.apply_rope(DL.rmsnorm(kk.reshape(B, 1, s.kv_heads, D), kw, 1e-6), cos[37:38], sin[37:38])[:, 0]
    assert (q.float() - rq.float()).abs().max().item() <= 2 ** -6 * rq.float().abs().max().item()
    assert (k.float() - rk.float()).abs().max().item() <= 2 ** -6 * rk.float().abs().max().item()
    assert torch.equal(v, vv.reshape(B, s.kv_heads, D))
    gu = torch.randn(B, 2 * s.ffn, generator=g, device=DEV).to(torch.bfloat16)
    out = torch.empty(B, s.ffn, dtype=torch.bfloat16, device=DEV)
    ops.silu_mul(gu, out)
    ref = (F.silu(gu[:, :s.ffn].float()) * gu[:, s.ffn:].float())
    assert ((out.float() - ref).abs() <= 2 ** -7 * ref.abs() + 1e-3).all()
