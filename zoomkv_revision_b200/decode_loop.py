"""Decode-loop caller of the sparse attention path (the benchmark's config 4).

The reference's loop is a Qwen3 decoder whose attention is the polar_cache
plugin: model_hub/LLM.py:208-294 (layer_decode, prefill/decode_forward),
:398-446 (inference_cot), :63-110 (sample_next_token) and model_hub/qwen.py:
429-612 (embedding, fused QKV with per-head q/k RMSNorm, neox RoPE, o_proj,
SwiGLU MLP, LM head).  This module is that caller around this package's
drop-in cache:

  * weights of the Qwen3-8B shape are random-initialised (no checkpoint is
    available), bf16; projections are library GEMMs (torch / cuBLAS);
  * per layer and step: RMSNorm -> QKV -> q/k RMSNorm -> RoPE ->
    cache.decode_update_kv_cache(k, v, layer) -> cache.compute(q, layer) ->
    o_proj + residual -> RMSNorm -> MLP + residual, as layer_decode does;
  * the dense segments between two attention calls (o_proj, MLP, the next
    layer's norm, QKV and RoPE) are replayed as one CUDA graph per layer, the
    RoPE position read from a device counter, so a step issues 36 graph
    launches plus the attention calls, whose arguments change every step;
  * sampling: temperature, top-k, top-p (nucleus), as sample_next_token,
    with a seeded generator.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn.functional as F

from . import ops


@dataclass
class Shape:
    hidden: int = 4096
    layers: int = 36
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 12288
    vocab: int = 151936
    rms_eps: float = 1e-6
    rope_theta: float = 1_000_000.0


QWEN3_8B = Shape()


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm in fp32, result in x's dtype (as flashinfer.rmsnorm)."""
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


def rope_tables(shape: Shape, max_pos: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """cos / sin [max_pos, head_dim/2] of the neox rotation (qwen.py:131-140)."""
    half = shape.head_dim // 2
    inv = 1.0 / (shape.rope_theta ** (torch.arange(0, half, device=device, dtype=torch.float32) / half))
    t = torch.arange(max_pos, device=device, dtype=torch.float32)
    f = torch.outer(t, inv)
    return f.cos(), f.sin()


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [..., seq, heads, head_dim]; cos/sin [seq, head_dim/2]: rotate_half
    form (qwen.py:579-592), computed in fp32."""
    half = x.shape[-1] // 2
    xf = x.float()
    x1, x2 = xf[..., :half], xf[..., half:]
    c = cos[:, None, :]
    s = sin[:, None, :]
    return torch.cat((x1 * c - x2 * s, x2 * c + x1 * s), dim=-1).to(x.dtype)


def sample_next_token(logits: torch.Tensor, temperature: float, top_p: float, top_k: int,
                      generator: Optional[torch.Generator] = None) -> torch.Tensor:
    """LLM.py:63-110: greedy below temperature 1e-5, else temperature, top-k
    mask, nucleus mask (tokens whose preceding cumulative probability already
    exceeds top_p are removed; the first is always kept), multinomial over
    the survivors."""
    if logits.dim() == 3:
        logits = logits.squeeze(1)
    if temperature < 1e-5:
        return logits.argmax(dim=-1)
    logits = logits / temperature
    if top_k > 0:
        # the top-k survivors, sorted; the nucleus mask over them equals the
        # mask over the whole row (masked tokens have probability 0), apart
        # from exact ties at the k-th logit
        vals, idx = torch.topk(logits, min(top_k, logits.size(-1)), dim=-1)
    else:
        vals, idx = torch.sort(logits, descending=True, dim=-1)
    if 0.0 < top_p < 1.0:
        cum = torch.cumsum(F.softmax(vals, dim=-1), dim=-1)
        remove = cum > top_p
        remove[..., 1:] = remove[..., :-1].clone()
        remove[..., 0] = False
        vals = vals.masked_fill(remove, float("-inf"))
    pick = torch.multinomial(F.softmax(vals, dim=-1), 1, generator=generator)
    return idx.gather(-1, pick).squeeze(-1)


class Weights:
    """Random-initialised Qwen3 weights (N(0, std), norms at 1), bf16."""

    def __init__(self, shape: Shape, device, seed: int = 0, std: float = 0.02):
        g = torch.Generator(device=device).manual_seed(seed)
        bf = torch.bfloat16
        H, D, KV = shape.hidden, shape.head_dim, shape.kv_heads

        def w(*s):
            return (torch.randn(*s, generator=g, device=device, dtype=torch.float32) * std).to(bf)

        self.embed = w(shape.vocab, H)
        self.lm_head = w(shape.vocab, H)
        self.norm = torch.ones(H, device=device, dtype=bf)
        self.layers = []
        for _ in range(shape.layers):
            self.layers.append(dict(
                in_norm=torch.ones(H, device=device, dtype=bf),
                post_norm=torch.ones(H, device=device, dtype=bf),
                q_norm=torch.ones(D, device=device, dtype=bf),
                k_norm=torch.ones(D, device=device, dtype=bf),
                wqkv=w((shape.heads + 2 * KV) * D, H),
                wo=w(H, shape.heads * D),
                gate_up=w(2 * shape.ffn, H),
                down=w(H, shape.ffn),
            ))


class DecodeLoop:
    """A Qwen3-shape decoder over `cache` (the polar_cache drop-in, built
    with the same layer count, batch and heads).  prefill(prompt) then
    step() per generated token; `use_graphs` replays the dense segments as
    CUDA graphs."""

    def __init__(self, shape: Shape, weights: Weights, cache, batch: int, max_pos: int, device,
                 use_graphs: bool = True, temperature: float = 0.6, top_p: float = 0.95, top_k: int = 20,
                 seed: int = 42):
        self.s, self.w, self.cache, self.B = shape, weights, cache, batch
        self.dev = torch.device(device)
        self.cos, self.sin = rope_tables(shape, max_pos, self.dev)
        self.temperature, self.top_p, self.top_k = temperature, top_p, top_k
        self.gen = torch.Generator(device=self.dev).manual_seed(seed)
        self.use_graphs = use_graphs
        bf = torch.bfloat16
        H, D = shape.hidden, shape.head_dim
        # static buffers of the decode step
        self.pos = torch.zeros(1, dtype=torch.long, device=self.dev)        # RoPE position of the new token
        self.hidden = torch.zeros(batch, 1, H, dtype=bf, device=self.dev)   # residual stream
        self.q = torch.zeros(batch, 1, shape.heads, D, dtype=bf, device=self.dev)
        self.k = torch.zeros(batch, 1, shape.kv_heads, D, dtype=bf, device=self.dev)
        self.v = torch.zeros_like(self.k)
        self.attn = torch.zeros(batch, 1, shape.heads, D, dtype=bf, device=self.dev)
        self.logits = torch.zeros(batch, shape.vocab, dtype=torch.float32, device=self.dev)
        self.h = torch.zeros(batch, H, dtype=bf, device=self.dev)                  # normed activations
        self.qkv = torch.zeros(batch, (shape.heads + 2 * shape.kv_heads) * D, dtype=bf, device=self.dev)
        self.gu = torch.zeros(batch, 2 * shape.ffn, dtype=bf, device=self.dev)
        self.act = torch.zeros(batch, shape.ffn, dtype=bf, device=self.dev)
        self.lg = torch.zeros(batch, shape.vocab, dtype=bf, device=self.dev)
        self.graphs: list = []
        self.position = 0

    # ------------------------------------------------------------------ pieces
    def _qkv(self, x: torch.Tensor, L: dict, pos_cos: torch.Tensor, pos_sin: torch.Tensor):
        """x [B, T, H] -> q [B, T, heads, D], k / v [B, T, kv, D] (qwen.py:439-453, :550-612)."""
        s = self.s
        B, T, _ = x.shape
        h = rmsnorm(x, L["in_norm"], s.rms_eps)
        qkv = F.linear(h, L["wqkv"])
        q, k, v = qkv.split([s.heads * s.head_dim, s.kv_heads * s.head_dim, s.kv_heads * s.head_dim], dim=-1)
        q = rmsnorm(q.reshape(B, T, s.heads, s.head_dim), L["q_norm"], s.rms_eps)
        k = rmsnorm(k.reshape(B, T, s.kv_heads, s.head_dim), L["k_norm"], s.rms_eps)
        v = v.reshape(B, T, s.kv_heads, s.head_dim)
        return apply_rope(q, pos_cos, pos_sin), apply_rope(k, pos_cos, pos_sin), v

    def _post_attn(self, x: torch.Tensor, attn: torch.Tensor, L: dict) -> torch.Tensor:
        """o_proj + residual, RMSNorm, SwiGLU MLP + residual (LLM.py:240-249)."""
        s = self.s
        B, T = attn.shape[:2]
        x = x + F.linear(attn.reshape(B, T, s.heads * s.head_dim), L["wo"])
        h = rmsnorm(x, L["post_norm"], s.rms_eps)
        gu = F.linear(h, L["gate_up"])
        g, u = gu.split(s.ffn, dim=-1)
        return x + F.linear(F.silu(g) * u, L["down"])

    def _lm(self, x: torch.Tensor) -> torch.Tensor:
        return F.linear(rmsnorm(x, self.w.norm, self.s.rms_eps), self.w.lm_head).float()

    # ------------------------------------------------------------------ prefill
    @torch.no_grad()
    def prefill(self, prompt: torch.Tensor) -> torch.Tensor:
        """prompt [B, T] token ids -> the first generated token [B]
        (prefill_forward, LLM.py:252-276, with causal attention over the
        prompt; the K/V go to the cache by prefill_update_kv_cache)."""
        s = self.s
        B, T = prompt.shape
        x = F.embedding(prompt, self.w.embed)
        cos, sin = self.cos[:T], self.sin[:T]
        for l, L in enumerate(self.w.layers):
            q, k, v = self._qkv(x, L, cos, sin)
            self.cache.prefill_update_kv_cache(None, k, v, l, 0)
            rep = s.heads // s.kv_heads
            o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2).repeat_interleave(rep, 1),
                                               v.transpose(1, 2).repeat_interleave(rep, 1), is_causal=True)
            x = self._post_attn(x, o.transpose(1, 2), L)
        logits = self._lm(x[:, -1:])
        self.position = T
        self.pos.fill_(T)
        return sample_next_token(logits, self.temperature, self.top_p, self.top_k, self.gen)

    # ------------------------------------------------------------------ decode
    def _segment(self, l: int) -> None:
        """Dense work between attention calls: layer l-1's post-attention
        part (l > 0) and layer l's pre-attention part (l < layers); with
        l == layers the final norm and LM head.  Library GEMMs (the residual
        adds in their epilogues) and this package's fused element-wise
        kernels; every tensor is a preallocated buffer."""
        s = self.s
        x = self.hidden.view(self.B, s.hidden)
        if l > 0:
            L = self.w.layers[l - 1]
            x.addmm_(self.attn.view(self.B, s.heads * s.head_dim), L["wo"].t())
            ops.rmsnorm(x, L["post_norm"], s.rms_eps, out=self.h)
            torch.matmul(self.h, L["gate_up"].t(), out=self.gu)
            ops.silu_mul(self.gu, self.act)
            x.addmm_(self.act, L["down"].t())
        if l < s.layers:
            L = self.w.layers[l]
            ops.rmsnorm(x, L["in_norm"], s.rms_eps, out=self.h)
            torch.matmul(self.h, L["wqkv"].t(), out=self.qkv)
            ops.qk_norm_rope(self.qkv, L["q_norm"], L["k_norm"], self.cos, self.sin, self.pos, s.heads, s.kv_heads,
                             s.rms_eps, self.q, self.k, self.v)
        else:
            ops.rmsnorm(x, self.w.norm, s.rms_eps, out=self.h)
            torch.matmul(self.h, self.w.lm_head.t(), out=self.lg)
            self.logits.copy_(self.lg)

    def _build_graphs(self) -> None:
        side = torch.cuda.Stream(device=self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(side):
            for l in range(self.s.layers + 1):   # warm-up on the capture stream
                self._segment(l)
        torch.cuda.current_stream(self.dev).wait_stream(side)
        torch.cuda.synchronize(self.dev)
        pool = None
        for l in range(self.s.layers + 1):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=pool):
                self._segment(l)
            pool = g.pool()
            self.graphs.append(g)

    @torch.no_grad()
    def step(self, token: torch.Tensor) -> torch.Tensor:
        """One decode step (decode_forward, LLM.py:279-294): token [B] -> next [B]."""
        s = self.s
        if self.use_graphs and not self.graphs:
            self._build_graphs()   # its warm-up pass writes the step buffers: before the embedding
        self.hidden.copy_(F.embedding(token.view(-1, 1), self.w.embed))
        run = (lambda l: self.graphs[l].replay()) if self.use_graphs else self._segment
        for l in range(s.layers):
            run(l)
            self.cache.decode_update_kv_cache(self.k, self.v, l)
            self.attn.copy_(self.cache.compute(self.q, l))
        run(s.layers)
        self.position += 1
        self.pos.add_(1)
        return sample_next_token(self.logits, self.temperature, self.top_p, self.top_k, self.gen)


def config4_cache_kwargs(shape: Shape, batch: int, prompt: int, max_new: int, device) -> dict:
    """polar_cache keywords of the benchmark's config 4: refresh every 512
    steps, dense below 2048 tokens, the reference run's sink 64 / local 256
    (run/eval_math_aime.py:202-206)."""
    return dict(valid_start=[0] * batch, layer_num=shape.layers, batch_size=batch, max_length=prompt + max_new,
                num_key_value_heads=shape.kv_heads, num_heads=shape.heads, head_dim=shape.head_dim,
                dtype=torch.bfloat16, layer_mapping={str(l): str(device) for l in range(shape.layers)},
                max_new_length=max_new, sink_size=64, local_size=256, final_topk=100,
                dynamic_update_interval=512, full_attention_threshold=2048, enable_offload=True)
