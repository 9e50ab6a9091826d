"""Restated reference forward of Qwen2.5-1.5B (test infrastructure only).

The reference model.py:43-207 with its CPU/SDPA attention branch: per layer
q/k/v projections, RoPE with bf16/fp32 per-op rounding in the activation
dtype (model.py:58-65, :151-155), KVCache write + dense gather
(kv_cache.py:108-121), SDPA over repeat_kv'd K/V with the mask selection of
model.py:181-195, o_proj, fp32 RMSNorm, SwiGLU MLP, tied lm_head on the last
position.  Parameter names match the reference, so one state dict loads into
the reference, this oracle and the product model.  Runs on CPU or CUDA.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from oracle.attention_ref import repeat_kv

HIDDEN, LAYERS, HEADS, KV_HEADS, HEAD_DIM, INTER, VOCAB = 1536, 28, 12, 2, 128, 8960, 151936
EPS, THETA = 1e-6, 1_000_000.0


class _Norm(nn.Module):
    def __init__(self):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(HIDDEN))

    def forward(self, x):
        dt = x.dtype
        x = x.float()
        x = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + EPS)
        return self.weight * x.to(dt)


class _Attn(nn.Module):
    def __init__(self):
        super().__init__()
        self.q_proj = nn.Linear(HIDDEN, HEADS * HEAD_DIM, bias=True)
        self.k_proj = nn.Linear(HIDDEN, KV_HEADS * HEAD_DIM, bias=True)
        self.v_proj = nn.Linear(HIDDEN, KV_HEADS * HEAD_DIM, bias=True)
        self.o_proj = nn.Linear(HEADS * HEAD_DIM, HIDDEN, bias=False)


class _MLP(nn.Module):
    def __init__(self):
        super().__init__()
        self.gate_proj = nn.Linear(HIDDEN, INTER, bias=False)
        self.up_proj = nn.Linear(HIDDEN, INTER, bias=False)
        self.down_proj = nn.Linear(INTER, HIDDEN, bias=False)


class _Block(nn.Module):
    def __init__(self):
        super().__init__()
        self.input_layernorm = _Norm()
        self.self_attn = _Attn()
        self.post_attention_layernorm = _Norm()
        self.mlp = _MLP()


def _rot(x):
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat((-x2, x1), dim=-1)


class RefQwen2(nn.Module):
    def __init__(self):
        super().__init__()
        self.embed_tokens = nn.Embedding(VOCAB, HIDDEN)
        self.layers = nn.ModuleList(_Block() for _ in range(LAYERS))
        self.norm = _Norm()
        self.register_buffer("inv_freq", 1.0 / (THETA ** (torch.arange(0, HEAD_DIM, 2).float() / HEAD_DIM)),
                             persistent=False)

    @torch.no_grad()
    def forward(self, input_ids, cache, seqs):
        """cache: oracle.kvcache_ref.RefKVCache whose pool lives on input_ids.device."""
        B, T = input_ids.shape
        dev = input_ids.device
        x = self.embed_tokens(input_ids)
        starts, slot, gather = cache.prepare(seqs, T)
        st = torch.tensor(starts, device=dev)
        pos = st[:, None] + torch.arange(T, device=dev)[None, :]
        freqs = pos.float()[..., None] * self.inv_freq[None, None, :]
        emb = torch.cat((freqs, freqs), dim=-1)
        cos, sin = emb.cos()[:, None].to(x.dtype), emb.sin()[:, None].to(x.dtype)
        same = all(s == starts[0] for s in starts)
        if same and (T == 1 or starts[0] == 0):
            mask, causal = None, starts[0] == 0
        else:
            S = max(starts) + T
            kp = torch.arange(S, device=dev)
            mask = (kp[None, None, :] <= pos[:, :, None]).unsqueeze(1)
            causal = False
        slot_t = torch.tensor(slot, dtype=torch.long, device=dev)
        gather_t = torch.tensor(gather, dtype=torch.long, device=dev)
        for li, blk in enumerate(self.layers):
            a = blk.self_attn
            h = blk.input_layernorm(x)
            q = a.q_proj(h).view(B, T, HEADS, HEAD_DIM).transpose(1, 2)
            k = a.k_proj(h).view(B, T, KV_HEADS, HEAD_DIM).transpose(1, 2)
            v = a.v_proj(h).view(B, T, KV_HEADS, HEAD_DIM).transpose(1, 2)
            q = (q * cos) + (_rot(q) * sin)
            k = (k * cos) + (_rot(k) * sin)
            if getattr(cache, "fp8", False):  # the FP8 pool's e4m3 round trip (not the reference's)
                from oracle.kvcache_ref import fp8_round_trip

                k, v = fp8_round_trip(k).to(k.dtype), fp8_round_trip(v).to(v.dtype)
            cache.buf[li, 0].index_copy_(0, slot_t, k.transpose(1, 2).reshape(B * T, KV_HEADS, HEAD_DIM))
            cache.buf[li, 1].index_copy_(0, slot_t, v.transpose(1, 2).reshape(B * T, KV_HEADS, HEAD_DIM))
            kd = cache.buf[li, 0][gather_t].transpose(1, 2)
            vd = cache.buf[li, 1][gather_t].transpose(1, 2)
            if mask is None:
                o = F.scaled_dot_product_attention(q, repeat_kv(kd, HEADS // KV_HEADS),
                                                   repeat_kv(vd, HEADS // KV_HEADS), is_causal=causal)
            else:
                o = F.scaled_dot_product_attention(q, repeat_kv(kd, HEADS // KV_HEADS),
                                                   repeat_kv(vd, HEADS // KV_HEADS), attn_mask=mask)
            x = x + a.o_proj(o.transpose(1, 2).reshape(B, T, HEADS * HEAD_DIM))
            hm = blk.post_attention_layernorm(x)
            x = x + blk.mlp.down_proj(F.silu(blk.mlp.gate_proj(hm)) * blk.mlp.up_proj(hm))
        cache.advance(seqs, T)
        x = self.norm(x[:, -1:])
        return x @ self.embed_tokens.weight.T
