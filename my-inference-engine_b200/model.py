"""Qwen2.5-1.5B with its attention call sites moved onto the paged-KV kernels
(drop-in for the reference's model.py:1-207).

Unchanged from the reference (consumed as-is, cuBLAS/torch): embeddings,
RMSNorm in fp32 (model.py:43-55), q/k/v/o projections with bias
(model.py:81-84), SwiGLU MLP (model.py:112-120), residual blocks
(model.py:123-138), last-position logits through the tied embedding
(model.py:204-206).

Changed (the hot path):
  * RoPE cos/sin come from a table built once, on the CPU, with exactly the
    reference's fp32 formula (model.py:148-155) and rounded to the
    activation dtype; the fused append kernel indexes it by position.
  * apply_rope + cache.write + cache.read + FA2 (model.py:92-103) become
    cache.append (RoPE on q and k, K/V into their blocks) and one paged
    attention launch that reads the blocks in place (kernels/fa2.py).
  * No mask or SDPA branch: there is no CPU fallback (model.py:102-107).
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

# Qwen2.5-1.5B architecture constants (model.py:18-27)
HIDDEN_SIZE = 1536
NUM_LAYERS = 28
NUM_HEADS = 12
NUM_KV_HEADS = 2
N_REP = NUM_HEADS // NUM_KV_HEADS
HEAD_DIM = HIDDEN_SIZE // NUM_HEADS
INTERMEDIATE_SIZE = 8960
VOCAB_SIZE = 151936
RMS_NORM_EPS = 1e-6
ROPE_THETA = 1_000_000.0


class RMSNorm(torch.nn.Module):
    def __init__(self, dim, eps):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x):
        input_dtype = x.dtype
        x = x.to(torch.float32)
        variance = x.pow(2).mean(-1, keepdim=True)
        x = x * torch.rsqrt(variance + self.eps)
        return self.weight * x.to(input_dtype)


def rotate_half(x):
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat((-x2, x1), dim=-1)


def apply_rope(q, k, cos, sin):
    """Unfused RoPE with the reference's op sequence (model.py:62-65); the
    engine uses the fused append kernel instead."""
    q = (q * cos) + (rotate_half(q) * sin)
    k = (k * cos) + (rotate_half(k) * sin)
    return q, k


def repeat_kv(x):
    if N_REP == 1:
        return x
    b, h, s, d = x.shape
    return x[:, :, None, :, :].expand(b, h, N_REP, s, d).reshape(b, h * N_REP, s, d)


def rope_table(num_positions, dtype, device):
    """cos/sin [num_positions, HEAD_DIM] for positions 0..num_positions-1,
    computed on the CPU exactly as rope_cos_sin (model.py:148-155) does:
    fp32 inv_freq, fp32 position * inv_freq, cat(freqs, freqs), cos/sin in
    fp32, then a cast to the activation dtype."""
    inv_freq = 1.0 / (ROPE_THETA ** (torch.arange(0, HEAD_DIM, 2).float() / HEAD_DIM))
    pos = torch.arange(num_positions, dtype=torch.int64).to(torch.float32)
    freqs = pos[:, None] * inv_freq[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype).to(device), emb.sin().to(dtype).to(device)


class QwenAttention(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.q_proj = torch.nn.Linear(HIDDEN_SIZE, NUM_HEADS * HEAD_DIM, bias=True)
        self.k_proj = torch.nn.Linear(HIDDEN_SIZE, NUM_KV_HEADS * HEAD_DIM, bias=True)
        self.v_proj = torch.nn.Linear(HIDDEN_SIZE, NUM_KV_HEADS * HEAD_DIM, bias=True)
        self.o_proj = torch.nn.Linear(NUM_HEADS * HEAD_DIM, HIDDEN_SIZE, bias=False)

    def forward(self, x, cos, sin, mask, is_causal, kv_lens, cache, layer_idx, slot_mapping, gather_idx):
        from kernels.fa2 import flash_attention

        B, T, _ = x.shape
        q = self.q_proj(x).view(B, T, NUM_HEADS, HEAD_DIM).transpose(1, 2)
        k = self.k_proj(x).view(B, T, NUM_KV_HEADS, HEAD_DIM).transpose(1, 2)
        v = self.v_proj(x).view(B, T, NUM_KV_HEADS, HEAD_DIM).transpose(1, 2)

        # RoPE on q and k + K/V into their pool blocks, one launch
        q_rot = torch.empty(B, T, NUM_HEADS, HEAD_DIM, device=x.device, dtype=x.dtype)
        cache.append(layer_idx, slot_mapping, q, k, v, cos, sin, q_rot.transpose(1, 2))
        k_blocks, v_blocks = cache.read(layer_idx, gather_idx)

        # paged attention straight from the blocks; O lands in [B, T, H, D]
        out = torch.empty(B, T, NUM_HEADS, HEAD_DIM, device=x.device, dtype=x.dtype)
        flash_attention(q_rot.transpose(1, 2), k_blocks, v_blocks, is_causal, kv_lens,
                        out=out.transpose(1, 2))
        return self.o_proj(out.view(B, T, NUM_HEADS * HEAD_DIM))


class QwenMLP(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.gate_proj = torch.nn.Linear(HIDDEN_SIZE, INTERMEDIATE_SIZE, bias=False)
        self.up_proj = torch.nn.Linear(HIDDEN_SIZE, INTERMEDIATE_SIZE, bias=False)
        self.down_proj = torch.nn.Linear(INTERMEDIATE_SIZE, HIDDEN_SIZE, bias=False)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class QwenBlock(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.input_layernorm = RMSNorm(HIDDEN_SIZE, RMS_NORM_EPS)
        self.self_attn = QwenAttention()
        self.post_attention_layernorm = RMSNorm(HIDDEN_SIZE, RMS_NORM_EPS)
        self.mlp = QwenMLP()

    def forward(self, x, cos, sin, mask, is_causal, kv_lens, cache, layer_idx, slot_mapping, gather_idx):
        attention_output = self.self_attn(
            self.input_layernorm(x), cos, sin, mask, is_causal, kv_lens,
            cache, layer_idx, slot_mapping, gather_idx,
        )
        x = x + attention_output
        x = x + self.mlp(self.post_attention_layernorm(x))
        return x


class Qwen2ForCausalLM(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.embed_tokens = torch.nn.Embedding(VOCAB_SIZE, HIDDEN_SIZE)
        self.layers = torch.nn.ModuleList(QwenBlock() for _ in range(NUM_LAYERS))
        self.norm = RMSNorm(HIDDEN_SIZE, RMS_NORM_EPS)

        inv_freq = 1.0 / (ROPE_THETA ** (torch.arange(0, HEAD_DIM, 2).float() / HEAD_DIM))
        self.register_buffer("inv_freq", inv_freq, persistent=False)
        self._rope = {}  # (device, dtype) -> (cos, sin) tables

    def rope_tables(self, num_positions, dtype, device):
        key = (str(device), dtype)
        tab = self._rope.get(key)
        if tab is None or tab[0].shape[0] < num_positions:
            n = max(num_positions, 2 * (tab[0].shape[0] if tab is not None else 0), 4096)
            tab = rope_table(n, dtype, device)
            self._rope[key] = tab
        return tab

    def forward(self, input_ids, cache, seqs):
        """input_ids: [B, T]. cache: a KVCache. seqs: that cache's sequence id for
        each batch item.  Returns logits for each row's last position: [B, 1, vocab]."""
        _, T = input_ids.shape
        x = self.embed_tokens(input_ids)

        starts_list, slot_mapping, gather_idx = cache.prepare(seqs, T)
        cos, sin = self.rope_tables(cache.table_pitch * cache.block_size, x.dtype, x.device)
        kv_lens = gather_idx.kv_lens
        is_causal = T > 1  # a single query row sees every key up to kv_lens anyway

        for layer_idx, layer in enumerate(self.layers):
            x = layer(x, cos, sin, None, is_causal, kv_lens, cache, layer_idx, slot_mapping, gather_idx)

        cache.advance(seqs, T)

        x = self.norm(x[:, -1:])
        logits = x @ self.embed_tokens.weight.T
        return logits
