"""RoPE with the reference's bf16 rounding, restated in numpy (test oracle).

TEST INFRASTRUCTURE ONLY.  The reference applies RoPE as five torch ops on
bf16 tensors (model.py:58-65): q*cos, rotate_half(q) = cat(-x2, x1),
rotate_half(q)*sin and the sum, each computed in fp32 and rounded to bf16
(round-to-nearest-even).  cos/sin come from model.py:148-155: fp32 inv_freq
(theta 1e6), fp32 position*inv_freq, cat(freqs, freqs), cos/sin in fp32, cast
to bf16.
"""
from __future__ import annotations

import numpy as np
import torch

ROPE_THETA = 1_000_000.0
HEAD_DIM = 128


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16, nearest-even (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = (u + 0x7FFF + lsb) >> 16
    return r.astype(np.uint16)


def rne(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest bf16, returned as fp32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def rope_bits(x_bits: np.ndarray, cos_bits: np.ndarray, sin_bits: np.ndarray) -> np.ndarray:
    """x [..., 128], cos/sin broadcastable [..., 128], all bf16 bit patterns.
    Returns bf16 bits of (x*cos) + (rotate_half(x)*sin), rounded per op."""
    x = bf16_bits_to_f32(x_bits)
    c = bf16_bits_to_f32(cos_bits)
    s = bf16_bits_to_f32(sin_bits)
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    xc = rne((x * c).astype(np.float32))
    rs = rne((rot * s).astype(np.float32))
    return f32_to_bf16_bits((xc + rs).astype(np.float32))


def rope_table_bits(positions: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """bf16 bits of cos/sin [len(positions), 128] by the reference's formula
    (evaluated with torch's fp32 CPU cos/sin, as the reference CPU path does)."""
    inv_freq = 1.0 / (ROPE_THETA ** (torch.arange(0, HEAD_DIM, 2).float() / HEAD_DIM))
    freqs = torch.as_tensor(positions).to(torch.float32)[:, None] * inv_freq[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    c = emb.cos().to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16)
    s = emb.sin().to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16)
    return c, s
