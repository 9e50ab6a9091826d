"""Attention oracles (test infrastructure only).

attention_np   -- numpy float64 restatement of what kernels/fa2.py:23-162
                  computes: per (row, query head) softmax(q.K^T/sqrt(d)).V over
                  the first kv_lens[b] keys of the row's KV head (GQA:
                  head // group, fa2.py:53), bottom-right causal when asked
                  (query i sits at key i + kv_len - T, fa2.py:110-111).
sdpa_reference -- the reference's own CPU path: fp32 SDPA over K/V expanded
                  with repeat_kv (model.py:70-75, :104-107) under an explicit
                  boolean mask; used as the timed CPU baseline.
bottom_right_mask -- model.py:191-195.
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F


def attention_np(q: np.ndarray, k: np.ndarray, v: np.ndarray, kv_lens, causal: bool) -> np.ndarray:
    """q [B,Hq,T,D], k/v [B,Hkv,S,D] (any float dtype) -> float64 [B,Hq,T,D].
    Rows with no visible key give NaN (0/0), like the reference kernel."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    B, Hq, T, D = q.shape
    Hkv = k.shape[1]
    group = Hq // Hkv
    out = np.zeros((B, Hq, T, D))
    scale = 1.0 / math.sqrt(D)
    for b in range(B):
        n = int(kv_lens[b])
        for h in range(Hq):
            kk, vv = k[b, h // group, :n], v[b, h // group, :n]
            s = q[b, h] @ kk.T * scale  # [T, n]
            if causal:
                qi = np.arange(T)[:, None] + (n - T)
                s = np.where(np.arange(n)[None, :] <= qi, s, -np.inf)
            with np.errstate(invalid="ignore", divide="ignore"):
                m = s.max(axis=1, keepdims=True) if n else np.full((T, 1), -np.inf)
                p = np.exp(s - m)
                out[b, h] = (p @ vv) / p.sum(axis=1, keepdims=True)
    return out


def repeat_kv(x: torch.Tensor, n_rep: int) -> torch.Tensor:
    """model.py:70-75"""
    if n_rep == 1:
        return x
    b, h, s, d = x.shape
    return x[:, :, None, :, :].expand(b, h, n_rep, s, d).reshape(b, h * n_rep, s, d)


def bottom_right_mask(starts, T, S=None) -> torch.Tensor:
    """model.py:191-195: key j visible to query t of row b iff j <= starts[b] + t."""
    S = S if S is not None else max(starts) + T
    key_pos = torch.arange(S)
    query_pos = torch.as_tensor(starts)[:, None] + torch.arange(T)[None, :]
    return (key_pos[None, None, :] <= query_pos[:, :, None]).unsqueeze(1)


def sdpa_reference(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask) -> torch.Tensor:
    """fp32 SDPA over GQA-expanded K/V (model.py:104-107)."""
    n_rep = q.shape[1] // k.shape[1]
    return F.scaled_dot_product_attention(q.float(), repeat_kv(k.float(), n_rep),
                                          repeat_kv(v.float(), n_rep), attn_mask=mask)
