"""FlashAttention2Function on the B200 paged-KV kernels (drop-in for the
reference's kernels/fa2.py:164-214).

`FlashAttention2Function.apply(Q, K, V, is_causal=False, kv_lens=None) -> O`
keeps the reference contract:
  * Q [B, Hq, T, D] bf16 CUDA, any strides; O is a new [B, Hq, T, D] tensor in
    Q's dtype (fa2.py:188).
  * kv_lens [B] int32 or None (= every row uses all of K/V, fa2.py:182-184);
    query i of row b sits at key i + kv_lens[b] - T when is_causal
    (bottom-right, fa2.py:110-111).
  * Precondition failures raise AssertionError with the reference's
    messages (fa2.py:177-185).  head_dim must be 128 here (the kernels are
    specialised for the Qwen2.5-1.5B path).
K and V may be
  * `PagedKV` handles from KVCache.read(): blocks are read in place through
    the device block table (no gather copy) -- the engine's path;
  * dense [B, Hkv, S, D] tensors, as the reference's own test passes them
    (kernels/test_fa2.py:44-52).
T == 1 runs the split-K decode kernel, T > 1 the prefill kernel.  There is no
SDPA/CPU fallback: non-CUDA inputs fail the reference's first assertion.
"""
from __future__ import annotations

import math

import torch

import pagedkv
from kv_cache import PagedKV


def flash_attention(Q, K, V, is_causal=False, kv_lens=None, out=None):
    """Forward attention; `out` (optional) receives O with any strides, e.g. a
    [B, T, Hq, D] buffer viewed as [B, Hq, T, D] so the caller's transpose is free."""
    batch_size, num_heads, seq_len, d = Q.shape
    paged = isinstance(K, PagedKV)
    seq_len_k = K.shape[2]
    d_v = V.shape[-1]
    sm_scale = 1.0 / math.sqrt(d)

    assert Q.is_cuda and K.is_cuda and V.is_cuda, "Expected CUDA tensors"
    num_kv_heads = K.shape[1]
    assert Q.shape[0] == K.shape[0] and Q.shape[-1] == K.shape[-1], "Q and K match in batch and head dim"
    assert num_heads % num_kv_heads == 0, "num_heads must be a multiple of num_kv_heads (GQA)"
    assert K.shape[:-1] == V.shape[:-1], "K and V are the same shape for all dimensions but the last"
    if kv_lens is None:
        kv_lens = K.step.kv_lens if paged else torch.full(
            (batch_size,), seq_len_k, device=Q.device, dtype=torch.int32)
    assert kv_lens.shape == (batch_size,) and kv_lens.dtype == torch.int32, "kv_lens is [batch] int32"
    assert (d & (d - 1) == 0) and (d_v & (d_v - 1) == 0), "d and d_v must be powers of 2 (Triton block_shape constraint)"
    assert d == pagedkv.HEAD_DIM and d_v == pagedkv.HEAD_DIM, "head_dim must be 128 (paged kernels)"
    assert Q.dtype == torch.bfloat16 and K.dtype == torch.bfloat16 and V.dtype == torch.bfloat16, \
        "bf16 Q/K/V expected"

    if out is None:
        out = torch.empty((batch_size, num_heads, seq_len, d_v), device=Q.device, dtype=Q.dtype)
    if batch_size == 0 or seq_len == 0:
        return out
    if paged:
        assert isinstance(V, PagedKV) and V.step is K.step, "K and V handles come from one read()"
        cache, step = K.cache, K.step
        if cache.fp8:
            if seq_len == 1:
                pagedkv.paged_decode_fp8(Q[:, :, 0], cache.pool8[K.layer_idx], cache.block_tables,
                                         step.rows, kv_lens, step.max_kv_len, out[:, :, 0],
                                         sm_scale, cache.err_flag)
            else:
                # prefill over an FP8 pool: the rows' K/V dequantised into bf16
                # planes (one block per 16 positions, identity tables), then
                # the bf16 tensor-core prefill kernel
                S = step.max_kv_len
                kd, vd = cache.dequant_step(K.layer_idx, step, S)
                S16 = kd.shape[0] // batch_size
                tables = cache.identity_tables(batch_size, S16, Q.device)
                pagedkv.paged_prefill(Q, kd, vd, tables, None, kv_lens, S, out, bool(is_causal),
                                      sm_scale, num_kv_heads, cache.err_flag, step.q_lens)
            return out
        if seq_len == 1:
            pagedkv.paged_decode(Q[:, :, 0], K.plane, V.plane, cache.block_tables, step.rows,
                                 kv_lens, step.max_kv_len, out[:, :, 0], sm_scale, num_kv_heads,
                                 cache.err_flag)
        else:
            pagedkv.paged_prefill(Q, K.plane, V.plane, cache.block_tables, step.rows, kv_lens,
                                  step.max_kv_len, out, bool(is_causal), sm_scale, num_kv_heads,
                                  cache.err_flag, step.q_lens)
        return out
    # dense K/V: TMA needs 16-byte aligned rows
    def aligned(x):
        return x.stride(-1) == 1 and all(s % 8 == 0 for s in x.stride()[:-1]) and x.data_ptr() % 16 == 0
    if not aligned(K):
        K = K.contiguous()
    if not aligned(V):
        V = V.contiguous()
    if not aligned(Q):
        Q = Q.contiguous()
    tgt = out if aligned(out) else torch.empty_like(out, memory_format=torch.contiguous_format)
    pagedkv.dense_attention(Q, K, V, kv_lens, tgt, bool(is_causal), sm_scale)
    if tgt is not out:
        out.copy_(tgt)
    return out


class FlashAttention2Function(torch.autograd.Function):
    @staticmethod
    def forward(ctx, Q, K, V, is_causal=False, kv_lens=None):
        O = flash_attention(Q, K, V, is_causal, kv_lens)
        ctx.is_causal = is_causal
        ctx.scale = 1.0 / math.sqrt(Q.shape[-1])
        return O

    @staticmethod
    def backward(ctx, *grads):
        raise NotImplementedError("forward-only kernel (the reference defines no backward either)")
