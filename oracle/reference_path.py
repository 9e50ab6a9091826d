"""The reference engine's CPU decode path, restated for timing (test
infrastructure / CPU baseline only).

One decode step exactly as the reference runs it off-CUDA (chat.py:34 picks
fp32 there): KVCache.prepare once per step (kv_cache.py:74-101), then per
layer KVCache.write (index_copy_, :108-115), KVCache.read (dense gather copy,
:117-121) and fp32 SDPA over repeat_kv'd K/V with the ragged-batch mask
(model.py:104-107, :186-195).  Projections/MLP are not part of the path and
are not timed.
"""
from __future__ import annotations

import torch

from oracle.attention_ref import bottom_right_mask, sdpa_reference
from oracle.kvcache_ref import RefKVCache


class CpuDecodePath:
    def __init__(self, lens, num_layers, seed=0, dtype=torch.float32, heads=12, kv_heads=2):
        g = torch.Generator().manual_seed(seed)
        nb = sum((n + 15) // 16 for n in lens) + 1
        self.cache = RefKVCache(nb, 16, dtype=dtype, num_layers=num_layers)
        self.cache.free_blocks = torch.randperm(nb, generator=g).tolist()
        self.cache.buf.normal_(generator=g)
        self.seqs = [self.cache.alloc() for _ in lens]
        for s, n in zip(self.seqs, lens):
            self.cache.ensure_capacity(s, n)
            self.cache.lengths[s] = n - 1  # history; this step appends token n-1
        B = len(lens)
        self.L = num_layers
        self.q = torch.randn(num_layers, B, heads, 1, 128, generator=g, dtype=dtype)
        self.k = torch.randn(num_layers, B, kv_heads, 1, 128, generator=g, dtype=dtype)
        self.v = torch.randn(num_layers, B, kv_heads, 1, 128, generator=g, dtype=dtype)

    def step(self):
        starts, slot, gather = self.cache.prepare(self.seqs, 1)
        mask = bottom_right_mask(starts, 1)
        out = None
        for l in range(self.L):
            self.cache.write(l, slot, self.k[l], self.v[l])
            kd, vd = self.cache.read(l, gather)
            out = sdpa_reference(self.q[l], kd, vd, mask)
        return out
