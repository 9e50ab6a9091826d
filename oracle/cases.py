"""Seeded input generators for the parity cases (test oracle).

TEST INFRASTRUCTURE ONLY.  The golden-fixture script and the tests both build
their inputs here, so a fixture can store only the reference's outputs plus a
hash of the inputs it was made from (tests check the hash before comparing).
All generation is on the CPU with explicit or documented seeds.
"""
from __future__ import annotations

import hashlib

import numpy as np
import torch

PAD_VALUE = 100.0  # kernels/test_fa2.py:24

# kernels/test_fa2.py:17-23: (name, T queries, each row's key count, is_causal)
FA2_CASES = [
    ("prefill", 300, [300, 300], True),
    ("decode", 1, [1000, 1000], False),
    ("chunked", 64, [500, 500], True),
    ("ragged decode", 1, [1000, 37, 512, 1], False),
    ("ragged prefill", 16, [16, 300, 100], True),
]


def bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 bit patterns (numpy)."""
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def from_bits(a: np.ndarray) -> torch.Tensor:
    """uint16 bit patterns -> bf16 tensor."""
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        if isinstance(a, torch.Tensor):
            a = bits(a) if a.dtype == torch.bfloat16 else a.contiguous().numpy()
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def fa2_cases():
    """The reference kernel test's inputs, generated exactly as
    kernels/test_fa2.py:39-50 does (global seed 0, q/k/v per case in order,
    PAD_VALUE written past each row's length).  Yields
    (name, q, k, v, lens, is_causal) with bf16 CPU tensors."""
    torch.manual_seed(0)
    out = []
    for name, T, lens, causal in FA2_CASES:
        B, S = len(lens), max(lens)
        q = torch.randn(B, 12, T, 128, dtype=torch.bfloat16)
        k = torch.randn(B, 2, S, 128, dtype=torch.bfloat16)
        v = torch.randn(B, 2, S, 128, dtype=torch.bfloat16)
        for b, n in enumerate(lens):
            k[b, :, n:] = PAD_VALUE
            v[b, :, n:] = PAD_VALUE
        out.append((name, q, k, v, list(lens), causal))
    return out


def decode_config0_inputs():
    """batch 4, contexts {37,128,511,1000}, 1024-block pool
    assigned from a seeded permutation, Q/K/V ~ N(0,1) rounded to bf16.
    Row b holds lens[b]-1 history tokens and appends one (T=1) this step."""
    g = torch.Generator().manual_seed(0)
    N, lens = 1024, [37, 128, 511, 1000]
    perm = torch.randperm(N, generator=g).tolist()
    hist_k, hist_v = [], []
    for n in lens:
        hist_k.append(torch.randn(1, 2, n - 1, 128, generator=g).to(torch.bfloat16))
        hist_v.append(torch.randn(1, 2, n - 1, 128, generator=g).to(torch.bfloat16))
    B = len(lens)
    q = torch.randn(B, 12, 1, 128, generator=g).to(torch.bfloat16)
    k_new = torch.randn(B, 2, 1, 128, generator=g).to(torch.bfloat16)
    v_new = torch.randn(B, 2, 1, 128, generator=g).to(torch.bfloat16)
    return dict(num_blocks=N, lens=lens, perm=perm, hist_k=hist_k, hist_v=hist_v, q=q,
                k_new=k_new, v_new=v_new)


def prefill_config1_inputs(prior=(0, 211, 57), T=90, num_blocks=256, seed=1):
    """Ragged causal prefill + append (BASELINE config 1 shapes): rows already
    hold `prior` tokens and append T each (one T per prepare call,
    kv_cache.py:74)."""
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(num_blocks, generator=g).tolist()
    hk, hv = [], []
    for n in prior:
        hk.append(torch.randn(1, 2, n, 128, generator=g).to(torch.bfloat16))
        hv.append(torch.randn(1, 2, n, 128, generator=g).to(torch.bfloat16))
    B = len(prior)
    q = torch.randn(B, 12, T, 128, generator=g).to(torch.bfloat16)
    k_new = torch.randn(B, 2, T, 128, generator=g).to(torch.bfloat16)
    v_new = torch.randn(B, 2, T, 128, generator=g).to(torch.bfloat16)
    return dict(num_blocks=num_blocks, prior=list(prior), T=T, perm=perm, hist_k=hk, hist_v=hv,
                q=q, k_new=k_new, v_new=v_new)
