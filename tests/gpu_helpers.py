"""Helpers shared by the GPU parity tests (CPU-side construction only)."""
import numpy as np
import torch

from oracle import cases

TOL = 2e-2  # max-abs for bf16 attention outputs, kernels/test_fa2.py:25


def build_cache(num_blocks, perm, device, **kw):
    from kv_cache import KVCache

    c = KVCache(num_blocks, 16, device, torch.bfloat16, **kw)
    c._free_blocks = list(perm)
    return c


def write_history(cache, seqs, hist_k, hist_v, layer=0):
    """Write each row's history through the product write() path, one row at a
    time (as the reference scheduler prefills)."""
    for s, kk, vv in zip(seqs, hist_k, hist_v):
        n = kk.shape[2]
        if n:
            _, step, _ = cache.prepare([s], n)
            cache.write(layer, step, kk.to(cache.device), vv.to(cache.device))
            cache.advance([s], n)


def max_err(got, want):
    """Max-abs difference over the elements that are finite in both, after
    requiring NaN in exactly the same places (a kv_len == 0 row is NaN in the
    reference too, fa2.py:151).  A NaN where the oracle is finite, or a finite
    value where the oracle is NaN, returns inf, so no tolerance can pass it."""
    g = got.float().cpu().numpy() if isinstance(got, torch.Tensor) else np.asarray(got)
    w = want.float().cpu().numpy() if isinstance(want, torch.Tensor) else np.asarray(want)
    g, w = np.broadcast_arrays(g.astype(np.float64), w.astype(np.float64))
    if not np.array_equal(np.isnan(g), np.isnan(w)):
        return float("inf")
    ok = ~np.isnan(g)
    if not ok.any():
        return 0.0
    return float(np.abs(g[ok] - w[ok]).max())
