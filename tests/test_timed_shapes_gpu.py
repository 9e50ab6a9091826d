"""Parity at the exact launch shapes the benchmark times.

The decode planner sizes split-K partitions by launch size (4, 16 or 32
blocks at least per partition), so small parity cases and the large timed
launches take different branches.  These tests run the timed shapes
themselves and compare sampled rows with the float64 oracle
(oracle/attention_ref.py, a restatement of kernels/fa2.py:23-162):

  * config 3: 256 rows, contexts U[2048, 8192] seeded as bench.py's
    context_lengths, fused RoPE + append of the step's token, then ONE paged
    decode launch over a pool whose unused slots hold PAD_VALUE (the leak
    check of kernels/test_fa2.py:47-49);
  * the engine's 128-row decode of ~2100-token rows (config 4), both with
    the true max_kv_len and with a CUDA graph's capacity as max_kv_len;
  * config 1 as bench.py times it: ONE paged, left-padded 8-row causal
    launch with starts = kv_len - T, through both tensor-core prefill kernels.
"""
import math

import numpy as np
import pytest
import torch

from gpu_helpers import TOL, max_err
from oracle import attention_ref, cases

pytestmark = pytest.mark.gpu

HQ, HKV, D = 12, 2, 128


def _decode_case(cuda, lens, seed, max_kv_len=None):
    """A one-layer pool holding every row's first n-1 tokens (random, written
    on the device), PAD_VALUE everywhere else; then the bench's per-layer
    call: append the step's token (RoPE on q and k), paged decode over it."""
    import model
    import pagedkv
    from kernels.fa2 import flash_attention
    from kv_cache import KVCache

    B = len(lens)
    need = sum(math.ceil(n / 16) for n in lens)
    N = need + 64
    pitch = math.ceil((max(max_kv_len or 0, max(lens)) + 1) / 16)
    # one layer is enough: the planner and the kernel never see the layer count
    cache = KVCache(N, 16, cuda, torch.bfloat16, max_seqs=B, max_blocks_per_seq=pitch,
                    num_layers=1)
    g = torch.Generator().manual_seed(seed)
    cache._free_blocks = torch.randperm(N, generator=g).tolist()
    seqs = [cache.alloc() for _ in lens]
    for s, n in zip(seqs, lens):
        cache.ensure_capacity(s, n)
        cache._lengths[s] = n - 1
    cache.buf.fill_(cases.PAD_VALUE)
    gd = torch.Generator(device=cuda).manual_seed(seed + 1)
    for which in (0, 1):
        plane = cache.buf[0, which].view(N, 16, HKV, D)
        for s, n in zip(seqs, lens):
            blocks = torch.tensor(cache._block_tables[s], device=cuda)
            vals = torch.randn(len(blocks) * 16, HKV, D, device=cuda, generator=gd)
            vals[n - 1:] = cases.PAD_VALUE  # past the history: poisoned
            plane[blocks] = vals.to(torch.bfloat16).view(len(blocks), 16, HKV, D)
    _, step, _ = cache.prepare(seqs, 1)
    if max_kv_len is not None:  # a captured graph sizes the grid for its capacity
        step.max_kv_len = max_kv_len
    cos, sin = model.rope_table(pitch * 16, torch.bfloat16, cuda)
    q = torch.randn(B, HQ, 1, D, device=cuda, generator=gd).to(torch.bfloat16)
    k = torch.randn(B, HKV, 1, D, device=cuda, generator=gd).to(torch.bfloat16)
    v = torch.randn(B, HKV, 1, D, device=cuda, generator=gd).to(torch.bfloat16)
    q_rot = torch.empty_like(q)
    out = torch.full_like(q, float("nan"))
    cache.append(0, step, q, k, v, cos, sin, q_rot)
    kh, vh = cache.read(0, step)
    flash_attention(q_rot, kh, vh, False, step.kv_lens, out=out)
    torch.cuda.synchronize()
    cache.check_errors()
    plan = pagedkv.decode_plan(B, HQ, HKV, step.max_kv_len)
    return cache, seqs, q_rot, out, plan


def _check_rows(cache, seqs, lens, q_rot, out, rows):
    """Oracle over the K/V a reference gather would read for each sampled row
    (slot = table[p // 16] * 16 + p % 16, kv_cache.py:88-95)."""
    for b in rows:
        n = lens[b]
        tbl = torch.tensor(cache._block_tables[seqs[b]], dtype=torch.long)
        pos = torch.arange(n)
        slots = (tbl[pos // 16] * 16 + pos % 16).to(cache.device)
        kk = cache.buf[0, 0][slots].permute(1, 0, 2)[None].float().cpu().numpy()
        vv = cache.buf[0, 1][slots].permute(1, 0, 2)[None].float().cpu().numpy()
        assert not (kk == cases.PAD_VALUE).all(-1).any(), "a visible key is still poisoned"
        want = attention_ref.attention_np(q_rot[b:b + 1].float().cpu().numpy(), kk, vv, [n], False)
        err = max_err(out[b:b + 1], want)
        assert err < TOL, (b, n, err)


def _sample_rows(lens, k, seed):
    order = np.argsort(lens)
    rng = np.random.default_rng(seed)
    pick = {int(order[0]), int(order[-1])}  # shortest and longest
    pick |= set(int(x) for x in rng.choice(len(lens), size=k - 2, replace=False))
    return sorted(pick)


def test_config3_decode_launch_vs_oracle(cuda):
    """BASELINE config 3's timed launch: 256 rows, ctx U[2048, 8192] drawn
    exactly as bench.py context_lengths(seed 0)."""
    g = torch.Generator().manual_seed(0)
    lens = torch.randint(2048, 8192 + 1, (256,), generator=g).tolist()
    cache, seqs, q_rot, out, plan = _decode_case(cuda, lens, seed=1)
    assert plan["min_blocks_per_part"] == 32 and plan["max_parts"] > 1, plan
    assert plan["blocks_per_part"] == 128 and plan["max_parts"] == 4, plan
    assert not torch.isnan(out.float()).any()
    _check_rows(cache, seqs, lens, q_rot, out, _sample_rows(lens, 18, 0))


@pytest.mark.parametrize("capacity", [None, 4352])
def test_engine_128_row_decode_launch_vs_oracle(cuda, capacity):
    """The engine's decode step at ~128 rows of ~2100 tokens (config 4);
    capacity = a graph's max_kv_len (grid planned for it, rows sized by their
    own length)."""
    g = torch.Generator().manual_seed(7)
    lens = torch.randint(2048, 2176, (128,), generator=g).tolist()
    cache, seqs, q_rot, out, plan = _decode_case(cuda, lens, seed=3, max_kv_len=capacity)
    assert plan["min_blocks_per_part"] == 32 and plan["max_parts"] > 1, plan
    if capacity is None:
        assert plan["max_parts"] == 5, plan
    assert not torch.isnan(out.float()).any()
    _check_rows(cache, seqs, lens, q_rot, out, _sample_rows(lens, 16, 1))


@pytest.mark.parametrize("kernel", ["one", "pair"])
def test_config1_bench_prefill_launch_vs_oracle(cuda, monkeypatch, kernel):
    """bench.py prefill_run's launch: 8 prompts U[16, 1024] (seed 42) in a
    shuffled pool, then ONE causal launch over the paged K/V with the queries
    left-padded to T = max(lens) and starts = kv_len - T (negative for the
    padded rows).  Real query rows must match the oracle; padded query rows
    see no key and are NaN, as the reference's 0/0 (fa2.py:151)."""
    from kernels.fa2 import flash_attention
    from kv_cache import KVCache, PagedStep

    monkeypatch.setenv("PKV_PREFILL_KERNEL", kernel)
    g = torch.Generator().manual_seed(42)
    lens = torch.randint(16, 1025, (8,), generator=g).tolist()
    T = max(lens)
    N = sum(math.ceil(n / 16) for n in lens) + 16
    cache = KVCache(N, 16, cuda, torch.bfloat16, num_layers=1)
    cache._free_blocks = torch.randperm(N, generator=g).tolist()
    cache.buf.fill_(cases.PAD_VALUE)
    seqs = [cache.alloc() for _ in lens]
    ks, vs = [], []
    for s_, n in zip(seqs, lens):
        k = torch.randn(1, HKV, n, D, generator=g).to(torch.bfloat16)
        v = torch.randn(1, HKV, n, D, generator=g).to(torch.bfloat16)
        _, st, _ = cache.prepare([s_], n)
        cache.write(0, st, k.to(cuda), v.to(cuda))
        cache.advance([s_], n)
        ks.append(k)
        vs.append(v)
    rows = torch.tensor([cache.table_row(x) for x in seqs], dtype=torch.int32, device=cuda)
    kvl = torch.tensor(lens, dtype=torch.int32, device=cuda)
    step = PagedStep(cache, T, [0] * len(lens), rows, kvl - T, kvl, T)
    q = torch.randn(len(lens), HQ, T, D, generator=g).to(torch.bfloat16)
    out = torch.full((len(lens), HQ, T, D), 3.0, dtype=torch.bfloat16, device=cuda)
    kh, vh = cache.read(0, step)
    flash_attention(q.to(cuda), kh, vh, True, kvl, out=out)
    torch.cuda.synchronize()
    cache.check_errors()
    for b, n in enumerate(lens):
        want = attention_ref.attention_np(q[b:b + 1].float().numpy(), ks[b].float().numpy(),
                                          vs[b].float().numpy(), [n], True)
        assert np.isnan(want[0, :, :T - n]).all() and not np.isnan(want[0, :, T - n:]).any()
        err = max_err(out[b:b + 1], want)  # NaN positions must agree, then max-abs
        assert err < TOL, (kernel, b, n, err)
