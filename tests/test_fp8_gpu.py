"""FP8 (e4m3) KV pool, opt-in (KVCache(kv_format="fp8_e4m3")).

The reference has no FP8 path (its pool holds the activation dtype,
kv_cache.py:20-22), so parity is pinned in two steps:
  * stored bytes and scales bit-exact against the numpy restatement of the
    format (oracle/fp8_ref.py), applied to the reference's bf16 RoPE'd k and
    v (taken from the bf16 append, itself bit-exact with the reference);
  * attention within the bf16 bar (max-abs 2e-2, kernels/test_fa2.py:25) of
    the float64 oracle over the DEQUANTISED K/V read back from the pool, and
    within a stated FP8 accuracy bar (FP8_TOL) of the oracle over the
    unquantised bf16 K/V (e4m3 keeps 3 mantissa bits).
"""
import math

import numpy as np
import pytest
import torch

from gpu_helpers import TOL, max_err
from oracle import attention_ref, cases, fp8_ref

pytestmark = pytest.mark.gpu

HQ, HKV, D = 12, 2, 128
# attention over e4m3 K/V vs over the bf16 originals, N(0,1) data.  A row is
# rounded to e4m3 with scale amax / 448, so an element moves by at most half
# the top-binade step, amax / 448 * 16; for N(0,1) rows amax is ~4, i.e. up to
# ~0.14.  A one-token context returns that V row itself (0.094 measured); long
# contexts average the errors down.
FP8_TOL = 0.15


def _caches(cuda, N, perm, B, pitch=None, layers=1):
    from kv_cache import KVCache

    out = []
    for fmt in ("bf16", "fp8_e4m3"):
        c = KVCache(N, 16, cuda, torch.bfloat16, max_seqs=max(B, 4), num_layers=layers,
                    max_blocks_per_seq=pitch, kv_format=fmt)
        c._free_blocks = list(perm)
        out.append(c)
    return out


def _append_both(cuda, caches, seqs, T, g, with_q=True):
    """One step of T tokens for every row through both caches' append (RoPE
    on q and k); returns (q_rot from bf16, q_rot from fp8, k, v, step pair)."""
    import model

    B = len(seqs[0])
    q = torch.randn(B, HQ, T, D, generator=g).to(torch.bfloat16).to(cuda)
    k = torch.randn(B, HKV, T, D, generator=g).to(torch.bfloat16).to(cuda)
    v = torch.randn(B, HKV, T, D, generator=g).to(torch.bfloat16).to(cuda)
    cos, sin = model.rope_table(16384, torch.bfloat16, cuda)
    outs, steps = [], []
    for c, ss in zip(caches, seqs):
        _, st, _ = c.prepare(ss, T)
        qr = torch.empty_like(q)
        c.append(0, st, q, k, v, cos, sin, qr)
        outs.append(qr)
        steps.append(st)
    return outs[0], outs[1], k, v, steps


def _expected_pool(c16, c8, seqs16, seqs8):
    """The FP8 pool the format predicts: every written slot of the bf16 pool
    (the reference's RoPE'd k and v) quantised by the restatement."""
    buf = c16.buf[0].float().cpu().numpy()  # [2, slots, Hkv, D]
    want = np.zeros(tuple(c8.pool8.shape[1:]), np.uint8)
    for s16, s8 in zip(seqs16, seqs8):
        n = c16.length(s16)
        t16, t8 = c16.host_table(s16), c8.host_table(s8)
        for p in range(n):
            slot = t16[p // 16] * 16 + p % 16
            for h in range(HKV):
                fp8_ref.write_token(want[t8[p // 16], h], p % 16, buf[0, slot, h], buf[1, slot, h])
    return want


@pytest.mark.parametrize("hist,T", [([0, 0, 0], 37), ([5, 16, 100], 1), ([31, 0], 20)])
def test_fp8_append_bytes_bit_exact(cuda, hist, T):
    g = torch.Generator().manual_seed(sum(hist) * 7 + T)
    B = len(hist)
    N = sum(math.ceil((h + T) / 16) for h in hist) + 6
    perm = torch.randperm(N, generator=g).tolist()
    c16, c8 = _caches(cuda, N, perm, B)
    s16 = [c16.alloc() for _ in hist]
    s8 = [c8.alloc() for _ in hist]
    for i, h in enumerate(hist):  # history, one row at a time
        if h:
            _append_both(cuda, (c16, c8), ([s16[i]], [s8[i]]), h, g)
            c16.advance([s16[i]], h)
            c8.advance([s8[i]], h)
    q16, q8, _, _, _ = _append_both(cuda, (c16, c8), (s16, s8), T, g)
    c16.advance(s16, T)
    c8.advance(s8, T)
    torch.cuda.synchronize()
    c16.check_errors()
    c8.check_errors()
    assert torch.equal(q16, q8), "roped q differs between the bf16 and FP8 appends"
    want = _expected_pool(c16, c8, s16, s8)
    got = c8.pool8[0].cpu().numpy()
    bad = np.argwhere(got != want)
    assert bad.size == 0, f"{len(bad)} FP8 pool bytes differ, first at {bad[:4].tolist()}"


def _decode_case(cuda, lens, seed, plan_len=None):
    """FP8 and bf16 caches with the same history (random, written through
    the appends), then one decode step: appended token + attention.
    plan_len: the max_kv_len the launches are planned for (default: the
    rows' real maximum; a captured graph plans for the cache's capacity)."""
    import dataclasses

    from kernels.fa2 import flash_attention

    g = torch.Generator().manual_seed(seed)
    B = len(lens)
    N = sum(math.ceil(n / 16) for n in lens) + 8
    perm = torch.randperm(N, generator=g).tolist()
    pitch = max(math.ceil(n / 16) for n in lens) + 1
    c16, c8 = _caches(cuda, N, perm, B, pitch=pitch)
    s16 = [c16.alloc() for _ in lens]
    s8 = [c8.alloc() for _ in lens]
    for i, n in enumerate(lens):
        if n > 1:
            _append_both(cuda, (c16, c8), ([s16[i]], [s8[i]]), n - 1, g)
            c16.advance([s16[i]], n - 1)
            c8.advance([s8[i]], n - 1)
    q16, q8, _, _, (st16, st8) = _append_both(cuda, (c16, c8), (s16, s8), 1, g)
    outs = []
    for c, st, q in ((c16, st16, q16), (c8, st8, q8)):
        if plan_len:
            st = dataclasses.replace(st, max_kv_len=plan_len)
        kh, vh = c.read(0, st)
        o = torch.full_like(q, float("nan"))
        flash_attention(q, kh, vh, False, st.kv_lens, out=o)
        outs.append(o)
    torch.cuda.synchronize()
    c16.check_errors()
    c8.check_errors()
    return c16, c8, s16, s8, q8, outs


@pytest.mark.parametrize("lens", [[1], [15, 16, 17], [1000, 37, 512, 1], [4096, 100],
                                  [8192, 8191, 3]])
def test_fp8_decode_vs_oracle(cuda, lens):
    _check_fp8_decode(lens, _decode_case(cuda, lens, seed=sum(lens) + 1))


@pytest.mark.parametrize("B,lo,hi", [(16, 480, 1000), (70, 60, 130)])
def test_fp8_capacity_planned_decode_vs_oracle(cuda, B, lo, hi):
    """FP8 decode planned for a 16k-token capacity over short rows (the
    per-row partition minimum and the one-wave cap, at the FP8 kernel's
    four CTAs per SM)."""
    g = torch.Generator().manual_seed(B * 1000 + hi)
    lens = torch.randint(lo, hi + 1, (B,), generator=g).tolist()
    _check_fp8_decode(lens, _decode_case(cuda, lens, seed=B + hi, plan_len=16384))


def _check_fp8_decode(lens, case):
    c16, c8, s16, s8, q, (o16, o8) = case
    pool = c8.pool8[0].cpu().numpy()
    worst_acc = 0.0
    for b, n in enumerate(lens):
        K = np.zeros((1, HKV, n, D), np.float32)
        V = np.zeros((1, HKV, n, D), np.float32)
        for h in range(HKV):
            K[0, h], V[0, h] = fp8_ref.gather_rows(pool, c8.host_table(s8[b]), n, h)
        want = attention_ref.attention_np(q[b:b + 1].float().cpu().numpy(), K, V, [n], False)
        assert max_err(o8[b:b + 1], want) < TOL, (b, n)
        worst_acc = max(worst_acc, max_err(o8[b:b + 1], o16[b:b + 1].float()))
    assert worst_acc < FP8_TOL, worst_acc


def test_fp8_decode_is_deterministic(cuda):
    *_, (_, a) = _decode_case(cuda, [6000, 5000, 300], seed=5)
    *_, (_, b) = _decode_case(cuda, [6000, 5000, 300], seed=5)
    assert torch.equal(a, b)


def test_fp8_config3_decode_launch(cuda):
    """The timed FP8 launch shape: 256 rows with contexts U[2048, 8192]
    (bench.py's seed), one layer; sampled rows against the oracle over the
    stored bytes."""
    from kernels.fa2 import flash_attention
    from kv_cache import KVCache

    g = torch.Generator().manual_seed(0)
    lens = torch.randint(2048, 8192 + 1, (256,), generator=g).tolist()
    N = sum(math.ceil(n / 16) for n in lens) + 64
    c8 = KVCache(N, 16, cuda, torch.bfloat16, max_seqs=256, num_layers=1,
                 max_blocks_per_seq=8192 // 16 + 2, kv_format="fp8_e4m3")
    c8._free_blocks = torch.randperm(N, generator=g).tolist()
    seqs = [c8.alloc() for _ in lens]
    for s, n in zip(seqs, lens):
        c8.ensure_capacity(s, n)
        c8._lengths[s] = n - 1
    # random history straight into the pool: valid e4m3 bytes (no NaN codes)
    # and positive scales
    gd = torch.Generator(device=cuda).manual_seed(3)
    body = torch.randint(0, 256, (N, HKV, 4096), device=cuda, generator=gd, dtype=torch.uint8)
    body[(body & 0x7F) == 0x7F] ^= 1
    c8.pool8[0, :, :, :4096] = body
    sc = (torch.rand(N, HKV, 32, device=cuda, generator=gd) * 0.01 + 0.001)
    c8.pool8[0, :, :, 4096:] = sc.view(torch.uint8).view(N, HKV, 128)
    import model

    _, st, _ = c8.prepare(seqs, 1)
    q = torch.randn(256, HQ, 1, D, device=cuda, generator=gd).to(torch.bfloat16)
    k = torch.randn(256, HKV, 1, D, device=cuda, generator=gd).to(torch.bfloat16)
    cos, sin = model.rope_table(8192 + 32, torch.bfloat16, cuda)
    qr = torch.empty_like(q)
    c8.append(0, st, q, k, k, cos, sin, qr)
    kh, vh = c8.read(0, st)
    out = torch.full_like(q, float("nan"))
    flash_attention(qr, kh, vh, False, st.kv_lens, out=out)
    torch.cuda.synchronize()
    c8.check_errors()
    assert not torch.isnan(out.float()).any()
    pool = c8.pool8[0].cpu().numpy()
    order = np.argsort(lens)
    for b in sorted({int(order[0]), int(order[-1]), 5, 77, 130, 200}):
        n = lens[b]
        K = np.zeros((1, HKV, n, D), np.float32)
        V = np.zeros((1, HKV, n, D), np.float32)
        for h in range(HKV):
            K[0, h], V[0, h] = fp8_ref.gather_rows(pool, c8.host_table(seqs[b]), n, h)
        want = attention_ref.attention_np(qr[b:b + 1].float().cpu().numpy(), K, V, [n], False)
        assert max_err(out[b:b + 1], want) < TOL, (b, n)


@pytest.mark.parametrize("prior,T", [([0, 0], 33), ([1000, 3], 64), ([17], 2)])
def test_fp8_prefill_vs_oracle(cuda, prior, T):
    """Chunked causal prefill over an FP8 pool (dequantised rows + the bf16
    tensor-core prefill): against the oracle over the stored bytes, and
    within FP8_TOL of the same prefill on a bf16 pool."""
    from kernels.fa2 import flash_attention

    g = torch.Generator().manual_seed(sum(prior) + T)
    B = len(prior)
    N = sum(math.ceil((n + T) / 16) for n in prior) + 8
    perm = torch.randperm(N, generator=g).tolist()
    c16, c8 = _caches(cuda, N, perm, B)
    s16 = [c16.alloc() for _ in prior]
    s8 = [c8.alloc() for _ in prior]
    for i, n in enumerate(prior):
        if n:
            _append_both(cuda, (c16, c8), ([s16[i]], [s8[i]]), n, g)
            c16.advance([s16[i]], n)
            c8.advance([s8[i]], n)
    q16, q8, _, _, (st16, st8) = _append_both(cuda, (c16, c8), (s16, s8), T, g)
    outs = []
    for c, st, q in ((c16, st16, q16), (c8, st8, q8)):
        kh, vh = c.read(0, st)
        outs.append(flash_attention(q, kh, vh, True, st.kv_lens))
    torch.cuda.synchronize()
    c8.check_errors()
    pool = c8.pool8[0].cpu().numpy()
    for b in range(B):
        n = prior[b] + T
        K = np.zeros((1, HKV, n, D), np.float32)
        V = np.zeros((1, HKV, n, D), np.float32)
        for h in range(HKV):
            K[0, h], V[0, h] = fp8_ref.gather_rows(pool, c8.host_table(s8[b]), n, h)
        # the prefill attends over bf16(e4m3 * scale): round like the kernel's input
        Kb = torch.from_numpy(K).to(torch.bfloat16).float().numpy()
        Vb = torch.from_numpy(V).to(torch.bfloat16).float().numpy()
        want = attention_ref.attention_np(q8[b:b + 1].float().cpu().numpy(), Kb, Vb, [n], True)
        assert max_err(outs[1][b:b + 1], want) < TOL, b
        assert max_err(outs[1][b:b + 1], outs[0][b:b + 1].float()) < FP8_TOL, b


def test_fp8_materialize_reads_back_dequantised_rows(cuda):
    from kv_cache import PagedStep

    c16, c8, s16, s8, q, _ = _decode_case(cuda, [40, 17], seed=9)

    rows = torch.tensor([c8.table_row(s) for s in s8], dtype=torch.int32, device=cuda)
    kvl = torch.tensor([c8.length(s) + 1 for s in s8], dtype=torch.int32, device=cuda)
    step = PagedStep(c8, 1, [0, 0], rows, kvl - 1, kvl, int(kvl.max()))
    kh, vh = c8.read(0, step)
    kd, vd = kh.materialize().float().cpu().numpy(), vh.materialize().float().cpu().numpy()
    pool = c8.pool8[0].cpu().numpy()
    for b, s in enumerate(s8):
        n = int(kvl[b])
        for h in range(HKV):
            K, V = fp8_ref.gather_rows(pool, c8.host_table(s), n, h)
            assert np.array_equal(kd[b, h, :n], torch.from_numpy(K).to(torch.bfloat16).float().numpy())
            assert np.array_equal(vd[b, h, :n], torch.from_numpy(V).to(torch.bfloat16).float().numpy())
