"""Paged decode attention through the C ABI vs the oracle and the reference's
golden outputs (bf16, max-abs 2e-2 as kernels/test_fa2.py:25)."""
import math

import numpy as np
import pytest
import torch

from gpu_helpers import TOL, build_cache, max_err, write_history
from oracle import attention_ref, cases

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("ci", [1, 3])  # "decode", "ragged decode"
def test_reference_fa2_decode_cases_dense(cuda, golden, ci):
    from kernels.fa2 import FlashAttention2Function

    fx = np.load(golden / "attention_cases.npz")
    name, q, k, v, lens, causal = cases.fa2_cases()[ci]
    assert cases.sha(q, k, v) == str(fx[f"c{ci}_input_sha"])
    kv_lens = torch.tensor(lens, dtype=torch.int32, device=cuda)
    out = FlashAttention2Function.apply(q.to(cuda), k.to(cuda), v.to(cuda), causal, kv_lens)
    torch.cuda.synchronize()
    assert out.shape == q.shape and out.dtype == torch.bfloat16
    assert max_err(out, fx[f"c{ci}_out"]) < TOL, name


def test_config0_paged_decode_matches_reference(cuda, golden):
    """BASELINE config 0 end to end through KVCache + FlashAttention2Function:
    bit-exact tables and pool, output within 2e-2 of the reference."""
    from kernels.fa2 import FlashAttention2Function

    fx = np.load(golden / "decode_config0.npz")
    inp = cases.decode_config0_inputs()
    assert cases.sha(inp["q"], inp["k_new"], inp["v_new"], *inp["hist_k"], *inp["hist_v"]) == \
        str(fx["input_sha"])
    cache = build_cache(inp["num_blocks"], inp["perm"], cuda)
    seqs = [cache.alloc() for _ in inp["lens"]]
    write_history(cache, seqs, inp["hist_k"], inp["hist_v"])
    starts, step, gidx = cache.prepare(seqs, 1)
    cache.write(0, step, inp["k_new"].to(cuda), inp["v_new"].to(cuda))
    k, v = cache.read(0, gidx)
    out = FlashAttention2Function.apply(inp["q"].to(cuda), k, v, False, step.kv_lens)
    torch.cuda.synchronize()
    cache.check_errors()
    assert starts == list(fx["starts"])
    for i, s in enumerate(seqs):
        t = [x for x in fx["tables"][i] if x >= 0]
        assert cache.block_tables[cache.table_row(s), :len(t)].tolist() == t
    assert cases.sha(cache.buf[0].cpu()) == str(fx["pool_sha"])
    assert max_err(out, fx["out"]) < TOL
    # and against the float64 restatement on the materialised history
    dense_k, dense_v = k.materialize().cpu(), v.materialize().cpu()
    want = attention_ref.attention_np(inp["q"].float().numpy(), dense_k.float().numpy(),
                                      dense_v.float().numpy(), [s + 1 for s in starts], False)
    assert max_err(out, want) < TOL


def _paged_case(cuda, lens, seed, Hq=12, num_blocks=None, poison=True, plan_len=None):
    """Random paged decode case through the raw binding; unused pool slots are
    poisoned with PAD_VALUE so a masking leak shows as a large error.
    plan_len: the max_kv_len the launch is planned for (default: the rows'
    real maximum)."""
    import pagedkv

    g = torch.Generator().manual_seed(seed)
    B = len(lens)
    nb = [math.ceil(n / 16) for n in lens]
    N = num_blocks or (sum(nb) + 8)
    perm = torch.randperm(N, generator=g).tolist()
    cache = build_cache(N, perm, cuda)
    if poison:
        cache.buf.fill_(cases.PAD_VALUE)
    seqs = [cache.alloc() for _ in lens]
    hk = [torch.randn(1, 2, n - 1, 128, generator=g).to(torch.bfloat16) for n in lens]
    hv = [torch.randn(1, 2, n - 1, 128, generator=g).to(torch.bfloat16) for n in lens]
    write_history(cache, seqs, hk, hv)
    q = torch.randn(B, 12, 1, 128, generator=g).to(torch.bfloat16)
    kn = torch.randn(B, 2, 1, 128, generator=g).to(torch.bfloat16)
    vn = torch.randn(B, 2, 1, 128, generator=g).to(torch.bfloat16)
    starts, step, _ = cache.prepare(seqs, 1)
    cache.write(0, step, kn.to(cuda), vn.to(cuda))
    out = torch.empty(B, 12, 128, dtype=torch.bfloat16, device=cuda)
    pagedkv.paged_decode(q[:, :, 0].to(cuda), cache.buf[0, 0], cache.buf[0, 1], cache.block_tables,
                         step.rows, step.kv_lens, plan_len or step.max_kv_len, out,
                         1 / math.sqrt(128), 2, cache.err_flag)
    torch.cuda.synchronize()
    cache.check_errors()
    kd = [torch.cat([a, b[i:i + 1]], 2) for i, (a, b) in enumerate(zip(hk, [kn] * B))]
    vd = [torch.cat([a, b[i:i + 1]], 2) for i, (a, b) in enumerate(zip(hv, [vn] * B))]
    errs = []
    for b in range(B):
        want = attention_ref.attention_np(q[b:b + 1].float().numpy(), kd[b].float().numpy(),
                                          vd[b].float().numpy(), [lens[b]], False)
        errs.append(max_err(out[b:b + 1, :, None], want))
    return max(errs), out


@pytest.mark.parametrize("lens", [
    [1], [15, 16, 17], [1, 2, 3, 31, 32, 33], [64] * 5, [255, 256, 257],
    [1000, 37, 512, 1],           # the reference's ragged decode lengths
    [4096, 100], [8192, 8191, 3],  # long rows split across partitions
])
def test_paged_decode_random_vs_oracle(cuda, lens):
    err, _ = _paged_case(cuda, lens, seed=sum(lens))
    assert err < TOL


@pytest.mark.parametrize("B,lo,hi", [(8, 300, 520), (16, 480, 1000), (64, 400, 520),
                                     (130, 60, 130), (40, 1500, 2100)])
def test_capacity_planned_decode_vs_oracle(cuda, B, lo, hi):
    """A grid planned for a 16k-token capacity (as a captured decode graph
    plans it) over rows far shorter: each row takes the partition minimum of
    its own length and a latency-bound launch about one wave of CTAs.  The
    output matches the oracle and, up to rounding, the launch planned for
    the rows' real maximum."""
    g = torch.Generator().manual_seed(B * 1000 + hi)
    lens = torch.randint(lo, hi + 1, (B,), generator=g).tolist()
    err_cap, out_cap = _paged_case(cuda, lens, seed=B + hi, plan_len=16384)
    err, out = _paged_case(cuda, lens, seed=B + hi)
    assert err_cap < TOL and err < TOL, (err_cap, err)
    assert max_err(out_cap, out.float()) < TOL


def test_paged_decode_is_deterministic(cuda):
    """Split-K partials merge in partition order: identical bits run to run."""
    _, a = _paged_case(cuda, [6000, 5000, 300], seed=5)
    _, b = _paged_case(cuda, [6000, 5000, 300], seed=5)
    assert torch.equal(a, b)


@pytest.mark.parametrize("hq,hkv", [(8, 8), (16, 1), (4, 2), (12, 2)])
def test_gqa_group_sizes_dense(cuda, hq, hkv):
    """Groups of 1..16 query heads per KV head (16 spans two CTAs)."""
    from kernels.fa2 import flash_attention

    g = torch.Generator().manual_seed(hq * 10 + hkv)
    lens = [700, 33, 2000]
    B, S = len(lens), max(lens)
    q = torch.randn(B, hq, 1, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(B, hkv, S, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(B, hkv, S, 128, generator=g).to(torch.bfloat16)
    for b, n in enumerate(lens):
        k[b, :, n:] = cases.PAD_VALUE
        v[b, :, n:] = cases.PAD_VALUE
    out = flash_attention(q.to(cuda), k.to(cuda), v.to(cuda), False,
                          torch.tensor(lens, dtype=torch.int32, device=cuda))
    want = attention_ref.attention_np(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                      lens, False)
    assert max_err(out, want) < TOL


def test_zero_length_row_gives_nan_like_reference(cuda):
    """kv_len == 0: fa2.py:151 divides 0 by 0; the other rows are unaffected."""
    from kernels.fa2 import flash_attention

    q = torch.randn(2, 12, 1, 128).to(torch.bfloat16).to(cuda)
    k = torch.randn(2, 2, 64, 128).to(torch.bfloat16).to(cuda)
    out = flash_attention(q, k, k, False, torch.tensor([0, 64], dtype=torch.int32, device=cuda))
    assert torch.isnan(out[0].float()).all()
    assert torch.isfinite(out[1].float()).all()


def test_bad_block_id_in_decode_is_flagged(cuda):
    import pagedkv

    cache = build_cache(16, list(range(16)), cuda)
    s = cache.alloc()
    _, step, _ = cache.prepare([s], 40)
    cache.advance([s], 40)
    cache.block_tables[cache.table_row(s), 1] = -5
    q = torch.randn(1, 12, 128, dtype=torch.bfloat16, device=cuda)
    out = torch.empty_like(q)
    pagedkv.paged_decode(q, cache.buf[0, 0], cache.buf[0, 1], cache.block_tables, step.rows,
                         step.kv_lens, 40, out, 0.088, 2, cache.err_flag)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="0x1"):
        cache.check_errors()
