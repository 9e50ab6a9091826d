"""Ragged causal prefill attention through the C ABI vs the oracle and the
reference's golden outputs (bf16, max-abs 2e-2)."""
import math

import numpy as np
import pytest
import torch

from gpu_helpers import TOL, build_cache, max_err, write_history
from oracle import attention_ref, cases

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("ci", [0, 2, 4])  # "prefill", "chunked", "ragged prefill"
def test_reference_fa2_prefill_cases_dense(cuda, golden, ci):
    from kernels.fa2 import FlashAttention2Function

    fx = np.load(golden / "attention_cases.npz")
    name, q, k, v, lens, causal = cases.fa2_cases()[ci]
    assert cases.sha(q, k, v) == str(fx[f"c{ci}_input_sha"])
    kv_lens = torch.tensor(lens, dtype=torch.int32, device=cuda)
    out = FlashAttention2Function.apply(q.to(cuda), k.to(cuda), v.to(cuda), causal, kv_lens)
    torch.cuda.synchronize()
    rows = fx[f"c{ci}_rows"]
    assert max_err(out[:, :, rows], fx[f"c{ci}_out"]) < TOL, name


def test_config1_paged_prefill_matches_reference(cuda, golden):
    from kernels.fa2 import FlashAttention2Function

    fx = np.load(golden / "prefill_config1.npz")
    inp = cases.prefill_config1_inputs()
    T = inp["T"]
    cache = build_cache(inp["num_blocks"], inp["perm"], cuda)
    seqs = [cache.alloc() for _ in inp["prior"]]
    write_history(cache, seqs, inp["hist_k"], inp["hist_v"])
    starts, step, gidx = cache.prepare(seqs, T)
    cache.write(0, step, inp["k_new"].to(cuda), inp["v_new"].to(cuda))
    k, v = cache.read(0, gidx)
    out = FlashAttention2Function.apply(inp["q"].to(cuda), k, v, True, step.kv_lens)
    torch.cuda.synchronize()
    cache.check_errors()
    assert cases.sha(cache.buf[0].cpu()) == str(fx["pool_sha"])
    for i, s in enumerate(seqs):
        t = [x for x in fx["tables"][i] if x >= 0]
        assert cache.block_tables[cache.table_row(s), :len(t)].tolist() == t
    assert max_err(out, fx["out"]) < TOL


def test_config1_full_batch8_from_empty(cuda):
    """BASELINE config 1 at full size: 8 rows, prompt lengths U[16,1024], empty
    caches, shuffled pool.  Each row prefilled on its own (one prompt per
    prepare, chat.py:_admit) and checked against the oracle."""
    from kernels.fa2 import flash_attention

    g = torch.Generator().manual_seed(42)
    lens = torch.randint(16, 1025, (8,), generator=g).tolist()
    N = sum(math.ceil(n / 16) for n in lens) + 16
    cache = build_cache(N, torch.randperm(N, generator=g).tolist(), cuda)
    cache.buf.fill_(cases.PAD_VALUE)
    for n in lens:
        s = cache.alloc()
        q = torch.randn(1, 12, n, 128, generator=g).to(torch.bfloat16)
        k = torch.randn(1, 2, n, 128, generator=g).to(torch.bfloat16)
        v = torch.randn(1, 2, n, 128, generator=g).to(torch.bfloat16)
        _, step, gidx = cache.prepare([s], n)
        cache.write(0, step, k.to(cuda), v.to(cuda))
        kh, vh = cache.read(0, gidx)
        out = flash_attention(q.to(cuda), kh, vh, True, step.kv_lens)
        torch.cuda.synchronize()
        want = attention_ref.attention_np(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                          [n], True)
        assert max_err(out, want) < TOL, n
    cache.check_errors()


@pytest.mark.parametrize("prior,T", [([0, 0], 33), ([5, 100, 16], 16), ([1000, 3], 64),
                                     ([0], 1024), ([17], 2), ([300, 0, 45, 1], 129)])
def test_paged_prefill_random_vs_oracle(cuda, prior, T):
    """Chunked prefill onto existing history (bottom-right causal), poisoned pool."""
    from kernels.fa2 import flash_attention

    g = torch.Generator().manual_seed(sum(prior) + T)
    B = len(prior)
    N = sum(math.ceil((n + T) / 16) for n in prior) + 8
    cache = build_cache(N, torch.randperm(N, generator=g).tolist(), cuda)
    cache.buf.fill_(cases.PAD_VALUE)
    seqs = [cache.alloc() for _ in prior]
    hk = [torch.randn(1, 2, n, 128, generator=g).to(torch.bfloat16) for n in prior]
    hv = [torch.randn(1, 2, n, 128, generator=g).to(torch.bfloat16) for n in prior]
    write_history(cache, seqs, hk, hv)
    q = torch.randn(B, 12, T, 128, generator=g).to(torch.bfloat16)
    kn = torch.randn(B, 2, T, 128, generator=g).to(torch.bfloat16)
    vn = torch.randn(B, 2, T, 128, generator=g).to(torch.bfloat16)
    _, step, gidx = cache.prepare(seqs, T)
    cache.write(0, step, kn.to(cuda), vn.to(cuda))
    kh, vh = cache.read(0, gidx)
    out = flash_attention(q.to(cuda), kh, vh, True, step.kv_lens)
    torch.cuda.synchronize()
    cache.check_errors()
    for b in range(B):
        kd = torch.cat([hk[b], kn[b:b + 1]], 2)
        vd = torch.cat([hv[b], vn[b:b + 1]], 2)
        want = attention_ref.attention_np(q[b:b + 1].float().numpy(), kd.float().numpy(),
                                          vd.float().numpy(), [prior[b] + T], True)
        assert max_err(out[b:b + 1], want) < TOL, (b, prior[b], T)


def test_non_causal_multi_query(cuda):
    """is_causal=False with T > 1: every query sees all kv_len keys."""
    from kernels.fa2 import flash_attention

    g = torch.Generator().manual_seed(9)
    lens = [50, 300]
    q = torch.randn(2, 12, 20, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(2, 2, 300, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(2, 2, 300, 128, generator=g).to(torch.bfloat16)
    out = flash_attention(q.to(cuda), k.to(cuda), v.to(cuda), False,
                          torch.tensor(lens, dtype=torch.int32, device=cuda))
    want = attention_ref.attention_np(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                      lens, False)
    assert max_err(out, want) < TOL


def test_left_padded_batched_prefill(cuda):
    """Ragged prompts in ONE call: rows left-padded to T, bottom-right causal
    aligns each row's real queries with its keys (fa2.py:110-111)."""
    from kernels.fa2 import flash_attention

    g = torch.Generator().manual_seed(77)
    lens = [16, 500, 1024, 77]
    T = max(lens)
    B = len(lens)
    q = torch.randn(B, 12, T, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(B, 2, T, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(B, 2, T, 128, generator=g).to(torch.bfloat16)
    out = flash_attention(q.to(cuda), k.to(cuda), v.to(cuda), True,
                          torch.tensor(lens, dtype=torch.int32, device=cuda))
    for b, n in enumerate(lens):
        want = attention_ref.attention_np(q[b:b + 1, :, T - n:].float().numpy(),
                                          k[b:b + 1, :, :n].float().numpy(),
                                          v[b:b + 1, :, :n].float().numpy(), [n], True)
        assert max_err(out[b:b + 1, :, T - n:], want) < TOL


def test_right_padded_rows_with_q_lens(cuda):
    """q_lens: row b has q_lens[b] real queries at the front of a padded T
    (query i sits at key i + kv_len - q_len); padded output rows are untouched."""
    import pagedkv

    g = torch.Generator().manual_seed(31)
    prior, qlen, T = [0, 300, 17, 64], [5, 130, 128, 1], 160
    B = len(prior)
    N = sum(math.ceil((p + T) / 16) for p in prior) + 8
    cache = build_cache(N, torch.randperm(N, generator=g).tolist(), cuda)
    cache.buf.fill_(cases.PAD_VALUE)
    seqs = [cache.alloc() for _ in prior]
    hk = [torch.randn(1, 2, n, 128, generator=g).to(torch.bfloat16) for n in prior]
    hv = [torch.randn(1, 2, n, 128, generator=g).to(torch.bfloat16) for n in prior]
    write_history(cache, seqs, hk, hv)
    kn = torch.randn(B, 2, T, 128, generator=g).to(torch.bfloat16)
    vn = torch.randn(B, 2, T, 128, generator=g).to(torch.bfloat16)
    q = torch.randn(B, 12, T, 128, generator=g).to(torch.bfloat16)
    starts, rows = cache.step_rows(seqs, T)
    cache.flush_tables()
    st = torch.tensor(starts, dtype=torch.int32, device=cuda)
    ql = torch.tensor(qlen, dtype=torch.int32, device=cuda)
    rows_d = torch.tensor(rows, dtype=torch.int32, device=cuda)
    pool_before = cache.buf[0].clone()
    pagedkv.append_rope(None, kn.to(cuda), vn.to(cuda), None, None, None, cache.buf[0, 0],
                        cache.buf[0, 1], cache.block_tables, rows_d, st, cache.err_flag, ql)
    out = torch.full((B, 12, T, 128), 7.0, dtype=torch.bfloat16, device=cuda)
    pagedkv.paged_prefill(q.to(cuda), cache.buf[0, 0], cache.buf[0, 1], cache.block_tables,
                          rows_d, st + ql, max(p + n for p, n in zip(prior, qlen)), out, True,
                          1 / math.sqrt(128), 2, cache.err_flag, ql)
    torch.cuda.synchronize()
    cache.check_errors()
    for b in range(B):
        n = qlen[b]
        kd = torch.cat([hk[b], kn[b:b + 1, :, :n]], 2)
        vd = torch.cat([hv[b], vn[b:b + 1, :, :n]], 2)
        want = attention_ref.attention_np(q[b:b + 1, :, :n].float().numpy(), kd.float().numpy(),
                                          vd.float().numpy(), [prior[b] + n], True)
        assert max_err(out[b:b + 1, :, :n], want) < TOL, b
        assert bool((out[b, :, n:] == 7.0).all()), "padded query rows must not be written"
    # padded tokens were not stored: only the real tokens' slots changed
    changed = (cache.buf[0] != pool_before).any(-1).any(-1).any(0)  # [slots]
    expect = sum(qlen)
    assert int(changed.sum()) <= expect


@pytest.mark.parametrize("hq,hkv,B,T,causal", [(12, 2, 3, 700, True), (32, 2, 2, 300, True),
                                               (4, 2, 5, 129, True), (12, 2, 2, 256, False),
                                               (12, 4, 2, 200, True)])
def test_prefill_kernels_give_identical_bits(cuda, monkeypatch, hq, hkv, B, T, causal):
    """Two tensor-core prefill kernels: one head per CTA (P in tensor memory)
    and two q-heads of an even GQA group per CTA over shared K/V tiles (P
    staged in shared memory).  The per-head arithmetic is the same, so both
    give the same bits (and match the oracle).  PKV_PREFILL_KERNEL pins the
    kernel."""
    import pagedkv

    g = torch.Generator().manual_seed(hq * 100 + T)
    S = T + 37
    q = torch.randn(B, hq, T, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(B, hkv, S, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(B, hkv, S, 128, generator=g).to(torch.bfloat16)
    kv_lens = [S - (b * 13) % 29 for b in range(B)]
    outs = []
    kernels = ("one", "pair") if (hq // hkv) % 2 == 0 else ("one",)
    for force in kernels:
        monkeypatch.setenv("PKV_PREFILL_KERNEL", force)
        out = torch.full((B, hq, T, 128), 5.0, dtype=torch.bfloat16, device=cuda)
        pagedkv.dense_attention(q.to(cuda), k.to(cuda), v.to(cuda),
                                torch.tensor(kv_lens, dtype=torch.int32, device=cuda), out,
                                causal, 1 / math.sqrt(128))
        torch.cuda.synchronize()
        outs.append(out)
    for o in outs[1:]:
        assert torch.equal(outs[0], o)
    for b in range(B):
        want = attention_ref.attention_np(q[b:b + 1].float().numpy(), k[b:b + 1].float().numpy(),
                                          v[b:b + 1].float().numpy(), [kv_lens[b]], causal)
        assert max_err(outs[0][b:b + 1], want) < TOL, b


@pytest.mark.parametrize("prior,T", [([0, 0, 7], 300), ([1000, 3], 129)])
def test_paged_prefill_kernels_give_identical_bits(cuda, monkeypatch, prior, T):
    """Both prefill kernels on block-table K/V (shuffled, poisoned pool)."""
    from kernels.fa2 import flash_attention

    g = torch.Generator().manual_seed(sum(prior) * 3 + T)
    B = len(prior)
    N = sum(math.ceil((n + T) / 16) for n in prior) + 8
    cache = build_cache(N, torch.randperm(N, generator=g).tolist(), cuda)
    cache.buf.fill_(cases.PAD_VALUE)
    seqs = [cache.alloc() for _ in prior]
    hk = [torch.randn(1, 2, n, 128, generator=g).to(torch.bfloat16) for n in prior]
    hv = [torch.randn(1, 2, n, 128, generator=g).to(torch.bfloat16) for n in prior]
    write_history(cache, seqs, hk, hv)
    q = torch.randn(B, 12, T, 128, generator=g).to(torch.bfloat16)
    kn = torch.randn(B, 2, T, 128, generator=g).to(torch.bfloat16)
    vn = torch.randn(B, 2, T, 128, generator=g).to(torch.bfloat16)
    _, step, gidx = cache.prepare(seqs, T)
    cache.write(0, step, kn.to(cuda), vn.to(cuda))
    kh, vh = cache.read(0, gidx)
    outs = []
    for force in ("one", "pair"):
        monkeypatch.setenv("PKV_PREFILL_KERNEL", force)
        outs.append(flash_attention(q.to(cuda), kh, vh, True, step.kv_lens))
    torch.cuda.synchronize()
    cache.check_errors()
    for o in outs[1:]:
        assert torch.equal(outs[0], o)
    kd = torch.cat([hk[0], kn[0:1]], 2)
    vd = torch.cat([hv[0], vn[0:1]], 2)
    want = attention_ref.attention_np(q[0:1].float().numpy(), kd.float().numpy(),
                                      vd.float().numpy(), [prior[0] + T], True)
    assert max_err(outs[1][0:1], want) < TOL
