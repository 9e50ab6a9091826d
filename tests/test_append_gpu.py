"""Fused RoPE + K/V append through the C ABI: bit-exact with the reference."""
import numpy as np
import pytest
import torch

from gpu_helpers import build_cache
from oracle import cases, rope_ref
from oracle.kvcache_ref import RefKVCache

pytestmark = pytest.mark.gpu


def test_append_rope_matches_reference_bits(cuda, golden):
    import model

    fx = np.load(golden / "rope_append.npz")
    N, layer, T = int(fx["num_blocks"]), int(fx["layer"]), int(fx["T"])
    cache = build_cache(N, fx["perm"], cuda)
    cache.buf[layer].copy_(cases.from_bits(fx["pool_before"]).view(cache.buf[layer].shape))
    starts = [int(x) for x in fx["starts"]]
    seqs = [cache.alloc() for _ in starts]
    for s, n in zip(seqs, starts):
        cache.ensure_capacity(s, n)
        cache._lengths[s] = n
    st, step, _ = cache.prepare(seqs, T)
    cos, sin = model.rope_table(cache.table_pitch * 16, torch.bfloat16, cuda)
    q = cases.from_bits(fx["q"]).to(cuda)
    k = cases.from_bits(fx["k"]).to(cuda)
    v = cases.from_bits(fx["v"]).to(cuda)
    q_out = torch.empty_like(q)
    cache.append(layer, step, q, k, v, cos, sin, q_out)
    torch.cuda.synchronize()
    cache.check_errors()
    assert np.array_equal(cases.bits(q_out.cpu()), fx["q_roped"])
    assert np.array_equal(cases.bits(cache.buf[layer].cpu()), fx["pool_after"])
    others = torch.cat([cache.buf[:layer], cache.buf[layer + 1:]])
    assert int(others.count_nonzero()) == 0
    # the device block tables equal the reference's host tables
    for i, s in enumerate(seqs):
        t = [x for x in fx["tables"][i] if x >= 0]
        assert cache.block_tables[cache.table_row(s), :len(t)].tolist() == t


@pytest.mark.parametrize("width", [128, 130])
@pytest.mark.parametrize("T,B", [(1, 7), (16, 3), (37, 2), (300, 1)])
def test_append_random_strided_inputs_vs_oracle(cuda, T, B, width):
    """Non-contiguous q/k/v (the projections' transposed views) and a table
    that crosses block boundaries mid-step; every pool byte is checked.
    width 128: 8-byte aligned rows (the one-warp-per-token kernel); width
    130: head rows 260 bytes apart (the one-warp-per-head kernel)."""
    import model

    g = torch.Generator().manual_seed(100 + T)
    N = 64
    perm = torch.randperm(N, generator=g).tolist()
    cache = build_cache(N, perm, cuda)
    ref = RefKVCache(N, 16, dtype=torch.bfloat16, num_layers=1)
    ref.free_blocks = list(perm)
    prior = [int(x) for x in torch.randint(0, 40, (B,), generator=g)]
    seqs = [cache.alloc() for _ in range(B)]
    rseqs = [ref.alloc() for _ in range(B)]
    for s, r, n in zip(seqs, rseqs, prior):
        cache.ensure_capacity(s, n)
        cache._lengths[s] = n
        ref.ensure_capacity(r, n)
        ref.lengths[r] = n
    x_full = (torch.randn(B, T, 12 + 2 + 2, width, generator=g) * 3).to(torch.bfloat16)
    x = x_full[..., :128]
    q, k, v = (t.transpose(1, 2) for t in x.split([12, 2, 2], dim=2))  # strided views
    st, step, _ = cache.prepare(seqs, T)
    rst, slot, _ = ref.prepare(rseqs, T)
    cos, sin = model.rope_table(cache.table_pitch * 16, torch.bfloat16, cuda)
    q_out = torch.empty(B, T, 12, 128, dtype=torch.bfloat16, device=cuda).transpose(1, 2)
    xd = x_full.to(cuda)[..., :128]  # keeps the padded row stride on the device
    qd, kd, vd = (t.transpose(1, 2) for t in xd.split([12, 2, 2], dim=2))
    cache.append(5, step, qd, kd, vd, cos, sin, q_out)
    torch.cuda.synchronize()
    cache.check_errors()
    pos = np.array(st)[:, None] + np.arange(T)[None, :]
    c, s = rope_ref.rope_table_bits(pos.reshape(-1))
    c = c.reshape(B, 1, T, 128)
    s = s.reshape(B, 1, T, 128)
    assert np.array_equal(cases.bits(q_out.cpu()), rope_ref.rope_bits(cases.bits(q), c, s))
    kr = cases.from_bits(rope_ref.rope_bits(cases.bits(k), c, s))
    ref.write(0, slot, kr, v)
    assert np.array_equal(cases.bits(cache.buf[5].cpu()), cases.bits(ref.buf[0]))


def test_write_without_rope_is_reference_index_copy(cuda):
    g = torch.Generator().manual_seed(3)
    N = 40
    perm = torch.randperm(N, generator=g).tolist()
    cache = build_cache(N, perm, cuda)
    ref = RefKVCache(N, 16, dtype=torch.bfloat16, num_layers=1)
    ref.free_blocks = list(perm)
    seqs, rseqs = [cache.alloc(), cache.alloc()], [ref.alloc(), ref.alloc()]
    for T in (5, 1, 17, 1, 40):
        k = torch.randn(2, 2, T, 128, generator=g).to(torch.bfloat16)
        v = torch.randn(2, 2, T, 128, generator=g).to(torch.bfloat16)
        _, step, _ = cache.prepare(seqs, T)
        _, slot, _ = ref.prepare(rseqs, T)
        cache.write(2, step, k.to(cuda), v.to(cuda))
        ref.write(0, slot, k, v)
        cache.advance(seqs, T)
        ref.advance(rseqs, T)
    torch.cuda.synchronize()
    cache.check_errors()
    assert np.array_equal(cases.bits(cache.buf[2].cpu()), cases.bits(ref.buf[0]))


def test_bad_block_id_is_flagged_not_faulted(cuda):
    """An out-of-range table entry is caught by the kernel's bounds check: the
    write is skipped and PKV_DEVERR_BLOCK_ID raised on the host."""
    cache = build_cache(8, list(range(8)), cuda)
    s = cache.alloc()
    _, step, _ = cache.prepare([s], 1)
    cache.block_tables[cache.table_row(s), 0] = 1_000_000  # corrupt the device copy
    k = torch.ones(1, 2, 1, 128, dtype=torch.bfloat16, device=cuda)
    before = cache.buf.clone()
    cache.write(0, step, k, k)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="device error bits 0x1"):
        cache.check_errors()
    assert torch.equal(cache.buf, before)
