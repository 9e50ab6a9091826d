"""Skinny tensor-core linear entries (pkv_linear*) on the GPU.

The plain GEMM is checked against an fp64 product of the same bf16 inputs
(the nn.Linear the reference runs, model.py:83-86 and :114-116, up to fp32
summation order and one bf16 rounding), for row counts that exercise one
split and cluster split-k reductions of up to 16 CTAs.  The fused entries
must equal, bit for bit, the plain GEMM followed by the separate kernel they
fuse (add_rmsnorm, silu_mul, append_rope).
"""
import ctypes
import math

import pytest
import torch
import torch.nn.functional as F

from gpu_helpers import build_cache

pytestmark = pytest.mark.gpu

# the Qwen2.5-1.5B projections (n, k): q/k/v merged, o, gate/up merged, down
SHAPES = [(2048, 1536), (1536, 1536), (17920, 1536), (1536, 8960)]
ROWS = [1, 7, 16, 33, 64, 100, 128, 200, 256]


def _operands(rows, n, k, device, seed, bias=True):
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(rows, k, device=device, generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn(n, k, device=device, generator=g)).to(torch.bfloat16)
    b = (0.02 * torch.randn(n, device=device, generator=g)).to(torch.bfloat16) if bias else None
    return x, w, b


def _ref(x, w, b):
    y = x.double() @ w.double().T
    if b is not None:
        y = y + b.double()
    return y


def _check_close(got, want):
    # fp32 accumulation of k products, then one bf16 rounding (2^-8 relative)
    d = (got.double() - want).abs()
    lim = 4e-3 + 2 ** -8 * want.abs()
    assert bool((d <= lim).all()), float((d - lim).max())


@pytest.mark.parametrize("n,k", SHAPES)
@pytest.mark.parametrize("rows", ROWS)
def test_linear_matches_fp64_product(cuda, rows, n, k):
    import pagedkv

    x, w, b = _operands(rows, n, k, cuda, rows * 7 + n)
    y = pagedkv.linear(x, w, b)
    torch.cuda.synchronize()
    _check_close(y, _ref(x, w, b))
    # deterministic: split-k partials are added in a fixed order
    assert torch.equal(pagedkv.linear(x, w, b), y)
    # and no worse than cuBLAS through F.linear
    ref = _ref(x, w, b)
    e_ours = float((y.double() - ref).abs().max())
    e_cublas = float((F.linear(x, w, b).double() - ref).abs().max())
    assert e_ours <= 2 * e_cublas + 1e-3


@pytest.mark.parametrize("n,k", SHAPES)
@pytest.mark.parametrize("rows", [1, 16, 128, 256])
def test_tiled_weight_gives_identical_results(cuda, rows, n, k):
    import pagedkv

    x, w, b = _operands(rows, n, k, cuda, rows + 3 * n)
    wt = pagedkv.TiledWeight(w)
    # the packed layout is exactly [n/128][k/64][128][64]
    want = w.view(n // 128, 128, k // 64, 64).permute(0, 2, 1, 3).reshape(-1)
    assert torch.equal(wt.data, want)
    assert torch.equal(pagedkv.linear(x, wt, b), pagedkv.linear(x, w, b))


def test_linear_strided_rows_and_out(cuda):
    import pagedkv

    x_big, w, b = _operands(24, 2048, 1536 + 64, cuda, 3)
    x = x_big[:, :1536]  # row stride 1600
    w = w[:, :1536].contiguous()
    out = torch.full((24, 2048 + 128), 7.0, device=cuda, dtype=torch.bfloat16)
    pagedkv.linear(x, w, b, out=out[:, :2048])
    torch.cuda.synchronize()
    _check_close(out[:, :2048], _ref(x, w, b))
    assert bool((out[:, 2048:] == 7.0).all())


@pytest.mark.parametrize("rows", [1, 16, 128, 256])
@pytest.mark.parametrize("k", [1536, 8960])
def test_linear_add_rmsnorm_equals_two_step(cuda, rows, k):
    import pagedkv

    x, w, _ = _operands(rows, 1536, k, cuda, rows + k, bias=False)
    g = torch.Generator(device=cuda).manual_seed(5)
    resid = (3 * torch.randn(rows, 1536, device=cuda, generator=g)).to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(1536, device=cuda, generator=g)).to(torch.bfloat16)
    r1, r2 = resid.clone(), resid.clone()
    want = pagedkv.add_rmsnorm(pagedkv.linear(x, w), r1, nw, 1e-6, resid_out=r1)
    got = pagedkv.linear_add_rmsnorm(x, w, r2, nw, 1e-6, resid_out=r2)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert torch.equal(r2, r1)


@pytest.mark.parametrize("rows", [1, 16, 128, 256])
def test_linear_silu_mul_equals_two_step(cuda, rows):
    import pagedkv

    x, w, _ = _operands(rows, 17920, 1536, cuda, rows, bias=False)
    want = pagedkv.silu_mul(pagedkv.linear(x, w))
    got = pagedkv.linear_silu_mul(x, w)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    # and the reference op sequence (model.py:120) within bf16 rounding
    gu = F.linear(x, w)
    ref = F.silu(gu[:, :8960]) * gu[:, 8960:]
    assert float((got.float() - ref.float()).abs().max()) < 2e-2


@pytest.mark.parametrize("rows", [1, 7, 16, 33, 64, 128, 256])
def test_paired_gate_up_swiglu_epilogue_equals_two_step(cuda, rows):
    """PKV_W_GATE_UP_PAIRED: SwiGLU finished in the GEMM's epilogue gives the
    bits of GEMM -> silu_mul on the original weight."""
    import pagedkv

    x, w, _ = _operands(rows, 17920, 1536, cuda, 40 + rows, bias=False)
    wp = pagedkv.PairedGateUp(w)
    gate = w[:8960].view(140, 64, 1536)
    up = w[8960:].view(140, 64, 1536)
    assert torch.equal(wp.data.view(140, 128, 1536), torch.cat([gate, up], dim=1))
    want = pagedkv.silu_mul(pagedkv.linear(x, w))
    out = torch.full((rows, 8960 + 64), 3.0, device=cuda, dtype=torch.bfloat16)
    got = pagedkv.linear_silu_mul(x, wp, out=out[:, :8960])
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert bool((out[:, 8960:] == 3.0).all())
    with pytest.raises(pagedkv.PagedKVError, match="silu_mul only"):
        pagedkv.linear(x, wp)


@pytest.mark.parametrize("q_layout", ["dense", "padded"])
@pytest.mark.parametrize("B,T", [(1, 1), (16, 1), (128, 1), (256, 1), (1, 200), (3, 40)])
def test_linear_rope_append_equals_two_step(cuda, B, T, q_layout):
    """dense q_out: RoPE + append run in the GEMM's epilogue; padded q_out
    rows (stride 130, not a multiple of 8): GEMM + append kernel.  Both must
    give the two-step result bit for bit."""
    import model as M
    import pagedkv

    x, w, b = _operands(B * T, 2048, 1536, cuda, B * 1000 + T)
    cos, sin = M.rope_table(8192, torch.bfloat16, cuda)
    caches, outs = [], []
    g = torch.Generator().manual_seed(B + T)
    lens = torch.randint(0, 3000, (B,), generator=g).tolist()
    N = sum(math.ceil((n + T) / 16) for n in lens) + 4
    perm = torch.randperm(N, generator=g).tolist()
    for fused in (False, True):
        cache = build_cache(N, perm, cuda)
        seqs = [cache.alloc() for _ in range(B)]
        for s, n in zip(seqs, lens):
            cache._lengths[s] = n  # a history of n tokens (contents irrelevant here)
        _, step, _ = cache.prepare(seqs, T)  # reserves blocks for n + T tokens
        width = 128 if q_layout == "dense" else 130
        q_rot = torch.full((B, T, 12, width), float("nan"), device=cuda,
                           dtype=torch.bfloat16)[..., :128]
        if fused:
            pagedkv.linear_rope_append(x, w, b, cos, sin, q_rot.transpose(1, 2),
                                       cache.buf[0, 0], cache.buf[0, 1], cache.block_tables,
                                       step.rows, step.starts, 2, err=cache.err_flag)
        else:
            qkv = pagedkv.linear(x, w, b).view(B, T, 16, 128)
            cache.append(0, step, qkv[:, :, :12].transpose(1, 2), qkv[:, :, 12:14].transpose(1, 2),
                         qkv[:, :, 14:].transpose(1, 2), cos, sin, q_rot.transpose(1, 2))
        torch.cuda.synchronize()
        cache.check_errors()
        caches.append(cache)
        outs.append(q_rot)
    assert torch.equal(outs[0], outs[1])
    assert torch.equal(caches[0].buf, caches[1].buf)


def test_linear_rejections(cuda):
    import pagedkv

    L = pagedkv.lib()
    x, w, _ = _operands(300, 2048, 1536, cuda, 1, bias=False)
    with pytest.raises(pagedkv.PagedKVError, match="rows"):
        pagedkv.linear(x, w)
    with pytest.raises(pagedkv.PagedKVError, match="multiple of 128"):
        pagedkv.linear(x[:16], w[:2000])
    # a fused entry with a workspace smaller than its bf16 intermediate:
    # refused before any launch
    x2, w2, _ = _operands(16, 1536, 8960, cuda, 2, bias=False)
    need = L.pkv_linear_workspace_size(16, 1536, 8960)
    assert need == 16 * 1536 * 2
    ws = torch.empty(need - 16, dtype=torch.uint8, device=cuda)
    resid = torch.zeros(16, 1536, device=cuda, dtype=torch.bfloat16)
    nw = torch.ones(1536, device=cuda, dtype=torch.bfloat16)
    out = torch.zeros(16, 1536, device=cuda, dtype=torch.bfloat16)
    st = L.pkv_linear_add_rmsnorm(
        x2.data_ptr(), x2.stride(0), w2.data_ptr(), w2.stride(0), 0, 16, 1536, 8960,
        resid.data_ptr(), 1536, resid.data_ptr(), 1536, nw.data_ptr(), 1e-6, out.data_ptr(), 1536,
        ws.data_ptr(), ws.numel(), None, torch.cuda.current_stream().cuda_stream)
    assert st == 6  # PKV_ERR_WORKSPACE
    torch.cuda.synchronize()
    assert int(out.count_nonzero()) == 0
