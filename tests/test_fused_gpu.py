"""Fused block kernels vs the reference's torch op sequences (model.py:49-55,
:120, :136-137) on the GPU."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _ref_rmsnorm(x, w, eps):
    # model.py:49-55 verbatim op order
    dt = x.dtype
    x = x.to(torch.float32)
    variance = x.pow(2).mean(-1, keepdim=True)
    x = x * torch.rsqrt(variance + eps)
    return w * x.to(dt)


@pytest.mark.parametrize("rows", [1, 16, 333])
def test_add_rmsnorm_matches_reference_ops(cuda, rows):
    import pagedkv

    g = torch.Generator(device=cuda).manual_seed(rows)
    a = (torch.randn(rows, 1536, device=cuda, generator=g) * 3).to(torch.bfloat16)
    r = (torch.randn(rows, 1536, device=cuda, generator=g) * 3).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(1536, device=cuda, generator=g)).to(torch.bfloat16)
    h_ref = r + a                       # bf16 residual add
    want = _ref_rmsnorm(h_ref, w, 1e-6)
    r_io = r.clone()
    got = pagedkv.add_rmsnorm(a, r_io, w, 1e-6, resid_out=r_io)
    assert torch.equal(r_io, h_ref), "residual stream must be the exact bf16 sum"
    # only the fp32 mean's summation order differs: at most 1 bf16 ulp, rarely
    d = (got.float() - want.float()).abs()
    ulp = want.float().abs().clamp_min(1e-30) * 2 ** -7
    assert bool((d <= ulp).all())
    assert float((d > 0).float().mean()) < 0.01
    # no residual: plain RMSNorm
    got2 = pagedkv.add_rmsnorm(a, None, w, 1e-6)
    d2 = (got2.float() - _ref_rmsnorm(a, w, 1e-6).float()).abs()
    assert float((d2 > 0).float().mean()) < 0.01


def test_add_rmsnorm_strided_rows(cuda):
    """Last-position rows of a [B, T, H] activation (row stride T*H)."""
    import pagedkv

    x = torch.randn(4, 7, 1536, device=cuda).to(torch.bfloat16)
    m = torch.randn(4, 7, 1536, device=cuda).to(torch.bfloat16)
    w = torch.ones(1536, device=cuda, dtype=torch.bfloat16)
    got = pagedkv.add_rmsnorm(m[:, -1], x[:, -1], w, 1e-6)
    want = _ref_rmsnorm(x[:, -1] + m[:, -1], w, 1e-6)
    assert float((got.float() - want.float()).abs().max()) < 0.05


@pytest.mark.parametrize("rows", [1, 16, 500])
def test_silu_mul_is_bit_exact(cuda, rows):
    import pagedkv

    g = torch.Generator(device=cuda).manual_seed(7)
    gu = (torch.randn(rows, 2 * 8960, device=cuda, generator=g) * 4).to(torch.bfloat16)
    want = F.silu(gu[:, :8960]) * gu[:, 8960:]
    got = pagedkv.silu_mul(gu)
    assert torch.equal(got, want)
