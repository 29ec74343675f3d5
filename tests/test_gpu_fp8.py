"""Block-scaled fp8: quantisation and the tcgen05 kind::mxf8f6f4 GEMM (GPU), against
plain PyTorch fp32 references."""

import math

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _ue8m0(amax: torch.Tensor) -> torch.Tensor:
    """Exponent of the smallest power of two s with amax / s <= 448, as integers: from
    the float's exponent and mantissa (no transcendental functions)."""
    m, ex = torch.frexp(amax.double().cpu())        # amax = m * 2^ex, 0.5 <= m < 1
    # amax <= 448 * 2^k  <=>  k >= log2(amax / 448); with amax = (2m) * 2^(ex-1) and 448 = 1.75 * 2^8
    k = (ex.to(torch.int64) - 1 - 8) + (2 * m > 1.75).to(torch.int64)
    e = (k + 127).clamp(1, 254)
    return torch.where(amax.cpu() > 0, e, torch.full_like(e, 127))


@pytest.mark.parametrize("rows,k", [(200, 256), (128, 1024), (8, 128)])
def test_quantize_act(device, native, rows, k):
    from sparknet.ops import fp8

    x = (torch.randn(rows, k, device=device) * torch.logspace(-3, 3, k, device=device)).to(torch.bfloat16)
    q, sf = fp8.quantize_act(x)
    torch.cuda.synchronize()
    amax = x.float().abs().view(rows, k // 128, 128).amax(-1)
    want_e = _ue8m0(amax)
    got_e = fp8.scale_exponents(sf, rows, k).to(torch.int64).cpu()
    assert torch.equal(got_e, want_e)
    deq = fp8.dequantize(q, sf)
    scale = fp8.scales_to_dense(sf, rows, k).repeat_interleave(128, 1)
    # e4m3: 3 mantissa bits -> relative error <= 2^-4, plus subnormal spacing 2^-9 * scale
    assert ((deq - x.float()).abs() <= x.float().abs() * 2 ** -4 + scale * 2 ** -9).all()


def test_quantize_weight(device, native):
    from sparknet.ops import fp8

    N, K = 384, 512
    w = (0.02 * torch.randn(N, K, device=device)).to(torch.bfloat16)
    w[:128, :128] *= 1000
    q, sf = fp8.quantize_weight(w)
    torch.cuda.synchronize()
    s = fp8.scales_to_dense(sf, N, K)
    amax = w.float().abs().view(N // 128, 128, K // 128, 128).amax((1, 3))
    want_e = _ue8m0(amax).repeat_interleave(128, 0)
    assert torch.equal(fp8.scale_exponents(sf, N, K).to(torch.int64).cpu(), want_e)
    deq = fp8.dequantize(q, sf)
    scale = s.repeat_interleave(128, 1)
    assert ((deq - w.float()).abs() <= w.float().abs() * 2 ** -4 + scale * 2 ** -9).all()


@pytest.mark.parametrize("M,N,K", [(256, 256, 512), (200, 384, 256), (1024, 2048, 4096), (128, 128, 128)])
def test_gemm_fp8(device, native, M, N, K):
    from sparknet.ops import fp8

    g = torch.Generator(device=device).manual_seed(M + N + K)
    x = torch.randn(M, K, generator=g, device=device).to(torch.bfloat16)
    w = (0.02 * torch.randn(N, K, generator=g, device=device)).to(torch.bfloat16)
    xq, sx = fp8.quantize_act(x)
    wq, sw = fp8.quantize_weight(w)
    y = fp8.gemm_fp8(xq, sx, wq, sw, check=True)
    want = fp8.dequantize(xq, sx) @ fp8.dequantize(wq, sw).T
    torch.testing.assert_close(y.float(), want, rtol=1e-2, atol=1e-2 * want.abs().max().item())
    # and close to the bf16 product (quantisation error only)
    ref = x.float() @ w.float().T
    rel = (y.float() - ref).norm() / ref.norm()
    assert rel < 0.08, rel


def test_gemm_fp8_scales_apply_per_block(device, native):
    """Blocks with very different magnitudes: a wrong scale placement shows at once."""
    from sparknet.ops import fp8

    M, N, K = 256, 256, 512
    x = torch.randn(M, K, device=device)
    x *= torch.exp2(torch.randint(-8, 8, (M, K // 128), device=device).float()).repeat_interleave(128, 1)
    w = 0.02 * torch.randn(N, K, device=device)
    w *= torch.exp2(torch.randint(-6, 6, (N // 128, K // 128), device=device).float()).repeat_interleave(
        128, 0).repeat_interleave(128, 1)
    xq, sx = fp8.quantize_act(x.to(torch.bfloat16))
    wq, sw = fp8.quantize_weight(w.to(torch.bfloat16))
    y = fp8.gemm_fp8(xq, sx, wq, sw, check=True)
    want = fp8.dequantize(xq, sx) @ fp8.dequantize(wq, sw).T
    err = ((y.float() - want).abs() / (want.abs() + 1e-3 * want.abs().max())).max().item()
    assert err < 2e-2, err
    assert not math.isnan(y.float().sum().item())
