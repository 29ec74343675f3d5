"""tcgen05 GEMM numerics against a plain PyTorch fp32 reference (GPU)."""

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 128), (1000, 1280, 1024), (384, 4096, 8192),
                                   (4096, 1280, 8192), (130, 96, 192), (1000, 1344, 1024), (4096, 7168, 512)])
@pytest.mark.parametrize("block_n", [256, 128, "pair"])
def test_gemm_matches_fp32(device, native, M, N, K, block_n):
    from sparknet.ops.gemm import gemm

    g = torch.Generator(device=device).manual_seed(M + N + K)
    a = torch.randn(M, K, generator=g, device=device).to(torch.bfloat16)
    b = torch.randn(N, K, generator=g, device=device).to(torch.bfloat16)
    c = gemm(a, b, block_n=block_n, check=True)
    ref = a.float() @ b.float().T
    err = (c.float() - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= 1e-2 * scale, (err, scale)


def test_gemm_throughput(device, native):
    """Not a threshold test: records TFLOP/s of a prefill-shaped GEMM next to cuBLAS."""
    from sparknet.ops.gemm import gemm

    M, N, K = 8192, 7168, 8192
    a = torch.randn(M, K, device=device).to(torch.bfloat16)
    b = torch.randn(N, K, device=device).to(torch.bfloat16)
    c = torch.empty(M, N, dtype=torch.bfloat16, device=device)
    for _ in range(3):
        gemm(a, b, c, block_n=256)
        gemm(a, b, c, block_n="pair")
        torch.mm(a, b.T)
    torch.cuda.synchronize()
    res = {}
    for name, fn in (("tcgen05", lambda: gemm(a, b, c, block_n=256)), ("tcgen05_pair", lambda: gemm(a, b, c, block_n="pair")),
                     ("cublas", lambda: torch.mm(a, b.T))):
        st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        st.record()
        for _ in range(10):
            fn()
        en.record()
        en.synchronize()
        res[name] = 2 * M * N * K * 10 / (st.elapsed_time(en) / 1000) / 1e12
    print(f"\nGEMM {M}x{N}x{K} TFLOP/s: {res}")
    gemm(a, b, c, block_n=256, check=True)
    gemm(a, b, c, block_n="pair", check=True)
    assert res["tcgen05"] > 100 and res["tcgen05_pair"] > 100


def test_fp8_gemm_throughput(device, native):
    """Block-scaled fp8 tcgen05 GEMM at a prefill shape; prints TFLOP/s beside bf16."""
    from sparknet.ops import fp8
    from sparknet.ops.gemm import gemm

    M, N, K = 8192, 7168, 8192
    x = torch.randn(M, K, device=device).to(torch.bfloat16)
    w = (0.02 * torch.randn(N, K, device=device)).to(torch.bfloat16)
    xq, sx = fp8.quantize_act(x)
    wq, sw = fp8.quantize_weight(w)
    y = torch.empty(M, N, dtype=torch.bfloat16, device=device)

    def t(fn, reps=10):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        st.record()
        for _ in range(reps):
            fn()
        en.record()
        en.synchronize()
        return st.elapsed_time(en) / reps

    f8 = 2 * M * N * K / (t(lambda: fp8.gemm_fp8(xq, sx, wq, sw, y)) * 1e-3) / 1e12
    bf = 2 * M * N * K / (t(lambda: gemm(x, w, y)) * 1e-3) / 1e12
    print(f"\nGEMM {M}x{N}x{K} TFLOP/s: fp8 block-scaled {f8:.0f}, bf16 {bf:.0f}")
    fp8.gemm_fp8(xq, sx, wq, sw, y, check=True)
    assert f8 > 0
