"""Decode-step kernels against plain PyTorch fp32 references (GPU)."""

import math
import os

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def rope_ref(x, cos, sin, pos):
    x = x.float()
    x1, x2 = x[..., :64], x[..., 64:]
    c, s = cos[pos][:, None, :], sin[pos][:, None, :]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def test_rope_qkv_cache(device, native):
    B, Hq, Hkv, L = 3, 8, 2, 40
    qkv = torch.randn(B, (Hq + 2 * Hkv) * 128, device=device).to(torch.bfloat16)
    ang = torch.arange(L, dtype=torch.float64)[:, None] / (5e5 ** (torch.arange(64, dtype=torch.float64) * 2 / 128))
    cos, sin = ang.cos().float().to(device), ang.sin().float().to(device)
    pos = torch.tensor([0, 7, 39], dtype=torch.int32, device=device)
    q = torch.empty(B, Hq, 128, dtype=torch.bfloat16, device=device)
    kc = torch.zeros(B, L, Hkv, 128, dtype=torch.bfloat16, device=device)
    vc = torch.zeros_like(kc)
    native.rope_qkv_cache(qkv, cos, sin, pos, q, kc, vc, Hq, Hkv)
    torch.cuda.synchronize()
    parts = qkv.view(B, Hq + 2 * Hkv, 128)
    p = pos.long()
    torch.testing.assert_close(q.float(), rope_ref(parts[:, :Hq], cos, sin, p), rtol=1e-2, atol=1e-2)
    for b in range(B):
        torch.testing.assert_close(kc[b, p[b]].float(), rope_ref(parts[b:b + 1, Hq:Hq + Hkv], cos, sin, p[b:b + 1])[0],
                                   rtol=1e-2, atol=1e-2)
        assert torch.equal(vc[b, p[b]], parts[b, Hq + Hkv:])


ATTENTION_SHAPES = [(1, 8, 1, 1025), (4, 8, 1, 300), (2, 64, 8, 129), (64, 8, 1, 1280), (3, 4, 4, 33),
                    (8, 8, 1, 1024), (2, 16, 1, 300), (1, 8, 1, 9000), (2, 8, 1, 128), (1, 1, 1, 200), (4, 16, 4, 257),
                    (32, 16, 2, 700), (8, 64, 8, 1024)]


@pytest.mark.parametrize("impl", [1, 2])
@pytest.mark.parametrize("B,Hq,Hkv,L", ATTENTION_SHAPES)
def test_decode_attention(device, native, B, Hq, Hkv, L, impl):
    """impl 1: the CUDA-core kernel; impl 2: the tensor-core kernel (tcgen05 QK^T and
    P V), where it takes the shape.  Both against fp32 attention, twice (PDL on the
    second call), counters and error word left at zero."""
    if impl == 2 and B * (L + 7) < 128:
        pytest.skip("the tensor-core kernel needs at least one 128-key tile of cache")
    Lmax = L + 7
    q = torch.randn(B, Hq, 128, device=device).to(torch.bfloat16)
    kc = torch.randn(B, Lmax, Hkv, 128, device=device).to(torch.bfloat16)
    vc = torch.randn(B, Lmax, Hkv, 128, device=device).to(torch.bfloat16)
    lengths = torch.randint(1, L + 1, (B,), dtype=torch.int32, device=device)
    lengths[0] = L
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    ws = torch.zeros(native.attention_workspace_floats(B, Hq, Hkv, L, sms), dtype=torch.float32, device=device)
    out = torch.empty(B, Hq, 128, dtype=torch.bfloat16, device=device)
    native.decode_attention(q, kc, vc, lengths, out, ws, L, 1 / math.sqrt(128), False, impl)
    again = torch.empty_like(out)
    # counters were left at zero; programmatic dependent launch computes the same
    native.decode_attention(q, kc, vc, lengths, again, ws, L, 1 / math.sqrt(128), True, impl)
    torch.cuda.synchronize()
    assert torch.equal(out, again)
    assert not ws[:4096].view(torch.int32).any()
    G = Hq // Hkv
    for b in range(B):
        n = int(lengths[b])
        k = kc[b, :n].float().repeat_interleave(G, dim=1)          # [n, Hq, 128]
        v = vc[b, :n].float().repeat_interleave(G, dim=1)
        s = torch.einsum("hd,nhd->hn", q[b].float(), k) / math.sqrt(128)
        ref = torch.einsum("hn,nhd->hd", s.softmax(-1), v)
        torch.testing.assert_close(out[b].float(), ref, rtol=2e-2, atol=2e-2)


def test_add_rmsnorm_silu_argmax(device, native):
    x = torch.randn(5, 8192, device=device).to(torch.bfloat16)
    r = torch.randn(5, 8192, device=device).to(torch.bfloat16)
    g = (1 + 0.02 * torch.randn(8192, device=device)).to(torch.bfloat16)
    out, rout = torch.empty_like(x), torch.empty_like(x)
    native.add_rmsnorm(x, r, rout, g, out, 1e-5)
    torch.cuda.synchronize()
    want_r = (x.float() + r.float()).to(torch.bfloat16)
    assert torch.equal(rout, want_r)
    want = (want_r.float() * torch.rsqrt(want_r.float().pow(2).mean(-1, keepdim=True) + 1e-5) * g.float())
    torch.testing.assert_close(out.float(), want, rtol=1e-2, atol=1e-2)
    gu = torch.randn(3, 2 * 1000, device=device).to(torch.bfloat16)
    act = torch.empty(3, 1000, dtype=torch.bfloat16, device=device)
    native.silu_mul(gu, act)
    torch.cuda.synchronize()
    g_, u_ = gu.float()[:, :1000], gu.float()[:, 1000:]
    torch.testing.assert_close(act.float(), torch.nn.functional.silu(g_) * u_, rtol=1e-2, atol=1e-2)
    # interleaved [64 gate | 64 up] column groups
    gu = torch.randn(3, 2 * 1024, device=device).to(torch.bfloat16)
    act = torch.empty(3, 1024, dtype=torch.bfloat16, device=device)
    native.silu_mul(gu, act, 64)
    torch.cuda.synchronize()
    v = gu.float().view(3, 16, 2, 64)
    want = (torch.nn.functional.silu(v[:, :, 0]) * v[:, :, 1]).reshape(3, 1024)
    torch.testing.assert_close(act.float(), want, rtol=1e-2, atol=1e-2)
    logits = torch.randn(4, 16032, device=device).to(torch.bfloat16)
    best = torch.empty(4, 2, dtype=torch.float32, device=device)
    native.row_argmax(logits, 1000, best)
    torch.cuda.synchronize()
    vals, idx = logits.float().max(-1)
    assert torch.equal(best[:, 0], vals) and torch.equal(best[:, 1].long(), idx + 1000)


@pytest.mark.parametrize("gemm", ["sparknet", "cublas"])
def test_tiny_model_step_matches_torch(device, native, gemm):
    from sparknet.models.llama import LlamaConfig, TPLlama

    cfg = LlamaConfig.tiny(layers=2)
    m = TPLlama(cfg, rank=0, world=1, device=device, batch=2, max_len=32, gemm=gemm)
    m.fill_prompt_cache(5)
    m.tokens.copy_(torch.tensor([3, 9], device=device))
    tokens0, pos0 = m.tokens.clone(), m.positions.clone().long()
    kcache0 = [L["k"].clone() for L in m.layers]
    vcache0 = [L["v"].clone() for L in m.layers]
    m.step_kernels()
    torch.cuda.synchronize()
    # fp32 reference of the same step
    f = lambda t: t.float()  # noqa: E731
    rms = lambda v, g: v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + cfg.eps) * f(g)  # noqa: E731
    res = f(m.embed[tokens0])
    x = rms(res, m.layers[0]["ln1"])
    from sparknet.ops.decode_gemm import split_gate_up

    for i, L in enumerate(m.layers):
        qkv = (x @ f(L["wqkv"]).T).view(2, -1, 128)
        q, k, v = qkv[:, :m.hq], qkv[:, m.hq:m.hq + m.hkv], qkv[:, m.hq + m.hkv:]
        q, k = rope_ref(q, m.cos, m.sin, pos0), rope_ref(k, m.cos, m.sin, pos0)
        outs = []
        for b in range(2):
            n = int(pos0[b]) + 1
            kk = torch.cat([f(kcache0[i][b, :n - 1]), k[b:b + 1]], 0).repeat_interleave(m.hq // m.hkv, 1)
            vv = torch.cat([f(vcache0[i][b, :n - 1]), v[b:b + 1]], 0).repeat_interleave(m.hq // m.hkv, 1)
            s = torch.einsum("hd,nhd->hn", q[b], kk) / math.sqrt(128)
            outs.append(torch.einsum("hn,nhd->hd", s.softmax(-1), vv))
        attn = torch.stack(outs).view(2, -1)
        res = res + attn @ f(L["wo"]).T
        x = rms(res, L["ln2"])
        gate, up = split_gate_up(L["wgu"])
        act = torch.nn.functional.silu(x @ f(gate).T) * (x @ f(up).T)
        res = res + act @ f(L["wdown"]).T
        x = rms(res, m.layers[i + 1]["ln1"] if i + 1 < len(m.layers) else m.norm)
    logits = x @ f(m.lm_head).T
    torch.testing.assert_close(m.logits.float(), logits, rtol=5e-2, atol=5e-2)
    assert torch.equal(m.positions.long(), pos0 + 1)


@pytest.mark.parametrize("M,N,K,swiglu,max_splits", [
    (1, 1280, 8192, False, 0), (8, 8192, 1024, False, 0), (8, 7168, 8192, True, 0), (33, 1000, 512, False, 0),
    (64, 2048, 3584, False, 0), (16, 512, 1024, False, 1), (200, 384, 256, True, 0), (8, 16032, 8192, False, 0),
    (64, 1000, 512, False, 1), (64, 1024, 512, True, 1), (37, 896, 2048, True, 3)])
def test_decode_gemm(device, native, M, N, K, swiglu, max_splits):
    from sparknet.ops.decode_gemm import DecodeGemm, split_gate_up

    gen = torch.Generator(device=device).manual_seed(M * 7 + N)
    x = torch.randn(M, K, generator=gen, device=device).to(torch.bfloat16)
    w = (0.02 * torch.randn(N, K, generator=gen, device=device)).to(torch.bfloat16)
    op = DecodeGemm(device, max_splits=max_splits)
    y = op(x, w, swiglu=swiglu)
    y2 = op(x, w, swiglu=swiglu)
    op.check()
    assert torch.equal(y, y2), "the split-K sum must not depend on CTA timing"
    if swiglu:
        gate, up = split_gate_up(w)
        want = torch.nn.functional.silu(x.float() @ gate.float().T) * (x.float() @ up.float().T)
    else:
        want = x.float() @ w.float().T
    torch.testing.assert_close(y.float(), want, rtol=2e-2, atol=2e-2)
    # programmatic dependent launch gives the same result
    y3 = DecodeGemm(device, max_splits=max_splits, pdl=True)(x, w, swiglu=swiglu)
    torch.cuda.synchronize()
    assert torch.equal(y, y3)


@pytest.mark.parametrize("B,Hq,Hkv", [(8, 8, 1), (3, 16, 2), (1, 8, 8)])
def test_decode_qkv_rope_epilogue(device, native, B, Hq, Hkv):
    from sparknet.ops.decode_gemm import DecodeGemm

    K, L = 1024, 48
    g = torch.Generator(device=device).manual_seed(B * 100 + Hq)
    x = torch.randn(B, K, generator=g, device=device).to(torch.bfloat16)
    w = (0.05 * torch.randn((Hq + 2 * Hkv) * 128, K, generator=g, device=device)).to(torch.bfloat16)
    ang = torch.arange(L, dtype=torch.float64)[:, None] / (5e5 ** (torch.arange(64, dtype=torch.float64) * 2 / 128))
    cos, sin = ang.cos().float().to(device), ang.sin().float().to(device)
    pos = torch.randint(0, L, (B,), dtype=torch.int32, device=device)
    q = torch.empty(B, Hq, 128, dtype=torch.bfloat16, device=device)
    kc = torch.zeros(B, L, Hkv, 128, dtype=torch.bfloat16, device=device)
    vc = torch.zeros_like(kc)
    op = DecodeGemm(device, pdl=True)
    op.qkv_rope(x, w, cos, sin, pos, q, kc, vc, Hq, Hkv)
    op.check()
    qkv = (x.float() @ w.float().T).view(B, Hq + 2 * Hkv, 128)
    p = pos.long()
    torch.testing.assert_close(q.float(), rope_ref(qkv[:, :Hq], cos, sin, p), rtol=2e-2, atol=2e-2)
    for b in range(B):
        torch.testing.assert_close(kc[b, p[b]].float(), rope_ref(qkv[b:b + 1, Hq:Hq + Hkv], cos, sin, p[b:b + 1])[0],
                                   rtol=2e-2, atol=2e-2)
        torch.testing.assert_close(vc[b, p[b]].float(), qkv[b, Hq + Hkv:], rtol=2e-2, atol=2e-2)
        others = torch.ones(L, dtype=torch.bool, device=device)
        others[p[b]] = False
        assert not kc[b, others].any() and not vc[b, others].any(), "wrote outside the token's position"


def test_attention_kernels_keep_the_step(device, native):
    """A decode step with the tensor-core attention gives the CUDA-core step's logits
    (within bf16): the two kernels are interchangeable inside the model."""
    from sparknet.models.llama import LlamaConfig, TPLlama

    cfg = LlamaConfig.tiny(layers=3)
    logits = []
    for attention in ("simt", "tcgen05"):
        m = TPLlama(cfg, rank=0, world=1, device=device, batch=4, max_len=256, attention=attention)
        m.fill_prompt_cache(150)
        m.tokens.copy_(torch.tensor([3, 9, 1, 4], device=device))
        m.step_kernels()
        m.step_kernels()
        torch.cuda.synchronize()
        logits.append(m.logits.float().clone())
    torch.testing.assert_close(logits[1], logits[0], rtol=5e-2, atol=5e-2)


def test_parallel_layer_decode_uses_the_decode_gemm(device, native):
    """ColumnParallelLinear.decode on few tokens: the tcgen05 decode GEMM, against fp32."""
    from sparknet.parallel.linear import ColumnParallelLinear

    w = (0.05 * torch.randn(1024, 512, device=device)).to(torch.bfloat16)
    x = torch.randn(8, 512, device=device).to(torch.bfloat16)
    layer = ColumnParallelLinear(w, runtime=None)
    y = layer.decode(x)
    torch.cuda.synchronize()
    torch.testing.assert_close(y.float(), x.float() @ w.float().T, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("variant", ["auto", "simt", "tcgen05"])
def test_ops_decode_attention_wrapper(device, native, variant):
    """sparknet.ops.decode_attention (its own workspace), every variant, against fp32, twice."""
    from sparknet.ops import decode_attention

    B, Hq, Hkv, L = 3, 16, 2, 200
    for _ in range(2):
        q = torch.randn(B, Hq, 128, device=device).to(torch.bfloat16)
        kc = torch.randn(B, L + 8, Hkv, 128, device=device).to(torch.bfloat16)
        vc = torch.randn(B, L + 8, Hkv, 128, device=device).to(torch.bfloat16)
        lengths = torch.tensor([L, 17, 150], dtype=torch.int32, device=device)
        out = decode_attention(q, kc, vc, lengths, L, variant=variant)
        torch.cuda.synchronize()
        G = Hq // Hkv
        for b in range(B):
            n = int(lengths[b])
            k = kc[b, :n].float().repeat_interleave(G, dim=1)
            v = vc[b, :n].float().repeat_interleave(G, dim=1)
            s = torch.einsum("hd,nhd->hn", q[b].float(), k) / math.sqrt(128)
            torch.testing.assert_close(out[b].float(), torch.einsum("hn,nhd->hd", s.softmax(-1), v),
                                       rtol=2e-2, atol=2e-2)
