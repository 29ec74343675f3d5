"""The tensor-parallel layers' routing on CPU: which runtime call each path makes, with
which arguments (a recording stand-in for the runtime; the kernels have GPU tests)."""

import pytest

torch = pytest.importorskip("torch")

from sparknet.parallel import linear as L  # noqa: E402


class Recorder:
    def __init__(self):
        self.calls = []

    def __getattr__(self, name):
        def call(*args, **kwargs):
            self.calls.append((name, args, kwargs))
            return name
        return call


def test_bf16_forward_routes_to_the_fused_kernels():
    rt = Recorder()
    w = torch.zeros(256, 512, dtype=torch.bfloat16)
    col = L.ColumnParallelLinear(w, rt)
    x = torch.zeros(128, 512, dtype=torch.bfloat16)
    assert col.forward(x) == "ag_gemm"
    name, args, kwargs = rt.calls[-1]
    assert args[1] is col.weight and kwargs == {"out": None}
    row = L.RowParallelLinear(w, rt)
    assert row.forward(x) == "gemm_rs" and rt.calls[-1][2] == {"out": None}


def test_fp8_forward_quantises_once_per_weight_and_per_call(monkeypatch):
    from sparknet.ops import fp8

    seen = []
    monkeypatch.setattr(fp8, "quantize_weight", lambda w: seen.append(("w", tuple(w.shape))) or ("wq", "sw"))
    monkeypatch.setattr(fp8, "quantize_act", lambda x: seen.append(("x", tuple(x.shape))) or ("xq", "sx"))
    rt = Recorder()
    w = torch.zeros(256, 512, dtype=torch.bfloat16)
    col = L.ColumnParallelLinear(w, rt, fp8=True)
    row = L.RowParallelLinear(w, rt, fp8=True)
    x = torch.zeros(128, 512, dtype=torch.bfloat16)
    col.forward(x)
    col.forward(x)
    row.forward(x)
    assert seen == [("w", (256, 512)), ("w", (256, 512)), ("x", (128, 512)), ("x", (128, 512)), ("x", (128, 512))]
    assert [c[0] for c in rt.calls] == ["ag_gemm_fp8", "ag_gemm_fp8", "gemm_rs_fp8"]
    assert rt.calls[0][1] == ("xq", "sx", "wq", "sw") and rt.calls[2][1] == ("xq", "sx", "wq", "sw")
    with pytest.raises(ValueError, match="multiple of 128"):
        L.ColumnParallelLinear(torch.zeros(200, 512, dtype=torch.bfloat16), rt, fp8=True)


def test_decode_product_outside_the_decode_gemm_limits_is_a_matmul():
    w = torch.randn(64, 96).to(torch.bfloat16)
    x = torch.randn(3, 96).to(torch.bfloat16)       # CPU tensors, K not a multiple of 64
    col = L.ColumnParallelLinear(w, Recorder())
    torch.testing.assert_close(col.decode(x).float(), (x.float() @ w.float().T), rtol=2e-2, atol=2e-2)
    rt = Recorder()
    row = L.RowParallelLinear(w, rt)
    res, gamma = torch.zeros(3, 64, dtype=torch.bfloat16), torch.ones(64, dtype=torch.bfloat16)
    assert row.decode(x, res, gamma) == "all_reduce_residual_rmsnorm"
    name, args, kwargs = rt.calls[-1]
    assert args[1] is res and kwargs == {"residual_out": res}


def test_weights_must_be_bf16_matrices():
    with pytest.raises(ValueError, match="bfloat16"):
        L.RowParallelLinear(torch.zeros(4, 4), Recorder())
