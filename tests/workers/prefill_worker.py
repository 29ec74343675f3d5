"""One rank of the fused prefill GEMM check and benchmark (AG->GEMM, GEMM->RS).

Correctness at small shapes against fp32 torch; then timing at the BASELINE prefill
shapes (8192 tokens, hidden 8192, FFN 28672, TP = world) of the fused kernels and of
the unfused NCCL + cuBLAS sequence, device-timed, max over ranks.  One JSON file per
rank into $SPARKNET_TEST_OUT (or stdout from rank 0 with --print).
"""

import json
import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def timed(fn, reps=5):
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record()
    for _ in range(reps):
        fn()
    en.record()
    en.synchronize()
    return st.elapsed_time(en) / reps


def gathered_fp32(shard):
    """Every rank's shard (NCCL all-gather of the bf16 values), stacked in rank order, in fp32."""
    parts = [torch.empty_like(shard) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, shard.contiguous())
    return torch.cat(parts).float()


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("cpu:gloo,cuda:nccl", timeout=timedelta(seconds=120), device_id=device)
    rank, world = dist.get_rank(), dist.get_world_size()
    cpu = dist.new_group(backend="gloo", timeout=timedelta(seconds=120))
    from sparknet.oneshot import AllReduce
    from sparknet.ops.prefill import ag_gemm_reference, gemm_rs_reference

    T, H, F = 8192, 8192, 28672
    shard_bytes = (T // world) * max(H, F // world) * 2
    rt = AllReduce.from_exchange_group(exchange_group=cpu, device=device, max_size=8 << 20,
                                       max_gather_bytes=max(16 << 20, shard_bytes))
    rt.set_timeout_ms(10000)
    failures, results = [], {"rank": rank, "world": world}
    g = torch.Generator(device=device).manual_seed(100 + rank)
    # -- correctness (small)
    t, k, n = 256 * world, 512, 768
    x = torch.randn(t // world, k, generator=g, device=device).to(torch.bfloat16)
    w = (0.05 * torch.randn(n, k, generator=g, device=device)).to(torch.bfloat16)
    got = rt.ag_gemm(x, w)
    want = gathered_fp32(x) @ w.float().T  # fp32 product of the gathered operands
    torch.cuda.synchronize()
    err = (got.float() - want).abs().max().item() / max(1e-6, want.abs().max().item())
    if err > 1e-2:  # bf16 output rounding is 2^-9 relative
        failures.append(f"ag_gemm relative error {err}")
    a = torch.randn(t, k, generator=g, device=device).to(torch.bfloat16)
    got = rt.gemm_rs(a, w[:512])
    full = [torch.empty_like(a) for _ in range(world)]
    dist.all_gather(full, a)
    ws = [torch.empty_like(w[:512]) for _ in range(world)]
    dist.all_gather(ws, w[:512].contiguous())
    ref = sum((full[s].float() @ ws[s].float().T) for s in range(world))[rank * (t // world):(rank + 1) * (t // world)]
    torch.cuda.synchronize()
    err = (got.float() - ref).abs().max().item() / max(1e-6, ref.abs().max().item())
    if err > 2e-2:
        failures.append(f"gemm_rs relative error {err}")
    if rt.gemm_error() or rt.failure():
        failures.append(f"error word {rt.gemm_error()} / {rt.failure()}")
    # -- block-scaled fp8 forms, against fp32 matmuls of the dequantised operands
    from sparknet.ops import fp8

    xq, sx = fp8.quantize_act(x)
    wq, sw = fp8.quantize_weight(w)
    got = rt.ag_gemm_fp8(xq, sx, wq, sw)
    xd = fp8.dequantize(xq, sx)
    parts = [torch.empty_like(xd) for _ in range(world)]
    dist.all_gather(parts, xd)
    want = torch.cat(parts) @ fp8.dequantize(wq, sw).T
    torch.cuda.synchronize()
    err = (got.float() - want).abs().max().item() / max(1e-6, want.abs().max().item())
    if err > 1e-2:
        failures.append(f"ag_gemm_fp8 relative error {err}")
    aq, sa = fp8.quantize_act(a)
    w2q, s2 = fp8.quantize_weight(w[:512].contiguous())
    got = rt.gemm_rs_fp8(aq, sa, w2q, s2)
    ad, wd = fp8.dequantize(aq, sa), fp8.dequantize(w2q, s2)
    fa = [torch.empty_like(ad) for _ in range(world)]
    fw = [torch.empty_like(wd) for _ in range(world)]
    dist.all_gather(fa, ad)
    dist.all_gather(fw, wd)
    ref = sum(fa[s] @ fw[s].T for s in range(world))[rank * (t // world):(rank + 1) * (t // world)]
    torch.cuda.synchronize()
    err = (got.float() - ref).abs().max().item() / max(1e-6, ref.abs().max().item())
    if err > 1e-2:
        failures.append(f"gemm_rs_fp8 relative error {err}")
    if rt.gemm_error() or rt.failure():
        failures.append(f"error word (fp8) {rt.gemm_error()} / {rt.failure()}")
    results["correct"] = not failures
    # -- timing at the prefill shapes
    if os.environ.get("SPARKNET_PREFILL_BENCH", "1") == "1" and not failures:
        cases = {}
        qkv_n, gu_n = (64 + 16) * 128 // world, 2 * F // world
        x = torch.randn(T // world, H, generator=g, device=device).to(torch.bfloat16)
        for name, n in (("ag_gemm_qkv", qkv_n), ("ag_gemm_gate_up", gu_n)):
            w = (0.02 * torch.randn(n, H, generator=g, device=device)).to(torch.bfloat16)
            out = torch.empty(T, n, dtype=torch.bfloat16, device=device)
            fused = timed(lambda: rt.ag_gemm(x, w, out=out))
            fused16 = timed(lambda: rt.ag_gemm(x, w, out=out, copy_ctas=16))
            base = timed(lambda: ag_gemm_reference(x, w))
            cases[name] = {"fused_ms": fused, "nccl_cublas_ms": base, "flops": 2 * T * H * n,
                           "nvlink_bytes_in": (world - 1) * (T // world) * H * 2}
            cases[name + "_copy16"] = {"fused_ms": fused16, "nccl_cublas_ms": base, "flops": 2 * T * H * n,
                                       "nvlink_bytes_in": (world - 1) * (T // world) * H * 2}
        for name, kk in (("gemm_rs_o", H // world), ("gemm_rs_down", F // world)):
            a = torch.randn(T, kk, generator=g, device=device).to(torch.bfloat16)
            w = (0.02 * torch.randn(H, kk, generator=g, device=device)).to(torch.bfloat16)
            out = torch.empty(T // world, H, dtype=torch.bfloat16, device=device)
            fused = timed(lambda: rt.gemm_rs(a, w, out=out))
            base = timed(lambda: gemm_rs_reference(a, w))
            cases[name] = {"fused_ms": fused, "nccl_cublas_ms": base, "flops": 2 * T * H * kk,
                           "nvlink_bytes_out": (world - 1) * (T // world) * H * 2}
        # fp8 block-scaled forms (operands quantised outside the timed region)
        from sparknet.ops import fp8

        xq, sx = fp8.quantize_act(x)
        for name, n in (("ag_gemm_qkv_fp8", qkv_n), ("ag_gemm_gate_up_fp8", gu_n)):
            wq, sw = fp8.quantize_weight((0.02 * torch.randn(n, H, generator=g, device=device)).to(torch.bfloat16))
            out = torch.empty(T, n, dtype=torch.bfloat16, device=device)
            fused = timed(lambda: rt.ag_gemm_fp8(xq, sx, wq, sw, out=out))
            cases[name] = {"fused_ms": fused, "nccl_cublas_ms": cases[name[:-4]]["nccl_cublas_ms"],
                           "flops": 2 * T * H * n, "nvlink_bytes_in": (world - 1) * (T // world) * H}
        for name, kk in (("gemm_rs_o_fp8", H // world), ("gemm_rs_down_fp8", F // world)):
            aq, sa = fp8.quantize_act(torch.randn(T, kk, generator=g, device=device).to(torch.bfloat16))
            wq, sw = fp8.quantize_weight((0.02 * torch.randn(H, kk, generator=g, device=device)).to(torch.bfloat16))
            out = torch.empty(T // world, H, dtype=torch.bfloat16, device=device)
            fused = timed(lambda: rt.gemm_rs_fp8(aq, sa, wq, sw, out=out))
            cases[name] = {"fused_ms": fused, "nccl_cublas_ms": cases[name[:-4]]["nccl_cublas_ms"],
                           "flops": 2 * T * H * kk, "nvlink_bytes_out": (world - 1) * (T // world) * H * 2}
        gathered = [None] * world
        dist.all_gather_object(gathered, cases, group=cpu)
        for name in cases:
            for key in ("fused_ms", "nccl_cublas_ms"):
                cases[name][key] = max(gg[name][key] for gg in gathered)
        results["cases"] = cases
        if rt.gemm_error() or rt.failure():
            failures.append(f"error word after timing {rt.gemm_error()} / {rt.failure()}")
    results["failures"] = failures
    torch.cuda.synchronize()
    dist.barrier(group=cpu)
    rt.close()
    dist.barrier(group=cpu)
    out_dir = os.environ.get("SPARKNET_TEST_OUT")
    if out_dir:
        Path(out_dir, f"rank{rank}.json").write_text(json.dumps(results))
    elif rank == 0:
        print(json.dumps(results), flush=True)
    dist.destroy_process_group()
    return 1 if failures else 0


if __name__ == "__main__":
    sys.exit(main())
