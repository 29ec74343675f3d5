"""One rank of the multi-GPU decode check: a tiny TP Llama decodes with the fused
NVLink epilogue and with NCCL; both arms must produce the same tokens on every rank
and close logits.  Writes one JSON file per rank to $SPARKNET_TEST_OUT."""

import json
import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def gemm_pushes_all_reduce(rt, cfg, rank, world, device, results):
    """The decode GEMM whose epilogue pushes into the all-reduce gives the unfused
    sequence's bits: eagerly on both slot parities, from a replayed graph, and as the
    O / down projections of the decode step."""
    from sparknet.models.llama import TPLlama
    from sparknet.ops.decode_gemm import linear

    g = torch.Generator(device=device).manual_seed(11 + rank)
    # 8 tokens: one-shot; 64 tokens x 8192: two-shot at 4 or more ranks (one-shot at 2)
    for tokens, n in ((8, 2048), (64, 8192)):
        xs = torch.randn(tokens, 1024, generator=g, device=device).to(torch.bfloat16)
        ws = (0.05 * torch.randn(n, 1024, generator=g, device=device)).to(torch.bfloat16)
        gs = (1 + 0.1 * torch.randn(n, device=device)).to(torch.bfloat16)
        rs = torch.randn(tokens, n, generator=torch.Generator(device=device).manual_seed(5), device=device)
        rs = rs.to(torch.bfloat16)
        if not rt.gemm_push_eligible(xs, ws):
            results["failures"].append(f"{tokens} x {n} not eligible for the pushing GEMM")
            continue
        for call in range(2):  # both slot parities
            partial = linear(xs, ws)
            want_out, want_res = rt.all_reduce_residual_rmsnorm(partial, rs.clone(), gs, 1e-5)
            got_out, got_res = rt.gemm_all_reduce_residual_rmsnorm(xs, ws, rs.clone(), gs, 1e-5)
            torch.cuda.synchronize()
            if not (torch.equal(got_out, want_out) and torch.equal(got_res, want_res)):
                results["failures"].append(f"pushing GEMM differs from the unfused sequence ({tokens} x {n}, "
                                           f"call {call})")
    x = torch.randn(8, 1024, generator=g, device=device).to(torch.bfloat16)
    w = (0.05 * torch.randn(2048, 1024, generator=g, device=device)).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(2048, device=device)).to(torch.bfloat16)
    res0 = torch.randn(8, 2048, generator=torch.Generator(device=device).manual_seed(5), device=device)
    res0 = res0.to(torch.bfloat16)
    res, out, part = res0.clone(), torch.empty_like(res0), torch.empty_like(res0)
    stream = torch.cuda.Stream(device=device)
    stream.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream), rt.capture(stream=stream):
        rt.gemm_all_reduce_residual_rmsnorm(x, w, res, gamma, 1e-5, partial=part, out=out, residual_out=res)
    want = res0.clone()
    for rep in range(3):
        graph.replay()
        want_out, want = rt.all_reduce_residual_rmsnorm(linear(x, w), want, gamma, 1e-5)
        torch.cuda.synchronize()
        if not (torch.equal(out, want_out) and torch.equal(res, want)):
            results["failures"].append(f"pushing GEMM graph replay {rep} differs")
    del graph
    logits = {}
    for fused in (False, True):
        m = TPLlama(cfg, rank=rank, world=world, device=device, batch=4, max_len=64, comm="sparknet", runtime=rt,
                    seed=3, fuse_gemm_ar=fused)
        m.fill_prompt_cache(10)
        m.tokens.copy_(torch.tensor([1, 2, 3, 4], device=device))
        m.capture()
        for _ in range(3):
            m.replay()
        torch.cuda.synchronize()
        logits[fused] = (m.logits.clone(), m.tokens.clone())
        m.release()
        del m
    if not (torch.equal(logits[True][0], logits[False][0]) and torch.equal(logits[True][1], logits[False][1])):
        results["failures"].append("decode step with pushing GEMMs differs from the unfused step")
    results["gemm_pushes_all_reduce_checked"] = True


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("cpu:gloo,cuda:nccl", timeout=timedelta(seconds=60), device_id=device)
    rank, world = dist.get_rank(), dist.get_world_size()
    cpu = dist.new_group(backend="gloo", timeout=timedelta(seconds=60))
    from sparknet.models.llama import LlamaConfig, TPLlama
    from sparknet.oneshot import AllReduce

    rt = AllReduce.from_exchange_group(exchange_group=cpu, device=device, max_size=4 << 20, max_gather_bytes=1 << 20)
    rt.prepare((torch.bfloat16,))
    cfg = LlamaConfig(hidden=2048, layers=3, heads=16, kv_heads=8, head_dim=128, ffn=4096, vocab=8192)
    results = {"rank": rank, "failures": []}
    outs = {}
    # Teacher-forced: every step starts from the same input tokens in both arms.  With
    # random weights the logits are nearly flat, so the arms' different GEMM rounding can
    # pick different argmax tokens; feeding those back would compare different sequences.
    forced = torch.tensor([[1, 2, 3, 4], [5, 6, 7, 8], [9, 10, 11, 12], [13, 14, 15, 16]], device=device)
    for comm in ("sparknet", "nccl"):
        m = TPLlama(cfg, rank=rank, world=world, device=device, batch=4, max_len=64, comm=comm, runtime=rt, seed=3)
        m.fill_prompt_cache(10)
        m.tokens.copy_(forced[0])
        m.capture()
        toks, xs = [], []
        for step in range(4):
            m.tokens.copy_(forced[step])
            m.replay()
            toks.append(m.tokens.clone())
            xs.append(m.x.float().clone())
        torch.cuda.synchronize()
        outs[comm] = (torch.stack(toks).cpu(), m.logits.float().cpu(), torch.stack(xs).cpu())
        m.release()
        del m
    t_s, l_s, x_s = outs["sparknet"]
    t_n, l_n, x_n = outs["nccl"]
    gathered = [None] * world
    dist.all_gather_object(gathered, t_s.tolist(), group=cpu)
    if any(g != gathered[0] for g in gathered):
        results["failures"].append("ranks sampled different tokens")
    if not torch.allclose(x_s, x_n, rtol=5e-2, atol=5e-2):
        results["failures"].append(f"hidden states differ between arms: {(x_s - x_n).abs().max().item()}")
    results["tokens_equal_between_arms"] = bool(torch.equal(t_s, t_n))
    if os.environ.get("SPARKNET_TEST_EXPERIMENTAL") == "1":
        gemm_pushes_all_reduce(rt, cfg, rank, world, device, results)
    results["rt_health"] = rt.failure()
    torch.cuda.synchronize()
    dist.barrier(group=cpu)
    rt.close()
    dist.barrier(group=cpu)
    Path(os.environ["SPARKNET_TEST_OUT"], f"rank{rank}.json").write_text(json.dumps(results))
    dist.destroy_process_group()
    return 1 if results["failures"] else 0


if __name__ == "__main__":
    sys.exit(main())
