#!/usr/bin/env python3
"""NVLink data-phase microbenchmark (K13): P2P store vs P2P load vs NVLS multimem.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 benchmarks/microbench_nvlink.py \
        --sizes 10240 491520 4194304 --blocks 8 32 148 --ppt 1 4 [--nvls] [--gemm] [--pattern pair|ring|all]

Each rank maps every peer's symmetric region (CUDA VMM, the runtime's transport) and
moves ``size`` bytes with ``sparknet._C.nvlink_move``:

* ``store``      local -> peer (P2P stores, the one-shot push)
* ``load``       peer -> local (P2P loads, the pull)
* ``mc_store``   local -> multicast alias (one ``multimem.st`` reaches every GPU)
* ``mc_reduce``  multicast alias -> local (``multimem.ld_reduce`` sums every GPU's copy)
* ``bulk``       local -> shared memory -> every target peer by bulk copies (one working
                 thread per CTA, ``--pieces`` bytes per copy): the push of the fused
                 all-gather -> GEMM done by the SM's copy engine instead of its threads

Patterns: ``pair`` (rank 0 <-> rank 1 only), ``ring`` (rank r -> r+1, all at once),
``all`` (rank r -> every peer in turn, all ranks at once).  Timing: CUDA events around
``--reps`` back-to-back launches on each rank, after a barrier; the slowest rank counts.
``--gemm`` runs a tcgen05 GEMM on a second stream during the timed loop (the
interference a fused compute+collective kernel sees).  One JSON receipt on rank 0.
Method after the reference's data-phase sweeps (``evidence/2026-10-20-wide-read``).
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

MODES = {"store": 0, "load": 1, "mc_store": 2, "mc_reduce": 3, "bulk": 4}


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--sizes", type=int, nargs="+", default=[10240, 61440, 491520, 2097152, 16 << 20])
    ap.add_argument("--blocks", type=int, nargs="+", default=[8, 32, 148])
    ap.add_argument("--threads", type=int, default=512)
    ap.add_argument("--ppt", type=int, nargs="+", default=[1, 4])
    ap.add_argument("--pieces", type=int, nargs="+", default=[16384, 32768],
                    help="bulk mode: bytes per bulk copy (ppt is ignored)")
    ap.add_argument("--modes", nargs="+", default=["store", "load"], choices=sorted(MODES))
    ap.add_argument("--pattern", default="ring", choices=["pair", "ring", "all"])
    ap.add_argument("--reps", type=int, default=50)
    ap.add_argument("--nvls", action="store_true", help="build the multicast object (needed for mc_* modes)")
    ap.add_argument("--gemm", action="store_true", help="tcgen05 GEMM co-runner on a second stream")
    ap.add_argument("--output", default="")
    args = ap.parse_args()

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("gloo", timeout=timedelta(seconds=120))
    rank, world = dist.get_rank(), dist.get_world_size()
    from sparknet import _native
    from sparknet.oneshot import symm

    C = _native.load()
    big = max(args.sizes)
    regions = symm.build_regions(C, group=dist.group.WORLD, device_index=local, region_bytes=2 * big,
                                 multicast_bytes=big if args.nvls else 0)
    src = torch.randn(big // 2, device=device).to(torch.bfloat16)
    dst = torch.empty_like(src)
    co = None
    if args.gemm:
        from sparknet.ops.gemm import gemm

        a = torch.randn(4096, 8192, device=device).to(torch.bfloat16)
        b = torch.randn(4096, 8192, device=device).to(torch.bfloat16)
        c = torch.empty(4096, 4096, device=device, dtype=torch.bfloat16)
        side = torch.cuda.Stream(device=device)
        co = (lambda: gemm(a, b, c), side)

    def targets():
        if args.pattern == "pair":
            return [1 - rank] if rank < 2 and world > 1 else []
        if args.pattern == "ring":
            return [(rank + 1) % world] if world > 1 else [rank]
        return [p for p in range(world) if p != rank] or [rank]

    err = torch.zeros(1, dtype=torch.int32, device=device)
    rows = []
    for mode in args.modes:
        if mode.startswith("mc_") and regions.multicast is None:
            continue
        for size in args.sizes:
            for blocks in args.blocks:
                for ppt in (args.pieces if mode == "bulk" else args.ppt):
                    peers = targets()

                    def once():
                        if mode == "bulk":
                            C.nvlink_bulk_fanout(src.data_ptr(), [regions.bases[p] for p in peers], size, blocks,
                                                 ppt, err, local)
                            return
                        for p in peers:
                            if mode == "store":
                                s_, d_ = src.data_ptr(), regions.bases[p]
                            elif mode == "load":
                                s_, d_ = regions.bases[p], dst.data_ptr()
                            elif mode == "mc_store":
                                s_, d_ = src.data_ptr(), regions.mc_ptr
                            else:
                                s_, d_ = regions.mc_ptr, dst.data_ptr()
                            C.nvlink_move(s_, d_, size, MODES[mode], blocks, args.threads, ppt, local)

                    once()
                    torch.cuda.synchronize()
                    dist.barrier()
                    if co is not None:
                        co[1].wait_stream(torch.cuda.current_stream())
                        with torch.cuda.stream(co[1]):
                            for _ in range(8):
                                co[0]()
                    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    st.record()
                    for _ in range(args.reps):
                        once()
                    en.record()
                    en.synchronize()
                    torch.cuda.synchronize()
                    us = st.elapsed_time(en) * 1000.0 / args.reps
                    per = [None] * world
                    dist.all_gather_object(per, us)
                    active = [per[r] for r in range(world) if (args.pattern != "pair" or r < 2)]
                    worst = max(active)
                    moved = size * max(1, len(peers))
                    row = {"mode": mode, "bytes": size, "blocks": blocks, "threads": args.threads, "ppt": ppt,
                           "us": round(worst, 3), "gbs_per_gpu": round(moved / worst / 1e3, 1)}
                    if mode == "bulk":
                        row.update(threads=32, piece=ppt, ppt=None, wait_error=int(err.item()))
                    rows.append(row)
    receipt = {"benchmark": "microbench_nvlink", "world": world, "pattern": args.pattern, "gemm_corunner": args.gemm,
               "nvls": regions.multicast is not None, "rows": rows,
               "gpu": torch.cuda.get_device_name(device)}
    if rank == 0:
        text = json.dumps(receipt)
        print(text, flush=True)
        if args.output:
            Path(args.output).write_text(text + "\n")
    torch.cuda.synchronize()
    dist.barrier()
    del regions
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
