"""The vLLM adapter's host logic with gloo ranks on CPU and a fake runtime: capability
vote, identical limits, fail-stop construction, rank-invariant dispatch surface.
(After the reference's adapter contract, sparknet/integration/vllm/roce_all_reduce.py.)"""

import sys
from pathlib import Path

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

ROOT = Path(__file__).resolve().parent.parent


class FakeRuntime:
    def __init__(self, *, exchange_group, device, max_size, max_gather_bytes):
        self.max_size, self.max_gather_bytes, self.dispatch_max_bytes = max_size, max_gather_bytes, 2 << 20
        self.prepared = None
        self.calls = []

    def prepare(self, dtypes, padded_gather=False):
        self.prepared = (tuple(dtypes), padded_gather)

    def should_allreduce(self, x):
        return x.numel() * x.element_size() <= self.dispatch_max_bytes

    def all_reduce(self, x):
        self.calls.append("ar")
        return x * 2

    def all_reduce_residual_rmsnorm(self, x, residual, weight, eps, residual_out=None):
        self.calls.append("fused")
        residual_out.add_(x)
        return residual_out * weight, residual_out

    def check_health(self):
        return None

    def failure(self):
        return None

    def close(self):
        self.calls.append("close")


def _worker(rank, world, store, mode, results):
    sys.path.insert(0, str(ROOT))
    import os

    dist.init_process_group("gloo", init_method=f"file://{store}", rank=rank, world_size=world)
    from sparknet.integration.vllm import nvlink_all_reduce as mod

    if mode == "mismatch" and rank == 1:
        os.environ["SPARKNET_ALLREDUCE_CAPACITY_BYTES"] = "4MB"
    mod.SparknetOneShotAllReduce._assess = lambda self: (
        mod.Readiness(self.rank, (), (mod.parse_byte_size(os.environ.get("SPARKNET_ALLREDUCE_CAPACITY_BYTES", "8MB")),
                                      16 << 20))
        if not (mode == "refuse" and self.rank == 1) else mod.Readiness(self.rank, ("no B200 here",), None))
    out = {}
    try:
        adapter = mod.SparknetOneShotAllReduce(dist.group.WORLD, object(), torch.device("cpu"),
                                               in_the_same_node=[True] * world, runtime_factory=FakeRuntime)
        x = torch.ones(4, 64)
        out["enabled"] = not adapter.disabled
        out["fused"] = adapter.supports_fused_add_rms_norm()
        out["should"] = adapter.should_custom_ar(x)
        out["ar"] = float(adapter.custom_all_reduce(x).sum())
        res = torch.zeros(4, 64)
        y, r = adapter.fused_add_rms_norm(x, res, torch.full((64,), 3.0), 1e-5)
        out["fused_residual_in_place"] = bool(r is res and float(res.sum()) == 256.0)
        out["limits"] = (adapter.all_reduce_max_bytes, adapter.all_reduce_capacity_bytes, adapter.all_gather_max_bytes)
        adapter.close()
        out["disabled_after_close"] = adapter.disabled
    except RuntimeError as exc:
        out["error"] = str(exc)
    results[rank] = out
    dist.destroy_process_group()


def run(mode, tmp_path, world=2):
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_worker, args=(world, str(tmp_path / "s"), mode, results), nprocs=world, join=True,
                       start_method="spawn")
    return dict(results)


def test_adapter_votes_and_routes(tmp_path):
    res = run("ok", tmp_path)
    for out in res.values():
        assert out["enabled"] and out["fused"] and out["should"] and out["ar"] == 512.0
        assert out["fused_residual_in_place"] and out["limits"] == (2 << 20, 8 << 20, 16 << 20)
        assert out["disabled_after_close"]


def test_a_refusing_rank_fails_every_rank(tmp_path):
    res = run("refuse", tmp_path)
    assert all("rank 1 cannot serve: no B200 here" in out.get("error", "") for out in res.values()), res


def test_differing_limits_fail_every_rank(tmp_path):
    res = run("mismatch", tmp_path)
    assert all("size limits disagree" in out.get("error", "") for out in res.values()), res


def test_parse_byte_size():
    from sparknet.integration.vllm import parse_byte_size

    assert parse_byte_size("2MB") == 2 << 20 and parse_byte_size(" 16 kb ") == 16 << 10
    with pytest.raises(ValueError):
        parse_byte_size("0")


def test_agreement_lists_every_blocker_and_limit_set():
    from sparknet.integration.vllm.nvlink_all_reduce import Readiness, agreement

    ok = [Readiness(r, (), (8 << 20, 16 << 20)) for r in range(4)]
    assert agreement(ok) is None
    blocked = ok[:2] + [Readiness(2, ("a", "b"), None), Readiness(3, ("c",), None)]
    text = agreement(blocked)
    assert "rank 2 cannot serve: a; b" in text and "rank 3 cannot serve: c" in text
    split = ok[:3] + [Readiness(3, (), (4 << 20, 16 << 20))]
    text = agreement(split)
    assert "ranks [0, 1, 2]" in text and "ranks [3]" in text and str(4 << 20) in text
