"""Policy boundaries (CPU only), after the reference's tests/test_policy.py."""

import pytest

from sparknet.policy import CollectivePolicy, crossover_from_timings
from sparknet.policy.policy import DEFAULT_ONESHOT_MAX


def make(**kw):
    base = dict(all_reduce_dispatch_bytes=2 << 20, all_reduce_capacity_bytes=8 << 20, all_gather_shard_bytes=16 << 20)
    base.update(kw)
    return CollectivePolicy(**base)


def test_limits_are_distinct_and_validated():
    assert make().problems() == []
    assert "dispatch" in " ".join(make(all_reduce_dispatch_bytes=16 << 20).problems())
    assert make(all_gather_shard_bytes=17).problems()
    assert make(force="bogus").problems()
    assert make(force="nvls").problems()  # NVLS is opt-in
    assert make(force="nvls", allow_nvls=True).problems() == []


@pytest.mark.parametrize("world", [2, 4, 8])
def test_all_reduce_backend_boundaries(world):
    p = make()
    limit = min(DEFAULT_ONESHOT_MAX[world], p.all_reduce_dispatch_bytes)
    assert p.all_reduce_backend(16, "bfloat16", world=world) == "oneshot"
    assert p.all_reduce_backend(limit, "bfloat16", world=world) == "oneshot"
    assert p.all_reduce_backend(limit + 16, "bfloat16", world=world) in ("twoshot", "nccl")
    assert p.all_reduce_backend(2 << 20, "bfloat16", world=world) in ("oneshot", "twoshot")
    assert p.all_reduce_backend((2 << 20) + 16, "bfloat16", world=world) == "nccl"
    assert p.all_reduce_backend(1024 + 8, "bfloat16", world=world) == "nccl"   # not a 16-byte multiple
    assert p.all_reduce_backend(1024, "int32", world=world) == "nccl"
    assert p.all_reduce_backend(1024, "bfloat16", contiguous=False, world=world) == "nccl"
    assert p.all_reduce_backend(0, "bfloat16", world=world) == "nccl"


def test_world_one_and_unlisted_worlds():
    p = make()
    assert p.all_reduce_backend(1 << 20, "float32", world=1) == "oneshot"
    assert p.oneshot_limit(6) == DEFAULT_ONESHOT_MAX[4]
    assert p.oneshot_limit(3) == DEFAULT_ONESHOT_MAX[2]


def test_nvls_only_when_allowed():
    assert make().all_reduce_backend(1 << 20, "bfloat16", world=8) == "twoshot"
    assert make(allow_nvls=True).all_reduce_backend(1 << 20, "bfloat16", world=8) == "nvls"
    assert make(allow_nvls=True).all_reduce_backend(4096, "bfloat16", world=8) == "oneshot"


def test_all_gather_backend_and_algorithm():
    p = make()
    assert p.all_gather_backend(1024, "bfloat16", dim=0, ndim=2) == "oneshot"
    assert p.all_gather_backend(1024, "bfloat16", dim=-1, ndim=3) == "oneshot"
    assert p.all_gather_backend(1024, "bfloat16", dim=1, ndim=3) == "nccl"
    assert p.all_gather_backend(1024, "bool", dim=0, ndim=1) == "nccl"
    assert p.all_gather_backend((16 << 20) + 16, "bfloat16", dim=0, ndim=1) == "nccl"
    assert p.all_gather_algorithm(1024, row_bytes=1024, nvls_available=False) == "ll"
    assert p.all_gather_algorithm(1 << 20, row_bytes=4096, nvls_available=True) == "ll"
    assert p.all_gather_algorithm(4 << 20, row_bytes=4096, nvls_available=True) == "ll"
    assert p.all_gather_algorithm((4 << 20) + 16, row_bytes=4096, nvls_available=True) == "push"
    assert make(allow_nvls=True).all_gather_algorithm(16 << 20, row_bytes=4096, nvls_available=True) == "nvls"
    assert p.all_gather_algorithm(1020, row_bytes=12, nvls_available=False) == "push"


def test_rank_invariance_ignores_everything_but_shape():
    """Same inputs, same answer, whatever else differs (nothing else is an argument)."""
    p = make()
    answers = {p.all_reduce_backend(n, "bfloat16", world=8) for _ in range(3) for n in [65536]}
    assert len(answers) == 1


def test_environment_round_trip():
    p = make(allow_nvls=True, oneshot_max_bytes={2: 1 << 20, 8: 128 << 10})
    q = CollectivePolicy.from_environment(p.environment())
    assert q.all_reduce_capacity_bytes == p.all_reduce_capacity_bytes
    assert q.allow_nvls and q.oneshot_limit(8) == 128 << 10
    with pytest.raises(ValueError):
        CollectivePolicy.from_environment({})


def test_crossover_from_timings():
    rows = [
        {"world_size": 8, "nbytes": 1 << 16, "algorithm": "oneshot", "p50_us": 5.0},
        {"world_size": 8, "nbytes": 1 << 16, "algorithm": "twoshot", "p50_us": 7.0},
        {"world_size": 8, "nbytes": 1 << 18, "algorithm": "oneshot", "p50_us": 9.0},
        {"world_size": 8, "nbytes": 1 << 18, "algorithm": "twoshot", "p50_us": 8.0},
    ]
    assert crossover_from_timings(rows) == {8: 1 << 16}


def test_ag_gemm_copy_ctas_balance():
    from sparknet.oneshot.runtime import copy_ctas_for

    T, H = 8192, 8192
    shard = T // 8 * H * 2
    small = copy_ctas_for(shard, 8, 2 * T * H * 1280)      # QKV: little GEMM per gathered byte
    large = copy_ctas_for(shard, 8, 2 * T * H * 7168)      # gate/up: GEMM-bound
    assert 16 <= large < small <= 74
    assert copy_ctas_for(shard, 1, 2 * T * H * 1280) == 0
    assert copy_ctas_for(1 << 30, 8, 1) == 74              # clamped to half the SMs
    assert copy_ctas_for(1, 8, 1 << 50) == 16


def test_derive_limits_stops_at_the_first_loss():
    from sparknet.policy import derive_limits

    def row(world, kib, arm, us):
        return {"world": world, "nbytes": kib << 10, "arm": arm, "p50_us": us}

    rows = [
        row(8, 4, "oneshot", 5), row(8, 4, "twoshot", 7), row(8, 4, "nccl", 20),
        row(8, 64, "oneshot", 6), row(8, 64, "twoshot", 7), row(8, 64, "nccl", 22),
        row(8, 512, "oneshot", 11), row(8, 512, "twoshot", 10), row(8, 512, "nccl", 30),
        row(8, 1024, "oneshot", 9), row(8, 1024, "twoshot", 15), row(8, 1024, "nccl", 35),  # one-shot wins again: ignored
        row(8, 4096, "twoshot", 40), row(8, 4096, "nccl", 38),                              # NCCL first wins
        row(8, 8192, "twoshot", 50), row(8, 8192, "nccl", 60),                              # after the first loss: ignored
        row(8, 512, "nvls", 9), row(8, 1024, "nvls", 8), row(8, 4096, "nvls", 30), row(8, 64, "nvls", 9),
    ]
    lim = derive_limits(rows)
    assert lim.oneshot_max[8] == 64 << 10
    assert lim.dispatch_max[8] == 1024 << 10
    assert lim.nvls_min[8] == 512 << 10


def test_sweep_rows_keep_cases_that_ran_on_their_arm():
    from sparknet.policy import sweep_rows

    receipt = {"timings": [
        {"operation": "all_reduce", "arm": "oneshot", "backend": "oneshot", "dtype": "torch.bfloat16",
         "elements_per_rank": 2048, "median_us": 5.0},
        {"operation": "all_reduce", "arm": "policy", "backend": "oneshot", "dtype": "torch.bfloat16",
         "elements_per_rank": 2048, "median_us": 5.0},
        {"operation": "all_gather", "arm": "oneshot", "backend": "oneshot", "dtype": "torch.bfloat16",
         "elements_per_rank": 2048, "median_us": 5.0},
        {"operation": "all_reduce", "arm": "nccl", "backend": "nccl", "dtype": "torch.float32",
         "elements_per_rank": 1024, "median_us": 9.0},
    ]}
    assert sweep_rows(receipt, 4) == [{"world": 4, "nbytes": 4096, "arm": "oneshot", "p50_us": 5.0},
                                     {"world": 4, "nbytes": 4096, "arm": "nccl", "p50_us": 9.0}]


def test_sweep_rows_take_the_all_gather_protocol_arms():
    from sparknet.policy import sweep_rows

    def ag(arm, elements, us, backend=None):
        return {"operation": "all_gather", "arm": arm, "backend": backend or arm, "dtype": "torch.bfloat16",
                "elements_per_rank": elements, "median_us": us}

    receipt = {"timings": [ag("ll", 2048, 4.5), ag("push", 2048, 9.7), ag("nccl", 2048, 12.7),
                           ag("oneshot", 2048, 5.0),              # the policy's pick, not a protocol arm
                           ag("nvls", 4096, 20.0, backend="push")]}  # ran elsewhere: dropped
    rows = sweep_rows(receipt, 2)
    assert [(r["arm"], r["nbytes"], r["operation"]) for r in rows] == [
        ("ll", 4096, "all_gather"), ("push", 4096, "all_gather"), ("nccl", 4096, "all_gather")]


def test_derive_ll_limit_from_the_protocol_sweep():
    from sparknet.policy import derive_limits

    def row(world, kib, arm, us, op="all_gather"):
        return {"world": world, "nbytes": kib << 10, "arm": arm, "p50_us": us, "operation": op}

    rows = [
        row(2, 4, "ll", 4.5), row(2, 4, "push", 9.7), row(2, 4, "nvls", 17.0), row(2, 4, "nccl", 12.7),
        row(2, 8, "nccl", 13.0),                                     # an NCCL-only size from another sweep
        row(2, 1024, "ll", 8.3), row(2, 1024, "push", 17.3), row(2, 1024, "nccl", 21.8),
        row(2, 4096, "ll", 20.7), row(2, 4096, "push", 23.1), row(2, 4096, "nccl", 39.5),
        row(2, 8192, "push", 30.7), row(2, 8192, "nccl", 51.2),     # beyond the LL slot
        row(8, 4, "nccl", 29.0),                                     # no protocol rows at W = 8
        row(4, 4, "ll", 6.0), row(4, 4, "push", 9.0),
        row(4, 64, "ll", 12.0), row(4, 64, "push", 10.0),            # LL loses: the limit stops at 4 KiB
        row(4, 128, "ll", 11.0), row(4, 128, "push", 14.0),
    ]
    lim = derive_limits(rows)
    assert lim.ll_max == {2: 4096 << 10, 4: 4 << 10}
    assert lim.oneshot_max == {} and lim.dispatch_max == {}         # all-gather rows leave the all-reduce limits alone


def test_committed_table_sets_the_ll_default():
    from sparknet.policy import load_measured, policy

    lim = load_measured()
    assert lim is not None and lim.ll_max
    assert policy.DEFAULT_LL_MAX == min(v for v in lim.ll_max.values() if v)
