"""NCCL control profiles (CPU only), after the reference's tests/test_nccl_profiles.py."""

import pytest

from sparknet import nccl
from sparknet.nccl import patchset
from sparknet.policy import policy_for_profile


@pytest.mark.parametrize("name", list(nccl.PROFILES))
def test_profiles_are_consistent(name):
    entry = nccl.profile(name)
    env = nccl.environment(name)
    for world in entry["node_counts"]:
        errors = nccl.problems(env, world=world)
        if name == "ib-forced-nccl-only" and world > 1:
            assert any("forced onto IB" in e for e in errors)
        else:
            assert errors == [], (name, world, errors)
    assert nccl.required_patches(env) == []
    for key, value in entry["nccl"].items():
        if value is None:
            assert key not in env


def test_reference_control_env_is_verbatim():
    env = nccl.environment("ib-forced-nccl-only")
    for key, value in nccl.REFERENCE_IB_ENV.items():
        assert env[key] == value


def test_profile_lookup_and_applicability():
    with pytest.raises(ValueError):
        nccl.profile("tp4-ring")
    assert nccl.profiles_for("nvlink", 8) == ["nvlink", "nvlink-8"]
    assert nccl.profiles_for("nvlink", 4) == ["nvlink"]
    assert "nvlink-nccl-only" in nccl.profiles_for("nccl-nvlink", 2)
    assert nccl.profile_problems("nvlink-nvls", "nvlink-nvls", 1)
    assert nccl.profile_problems("nvlink", "nccl-nvlink", 8)


def test_limits_and_contradictions():
    env = nccl.environment("nvlink")
    assert nccl.problems(dict(env, SPARKNET_ALLREDUCE_DISPATCH_MAX_BYTES="16777216"), world=8)
    assert nccl.problems(dict(env, SPARKNET_ALLGATHER_MAX_BYTES="1000"), world=8)
    assert nccl.problems(dict(env, NCCL_MIN_NCHANNELS="8", NCCL_MAX_NCHANNELS="4"), world=8)
    assert nccl.problems(dict(env, SPARKNET_NVLS="1", NCCL_NVLS_ENABLE="0"), world=8)
    assert nccl.problems(env, world=3)


def test_policy_for_profile():
    p = policy_for_profile("nvlink")
    assert p.all_reduce_dispatch_bytes == 2 << 20 and p.all_reduce_capacity_bytes == 8 << 20
    assert policy_for_profile("nvlink-nccl-only") is None


def test_size_bytes():
    assert nccl.size_bytes("2MB") == 2 << 20 and nccl.size_bytes("16") == 16
    with pytest.raises(ValueError):
        nccl.size_bytes("0")


def test_empty_patch_series(tmp_path):
    assert patchset.series() == [] and patchset.missing() == []
    files = patchset.export(tmp_path)
    assert (tmp_path / "series").read_text() == "" and len(files) == 2


def test_recipes_are_current():
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    out = subprocess.run([sys.executable, str(root / "recipes" / "generate.py"), "--check"], capture_output=True,
                         text=True)
    assert out.returncode == 0, out.stdout + out.stderr


def test_full_box_profile_carries_the_measured_dispatch_ceiling():
    from sparknet.policy import policy_for_profile
    from sparknet.policy.policy import default_dispatch_bytes

    pol = policy_for_profile("nvlink-8")
    assert pol.all_reduce_dispatch_bytes == default_dispatch_bytes(8)
    assert pol.all_reduce_capacity_bytes >= pol.all_reduce_dispatch_bytes
    assert not nccl.problems(nccl.environment("nvlink-8"), world=8)
    general = policy_for_profile("nvlink")
    assert general.all_reduce_dispatch_bytes == 2 << 20   # valid at every world size, W = 4 unmeasured
