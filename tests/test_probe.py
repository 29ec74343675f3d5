"""Probe planning and read-only checks with a fake NVML (CPU only), after the
reference's tests/test_probe.py."""

import copy
import importlib
import json
from pathlib import Path

import pytest

from sparknet.probe import container, counters, doctor, failstop, fleet, summary
from sparknet.topology import gpumap
from tests.fake_nvml import FakeNVML

nvlink_report = importlib.import_module("sparknet.probe.nvlink_report")  # the package exports a same-named function

EX = Path(__file__).resolve().parent.parent / "sparknet" / "topology" / "examples"


@pytest.fixture
def box():
    return gpumap.load(EX / "hgx-b200.json")


def fake_box_map():
    from sparknet.topology import discover

    return discover.generate_map(discover.local_inventory(FakeNVML(), multicast=lambda i: True), name="box",
                                 management_ip="192.0.2.1", management_interface="eno1")


def test_doctor_clean_and_findings():
    gmap = fake_box_map()
    gmap["nodes"][0]["driver"] = "580.159"
    nv = FakeNVML()
    ok = doctor.local_problems(gmap, "box", "nvlink", nvml=nv, fabricmanager=lambda: True, which=lambda x: "/x")
    assert ok == []
    nv.links[2] = 12
    nv.persistence[4] = 0
    nv.procs[5] = [object()]
    nv.ecc[6] = 3
    nv.p2p_broken.add((0, 7))
    errors = doctor.local_problems(gmap, "box", "nvlink", nvml=nv, fabricmanager=lambda: False, which=lambda x: None)
    text = "\n".join(errors)
    for needle in ("12 NVLinks active", "persistence mode is off", "already hold this GPU", "uncorrectable ECC",
                   "no NVLink peer-to-peer path", "fabricmanager", "nvcc not found"):
        assert needle in text, needle


def test_doctor_missing_gpu_and_bad_map():
    gmap = fake_box_map()
    gmap["nodes"][0]["gpus"][1]["uuid"] = "GPU-ffffffff-0000-4000-8000-ffffffffffff"
    errors = doctor.local_problems(gmap, "box", "nvlink", nvml=FakeNVML(), fabricmanager=lambda: True,
                                   which=lambda x: "/x")
    assert any("not present" in e for e in errors)
    assert doctor.local_problems({"nodes": []}, "box", "nvlink", nvml=FakeNVML())


def test_counters_and_deltas():
    nv = FakeNVML()
    before = counters.nvlink_counters(nv)
    nv.tx[0] += 100
    nv.errors[3] += 2
    after = counters.nvlink_counters(nv)
    d = counters.deltas(before, after)
    assert d["gpu0.nvlink_tx_kib"] == 100 and d["gpu0.nvlink_rx_kib"] == 100
    assert counters.error_deltas(before, after) == {f"gpu3.nvlink_{k}": 2 for k in counters.ERROR_COUNTERS}


def test_nvlink_report(tmp_path):
    (tmp_path / "nvidia-caps-imex-channels").mkdir()
    (tmp_path / "nvidia-caps-imex-channels" / "channel0").write_text("")
    rep = nvlink_report.nvlink_report(nvml=FakeNVML(), cuda_attr=lambda i, a: 1, fabricmanager=lambda: True,
                                      dev_root=str(tmp_path))
    assert rep["ready"] == {"p2p": True, "nvls": True, "fabric": True}
    assert "P2P over NVLink" in nvlink_report.render(rep)
    nv = FakeNVML()
    nv.p2p_broken.add((2, 3))
    rep = nvlink_report.nvlink_report(nvml=nv, cuda_attr=lambda i, a: 0, fabricmanager=lambda: None,
                                      dev_root=str(tmp_path / "none"))
    assert rep["ready"] == {"p2p": False, "nvls": False, "fabric": False}


def test_container_command():
    cmd = container.docker_probe_command(image="img", environment={"A": "1"}, nproc=8, master_port=1234,
                                         extra_args=("--benchmark",))
    assert "--ipc=host" in cmd and "--nproc-per-node=8" in cmd and cmd[-1] == "--benchmark"
    assert "SPARKNET_TRANSPORT=nvlink" in cmd


class FakeProc:
    def __init__(self, rc, text, stdout):
        self.rc = rc
        stdout.write(text)

    def wait(self, timeout=None):
        return self.rc

    def terminate(self):
        pass

    def kill(self):
        pass


def test_fleet_plan_and_run(tmp_path):
    fleet_map = gpumap.load(EX / "hgx-b200-fleet2.json")
    envs = {n["name"]: {"X": "1"} for n in fleet_map["nodes"]}
    plans = fleet.plan(fleet_map, envs, transport="nvlink", image="img", port=29650, probe_args=("--benchmark",),
                       local_box="hgx-b200-1")
    assert [p.node_rank for p in plans] == [0, 1] and plans[0].local and not plans[1].local
    assert fleet.ssh_command(plans[1])[0] == "ssh"
    assert fleet.bootstrap_warnings(fleet_map, envs)
    result = {"passed": True, "timings": [{"operation": "all_reduce", "dtype": "bfloat16", "elements_per_rank": 8,
                                           "arm": "policy", "microseconds_per_call": [1.0, 2.0, 3.0]}]}

    def popen(cmd, stdout, stderr):
        return FakeProc(0, "noise\n" + json.dumps(result) + "\n", stdout)

    outcomes = fleet.run(plans, tmp_path, popen=popen)
    assert all(o.passed for o in outcomes)
    table = summary.cases(summary.load_results(tmp_path))
    assert table[("all_reduce", "bfloat16", 16, "policy")]["slowest_rank_median_us"] == 2.0


def test_summary_slowest_box():
    results = {"a": {"timings": [{"operation": "all_reduce", "dtype": "torch.bfloat16", "elements_per_rank": 5120,
                                  "microseconds_per_call": [1, 5, 3]}]},
               "b": {"timings": [{"operation": "all_reduce", "dtype": "torch.bfloat16", "elements_per_rank": 5120,
                                  "microseconds_per_call": [4, 2, 2]}]}}
    table = summary.cases(results)
    assert table[("all_reduce", "bfloat16", 10240, "policy")]["slowest_rank_median_us"] == 4
    md = summary.markdown({"x": table})
    assert "10 KiB" in md and "4.0 us" in md


def test_failstop_bounds():
    good = {"rank": 0, "victim": 1, "eager": {"victim": False, "detected": True, "seconds": 1.1,
                                                 "report": "... waiting for rank 1 (block 0) ...", "recovered": True}}
    assert failstop.problems(good, 1000) == []
    slow = copy.deepcopy(good)
    slow["eager"]["seconds"] = 9.0
    assert failstop.problems(slow, 1000)
    early = copy.deepcopy(good)
    early["eager"]["seconds"] = 0.2
    assert failstop.problems(early, 1000)
    unnamed = copy.deepcopy(good)
    unnamed["eager"]["report"] = "something"
    assert failstop.problems(unnamed, 1000)
    victim = {"rank": 1, "victim": 1, "eager": {"victim": True, "recovered": True}}
    assert failstop.problems(victim, 1000) == []


def test_reference_report_names():
    import sparknet.probe as probe
    from sparknet.integration.vllm import REQUIRED_API_VERSION
    from sparknet.oneshot.runtime import API_VERSION

    assert probe.gpudirect_report is probe.nvlink_report
    assert REQUIRED_API_VERSION == API_VERSION


def test_runtime_counters_held_to_routing():
    from sparknet.probe.collectives import Route, check_runtime_counters, nvlink_bytes_expected

    ledger0 = {("all_reduce", "oneshot"): [2, 64]}
    ledger1 = {("all_reduce", "oneshot"): [5, 160], ("all_gather", "oneshot"): [1, 32], ("all_reduce", "nccl"): [4, 8]}
    want = check_runtime_counters({"oneshot": 2}, {"oneshot": 5, "all_gather": 1}, ledger0, ledger1, what="case")
    assert want == {"oneshot": 3, "all_gather": 1}
    with pytest.raises(RuntimeError, match="runtime counters moved"):
        # an NCCL-routed call that moved a runtime counter
        check_runtime_counters({}, {"twoshot": 1}, {}, {("all_reduce", "nccl"): [1, 16]}, what="case")
    with pytest.raises(RuntimeError, match="runtime counters moved"):
        # an NVLink-routed call the runtime never counted
        check_runtime_counters({}, {}, {}, {("reduce_scatter", "oneshot"): [1, 16]}, what="case")
    assert nvlink_bytes_expected(Route("all_reduce", "oneshot", 1024), 8) == 7 * 1024
    assert nvlink_bytes_expected(Route("all_reduce", "twoshot", 1024), 8) == 2 * 1024 * 7 // 8
    assert nvlink_bytes_expected(Route("all_reduce", "nccl", 1024), 8) == 0
    assert nvlink_bytes_expected(Route("all_gather", "oneshot", 1024), 4) == 3 * 1024
    assert nvlink_bytes_expected(Route("all_gather", "nvls", 1024), 4) == 1024  # one copy, fanned out by the switch
    assert nvlink_bytes_expected(Route("all_gather", "ll", 1024), 4) == 3 * 1024
