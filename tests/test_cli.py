"""The CLI end to end, in process (CPU only), after the reference's tests/test_cli.py."""

import json
import subprocess
import sys
from pathlib import Path

import pytest

from sparknet import cli

ROOT = Path(__file__).resolve().parent.parent
EX = ROOT / "sparknet" / "topology" / "examples" / "hgx-b200.json"


def run(capsys, *argv):
    code = cli.main(list(argv))
    out = capsys.readouterr()
    return code, out.out, out.err


def test_topology_commands(capsys, tmp_path):
    assert run(capsys, "topology", "validate", str(EX), "--transport", "nvlink")[0] == 0
    code, out, _ = run(capsys, "topology", "render", str(EX), "hgx-b200-1", "--transport", "nvlink",
                       "--profile", "nvlink", "--json", "--by", "index")
    assert code == 0 and json.loads(out)["CUDA_VISIBLE_DEVICES"] == "0,1,2,3,4,5,6,7"
    code, out, _ = run(capsys, "topology", "example", "hgx-b200")
    assert code == 0 and json.loads(out)["schema_version"] == 2
    assert run(capsys, "topology", "example", "nope")[0] == 1
    target = tmp_path / "pair.json"
    assert run(capsys, "topology", "subset", str(EX), "hgx-b200-1", "2", "3", "--out", str(target))[0] == 0
    assert run(capsys, "topology", "validate", str(target), "--transport", "nvlink")[0] == 0
    assert run(capsys, "topology", "subset", str(EX), "hgx-b200-1", "0", "1", "2")[0] == 1


def test_nccl_and_policy_commands(capsys, tmp_path):
    code, out, _ = run(capsys, "nccl", "env", "--profile", "nvlink-nccl-only")
    assert code == 0 and "TORCH_NCCL_ASYNC_ERROR_HANDLING=1" in out
    assert run(capsys, "nccl", "validate", "--profile", "nvlink")[0] == 0
    envf = tmp_path / "e.env"
    envf.write_text("# override\nSPARKNET_ALLGATHER_MAX_BYTES=17\n")
    assert run(capsys, "nccl", "validate", "--profile", "nvlink", "--env-file", str(envf))[0] == 1
    code, out, _ = run(capsys, "nccl", "profiles")
    assert code == 0 and "ib-forced-nccl-only" in out
    assert run(capsys, "nccl", "patches", "--export", str(tmp_path / "p"))[0] == 0
    code, out, _ = run(capsys, "policy", "show", "--profile", "nvlink")
    assert code == 0 and json.loads(out)["all_reduce_capacity_bytes"] == 8 << 20
    code, out, _ = run(capsys, "policy", "show", "--profile", "nvlink-nccl-only")
    assert "every collective on NCCL" in out


def test_probe_planning_commands(capsys, tmp_path):
    code, out, _ = run(capsys, "probe", "render-command", str(EX), "hgx-b200-1", "--transport", "nvlink",
                       "--image", "img:1", "--", "--benchmark")
    assert code == 0 and "--nproc-per-node=8" in out and out.strip().endswith("--benchmark")
    code, out, _ = run(capsys, "probe", "fleet", str(EX), "--transport", "nvlink", "--image", "img:1", "--dry-run")
    assert code == 0 and "ssh" in out
    receipts = tmp_path / "r"
    receipts.mkdir()
    (receipts / "box.json").write_text(json.dumps({"timings": [
        {"operation": "all_reduce", "dtype": "torch.bfloat16", "elements_per_rank": 5120, "arm": "policy",
         "microseconds_per_call": [5.0, 4.0, 6.0]}]}))
    code, out, _ = run(capsys, "probe", "summarize", f"a={receipts}", f"b={receipts}")
    assert code == 0 and "10 KiB" in out and "5.0 us" in out and "+0.0%" in out


def test_split_pass_through():
    assert cli.split_pass_through(["a", "--", "b"]) == (["a"], ["b"])
    assert cli.split_pass_through(["a"]) == (["a"], None)


def test_cpu_commands_do_not_import_torch():
    code = "import sys, sparknet.cli, sparknet.topology, sparknet.policy, sparknet.nccl, sparknet.probe; " \
           "print('torch' in sys.modules)"
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, cwd=ROOT)
    assert out.stdout.strip() == "False", out.stderr


def test_version(capsys):
    with pytest.raises(SystemExit):
        cli.main(["--version"])
    assert "sparknet" in capsys.readouterr().out


def test_probe_counters_snapshot_and_deltas(capsys, monkeypatch):
    from sparknet.probe import nvml as nvml_mod
    from tests.fake_nvml import FakeNVML

    nv = FakeNVML()
    monkeypatch.setattr(nvml_mod, "load", lambda: nv)
    code, out, _ = run(capsys, "probe", "counters")
    snap = json.loads(out)
    assert code == 0 and "gpu0.nvlink_tx_kib" in snap and snap["gpu7.nvlink_replay"] == 0
    # an interval over which only throughput moves: exit 0; an error counter that moves: exit 1
    import time as time_mod

    def step(seconds):
        nv.tx[1] += 64

    monkeypatch.setattr(time_mod, "sleep", step)
    code, out, _ = run(capsys, "probe", "counters", "--interval", "0.1")
    report = json.loads(out)
    assert code == 0 and report["deltas"]["gpu1.nvlink_tx_kib"] == 64 and not report["error_counters_moved"]

    def fault(seconds):
        nv.errors[2] += 1

    monkeypatch.setattr(time_mod, "sleep", fault)
    code, out, _ = run(capsys, "probe", "counters", "--interval", "0.1", "--errors-only")
    report = json.loads(out)
    assert code == 1 and report["deltas"] == {f"gpu2.nvlink_{k}": 1 for k in ("replay", "recovery", "crc_flit",
                                                                                "crc_data")}
