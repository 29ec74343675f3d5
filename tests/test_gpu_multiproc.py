"""Multi-process NVLink tests: one rank per GPU via torch.distributed.run (skipped on
boxes with fewer than two GPUs).  Mirrors the reference's GPU suite
(reference tests/gpu/test_oneshot_gpu.py) on the real peer-to-peer path."""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

torch = pytest.importorskip("torch")

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]
ROOT = Path(__file__).resolve().parent.parent


def _world():
    return min(torch.cuda.device_count(), 8) if torch.cuda.is_available() else 0


def run_workers(world, extra_env=None, timeout=600, script="mp_worker.py"):
    import tempfile

    out_dir = tempfile.mkdtemp(prefix="sparknet-mp-")
    env = dict(os.environ)
    env.update(extra_env or {})
    env["SPARKNET_TEST_OUT"] = out_dir
    env.setdefault("NCCL_NVLS_ENABLE", "0")
    cmd = ["timeout", "-k", "30", str(timeout), sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", str(29500 + os.getpid() % 1000),
           str(ROOT / "tests" / "workers" / script)]
    proc = subprocess.run(cmd, env=env, cwd=ROOT, capture_output=True, text=True, timeout=timeout + 60)
    lines = [json.loads(p.read_text()) for p in sorted(Path(out_dir).glob("rank*.json"))]
    failures = [l.get("failures") for l in lines]
    assert proc.returncode == 0, f"failures={failures}\n" + proc.stdout[-3000:] + proc.stderr[-5000:]
    return lines


@pytest.mark.skipif(_world() < 2, reason="needs two or more GPUs")
def test_multiprocess_collectives():
    lines = run_workers(_world())
    assert len(lines) == _world() and all(l["checks"] > 10 and not l["failures"] for l in lines), lines


@pytest.mark.skipif(_world() < 2 or os.environ.get("SPARKNET_TEST_NVLS") != "1",
                    reason="needs two or more GPUs and SPARKNET_TEST_NVLS=1")
def test_multiprocess_collectives_nvls():
    lines = run_workers(_world(), {"SPARKNET_NVLS": "1"})
    assert len(lines) == _world() and all(not l["failures"] for l in lines), lines


@pytest.mark.skipif(_world() < 2, reason="needs two or more GPUs")
def test_multiprocess_tp_decode_arms_agree():
    lines = run_workers(_world(), script="decode_worker.py")
    assert len(lines) == _world() and all(not l["failures"] and l["rt_health"] is None for l in lines), lines


@pytest.mark.skipif(_world() < 2, reason="needs two or more GPUs")
def test_multiprocess_fused_prefill_gemms():
    lines = run_workers(_world(), {"SPARKNET_PREFILL_BENCH": "0"}, script="prefill_worker.py")
    assert len(lines) == _world() and all(l["correct"] and not l["failures"] for l in lines), lines


@pytest.mark.skipif(_world() < 2, reason="needs two or more GPUs")
def test_multiprocess_trace_records_peer_arrivals():
    lines = run_workers(_world(), {"SPARKNET_TRACE": "1"})
    assert len(lines) == _world() and all(not l["failures"] and l["trace"]["collectives"] > 10 for l in lines), lines


@pytest.mark.skipif(_world() < 2, reason="needs two or more GPUs")
def test_failstop_qualification_two_gpus():
    """The fail-stop probe on 2 GPUs, NVLS off: the victim skips one collective on the
    host (it stays alive, launches nothing); the survivor's bounded wait must end within
    0.9 x timeout .. 3 x timeout + 2 s with a report naming the victim, then every rank
    re-arms and a healthy all-reduce is exact, eagerly and from a CUDA graph."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", SPARKNET_NVLS="0")
    cmd = ["timeout", "-k", "30", "400", sys.executable, "-m", "sparknet.probe.failstop", "--world", "2",
           "--timeout-ms", "1000", "--victim", "1", "--port", str(29300 + os.getpid() % 500)]
    proc = subprocess.run(cmd, env=env, cwd=ROOT, capture_output=True, text=True, timeout=460)
    lines = [l for l in proc.stdout.splitlines() if l.startswith("{")]
    assert lines, proc.stdout[-2000:] + proc.stderr[-3000:]
    result = json.loads(lines[-1])
    out_dir = os.environ.get("SPARKNET_TEST_OUT")
    if out_dir:
        Path(out_dir, "failstop_w2.json").write_text(json.dumps(result, indent=1))
    assert proc.returncode == 0 and result["passed"], result
    survivor = next(r for r in result["results"] if r["rank"] == 0)
    assert survivor["eager"]["detected"] and "waiting for rank 1" in survivor["eager"]["report"]
