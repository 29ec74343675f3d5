"""The one-rank runtime on a real GPU: the ``local`` all-reduce (a copy kernel with
programmatic dependent launch) returns the input's exact bits, eagerly and as a
chain of graph-captured calls that each read the previous call's output."""

import json
import os
import subprocess
import sys
import tempfile
from pathlib import Path

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def test_one_rank_all_reduce_is_an_exact_copy():
    out_dir = tempfile.mkdtemp(prefix="sparknet-1r-")
    env = dict(os.environ, SPARKNET_TEST_OUT=out_dir)
    env.pop("SPARKNET_TRACE", None)
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=1", "--master-addr", "127.0.0.1", "--master-port", str(28500 + os.getpid() % 1000),
           str(ROOT / "tests" / "workers" / "single_rank_worker.py")]
    proc = subprocess.run(cmd, env=env, cwd=ROOT, capture_output=True, text=True, timeout=400)
    files = list(Path(out_dir).glob("rank0.json"))
    result = json.loads(files[0].read_text()) if files else None
    assert proc.returncode == 0 and result is not None, (result, proc.stdout[-3000:], proc.stderr[-5000:])
    assert not result["failures"] and result["checks"] >= 20, result
