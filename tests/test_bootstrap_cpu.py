"""Host side of the symmetric-memory bootstrap with real gloo ranks on CPU.

The descriptor exchange (abstract unix sockets, SCM_RIGHTS, world rounds) and the
collective verdicts run exactly as on a GPU box; memfds stand in for VMM handles.
Failures are made on the host: a rank that reports an error, a rank that never
serves its descriptor.
"""

import os
import sys
from pathlib import Path

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

ROOT = Path(__file__).resolve().parent.parent


def _init(rank, world, store_path):
    sys.path.insert(0, str(ROOT))
    dist.init_process_group("gloo", init_method=f"file://{store_path}", rank=rank, world_size=world)


def _fd_worker(rank, world, store_path, results):
    _init(rank, world, store_path)
    from sparknet import _native
    from sparknet.oneshot import symm

    C = _native.load()
    fd = os.memfd_create(f"r{rank}")
    os.write(fd, f"payload-from-{rank}".encode())
    fds = symm._pass_descriptors(C, fd, dist.group.WORLD, rank, world, "tok" + store_path[-6:])
    got = {}
    for peer, pfd in enumerate(fds):
        if peer != rank:
            got[peer] = os.pread(pfd, 64, 0).decode()
            os.close(pfd)
    root = symm._share_from_root(C, fd if rank == 0 else -1, dist.group.WORLD, rank, world,
                                 "root" + store_path[-6:])
    got["root"] = os.pread(root, 64, 0).decode() if rank else "self"
    results[rank] = got
    dist.destroy_process_group()


def _verdict_worker(rank, world, store_path, results):
    _init(rank, world, store_path)
    from sparknet.oneshot import symm

    try:
        symm.collective_check("no device" if rank == 1 else None, dist.group.WORLD, "setup")
        results[rank] = "passed"
    except RuntimeError as exc:
        results[rank] = str(exc)
    dist.destroy_process_group()


def _fetch_without_server_worker(rank, world, store_path, results):
    _init(rank, world, store_path)
    from sparknet import _native

    C = _native.load()
    try:
        C.fd_fetch("sparknet-nobody-serves-this-" + store_path[-6:], 300)
        results[rank] = "fetched?"
    except RuntimeError as exc:
        results[rank] = str(exc)
    dist.destroy_process_group()


def spawn(fn, world, tmp_path):
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    store = str(tmp_path / "store")
    mp.start_processes(fn, args=(world, store, results), nprocs=world, join=True, start_method="spawn")
    return dict(results)


@pytest.mark.parametrize("world", [2, 4])
def test_descriptor_exchange(tmp_path, world):
    results = spawn(_fd_worker, world, tmp_path)
    for rank in range(world):
        got = results[rank]
        for peer in range(world):
            if peer != rank:
                assert got[peer] == f"payload-from-{peer}"
        assert got["root"] in ("self", "payload-from-0")


def test_collective_verdict_names_the_failing_rank(tmp_path):
    results = spawn(_verdict_worker, 3, tmp_path)
    assert all("rank 1: no device" in v for v in results.values()), results


def test_fetch_gives_up_when_nobody_serves(tmp_path):
    results = spawn(_fetch_without_server_worker, 1, tmp_path)
    assert "cannot connect" in results[0] or "no descriptor" in results[0]
