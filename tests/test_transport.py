"""The transport seam (CPU only): geometry validation, capability reports, and the
host-staged double mapping peers' regions across real gloo ranks."""

import sys
from pathlib import Path

import pytest

from sparknet.transport import (Geometry, HostStagedTransport, NvlinkP2PTransport, NvlsTransport, Transport,
                                host_staged_capability)

ROOT = Path(__file__).resolve().parent.parent


def test_geometry_validation():
    assert Geometry(8, 3, 0, 1 << 20).validate() == []
    assert Geometry(9, 0, 0, 1 << 20).validate()
    assert Geometry(2, 2, 0, 1 << 20).validate()
    assert Geometry(2, 0, 0, 1000).validate()
    assert Geometry(2, 0, 0, 4096, multicast_bytes=100).validate()
    with pytest.raises(ValueError):
        NvlinkP2PTransport(Geometry(2, 5, 0, 4096))


def test_protocol_conformance():
    t = HostStagedTransport(Geometry(1, 0, 0, 4096))
    try:
        assert isinstance(t, Transport)
        assert host_staged_capability().available
    finally:
        t.close()
    for cls in (NvlinkP2PTransport, NvlsTransport):
        assert isinstance(cls(Geometry(2, 0, 0, 4096)), Transport)


def _worker(rank, world, store, results):
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"file://{store}", rank=rank, world_size=world)
    t = HostStagedTransport(Geometry(world, rank, 0, 8192))
    t.connect(dist.group.WORLD)
    t.start()
    # write a byte into slot [rank] of every peer's region
    for peer in range(world):
        t.buffer(peer)[rank] = 100 + rank
    dist.barrier()
    mine = bytes(t.buffer(rank)[:world])
    results[rank] = (list(mine), len(t.bases()), t.stats()["transport"])
    dist.barrier()
    t.stop()
    t.close()
    dist.destroy_process_group()


def test_host_staged_regions_shared_across_ranks(tmp_path):
    import torch.multiprocessing as mp

    world = 3
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_worker, args=(world, str(tmp_path / "s"), results), nprocs=world, join=True,
                       start_method="spawn")
    for rank in range(world):
        seen, nbases, name = results[rank]
        assert seen == [100 + r for r in range(world)] and nbases == world and name == "host-staged"
