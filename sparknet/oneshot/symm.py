"""Collective bootstrap of the NVLink symmetric regions (host side of N1).

Every rank of the exchange group (a gloo/CPU process group) calls
``build_regions`` together.  It allocates this rank's region in device memory
(``LocalRegion``: CUDA VMM, exported as a POSIX descriptor), hands descriptors to
every peer over abstract unix sockets in ``world`` rounds (rank k serves in round
k, the others fetch), maps every peer's region, and optionally builds the NVLS
multicast object (created by rank 0, joined by every rank's device, bound and
mapped).  Every failure is reported collectively: all ranks raise the same verdict.

Replaces the reference's blob exchange and queue-pair connection
(``sparknet/oneshot/runtime.py:595-676``, ``_roce_proxy.c:600-729``).
"""

from __future__ import annotations

import uuid
from dataclasses import dataclass, field
from typing import Any

import torch.distributed as dist

FD_TIMEOUT_MS = 60_000


def exchange(local: object, group) -> list[object]:
    """All-gather one picklable object from every rank of ``group``."""
    out: list[object] = [None] * dist.get_world_size(group=group)
    dist.all_gather_object(out, local, group=group)
    return out


def collective_check(error: str | None, group, what: str) -> None:
    """Raise on every rank if any rank reported an error."""
    verdicts = exchange(error, group)
    failures = [f"rank {i}: {v}" for i, v in enumerate(verdicts) if v is not None]
    if failures:
        raise RuntimeError(f"{what} failed: " + "; ".join(failures))


@dataclass
class Regions:
    local: Any
    bases: list[int]
    multicast: Any = None
    keep: list = field(default_factory=list)

    @property
    def mc_ptr(self) -> int:
        return int(self.multicast.mc_ptr) if self.multicast is not None else 0

    @property
    def mc_uc_ptr(self) -> int:
        return int(self.multicast.uc_ptr) if self.multicast is not None else 0

    @property
    def mc_bytes(self) -> int:
        return int(self.multicast.bytes) if self.multicast is not None else 0


def _pass_descriptors(C, fd: int, group, rank: int, world: int, token: str) -> list[int]:
    """Every rank's descriptor for ``fd`` (this rank's slot holds -1)."""
    names = [f"sparknet-{token}-{r}" for r in range(world)]
    listener = C.fd_listen(names[rank])
    fds = [-1] * world
    try:
        dist.barrier(group=group)
        for server in range(world):
            error = None
            try:
                if server == rank:
                    C.fd_serve(listener, fd, world - 1, FD_TIMEOUT_MS)
                else:
                    fds[server] = C.fd_fetch(names[server], FD_TIMEOUT_MS)
            except Exception as exc:  # noqa: BLE001 - reported collectively
                error = str(exc)
            collective_check(error, group, f"descriptor exchange round {server}")
    finally:
        C.fd_close(listener)
    return fds


def build_regions(C, *, group, device_index: int, region_bytes: int, multicast_bytes: int = 0) -> Regions:
    rank = dist.get_rank(group=group)
    world = dist.get_world_size(group=group)
    error, local = None, None
    try:
        local = C.LocalRegion(device_index, region_bytes, 0)
    except Exception as exc:  # noqa: BLE001
        error = str(exc)
    collective_check(error, group, "symmetric region allocation")
    sizes = exchange(int(local.bytes), group)
    if len(set(sizes)) != 1:
        raise RuntimeError(f"symmetric region sizes differ across ranks: {sizes}")
    bases = [0] * world
    bases[rank] = int(local.ptr)
    if world == 1:
        return Regions(local=local, bases=bases)
    token = exchange(uuid.uuid4().hex[:16] if rank == 0 else None, group)[0]
    fd = local.export_fd()
    try:
        fds = _pass_descriptors(C, fd, group, rank, world, token)
    finally:
        C.fd_close(fd)
    error = None
    try:
        for peer in range(world):
            if peer != rank:
                bases[peer] = int(local.map_peer(fds[peer], int(local.bytes)))
    except Exception as exc:  # noqa: BLE001
        error = str(exc)
    finally:
        for peer_fd in fds:
            if peer_fd >= 0:
                C.fd_close(peer_fd)
    collective_check(error, group, "peer mapping")
    regions = Regions(local=local, bases=bases)
    if multicast_bytes > 0:
        regions.multicast = _build_multicast(C, group=group, device_index=device_index, nbytes=multicast_bytes,
                                             rank=rank, world=world, token=token)
    return regions


def _share_from_root(C, fd: int, group, rank: int, world: int, name: str) -> int:
    """Rank 0's descriptor ``fd`` on every other rank (-1 on rank 0)."""
    listener = C.fd_listen(name) if rank == 0 else None
    got, error = -1, None
    try:
        dist.barrier(group=group)
        try:
            if rank == 0:
                C.fd_serve(listener, fd, world - 1, FD_TIMEOUT_MS)
            else:
                got = C.fd_fetch(name, FD_TIMEOUT_MS)
        except Exception as exc:  # noqa: BLE001 - reported collectively
            error = str(exc)
    finally:
        if listener is not None:
            C.fd_close(listener)
    collective_check(error, group, "descriptor broadcast")
    return got


def _build_multicast(C, *, group, device_index: int, nbytes: int, rank: int, world: int, token: str):
    """The NVLS multicast object, or None if any rank's device cannot join one."""
    error = None
    supported = False
    try:
        supported = bool(C.multicast_supported(device_index))
    except Exception as exc:  # noqa: BLE001
        error = str(exc)
    votes = exchange((error, supported), group)
    if any(v[0] for v in votes) or not all(v[1] for v in votes):
        return None
    error, fd, mc = None, -1, None
    try:
        mc = C.Multicast(device_index, nbytes, world)
        if rank == 0:
            fd = mc.create_and_export()
    except Exception as exc:  # noqa: BLE001
        error = str(exc)
    collective_check(error, group, "multicast creation")
    peer_fd = _share_from_root(C, fd, group, rank, world, f"sparknet-{token}-mc")
    error = None
    try:
        if rank != 0:
            mc.import_handle(peer_fd)
        mc.add_device()
    except Exception as exc:  # noqa: BLE001
        error = str(exc)
    finally:
        C.fd_close(fd)
        C.fd_close(peer_fd)
    collective_check(error, group, "multicast join")
    error = None
    try:
        mc.bind_and_map()
    except Exception as exc:  # noqa: BLE001
        error = str(exc)
    collective_check(error, group, "multicast bind")
    return mc
