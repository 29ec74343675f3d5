"""GPU map schema and validation for NVSwitch boxes (replaces the reference's cabled
node maps, ``sparknet/topology/nodes.py:1-399``).

A map (``gpumap.json``) describes one or more boxes ("nodes"); each lists its GPUs
with their identity (UUID, PCI bus ID), NUMA node, active NVLink count, which peers
it reaches peer-to-peer over NVLink, and whether it can join an NVLS multicast
object.  A tensor-parallel group lives inside one box.  Every check here runs before
a process starts or a region is mapped: it reports configuration mistakes, not
whether NVLink actually delivers (the collective probe checks that).

Peers are identified by what they are (UUID / PCI bus ID from NVML), never by a
device index alone: the map fixes the rank -> GPU order that ``CUDA_VISIBLE_DEVICES``
then renders.
"""

from __future__ import annotations

import copy
import ipaddress
import json
import re
from pathlib import Path

SCHEMA_VERSION = 2
TRANSPORTS = (
    "nvlink",            # sparknet kernels (one-shot / two-shot) below dispatch, NCCL above
    "nvlink-nvls",       # as nvlink, with NVLS multicast enabled (opt-in, not rank-order sums)
    "nccl-nvlink",       # every collective on stock NCCL over NVLink (the control arm)
)
ONESHOT_TRANSPORTS = ("nvlink", "nvlink-nvls")
WORLD_SIZES = (1, 2, 4, 8)
MAX_GPUS_PER_NODE = 8
EXPECTED_NVLINKS = 18          # NVLink 5 on B200: 18 links per GPU
_GPU_FIELDS = {"index", "rank", "uuid", "pci_bus_id", "numa_node", "nvlinks_active", "p2p_peers", "multicast",
               "name"}
_NODE_FIELDS = {"name", "management_ip", "management_interface", "head", "nvswitch", "gpus", "driver", "cuda"}
_RETIRED_FIELDS = {
    "roce_peer_hcas": "NVSwitch connects every GPU to every peer: there are no per-peer routes; delete the field",
    "roce_subnets": "there is no RDMA fabric: peers are identified by GPU UUID; delete the field",
    "roce_hcas": "there is no RDMA fabric; delete the field",
    "nccl_hcas": "NCCL uses NVLink inside the box; delete the field",
    "roce_traffic_class": "there is no RoCE traffic; delete the field",
    "roce_gid_index": "there are no GIDs; delete the field",
    "mesh_ports": "there is no mesh forwarding on NVSwitch; delete the field",
}
REMOVED_NODE_FIELDS = _RETIRED_FIELDS
VIRTUAL_INTERFACES = ("lo", "docker", "br-", "veth", "virbr", "tailscale", "wl")
_INTERFACE_NAME = re.compile(r"[a-zA-Z0-9_.-]{1,15}")
_PCI = re.compile(r"[0-9a-fA-F]{4,8}:[0-9a-fA-F]{2}:[0-9a-fA-F]{2}\.[0-7]")
_UUID = re.compile(r"GPU-[0-9a-fA-F]{8}-[0-9a-fA-F]{4}-[0-9a-fA-F]{4}-[0-9a-fA-F]{4}-[0-9a-fA-F]{12}")


def load(path: str | Path) -> dict:
    """A GPU map from a JSON file."""
    return json.loads(Path(path).read_text())


def normalize_pci(bus_id: str) -> str:
    """``00000000:18:00.0`` and ``0000:18:00.0`` name the same function: 4-digit domain, lower case."""
    domain, rest = bus_id.strip().split(":", 1)
    return f"{int(domain, 16):04x}:{rest.lower()}"


def node_by_name(gmap: dict, name: str) -> dict:
    """The node called ``name`` (KeyError otherwise)."""
    for node in gmap.get("nodes", []):
        if node.get("name") == name:
            return node
    raise KeyError(f"node {name!r} is not in the map")


def head_node(gmap: dict) -> dict:
    """The map's one head node (ValueError unless exactly one)."""
    heads = [n for n in gmap.get("nodes", []) if n.get("head")]
    if len(heads) != 1:
        raise ValueError("exactly one head node is required")
    return heads[0]


def gpu_by_rank(node: dict, rank: int) -> dict:
    """The GPU entry of ``node`` with tensor-parallel rank ``rank``."""
    for gpu in node.get("gpus", []):
        if gpu.get("rank") == rank:
            return gpu
    raise KeyError(f"rank {rank} is not in node {node.get('name')!r}")


def ranked_gpus(node: dict) -> list[dict]:
    """The node's GPUs that carry a rank, in rank order."""
    return sorted((g for g in node.get("gpus", []) if g.get("rank") is not None), key=lambda g: g["rank"])


def uses_oneshot(transport: str) -> bool:
    """Whether ``transport`` runs this library's NVLink kernels (not NCCL only)."""
    return transport in ONESHOT_TRANSPORTS


def uses_nvls(transport: str) -> bool:
    """Whether ``transport`` uses the NVLS multicast kernels."""
    return transport == "nvlink-nvls"


def world_size(node: dict) -> int:
    """The number of ranked GPUs of ``node``."""
    return len(ranked_gpus(node))


def _interface_problems(label: str, name) -> list[str]:
    if name is None:
        return []
    if not isinstance(name, str) or not _INTERFACE_NAME.fullmatch(name):
        return [f"{label}: management_interface {name!r} is not an interface name"]
    if name.startswith(VIRTUAL_INTERFACES):
        return [f"{label}: management_interface {name!r} is virtual; name the wired interface"]
    return []


def node_problems(node: dict, transport: str) -> list[str]:
    """What is wrong with one node of the map for ``transport`` (empty when nothing)."""
    label = f"node {node.get('name', '?')}"
    errors: list[str] = []
    for field, why in _RETIRED_FIELDS.items():
        if field in node:
            errors.append(f"{label}: {field} is not read by this build: {why}")
    unknown = set(node) - _NODE_FIELDS - set(_RETIRED_FIELDS)
    if unknown:
        errors.append(f"{label}: unknown fields {sorted(unknown)}")
    if node.get("management_ip") is not None:
        try:
            ipaddress.IPv4Address(node["management_ip"])
        except (ValueError, ipaddress.AddressValueError):
            errors.append(f"{label}: management_ip {node['management_ip']!r} is not an IPv4 address")
    errors += _interface_problems(label, node.get("management_interface"))
    gpus = node.get("gpus")
    if not isinstance(gpus, list) or not gpus:
        return errors + [f"{label}: needs a non-empty gpus list"]
    if len(gpus) > MAX_GPUS_PER_NODE:
        errors.append(f"{label}: at most {MAX_GPUS_PER_NODE} GPUs per box")
    indices, uuids, pcis = [], [], []
    for gpu in gpus:
        glabel = f"{label} gpu {gpu.get('index', '?')}"
        unknown = set(gpu) - _GPU_FIELDS
        if unknown:
            errors.append(f"{glabel}: unknown fields {sorted(unknown)}")
        if not isinstance(gpu.get("index"), int) or gpu["index"] < 0:
            errors.append(f"{glabel}: index must be a non-negative integer")
        indices.append(gpu.get("index"))
        if not isinstance(gpu.get("uuid"), str) or not _UUID.fullmatch(gpu["uuid"]):
            errors.append(f"{glabel}: uuid must look like GPU-xxxxxxxx-xxxx-xxxx-xxxx-xxxxxxxxxxxx")
        uuids.append(gpu.get("uuid"))
        if not isinstance(gpu.get("pci_bus_id"), str) or not _PCI.fullmatch(gpu["pci_bus_id"]):
            errors.append(f"{glabel}: pci_bus_id must look like 0000:18:00.0")
            pcis.append(None)
        else:
            pcis.append(normalize_pci(gpu["pci_bus_id"]))
        links = gpu.get("nvlinks_active")
        if not isinstance(links, int) or links < 0:
            errors.append(f"{glabel}: nvlinks_active must be a non-negative integer")
    for what, values in (("index", indices), ("uuid", uuids), ("pci_bus_id", pcis)):
        seen = [v for v in values if v is not None]
        if len(set(seen)) != len(seen):
            errors.append(f"{label}: repeated GPU {what}")
    ranked = [g for g in gpus if g.get("rank") is not None]
    ranks = sorted(g["rank"] for g in ranked if isinstance(g.get("rank"), int))
    if len(ranks) != len(ranked) or ranks != list(range(len(ranks))):
        errors.append(f"{label}: GPU ranks must be 0..N-1 without gaps or repeats")
    if transport in TRANSPORTS and ranked and len(ranked) not in WORLD_SIZES:
        errors.append(f"{label}: a tensor-parallel group has {WORLD_SIZES} GPUs, not {len(ranked)}")
    if transport in ONESHOT_TRANSPORTS and len(ranked) > 1:
        if not node.get("nvswitch"):
            errors.append(f"{label}: the NVLink collectives need an NVSwitch box (nvswitch: true)")
        link_counts = {g.get("nvlinks_active") for g in ranked}
        if len(link_counts) != 1:
            errors.append(f"{label}: NVLink counts differ between GPUs {sorted(link_counts, key=str)} "
                          "(a degraded link halves the slowest rank)")
        elif 0 in link_counts:
            errors.append(f"{label}: no active NVLink on the tensor-parallel GPUs")
        by_index = {g.get("index"): g for g in gpus}
        for g in ranked:
            peers = set(g.get("p2p_peers", []))
            for h in ranked:
                if h is g:
                    continue
                if h.get("index") not in peers:
                    errors.append(f"{label}: gpu {g.get('index')} cannot reach gpu {h.get('index')} peer-to-peer")
            for p in peers:
                if p not in by_index:
                    errors.append(f"{label}: gpu {g.get('index')} lists unknown peer {p}")
        if uses_nvls(transport) and not all(g.get("multicast") for g in ranked):
            errors.append(f"{label}: nvlink-nvls needs every tensor-parallel GPU to support multicast")
    return errors


def problems(gmap: dict, transport: str) -> list[str]:
    """Every configuration mistake the map and transport selection contain."""
    errors: list[str] = []
    if transport not in TRANSPORTS:
        return [f"unknown transport {transport!r}; choose one of {', '.join(TRANSPORTS)}"]
    if gmap.get("schema_version") != SCHEMA_VERSION:
        errors.append(f"schema_version must be {SCHEMA_VERSION}")
    nodes = gmap.get("nodes")
    if not isinstance(nodes, list) or not nodes:
        return errors + ["the map needs a non-empty nodes list"]
    names = [n.get("name") for n in nodes]
    if len(set(names)) != len(names) or not all(isinstance(n, str) and n for n in names):
        errors.append("node names must be unique non-empty strings")
    heads = [n for n in nodes if n.get("head")]
    if len(heads) != 1:
        errors.append("exactly one head node is required")
    for node in nodes:
        errors += node_problems(node, transport)
    if len(nodes) > 1:
        sizes = {world_size(n) for n in nodes}
        if len(sizes) != 1:
            errors.append(f"every box must run the same tensor-parallel size, got {sorted(sizes)}")
        for node in nodes:
            if node.get("management_ip") is None:
                errors.append(f"node {node.get('name')}: a fleet of boxes needs management_ip on every node")
    return errors


def subset(gmap: dict, node_name: str, gpu_indices: list[int]) -> dict:
    """Carve a 1/2/4-GPU tensor-parallel group out of one box, ranks in the order given.

    The carved map keeps only that node and only those GPUs (re-ranked 0..N-1) and is
    validated like any other map.
    """
    if len(gpu_indices) not in WORLD_SIZES:
        raise ValueError(f"a subset has {WORLD_SIZES} GPUs, not {len(gpu_indices)}")
    if len(set(gpu_indices)) != len(gpu_indices):
        raise ValueError("a GPU appears twice in the subset")
    node = copy.deepcopy(node_by_name(gmap, node_name))
    by_index = {g["index"]: g for g in node["gpus"]}
    missing = [i for i in gpu_indices if i not in by_index]
    if missing:
        raise ValueError(f"node {node_name} has no GPU {missing}")
    keep = set(gpu_indices)
    gpus = []
    for rank, index in enumerate(gpu_indices):
        g = by_index[index]
        g["rank"] = rank
        g["p2p_peers"] = sorted(p for p in g.get("p2p_peers", []) if p in keep)
        gpus.append(g)
    node["gpus"] = gpus
    node["head"] = True
    out = {k: v for k, v in gmap.items() if k != "nodes"}
    out["nodes"] = [node]
    return out


__all__ = [
    "EXPECTED_NVLINKS", "ONESHOT_TRANSPORTS", "REMOVED_NODE_FIELDS", "SCHEMA_VERSION", "TRANSPORTS", "WORLD_SIZES",
    "gpu_by_rank", "head_node", "load", "node_by_name", "node_problems", "normalize_pci", "problems", "ranked_gpus",
    "subset", "uses_nvls", "uses_oneshot", "world_size",
]
