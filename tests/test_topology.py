"""GPU maps: schema, validation, subsets, rendering and NVML discovery (CPU only).
After the reference's tests/test_topology.py, for NVSwitch boxes."""

import copy
import json
from pathlib import Path

import pytest

from sparknet import topology
from sparknet.topology import discover, gpumap
from tests.fake_nvml import FakeNVML

EX = Path(__file__).resolve().parent.parent / "sparknet" / "topology" / "examples"


@pytest.fixture
def box():
    return gpumap.load(EX / "hgx-b200.json")


@pytest.mark.parametrize("transport", gpumap.TRANSPORTS)
def test_examples_validate(box, transport):
    assert gpumap.problems(box, transport) == []
    assert gpumap.problems(gpumap.load(EX / "hgx-b200-fleet2.json"), transport) == []


def test_unknown_transport_and_schema(box):
    assert "unknown transport" in gpumap.problems(box, "oneshot-ring4")[0]
    bad = dict(box, schema_version=1)
    assert any("schema_version" in e for e in gpumap.problems(bad, "nvlink"))


def test_retired_reference_fields_are_refused(box):
    bad = copy.deepcopy(box)
    bad["nodes"][0]["roce_peer_hcas"] = {"1": ["rocep1s0f0"]}
    errors = gpumap.problems(bad, "nvlink")
    assert any("roce_peer_hcas is not read" in e for e in errors)


def test_ranks_must_be_dense_and_world_allowed(box):
    bad = copy.deepcopy(box)
    bad["nodes"][0]["gpus"][3]["rank"] = 9
    assert any("ranks must be 0..N-1" in e for e in gpumap.problems(bad, "nvlink"))
    three = copy.deepcopy(box)
    for g in three["nodes"][0]["gpus"][3:]:
        g["rank"] = None
    assert any("tensor-parallel group has" in e for e in gpumap.problems(three, "nvlink"))


def test_degraded_link_and_missing_p2p(box):
    bad = copy.deepcopy(box)
    bad["nodes"][0]["gpus"][5]["nvlinks_active"] = 17
    assert any("NVLink counts differ" in e for e in gpumap.problems(bad, "nvlink"))
    assert gpumap.problems(bad, "nccl-nvlink") == []   # the control arm does not need uniform links
    bad = copy.deepcopy(box)
    bad["nodes"][0]["gpus"][2]["p2p_peers"].remove(6)
    assert any("cannot reach gpu 6" in e for e in gpumap.problems(bad, "nvlink"))


def test_nvls_needs_multicast_everywhere(box):
    bad = copy.deepcopy(box)
    bad["nodes"][0]["gpus"][0]["multicast"] = False
    assert gpumap.problems(bad, "nvlink") == []
    assert any("multicast" in e for e in gpumap.problems(bad, "nvlink-nvls"))


def test_identity_checks(box):
    bad = copy.deepcopy(box)
    bad["nodes"][0]["gpus"][1]["uuid"] = bad["nodes"][0]["gpus"][0]["uuid"]
    assert any("repeated GPU uuid" in e for e in gpumap.problems(bad, "nvlink"))
    bad = copy.deepcopy(box)
    bad["nodes"][0]["gpus"][1]["pci_bus_id"] = "00000000:1B:00.0"   # same function as gpu 0, other spelling
    assert any("repeated GPU pci_bus_id" in e for e in gpumap.problems(bad, "nvlink"))
    assert gpumap.normalize_pci("00000000:1B:00.0") == "0000:1b:00.0"


def test_interfaces_and_fleet_rules():
    fleet = gpumap.load(EX / "hgx-b200-fleet2.json")
    bad = copy.deepcopy(fleet)
    bad["nodes"][1]["management_interface"] = "docker0"
    assert any("virtual" in e for e in gpumap.problems(bad, "nvlink"))
    bad = copy.deepcopy(fleet)
    bad["nodes"][1]["head"] = True
    assert any("exactly one head" in e for e in gpumap.problems(bad, "nvlink"))
    bad = copy.deepcopy(fleet)
    del bad["nodes"][1]["management_ip"]
    assert any("needs management_ip" in e for e in gpumap.problems(bad, "nvlink"))


@pytest.mark.parametrize("gpus", [[4, 5], [0, 2, 4, 6], [7], [3, 1]])
def test_subset(box, gpus):
    carved = gpumap.subset(box, "hgx-b200-1", gpus)
    assert gpumap.problems(carved, "nvlink") == []
    node = carved["nodes"][0]
    assert [g["index"] for g in gpumap.ranked_gpus(node)] == gpus
    assert topology.visible_devices(node, by="index") == ",".join(map(str, gpus))


def test_subset_refusals(box):
    with pytest.raises(ValueError):
        gpumap.subset(box, "hgx-b200-1", [0, 1, 2])
    with pytest.raises(ValueError):
        gpumap.subset(box, "hgx-b200-1", [1, 1])
    with pytest.raises(ValueError):
        gpumap.subset(box, "hgx-b200-1", [0, 9])


def test_render_environment(box):
    env = topology.node_environment(box, "hgx-b200-1", "nvlink", profile="nvlink")
    assert env["CUDA_VISIBLE_DEVICES"].count("GPU-") == 8
    assert env["SPARKNET_ALLREDUCE_CAPACITY_BYTES"] == "8388608"
    assert env["NCCL_SOCKET_IFNAME"] == env["GLOO_SOCKET_IFNAME"] == "eno1"
    assert env["MASTER_ADDR"] == "192.0.2.10"
    control = topology.node_environment(box, "hgx-b200-1", "nccl-nvlink", profile="nvlink-nccl-only")
    assert not any(k.startswith("SPARKNET_ALL") for k in control)
    nvls = topology.node_environment(box, "hgx-b200-1", "nvlink-nvls", profile="nvlink-nvls")
    assert nvls["SPARKNET_NVLS"] == "1" and nvls["NCCL_NVLS_ENABLE"] == "1"
    with pytest.raises(ValueError):
        topology.node_environment(box, "hgx-b200-1", "nvlink", base={"CUDA_VISIBLE_DEVICES": "0"})
    with pytest.raises(ValueError):
        topology.node_environment(box, "hgx-b200-1", "nvlink", profile="nvlink-nccl-only")
    assert topology.environment_problems({"SPARKNET_NVLS": "1", "NCCL_NVLS_ENABLE": "0"})


def test_discovery_from_fake_nvml():
    nv = FakeNVML()
    inventory = discover.local_inventory(nv, multicast=lambda i: True)
    assert inventory["nvswitch"] and len(inventory["gpus"]) == 8
    assert all(g["nvlinks_active"] == 18 and len(g["p2p_peers"]) == 7 for g in inventory["gpus"])
    gmap = discover.generate_map(inventory, name="box", management_ip="192.0.2.9", management_interface="eno1")
    assert gpumap.problems(gmap, "nvlink-nvls") == []
    gmap = discover.generate_map(inventory, name="box", ranks=[6, 7])
    assert gpumap.problems(gmap, "nvlink") == []
    assert [g["index"] for g in gpumap.ranked_gpus(gmap["nodes"][0])] == [6, 7]
    nv.links[3] = 9
    nv.p2p_broken.add((1, 5))
    broken = discover.generate_map(discover.local_inventory(nv), name="box")
    errors = gpumap.problems(broken, "nvlink")
    assert any("NVLink counts differ" in e for e in errors) and any("cannot reach" in e for e in errors)
    json.dumps(broken)
