"""Run the collective probe on every box of a map at once and keep the receipts
(after the reference's ``sparknet/probe/fleet.py``).

Inside one box the probe is one container running ``torch.distributed.run`` with a
rank per GPU; a fleet of boxes runs one container per box over ssh, rendezvousing on
the head box.  Output per box: ``<out>/<box>.log`` and, when the probe printed its
result, ``<out>/<box>.json``.  The runner starts processes and waits; it changes
nothing else on a node.
"""

from __future__ import annotations

import json
import shlex
import subprocess
import time
from dataclasses import dataclass, field
from pathlib import Path
from typing import Callable

from sparknet.topology import gpumap

from .container import docker_probe_command

DEFAULT_SSH = ("ssh", "-o", "BatchMode=yes", "-o", "ConnectTimeout=15")


@dataclass
class BoxPlan:
    name: str
    node_rank: int
    target: str
    command: list[str]
    local: bool = False


@dataclass
class BoxOutcome:
    name: str
    returncode: int | None
    log: Path
    result: dict | None = None
    problems: list[str] = field(default_factory=list)

    @property
    def passed(self) -> bool:
        return self.returncode == 0 and self.result is not None and bool(self.result.get("passed")) \
            and not self.problems


def plan(gmap: dict, environments: dict[str, dict[str, str]], *, transport: str, image: str, port: int,
         probe_args: tuple[str, ...] = (), package_source: str | None = None,
         extra_env: dict[str, str] | None = None, ssh_user: str | None = None,
         target_field: str = "name", local_box: str | None = None) -> list[BoxPlan]:
    """One probe command per box of the map, with its rendered environment and ssh target."""
    head = gpumap.head_node(gmap)
    user = ssh_user or gmap.get("ssh_user")
    nodes = sorted(gmap["nodes"], key=lambda n: (not n.get("head"), n["name"]))
    plans = []
    for node_rank, node in enumerate(nodes):
        env = dict(environments[node["name"]])
        env.update(extra_env or {})
        command = docker_probe_command(image=image, environment=env, nproc=gpumap.world_size(node),
                                       node_rank=node_rank, nnodes=len(nodes),
                                       master_addr=head.get("management_ip") or "127.0.0.1", master_port=port,
                                       transport=transport, package_source=package_source,
                                       extra_args=tuple(probe_args))
        host = node[target_field] if target_field != "name" else node["name"]
        plans.append(BoxPlan(node["name"], node_rank, f"{user}@{host}" if user else host, command,
                             local=(node["name"] == local_box)))
    return plans


def ssh_command(p: BoxPlan, ssh: tuple[str, ...] = DEFAULT_SSH) -> list[str]:
    """The command that runs a box's probe: as is on the local box, through ssh otherwise."""
    if p.local:
        return list(p.command)
    return [*ssh, p.target, " ".join(shlex.quote(c) for c in p.command)]


def parse_result(text: str) -> dict | None:
    """The probe's JSON result line from a box's output, or None."""
    for line in reversed(text.splitlines()):
        line = line.strip()
        if line.startswith("{") and '"timings"' in line:
            try:
                return json.loads(line)
            except json.JSONDecodeError:
                continue
    return None


def run(plans: list[BoxPlan], out: str | Path, *, ssh: tuple[str, ...] = DEFAULT_SSH, timeout: float = 900.0,
        popen: Callable[..., subprocess.Popen] = subprocess.Popen) -> list[BoxOutcome]:
    """Start every box's probe at once, wait (bounded), and keep each box's log and result."""
    out = Path(out)
    out.mkdir(parents=True, exist_ok=True)
    running = []
    for p in plans:
        log = out / f"{p.name}.log"
        handle = log.open("w")
        running.append((p, log, handle, popen(ssh_command(p, ssh), stdout=handle, stderr=subprocess.STDOUT)))
    deadline = time.monotonic() + timeout
    outcomes = []
    for p, log, handle, proc in running:
        left = max(0.0, deadline - time.monotonic())
        try:
            rc = proc.wait(timeout=left)
        except subprocess.TimeoutExpired:
            proc.terminate()
            try:
                proc.wait(timeout=10)
            except subprocess.TimeoutExpired:
                proc.kill()
            rc = None
        handle.close()
        result = parse_result(log.read_text(errors="replace"))
        outcome = BoxOutcome(p.name, rc, log, result)
        if rc is None:
            outcome.problems.append("timed out")
        if result is not None:
            (out / f"{p.name}.json").write_text(json.dumps(result) + "\n")
        else:
            outcome.problems.append("no result line")
        outcomes.append(outcome)
    return outcomes


def bootstrap_warnings(gmap: dict, environments: dict[str, dict[str, str]]) -> list[str]:
    """A multi-box fleet without a socket interface often bootstraps gloo over the wrong NIC."""
    if len(gmap.get("nodes", [])) < 2:
        return []
    return [f"box {name}: no GLOO_SOCKET_IFNAME; gloo may pick a virtual interface"
            for name, env in environments.items() if not env.get("GLOO_SOCKET_IFNAME")]


__all__ = ["BoxOutcome", "BoxPlan", "bootstrap_warnings", "parse_result", "plan", "run", "ssh_command"]
