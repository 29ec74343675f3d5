"""The bounded container command that runs the collective probe on one box: a plan,
never executed here (after the reference's ``sparknet/probe/container.py:10-56``).

One container per box runs ``torch.distributed.run`` with one rank per GPU.  It
needs ``--ipc=host`` and the host network: ranks hand each other VMM descriptors over
abstract unix sockets and map peers' GPU memory, which a private IPC namespace per
rank would prevent.  Memory and lifetime are bounded.
"""

from __future__ import annotations

PROBE_CONTAINER = "sparknet-collective-probe"
DEFAULT_PACKAGE_TARGET = "/usr/local/lib/python3.12/dist-packages/sparknet"


def docker_probe_command(*, image: str, environment: dict[str, str], nproc: int, node_rank: int = 0,
                         nnodes: int = 1, master_addr: str = "127.0.0.1", master_port: int = 29650,
                         transport: str = "nvlink", package_source: str | None = None,
                         package_target: str = DEFAULT_PACKAGE_TARGET, memory: str = "64g",
                         timeout_seconds: int = 900, extra_args: tuple[str, ...] = ()) -> list[str]:
    """The bounded ``docker run`` command that runs the collective probe on one box (memory
    and time limits, the rendered environment, the GPUs and IPC it needs)."""
    env = dict(environment)
    env.setdefault("NCCL_DEBUG", "INFO")
    env.setdefault("NCCL_DEBUG_SUBSYS", "INIT,GRAPH")
    env["SPARKNET_TRANSPORT"] = transport
    command = ["docker", "run", "--rm", f"--name={PROBE_CONTAINER}", "--network=host", "--ipc=host", "--gpus=all",
               f"--memory={memory}", f"--memory-swap={memory}", "--ulimit=memlock=-1:-1", "--shm-size=8g",
               "--entrypoint=/usr/bin/timeout"]
    for key, value in sorted(env.items()):
        command.extend(["--env", f"{key}={value}"])
    if package_source:
        command.extend(["--volume", f"{package_source}:{package_target}:ro"])
    command.extend([image, "--signal=TERM", "--kill-after=30s", f"{timeout_seconds}s",
                    "python3", "-m", "torch.distributed.run", f"--nnodes={nnodes}", f"--node-rank={node_rank}",
                    f"--nproc-per-node={nproc}", f"--master-addr={master_addr}", f"--master-port={master_port}",
                    "-m", "sparknet.probe.collectives", *extra_args])
    return command


__all__ = ["DEFAULT_PACKAGE_TARGET", "PROBE_CONTAINER", "docker_probe_command"]
