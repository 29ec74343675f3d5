"""Per-node environment for a transport and profile (replaces the reference's
``sparknet/topology/render.py:57-153``).

On an NVSwitch box the environment fixes the rank -> GPU order through
``CUDA_VISIBLE_DEVICES`` (ranks in map order, GPUs named by UUID so an index
renumbering cannot reorder them), the collective limits (``SPARKNET_*``), the NCCL
control settings of the profile, and the bootstrap interface for gloo/NCCL sockets.
Keys the renderer owns are refused in a base environment instead of silently
overridden.
"""

from __future__ import annotations

from . import gpumap

OWNED_KEYS = ("CUDA_VISIBLE_DEVICES", "NCCL_SOCKET_IFNAME", "GLOO_SOCKET_IFNAME", "MASTER_ADDR",
              "SPARKNET_WORLD_SIZE")


def base_problems(base: dict[str, str]) -> list[str]:
    """Keys a base environment must not set: the renderer owns them."""
    return [f"{key} is rendered from the map; remove it from the base environment" for key in OWNED_KEYS
            if key in base]


def visible_devices(node: dict, *, by: str = "uuid") -> str:
    """``CUDA_VISIBLE_DEVICES`` in rank order (local rank r sees the rank-r GPU as cuda:r)."""
    gpus = gpumap.ranked_gpus(node)
    if by == "index":
        return ",".join(str(g["index"]) for g in gpus)
    return ",".join(g["uuid"] for g in gpus)


def node_environment(gmap: dict, node_name: str, transport: str, *, profile: str | None = None,
                     base: dict[str, str] | None = None, by: str = "uuid") -> dict[str, str]:
    """The environment every rank process on ``node_name`` starts with."""
    errors = gpumap.problems(gmap, transport)
    if errors:
        raise ValueError("; ".join(errors))
    base = dict(base or {})
    errors = base_problems(base)
    if errors:
        raise ValueError("; ".join(errors))
    node = gpumap.node_by_name(gmap, node_name)
    head = gpumap.head_node(gmap)
    env = dict(base)
    if profile is not None:
        from sparknet.nccl.profiles import environment as profile_env, profile_problems

        problems = profile_problems(profile, transport, gpumap.world_size(node))
        if problems:
            raise ValueError("; ".join(problems))
        env.update(profile_env(profile))
    env["CUDA_VISIBLE_DEVICES"] = visible_devices(node, by=by)
    env["SPARKNET_WORLD_SIZE"] = str(gpumap.world_size(node))
    iface = node.get("management_interface")
    if iface:
        env["NCCL_SOCKET_IFNAME"] = iface
        env["GLOO_SOCKET_IFNAME"] = iface
    env["MASTER_ADDR"] = head.get("management_ip") or "127.0.0.1"
    if not gpumap.uses_oneshot(transport):
        for key in [k for k in env if k.startswith("SPARKNET_ALL")]:
            env.pop(key)
    if gpumap.uses_nvls(transport):
        env["SPARKNET_NVLS"] = "1"
        env.setdefault("NCCL_NVLS_ENABLE", "1")
    return env


def environment_problems(env: dict[str, str]) -> list[str]:
    """Settings that contradict each other in a rendered environment."""
    errors = []
    if env.get("SPARKNET_NVLS") == "1" and env.get("NCCL_NVLS_ENABLE") == "0":
        errors.append("SPARKNET_NVLS=1 with NCCL_NVLS_ENABLE=0: a box without NVLS for NCCL is unlikely to have it "
                      "for sparknet; enable both or neither")
    devices = env.get("CUDA_VISIBLE_DEVICES", "")
    if devices and len(set(devices.split(","))) != len(devices.split(",")):
        errors.append("CUDA_VISIBLE_DEVICES repeats a GPU")
    return errors


__all__ = ["OWNED_KEYS", "base_problems", "environment_problems", "node_environment", "visible_devices"]
