#!/usr/bin/env python3
"""Render the recipe files: one JSON per (profile, example map) with the per-box
environment every rank starts with.  ``python recipes/generate.py`` rewrites them;
``--check`` exits 1 if a committed recipe is stale (after the reference's
``recipes/*.json``, rendered from the same sources)."""

from __future__ import annotations

import json
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

from sparknet import nccl, topology  # noqa: E402
from sparknet.topology import gpumap  # noqa: E402

EXAMPLE = ROOT / "sparknet" / "topology" / "examples" / "hgx-b200.json"
TRANSPORT_OF = {name: entry["transport"] for name, entry in nccl.PROFILES.items()}


def recipes() -> dict[str, dict]:
    gmap = gpumap.load(EXAMPLE)
    box = gmap["nodes"][0]["name"]
    out = {}
    for name, entry in nccl.PROFILES.items():
        transport = TRANSPORT_OF[name]
        env = topology.node_environment(gmap, box, transport, profile=name, by="index")
        out[name] = {
            "profile": name, "transport": transport, "gpus": list(entry["node_counts"]),
            "map_example": str(EXAMPLE.relative_to(ROOT)), "status": entry["status"],
            "evidence": entry["evidence"], "required_nccl_patches": nccl.required_patches(env),
            "environment": env, "problems": nccl.problems(env, world=gpumap.world_size(gmap["nodes"][0])),
        }
    return out


def main(argv=None) -> int:
    check = "--check" in (argv or sys.argv[1:])
    stale = []
    for name, recipe in recipes().items():
        path = ROOT / "recipes" / f"{name}.json"
        text = json.dumps(recipe, indent=2, sort_keys=True) + "\n"
        if check:
            if not path.exists() or path.read_text() != text:
                stale.append(path.name)
        else:
            path.write_text(text)
    if stale:
        print("stale recipes: " + ", ".join(stale))
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
