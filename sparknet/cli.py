"""sparknet: GPU maps, NCCL control profiles, the collective policy and the fabric probe
for tensor-parallel inference on NVSwitch (B200) boxes.

Command tree after the reference's (``sparknet/cli.py:332-462``):

  sparknet topology validate|render|example|discover|subset|inventory
  sparknet nccl env|validate|profiles|patches
  sparknet policy show
  sparknet probe doctor|nvlink|gpudirect|counters|render-command|fleet|summarize|collectives|failstop

Everything except ``probe collectives`` and ``probe failstop`` runs without torch.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

from sparknet import __version__
from sparknet import nccl as nccl_profiles
from sparknet import topology
from sparknet.topology import gpumap

EXAMPLES = Path(__file__).resolve().parent / "topology" / "examples"


def _print_env(env: dict[str, str], as_json: bool) -> None:
    """An environment as one JSON object, or as ``export``-ready ``KEY=value`` lines in
    key order (values quoted for a POSIX shell only where they need it)."""
    import shlex

    text = json.dumps(env, indent=2, sort_keys=True) if as_json else \
        "\n".join(f"{k}={shlex.quote(str(v))}" for k, v in sorted(env.items()))
    if text:
        print(text)


def cmd_topology_validate(args) -> int:
    errors = gpumap.problems(gpumap.load(args.map), args.transport)
    for e in errors:
        print(f"error: {e}", file=sys.stderr)
    if not errors:
        print(f"{args.map}: valid for {args.transport}")
    return 1 if errors else 0


def cmd_topology_render(args) -> int:
    try:
        env = topology.node_environment(gpumap.load(args.map), args.node, args.transport, profile=args.profile,
                                        by=args.by)
    except (KeyError, ValueError) as exc:
        print(f"error: {exc}", file=sys.stderr)
        return 1
    _print_env(env, args.json)
    return 0


def cmd_topology_example(args) -> int:
    path = EXAMPLES / f"{args.name}.json"
    if not path.exists():
        names = ", ".join(sorted(p.stem for p in EXAMPLES.glob("*.json")))
        print(f"error: no example {args.name!r}; choose {names}", file=sys.stderr)
        return 1
    print(path.read_text(), end="")
    return 0


def cmd_topology_discover(args) -> int:
    from sparknet.topology import discover

    multicast = None
    if not args.no_cuda:
        multicast = discover.cuda_multicast_query
    try:
        inventory = discover.local_inventory(multicast=multicast)
    except Exception as exc:  # noqa: BLE001
        print(f"error: NVML discovery failed: {exc}", file=sys.stderr)
        return 1
    ranks = [int(r) for r in args.ranks.split(",")] if args.ranks else None
    gmap = discover.generate_map(inventory, name=args.name, management_ip=args.management_ip,
                                 management_interface=args.management_interface, ranks=ranks)
    text = json.dumps(gmap, indent=2) + "\n"
    if args.out:
        Path(args.out).write_text(text)
    else:
        print(text, end="")
    errors = gpumap.problems(gmap, args.transport)
    for e in errors:
        print(f"warning: {e}", file=sys.stderr)
    return 0


def cmd_topology_subset(args) -> int:
    try:
        carved = gpumap.subset(gpumap.load(args.map), args.node, [int(i) for i in args.gpus])
    except (KeyError, ValueError) as exc:
        print(f"error: {exc}", file=sys.stderr)
        return 1
    text = json.dumps(carved, indent=2) + "\n"
    if args.out:
        Path(args.out).write_text(text)
    else:
        print(text, end="")
    return 0


def cmd_topology_inventory(args) -> int:
    from sparknet.topology import discover

    try:
        inventory = discover.local_inventory(multicast=None if args.no_cuda else discover.cuda_multicast_query)
    except Exception as exc:  # noqa: BLE001
        print(f"error: NVML discovery failed: {exc}", file=sys.stderr)
        return 1
    print(json.dumps(inventory, indent=2))
    return 0


def cmd_nccl_env(args) -> int:
    _print_env(nccl_profiles.environment(args.profile), args.json)
    return 0


def _read_env_file(path: str) -> dict[str, str]:
    env = {}
    for line in Path(path).read_text().splitlines():
        line = line.strip()
        if not line or line.startswith("#"):
            continue
        key, _, value = line.partition("=")
        env[key.strip()] = value.strip()
    return env


def cmd_nccl_validate(args) -> int:
    env = nccl_profiles.environment(args.profile)
    if args.env_file:
        env.update(_read_env_file(args.env_file))
    world = args.gpus or nccl_profiles.profile(args.profile)["node_counts"][-1]
    errors = nccl_profiles.problems(env, world=world)
    for e in errors:
        print(f"error: {e}", file=sys.stderr)
    if not errors:
        print(f"profile {args.profile}: consistent for {world} GPUs")
    return 1 if errors else 0


def cmd_nccl_profiles(args) -> int:
    for name, entry in nccl_profiles.PROFILES.items():
        print(f"{name:22s} {entry['transport']:12s} GPUs {','.join(map(str, entry['node_counts']))}: "
              f"{entry['status']}")
    return 0


def cmd_nccl_patches(args) -> int:
    from sparknet.nccl import patchset

    if args.export:
        for path in patchset.export(args.export):
            print(path)
        return 0
    print(patchset.README, end="")
    return 0


def cmd_policy_show(args) -> int:
    from sparknet.policy import CollectivePolicy, policy_for_profile

    if args.profile:
        policy = policy_for_profile(args.profile)
        if policy is None:
            print(f"profile {args.profile}: every collective on NCCL")
            return 0
    else:
        try:
            policy = CollectivePolicy.from_environment(dict(os.environ))
        except ValueError as exc:
            print(f"error: {exc}", file=sys.stderr)
            return 1
    print(json.dumps({
        "all_reduce_dispatch_bytes": policy.all_reduce_dispatch_bytes,
        "all_reduce_capacity_bytes": policy.all_reduce_capacity_bytes,
        "all_gather_shard_bytes": policy.all_gather_shard_bytes,
        "oneshot_max_bytes": {str(k): v for k, v in policy.oneshot_max_bytes.items() if v < (1 << 62)},
        "ll_max_bytes": policy.ll_max_bytes, "allow_nvls": policy.allow_nvls,
        "examples": {f"{w} GPUs, {n} B bf16": policy.all_reduce_backend(n, "bfloat16", world=w)
                     for w in (2, 4, 8) for n in (10240, 491520, 2097152, 4194304)},
    }, indent=2))
    return 0


def cmd_policy_derive(args) -> int:
    """Sweep receipts (one ``W=<world>:<receipt.json>`` per world size) -> the measured
    table the policy's defaults are derived from, plus the limits it implies."""
    from sparknet.policy import derive_limits, sweep_rows

    rows = []
    for item in args.receipts:
        world, _, path = item.partition(":")
        if not world.startswith("W=") or not path:
            print(f"error: expected W=<world>:<receipt.json>, got {item!r}", file=sys.stderr)
            return 2
        rows += sweep_rows(json.loads(Path(path).read_text()), int(world[2:]))
    if not rows:
        print("error: no all-reduce or all-gather sweep rows in the receipts", file=sys.stderr)
        return 1
    limits = derive_limits(rows)
    order = lambda r: (r.get("operation", "all_reduce"), r["world"], r["nbytes"], r["arm"])  # noqa: E731
    table = {"source": args.source, "rows": sorted(rows, key=order),
             "derived": {"oneshot_max": limits.oneshot_max, "dispatch_max": limits.dispatch_max,
                         "nvls_min": limits.nvls_min, "ll_max": limits.ll_max}}
    text = json.dumps(table, indent=1, sort_keys=False)
    if args.output:
        Path(args.output).write_text(text + "\n")
    print(json.dumps(table["derived"], indent=2))
    return 0


def cmd_probe_doctor(args) -> int:
    from sparknet.probe.doctor import local_problems

    errors = local_problems(gpumap.load(args.map), args.node, args.transport)
    for e in errors:
        print(f"error: {e}", file=sys.stderr)
    if not errors:
        print(f"{args.node}: ready for {args.transport}")
    return 1 if errors else 0


def cmd_probe_nvlink(args) -> int:
    from sparknet.probe.nvlink_report import nvlink_report, render

    report = nvlink_report()
    print(json.dumps(report, indent=2) if args.json else render(report), end="" if not args.json else "\n")
    return 0 if report.get("ready", {}).get("p2p") else 1


def cmd_probe_counters(args) -> int:
    """NVLink counters of every GPU (NVML, read-only): a snapshot, or with --interval the
    counters that moved over that many seconds; exit 1 if an error counter moved."""
    import time

    from sparknet.probe import counters

    before = counters.nvlink_counters()
    if args.interval <= 0:
        print(json.dumps(before, indent=2, sort_keys=True))
        return 0
    time.sleep(args.interval)
    after = counters.nvlink_counters()
    errors = counters.error_deltas(before, after)
    moved = errors if args.errors_only else counters.deltas(before, after)
    print(json.dumps({"interval_s": args.interval, "deltas": moved, "error_counters_moved": bool(errors)},
                     indent=2, sort_keys=True))
    return 1 if errors else 0


def _environments(gmap: dict, transport: str, profile: str | None) -> dict[str, dict[str, str]]:
    return {node["name"]: topology.node_environment(gmap, node["name"], transport, profile=profile)
            for node in gmap["nodes"]}


def _extra_env(pairs) -> dict[str, str]:
    out = {}
    for pair in pairs or []:
        key, sep, value = pair.partition("=")
        if not sep:
            raise ValueError(f"--env takes KEY=VALUE, got {pair!r}")
        out[key] = value
    return out


def cmd_probe_render_command(args) -> int:
    from sparknet.probe.container import docker_probe_command

    gmap = gpumap.load(args.map)
    env = topology.node_environment(gmap, args.node, args.transport, profile=args.profile)
    env.update(_extra_env(args.env))
    node = gpumap.node_by_name(gmap, args.node)
    head = gpumap.head_node(gmap)
    names = [n["name"] for n in sorted(gmap["nodes"], key=lambda n: (not n.get("head"), n["name"]))]
    command = docker_probe_command(image=args.image, environment=env, nproc=gpumap.world_size(node),
                                   node_rank=names.index(args.node), nnodes=len(names),
                                   master_addr=head.get("management_ip") or "127.0.0.1", master_port=args.port,
                                   transport=args.transport, package_source=args.package_source,
                                   extra_args=tuple(args.probe_args))
    import shlex

    print(" ".join(shlex.quote(c) for c in command))
    return 0


def cmd_probe_fleet(args) -> int:
    from sparknet.probe import fleet, summary

    gmap = gpumap.load(args.map)
    errors = gpumap.problems(gmap, args.transport)
    if errors:
        for e in errors:
            print(f"error: {e}", file=sys.stderr)
        return 1
    environments = _environments(gmap, args.transport, args.profile)
    for warning in fleet.bootstrap_warnings(gmap, environments):
        print(f"warning: {warning}", file=sys.stderr)
    plans = fleet.plan(gmap, environments, transport=args.transport, image=args.image, port=args.port,
                       probe_args=tuple(args.probe_args), package_source=args.package_source,
                       extra_env=_extra_env(args.env), ssh_user=args.ssh_user, target_field=args.target,
                       local_box=args.local)
    ssh = tuple(args.ssh.split()) if args.ssh else fleet.DEFAULT_SSH
    if args.dry_run:
        import shlex

        for p in plans:
            print(" ".join(shlex.quote(c) for c in fleet.ssh_command(p, ssh)))
        return 0
    outcomes = fleet.run(plans, args.out, ssh=ssh, timeout=args.timeout)
    for o in outcomes:
        print(f"{o.name}: {'passed' if o.passed else 'FAILED'} (rc={o.returncode}) {'; '.join(o.problems)}")
    if all(o.result for o in outcomes):
        print(summary.markdown({args.label: summary.cases(summary.load_results(args.out))}), end="")
    return 0 if all(o.passed for o in outcomes) else 1


def cmd_probe_summarize(args) -> int:
    from sparknet.probe import summary

    labelled = {}
    for item in args.receipts:
        label, sep, directory = item.partition("=")
        if not sep:
            label, directory = Path(item).name, item
        labelled[label] = summary.cases(summary.load_results(directory))
    print(summary.markdown(labelled, dtype=args.dtype), end="")
    return 0


def cmd_probe_collectives(args) -> int:
    from sparknet.probe.collectives import main as probe_main

    return probe_main(args.probe_args)


def cmd_probe_failstop(args) -> int:
    from sparknet.probe.failstop import main as failstop_main

    return failstop_main(args.probe_args)


def parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(prog="sparknet", description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--version", action="version", version=f"sparknet {__version__}")
    sub = p.add_subparsers(dest="command", required=True)
    profiles = list(nccl_profiles.PROFILES)

    t = sub.add_parser("topology", help="GPU maps").add_subparsers(dest="subcommand", required=True)
    v = t.add_parser("validate", help="check a GPU map for a transport")
    v.add_argument("map")
    v.add_argument("--transport", required=True, choices=topology.TRANSPORTS)
    v.set_defaults(func=cmd_topology_validate)
    r = t.add_parser("render", help="per-box environment for a transport and profile")
    r.add_argument("map")
    r.add_argument("node")
    r.add_argument("--transport", required=True, choices=topology.TRANSPORTS)
    r.add_argument("--profile", choices=profiles)
    r.add_argument("--by", choices=("uuid", "index"), default="uuid", help="how CUDA_VISIBLE_DEVICES names GPUs")
    r.add_argument("--json", action="store_true")
    r.set_defaults(func=cmd_topology_render)
    e = t.add_parser("example", help="print an example GPU map")
    e.add_argument("name")
    e.set_defaults(func=cmd_topology_example)
    d = t.add_parser("discover", help="read this box's GPUs, NVLinks and P2P matrix through NVML")
    d.add_argument("--name")
    d.add_argument("--ranks", help="GPU indices in rank order, comma separated (default: all)")
    d.add_argument("--management-ip")
    d.add_argument("--management-interface")
    d.add_argument("--transport", choices=topology.TRANSPORTS, default="nvlink")
    d.add_argument("--no-cuda", action="store_true", help="skip the CUDA multicast query")
    d.add_argument("--out")
    d.set_defaults(func=cmd_topology_discover)
    ts = t.add_parser("subset", help="carve a 1/2/4-GPU group out of a box (ranks in the order given)")
    ts.add_argument("map")
    ts.add_argument("node")
    ts.add_argument("gpus", nargs="+", metavar="GPU")
    ts.add_argument("--out")
    ts.set_defaults(func=cmd_topology_subset)
    i = t.add_parser("inventory", help="this host's GPUs as NVML sees them")
    i.add_argument("--no-cuda", action="store_true")
    i.set_defaults(func=cmd_topology_inventory)

    n = sub.add_parser("nccl", help="NCCL control profiles").add_subparsers(dest="subcommand", required=True)
    ne = n.add_parser("env", help="print a profile's environment")
    ne.add_argument("--profile", required=True, choices=profiles)
    ne.add_argument("--json", action="store_true")
    ne.set_defaults(func=cmd_nccl_env)
    nv = n.add_parser("validate", help="check a profile, optionally with overrides from an env file")
    nv.add_argument("--profile", required=True, choices=profiles)
    nv.add_argument("--env-file")
    nv.add_argument("--gpus", type=int)
    nv.set_defaults(func=cmd_nccl_validate)
    n.add_parser("profiles", help="list profiles").set_defaults(func=cmd_nccl_profiles)
    np_ = n.add_parser("patches", help="the NCCL patch series (empty on B200)")
    np_.add_argument("--export", metavar="DIR")
    np_.set_defaults(func=cmd_nccl_patches)

    po = sub.add_parser("policy", help="collective policy").add_subparsers(dest="subcommand", required=True)
    ps = po.add_parser("show", help="the policy of a profile, or of this environment")
    ps.add_argument("--profile", choices=profiles)
    ps.set_defaults(func=cmd_policy_show)
    pv = po.add_parser("derive", help="measured policy table from probe sweep receipts")
    pv.add_argument("receipts", nargs="+", metavar="W=<world>:<receipt.json>")
    pv.add_argument("--output", default="", help="write the table (sparknet/policy/measured_b200.json)")
    pv.add_argument("--source", default="sparknet probe collectives --benchmark --sweep --counter-samples",
                    help="how the receipts were made (recorded in the table)")
    pv.set_defaults(func=cmd_policy_derive)

    pr = sub.add_parser("probe", help="fabric checks and the collective probe").add_subparsers(
        dest="subcommand", required=True)
    pd = pr.add_parser("doctor", help="GPU map against this host, read-only (NVML)")
    pd.add_argument("map")
    pd.add_argument("--node", required=True)
    pd.add_argument("--transport", required=True, choices=topology.TRANSPORTS)
    pd.set_defaults(func=cmd_probe_doctor)
    for name in ("nvlink", "gpudirect"):
        pg = pr.add_parser(name, help="what this host offers the NVLink transport (P2P, NVLS, fabric)")
        pg.add_argument("--json", action="store_true")
        pg.set_defaults(func=cmd_probe_nvlink)
    pc = pr.add_parser("counters", help="NVLink throughput and error counters (NVML, read-only)")
    pc.add_argument("--interval", type=float, default=0.0, help="seconds between two snapshots (0: one snapshot)")
    pc.add_argument("--errors-only", action="store_true", help="with --interval: only the error counters")
    pc.set_defaults(func=cmd_probe_counters)

    def probe_options(parser_):
        parser_.add_argument("--transport", required=True, choices=topology.TRANSPORTS)
        parser_.add_argument("--profile", choices=profiles)
        parser_.add_argument("--image", required=True)
        parser_.add_argument("--port", type=int, default=29650)
        parser_.add_argument("--package-source", metavar="DIR")
        parser_.add_argument("--env", action="append", metavar="KEY=VALUE")
        parser_.add_argument("probe_args", nargs="*", help="arguments after -- go to the probe (e.g. --benchmark)")

    rc = pr.add_parser("render-command", help="the bounded container command for one box's probe")
    rc.add_argument("map")
    rc.add_argument("node")
    probe_options(rc)
    rc.set_defaults(func=cmd_probe_render_command)
    pf = pr.add_parser("fleet", help="run every box's probe at once and keep the receipts")
    pf.add_argument("map")
    probe_options(pf)
    pf.add_argument("--out", default="probe-receipts")
    pf.add_argument("--label", default="probe")
    pf.add_argument("--ssh-user")
    pf.add_argument("--target", choices=("name", "management_ip"), default="name")
    pf.add_argument("--ssh")
    pf.add_argument("--local", help="run this box's probe locally instead of over ssh")
    pf.add_argument("--timeout", type=float, default=900.0)
    pf.add_argument("--dry-run", action="store_true")
    pf.set_defaults(func=cmd_probe_fleet)
    psm = pr.add_parser("summarize", help="latency tables from probe receipts (LABEL=DIR ...)")
    psm.add_argument("receipts", nargs="+", metavar="[LABEL=]DIR")
    psm.add_argument("--dtype", default="bfloat16")
    psm.set_defaults(func=cmd_probe_summarize)
    pc = pr.add_parser("collectives", help="run the probe on this rank (needs torch)")
    pc.add_argument("probe_args", nargs=argparse.REMAINDER)
    pc.set_defaults(func=cmd_probe_collectives)
    pfs = pr.add_parser("failstop", help="fail-stop qualification on 2 or 4 GPUs (needs torch)")
    pfs.add_argument("probe_args", nargs=argparse.REMAINDER)
    pfs.set_defaults(func=cmd_probe_failstop)
    return p


def split_pass_through(argv: list[str]) -> tuple[list[str], list[str] | None]:
    """``(own words, pass-through words)``: everything after the first bare ``--`` is
    handed to the wrapped program verbatim (``None`` when there is no ``--``), so the
    probe's own flags never reach this parser."""
    for position, word in enumerate(argv):
        if word == "--":
            return argv[:position], argv[position + 1:]
    return argv, None


def main(argv: list[str] | None = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    head, passed = split_pass_through(argv)
    args = parser().parse_args(head)
    if passed is not None:
        if hasattr(args, "probe_args"):
            args.probe_args = [*args.probe_args, *passed]
        else:
            parser().error(f"unexpected arguments after --: {' '.join(passed)}")
    return args.func(args)


if __name__ == "__main__":
    sys.exit(main())
