"""Static checks over the native sources (CPU only), after the reference's header and
PTX-string checks (reference tests/test_oneshot_cpu.py: required PTX present,
record-then-fence-then-trap ordering).  Here they guard the rules the device code
keeps on a shared GPU pool:

* nothing traps: no ``trap`` instruction, ``__trap()``, ``__brkpt()`` or device
  ``assert`` (a failed wait ends in a status word and the context stays usable);
* every bulk copy is a plain per-CTA copy: its qualifiers come from a short
  allow-list (the collective and fused GEMM kernels run on several GPUs, so each CTA
  loads its own tiles);
* the protocols' memory-ordering and NVLS instructions are where the runtime
  expects them.
"""

import re
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
SOURCES = sorted(p for p in (ROOT / "csrc").rglob("*") if p.suffix in (".cu", ".cuh", ".h", ".cpp"))

BULK_COPY = re.compile(r"cp\.async\.bulk[\w.:]*")
# The qualifiers a bulk copy here may carry.  Anything else (a new state space, a
# cluster-wide delivery mode, a gather form) fails the check until reviewed.
ALLOWED_BULK_QUALIFIERS = {
    "cp", "async", "bulk", "tensor", "1d", "2d", "3d", "4d", "5d", "tile",
    "shared::cluster", "shared::cta", "global", "mbarrier::complete_tx::bytes",
    "bulk_group", "prefetch", "L2", "L2::cache_hint", "commit_group", "wait_group", "read",
    # a CTA-pair GEMM's tile load: into the issuing CTA's own shared memory, completing
    # on an mbarrier that may sit in the other CTA of the pair
    "cta_group::2",
}


def code_lines(path):
    """(line number, text) with // comments and /* */ blocks removed."""
    text = path.read_text()
    text = re.sub(r"/\*.*?\*/", lambda m: "\n" * m.group(0).count("\n"), text, flags=re.S)
    for number, line in enumerate(text.splitlines(), 1):
        yield number, line.split("//", 1)[0]


def test_sources_found():
    names = {p.name for p in SOURCES}
    assert {"proto.h", "dev_mem.cuh", "collectives.cu", "gemm_tcgen05.cu", "gemm_skinny.cu"} <= names


def test_nothing_traps():
    banned = re.compile(r"\btrap\s*;|__trap\s*\(|__brkpt\s*\(|(?<!static_)\bassert\s*\(")
    hits = [f"{p.relative_to(ROOT)}:{n}: {line.strip()}" for p in SOURCES for n, line in code_lines(p)
            if banned.search(line)]
    assert not hits, hits


def _qualifiers(instruction):
    """Split ``cp.async.bulk.x.y::z`` into its dot-separated parts (``::`` stays inside a part)."""
    return instruction.split(".")


def test_bulk_copies_are_per_cta():
    found, hits = 0, []
    for p in SOURCES:
        for n, line in code_lines(p):
            for m in BULK_COPY.finditer(line):
                found += 1
                extra = set(_qualifiers(m.group(0))) - ALLOWED_BULK_QUALIFIERS
                if extra:
                    hits.append(f"{p.relative_to(ROOT)}:{n}: {sorted(extra)}")
    assert found >= 2 and not hits, hits


def test_protocol_instructions_present():
    dev_mem = (ROOT / "csrc" / "include" / "sparknet" / "dev_mem.cuh").read_text()
    for instruction in ("ld.acquire.sys", "st.release.sys", "fence.acq_rel.sys", "ld.volatile",
                        "multimem.ld_reduce", "multimem.st"):
        assert instruction in dev_mem, instruction
    gemm = (ROOT / "csrc" / "include" / "sparknet" / "tc_gemm.cuh").read_text()
    for instruction in ("tcgen05.mma", "tcgen05.alloc", "tcgen05.ld", "cp.async.bulk.tensor"):
        assert instruction in gemm, instruction


def test_every_poll_loop_is_bounded():
    """The protocol's waits go through keep_waiting (clock, poison and timeout checks)."""
    proto = (ROOT / "csrc" / "include" / "sparknet" / "proto.h").read_text()
    loops = len(re.findall(r"while \(pending\)", proto))
    assert loops >= 3 and proto.count("keep_waiting(m, w, c,") >= loops


def test_mbarrier_waits_are_bounded():
    """The one mbarrier wait loop (mbar_wait) gives up after kWaitLimit tries, setting the
    error word; every tcgen05 kernel waits through it."""
    users = [p for p in SOURCES if any("mbarrier.try_wait" in line or "mbarrier.test_wait" in line
                                       for _, line in code_lines(p))]
    assert [p.name for p in users] == ["tc_gemm.cuh"], users
    gemm = (ROOT / "csrc" / "include" / "sparknet" / "tc_gemm.cuh").read_text()
    assert "for (uint32_t i = 0; i < kWaitLimit; ++i)" in gemm and "*err = kTcWaitTimeout;" in gemm
