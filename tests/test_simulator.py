"""The protocol simulator: the production protocol bodies (proto.h) compiled for the
host and run with simulated ranks as threads (CPU only).

Covers BASELINE config 1: world 4, direct and ring4-like delivery, bf16 inputs of 5120
elements (10 KiB) per rank drawn N(0,1) from seed 0 per rank; every rank's output is
bit-identical and equal to the sequential rank-0..3 fp32-accumulate reference.
"""

import ctypes
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
SRC = ROOT / "tests" / "sim" / "simulate.cpp"
INCLUDES = ["-I" + str(ROOT / "csrc" / "include"), "-I" + str(ROOT / "tests" / "sim")]

pytestmark = pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")


def build(tmp: Path, name: str, flags: list[str], shared: bool) -> Path:
    out = tmp / name
    # every simulated collective runs with the slot bounds checks of the protocol header on
    cmd = ["g++", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-g", "-DSN_BOUNDS_CHECK", *flags, *INCLUDES, str(SRC),
           "-o", str(out), "-lpthread"]
    if shared:
        cmd[1:1] = ["-shared", "-fPIC"]
    else:
        cmd.insert(1, "-DSIM_MAIN")
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return out


@pytest.fixture(scope="module")
def sim_lib(tmp_path_factory):
    path = build(tmp_path_factory.mktemp("sim"), "libsim.so", ["-O2"], shared=True)
    lib = ctypes.CDLL(str(path))
    lib.sim_group_create.restype = ctypes.c_void_p
    lib.sim_group_create.argtypes = [ctypes.c_int, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64]
    lib.sim_group_destroy.argtypes = [ctypes.c_void_p]
    lib.sim_group_chaos.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_int]
    lib.sim_collective.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_uint32, ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p),
                                   ctypes.POINTER(ctypes.c_void_p), ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64,
                                   ctypes.c_uint64, ctypes.c_int, ctypes.c_uint32]
    lib.sim_lam_offset.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32]
    lib.sim_lam_offset.restype = ctypes.c_uint64
    lib.sim_ll_offset.argtypes = [ctypes.c_void_p]
    lib.sim_ll_offset.restype = ctypes.c_uint64
    lib.sim_read.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_uint64]
    for name in ("sim_failed_kind", "sim_failed_peer", "sim_poison"):
        getattr(lib, name).argtypes = [ctypes.c_void_p, ctypes.c_int]
        getattr(lib, name).restype = ctypes.c_uint32
    lib.sim_f32_to_bf16.argtypes = [ctypes.c_float]
    lib.sim_f32_to_bf16.restype = ctypes.c_uint16
    lib.sim_f32_to_f16.argtypes = [ctypes.c_float]
    lib.sim_f32_to_f16.restype = ctypes.c_uint16
    lib.sim_f16_to_f32.argtypes = [ctypes.c_uint16]
    lib.sim_f16_to_f32.restype = ctypes.c_float
    return lib


@pytest.fixture(scope="module")
def sanitized(tmp_path_factory):
    tmp = tmp_path_factory.mktemp("san")
    return {"asan": build(tmp, "sim_asan", ["-O1", "-fsanitize=address,undefined", "-fno-omit-frame-pointer",
                                             "-fno-sanitize-recover=all"], shared=False),
            "tsan": build(tmp, "sim_tsan", ["-O1", "-fsanitize=thread"], shared=False)}


def run_sim(lib, group, op, algo, dtype_code, blocks, tensors_in, tensors_out, nbytes, seed=1, timeout_us=5_000_000):
    ins = (ctypes.c_void_p * len(tensors_in))(*[t.data_ptr() for t in tensors_in])
    outs = (ctypes.c_void_p * len(tensors_out))(*[t.data_ptr() for t in tensors_out])
    return lib.sim_collective(group, op, algo, dtype_code, blocks, seed, nbytes, ins, outs, 0, 0, nbytes, nbytes, -1,
                              timeout_us)


@pytest.mark.parametrize("ring4", [0, 1])
@pytest.mark.parametrize("algo", [0, 1])
def test_baseline_config_one(sim_lib, ring4, algo):
    torch = pytest.importorskip("torch")
    world = 4
    # N(0,1) per rank from seeds counted from 0 (rank r draws from seed r)
    xs = [torch.randn(5120, generator=torch.Generator().manual_seed(r), dtype=torch.float32).to(torch.bfloat16)
          for r in range(world)]
    outs = [torch.empty_like(x) for x in xs]
    g = sim_lib.sim_group_create(world, 1 << 20, 1 << 18, 1 << 18)
    try:
        sim_lib.sim_group_chaos(g, 100, 8, 16, ring4)
        failed = run_sim(sim_lib, g, 1, algo, 1, 4, xs, outs, 5120 * 2)
    finally:
        sim_lib.sim_group_destroy(g)
    assert failed == 0
    acc = torch.zeros(5120, dtype=torch.float32)
    for x in xs:
        acc = acc + x.float()
    want = acc.to(torch.bfloat16)
    for o in outs:
        assert torch.equal(o.view(torch.int16), want.view(torch.int16))


def test_all_gather_ll_and_push(sim_lib):
    torch = pytest.importorskip("torch")
    world = 4
    xs = [torch.randn(5120, generator=torch.Generator().manual_seed(r)).to(torch.bfloat16) for r in range(world)]
    for algo in (0, 1):
        outs = [torch.empty(world * 5120, dtype=torch.bfloat16) for _ in range(world)]
        g = sim_lib.sim_group_create(world, 1 << 20, 1 << 18, 1 << 18)
        try:
            sim_lib.sim_group_chaos(g, 100, 8, 0, 0)
            assert run_sim(sim_lib, g, 2, algo, 1, 3, xs, outs, 5120 * 2) == 0
        finally:
            sim_lib.sim_group_destroy(g)
        for o in outs:
            assert torch.equal(o, torch.cat(xs))


def test_host_conversions_match_torch(sim_lib):
    torch = pytest.importorskip("torch")
    vals = torch.cat([torch.randn(4000) * 10 ** torch.randint(-40, 38, (4000,)).float(),
                      torch.tensor([0.0, -0.0, float("inf"), -float("inf"), 65504.0, 65520.0, 1e-8, 5.96e-8,
                                    2.98e-8, 3.0e-8, -1e-45, 3.4e38])])
    vals = vals[torch.isfinite(vals) | torch.isinf(vals)]
    for v in vals.tolist():
        bf = torch.tensor([v], dtype=torch.float32).to(torch.bfloat16).view(torch.int16).item() & 0xFFFF
        assert sim_lib.sim_f32_to_bf16(v) == bf, v
        h = torch.tensor([v], dtype=torch.float32).to(torch.float16).view(torch.int16).item() & 0xFFFF
        assert sim_lib.sim_f32_to_f16(v) == h, v
    for bits in range(0, 1 << 16, 7):
        want = torch.tensor([bits], dtype=torch.int32).to(torch.int16).view(torch.float16).float().item()
        got = sim_lib.sim_f16_to_f32(bits)
        assert (got == want) or (got != got and want != want), bits


@pytest.mark.parametrize("world,blocks,ring4", [(2, 1, 0), (4, 4, 0), (4, 3, 1), (8, 2, 0)])
def test_random_sequences_under_asan(sanitized, world, blocks, ring4):
    out = subprocess.run([str(sanitized["asan"]), "check", str(world), str(blocks), "120", str(world * 10 + blocks),
                          "60", str(ring4)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "passed" in out.stdout


def test_random_sequences_under_tsan(sanitized):
    out = subprocess.run([str(sanitized["tsan"]), "check", "4", "2", "60", "5", "60", "1"], capture_output=True,
                         text=True, timeout=300)
    assert out.returncode == 0 and "WARNING: ThreadSanitizer" not in out.stderr, out.stdout + out.stderr


def test_missing_rank_times_out_and_reset_recovers(sanitized):
    for world in (2, 4):
        out = subprocess.run([str(sanitized["asan"]), "timeout", str(world)], capture_output=True, text=True,
                             timeout=60)
        assert out.returncode == 0, out.stdout + out.stderr


def test_sequence_wrap_keeps_parity_alternating(sanitized):
    """Start 40 collectives before the 32-bit sequence wraps and run past it: results stay
    exact, every rank keeps the same epoch, and each collective's slot parity differs
    from the previous one's (0 is skipped by jumping to 2)."""
    out = subprocess.run([str(sanitized["asan"]), "check", "4", "2", "100", "77", "60", "0", str(0xFFFFFFFF - 40)],
                         capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "passed" in out.stdout


def test_slot_overflow_is_caught_by_the_bounds_checks(sim_lib):
    """A message two packs longer than the Lamport slot (the host-side capacity check
    bypassed): with the bounds checks on, each rank records kind 4 (bounds) for the
    Lamport slot check and is poisoned, and the area after each written slot keeps its
    idle contents: rank 0's pushes fill slot [1][0] of rank 1, followed by the
    never-written slot [1][1] (sentinel); rank 1's fill slot [1][1] of rank 0, the
    last Lamport slot, followed by the LL area (zeros).  Without the checks the same
    call reports success, and the first LL units of rank 0 end up all-ones: the
    overflow landed there and its consumer re-armed it with the sentinel."""
    torch = pytest.importorskip("torch")
    world, lam_cap = 2, 1 << 16
    n = (lam_cap + 32) // 2
    xs = [torch.randn(n, generator=torch.Generator().manual_seed(r)).to(torch.bfloat16) for r in range(world)]
    outs = [torch.empty_like(x) for x in xs]
    g = sim_lib.sim_group_create(world, lam_cap, 1 << 16, 1 << 16)
    try:
        failed = run_sim(sim_lib, g, 1, 0, 1, 2, xs, outs, n * 2, timeout_us=200_000)
        kinds = [sim_lib.sim_failed_kind(g, r) for r in range(world)]
        checks = [sim_lib.sim_failed_peer(g, r) for r in range(world)]
        poisoned = [sim_lib.sim_poison(g, r) for r in range(world)]
        after_slot = ctypes.create_string_buffer(256)
        sim_lib.sim_read(g, 1, sim_lib.sim_lam_offset(g, 1, 1), after_slot, 256)
        after_last = ctypes.create_string_buffer(256)
        sim_lib.sim_read(g, 0, sim_lib.sim_ll_offset(g), after_last, 256)
    finally:
        sim_lib.sim_group_destroy(g)
    assert failed == world and kinds == [4] * world and checks == [1] * world and poisoned == [1] * world
    assert after_slot.raw == b"\xff" * 256
    assert after_last.raw == b"\x00" * 256
