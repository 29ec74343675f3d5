"""Host-side rules of the runtime that need no GPU: refused settings, timeout bounds,
device normalisation, support detection, alignment (CPU only)."""

import pytest

torch = pytest.importorskip("torch")


def test_reference_settings_are_refused_with_a_reason():
    from sparknet.oneshot.runtime import REMOVED_SETTINGS, removed_setting_problems

    assert removed_setting_problems({}) == []
    env = {"SPARKNET_ROCE_HCA": "mlx5_0", "SPARKNET_ROCE_TIMEOUT_MS": "100", "SPARKNET_TIMEOUT_MS": "100"}
    problems = removed_setting_problems(env)
    assert len(problems) == 2
    assert any("SPARKNET_ROCE_HCA" in p and "NVLink" in p for p in problems)
    assert any("renamed: set SPARKNET_TIMEOUT_MS" in p for p in problems)
    assert all(name.startswith("SPARKNET_ROCE_") for name in REMOVED_SETTINGS)


def test_timeout_bounds():
    from sparknet.oneshot.runtime import MAX_TIMEOUT_MS, checked_timeout_ms

    assert checked_timeout_ms(1) == 1 and checked_timeout_ms("250") == 250
    assert checked_timeout_ms(MAX_TIMEOUT_MS) == MAX_TIMEOUT_MS  # microseconds fit 32 bits
    for bad in (0, -5, MAX_TIMEOUT_MS + 1):
        with pytest.raises(ValueError):
            checked_timeout_ms(bad)


def test_devices_and_support_on_a_cpu_host():
    from sparknet.oneshot.runtime import align_up, is_supported, normalize_device

    assert normalize_device(3) == torch.device("cuda", 3)
    assert normalize_device("cuda:1") == torch.device("cuda", 1)
    with pytest.raises(ValueError):
        normalize_device("cpu")
    if not torch.cuda.is_available():
        assert is_supported() is False
    assert align_up(0, 16) == 0 and align_up(1, 16) == 16 and align_up(4096, 4096) == 4096


def test_codes_match_the_native_protocol():
    """The op and algorithm codes the runtime passes are the ones the kernels read."""
    from sparknet import _native
    from sparknet.oneshot.runtime import ALGO_CODES, GATHER_CODES

    assert ALGO_CODES == {"oneshot": 0, "twoshot": 1, "nvls": 2, "local": 3}
    assert GATHER_CODES == {"ll": 0, "push": 1, "nvls": 2}
    if _native.available():
        C = _native.load()
        assert int(C.MAX_RANKS) == 8 and int(C.ABI_VERSION) >= 5


def test_one_rank_all_reduce_is_the_local_copy():
    """At world size 1 the policy's choice becomes the copy kernel (an explicit
    algorithm passed to all_reduce still wins)."""
    from sparknet.oneshot.runtime import NvlinkAllReduce
    from sparknet.policy import NVLINK_POLICY

    rt = NvlinkAllReduce.__new__(NvlinkAllReduce)
    rt.policy = NVLINK_POLICY
    rt.has_multicast = False
    for world, want in ((1, "local"), (2, "oneshot"), (8, "oneshot")):
        rt.world_size = world
        assert rt.algorithm_for(10240, torch.bfloat16) == want
    rt.world_size = 1
    assert rt.algorithm_for(8 << 20, torch.bfloat16) == "local"


def test_algorithm_choice_is_memoised_per_policy():
    from sparknet.oneshot.runtime import NvlinkAllReduce
    from sparknet.policy import NVLINK_POLICY, CollectivePolicy

    rt = NvlinkAllReduce.__new__(NvlinkAllReduce)
    rt.policy, rt.has_multicast, rt.world_size = NVLINK_POLICY, False, 8
    rt._algo_cache, rt._algo_cache_policy = {}, None
    first = rt.algorithm_for(2 << 20, torch.bfloat16)
    assert rt.algorithm_for(2 << 20, torch.bfloat16) == first and len(rt._algo_cache) == 1
    # a different policy object is consulted afresh, not answered from the old entries
    rt.policy = CollectivePolicy(2 << 20, 8 << 20, 16 << 20, force="twoshot")
    assert rt.algorithm_for(10240, torch.bfloat16) == "twoshot" and len(rt._algo_cache) == 1


def test_stream_switch_orders_after_the_previous_stream(monkeypatch):
    """Eager calls on one stream record nothing; the first call on another stream first
    records an event on the previous stream and waits for it (everything the previous
    stream holds, the last collective included)."""
    from sparknet.oneshot.runtime import NvlinkAllReduce

    log = []

    class FakeStream:
        def __init__(self, name):
            self.name = name

        def wait_event(self, event):
            log.append(("wait", self.name, event))

    class FakeEvent:
        def record(self, stream):
            log.append(("record", stream.name))

    a, b = FakeStream("a"), FakeStream("b")
    current = {"s": a}
    monkeypatch.setattr(torch.cuda, "current_stream", lambda device=None: current["s"])
    rt = NvlinkAllReduce.__new__(NvlinkAllReduce)
    rt.device = torch.device("cuda", 0)
    rt._last_stream = rt._current_stream = rt._capture_stream = None
    rt._capture_id = 0
    rt._stream_event = FakeEvent()

    def call(stream):
        current["s"] = stream
        rt._order_stream(False)
        rt._mark_stream(False)

    call(a)
    call(a)
    call(a)
    assert log == []
    call(b)
    assert log == [("record", "a"), ("wait", "b", rt._stream_event)]
    call(b)
    assert len(log) == 2
    call(a)
    assert log[2:] == [("record", "b"), ("wait", "a", rt._stream_event)]


def test_entry_point_imports_the_built_extension_in_a_fresh_interpreter():
    """What the build check runs after compiling: a new interpreter that has not
    imported torch yet must still import the extension."""
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    if not list((root / "sparknet").glob("_C*.so")):
        pytest.skip("extension not built")
    proc = subprocess.run([sys.executable, "-c", "import __graft_entry__ as g; g.import_package(); print('ok')"],
                          cwd=root, capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0 and proc.stdout.strip().endswith("ok"), proc.stderr[-2000:]


def test_reference_exports_are_importable():
    """Every name the reference's sparknet.oneshot exports imports here too; on an
    NVSwitch box no RDMA device takes part, so discover_hcas() finds none."""
    import sparknet.oneshot as oneshot

    for name in ("API_VERSION", "AllReduce", "DEFAULT_MAX_GATHER_BYTES", "DEFAULT_MAX_SIZE",
                 "KernelResolutionFrozenError", "SUPPORTED_DTYPES", "SUPPORTED_WORLD_SIZES", "TOPOLOGIES",
                 "discover_hcas", "freeze_kernel_resolution", "is_supported", "thaw_kernel_resolution"):
        assert hasattr(oneshot, name), name
    assert oneshot.discover_hcas() == ()
    assert oneshot.discover_nvlink_gpus() == ()  # no CUDA device on this host


def test_attention_wrapper_rejects_unknown_variants():
    from sparknet.ops import decode_attention

    q = torch.zeros(1, 8, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="variant"):
        decode_attention(q, q, q, torch.ones(1, dtype=torch.int32), 1, variant="paged")


def test_freeze_gate_refuses_lazy_setup_and_counts():
    from sparknet.oneshot import _freeze

    _freeze.thaw_kernel_resolution()
    _freeze.raise_if_kernel_resolution_frozen("gather scratch allocation")  # open: no error
    before = _freeze.refused_resolutions()
    _freeze.freeze_kernel_resolution("serving warm-up done")
    try:
        assert _freeze.kernel_resolution_frozen()
        with pytest.raises(_freeze.KernelResolutionFrozenError) as info:
            _freeze.raise_if_kernel_resolution_frozen("alignment scratch allocation", target=object(), cache_key=(8, 2))
        text = str(info.value)
        assert "alignment scratch allocation for object" in text and "(8, 2)" in text
        assert "serving warm-up done" in text
        assert _freeze.refused_resolutions() == before + 1
    finally:
        _freeze.thaw_kernel_resolution()
    assert not _freeze.kernel_resolution_frozen()


def _bare_runtime(**attrs):
    """An NvlinkAllReduce shell with only the attributes a host-side rule reads."""
    from sparknet.oneshot.runtime import NvlinkAllReduce

    rt = object.__new__(NvlinkAllReduce)
    for name, value in attrs.items():
        setattr(rt, name, value)
    return rt


def test_forced_gather_protocol_must_fit():
    rt = _bare_runtime(world_size=8, _caps=(2 << 20, 4 << 20), _mc=(0, 0, 16 << 20), has_multicast=True)
    assert rt._gather_algorithm_fits("ll", 4 << 20) and not rt._gather_algorithm_fits("ll", (4 << 20) + 16)
    assert rt._gather_algorithm_fits("nvls", 2 << 20)                    # 8 x 2 MiB fills the 16 MiB window
    assert not rt._gather_algorithm_fits("nvls", (2 << 20) + 16)
    assert rt._gather_algorithm_fits("push", 1 << 30)
    assert not _bare_runtime(world_size=8, _caps=(0, 0), _mc=(0, 0, 16 << 20),
                             has_multicast=False)._gather_algorithm_fits("nvls", 4096)


def test_fused_norm_token_limit_by_world():
    from sparknet.oneshot.runtime import FUSED_NORM_MAX_TOKENS

    limits = {w: _bare_runtime(world_size=w).fused_norm_max_tokens() for w in (1, 2, 4, 8)}
    assert limits == {1: FUSED_NORM_MAX_TOKENS[1], 2: FUSED_NORM_MAX_TOKENS[2], 4: FUSED_NORM_MAX_TOKENS[2],
                      8: FUSED_NORM_MAX_TOKENS[8]}
    assert limits[1] == 0 and limits[2] < limits[8]
