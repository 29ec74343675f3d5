"""Protocol tests on one GPU: every rank of a collective runs inside one cooperative
launch (``EmulatedGroup``), executing the same device code as the multi-process path.

Oracle: sequential fp32 accumulation in rank order 0..W-1, one rounding to the dtype
(bit-exact), as the reference's simulator and GPU tests check
(reference tests/test_oneshot_cpu.py:35-48, tests/gpu/test_oneshot_gpu.py:142-206).
"""

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

DTYPES = [torch.bfloat16, torch.float16, torch.float32]


def rank_order_sum(xs):
    acc = torch.zeros_like(xs[0], dtype=torch.float32)
    for x in xs:
        acc = acc + x.float()
    return acc.to(xs[0].dtype)


def inputs(world, numel, dtype, device, seed=0):
    out = []
    for r in range(world):
        g = torch.Generator(device=device).manual_seed(seed * 100 + r)
        out.append(torch.randn(numel, generator=g, device=device, dtype=torch.float32).to(dtype))
    return out


@pytest.fixture(scope="module")
def groups(device, native):
    from sparknet.oneshot.emulate import EmulatedGroup

    made = {w: EmulatedGroup(w, device, max_size=8 << 20, max_gather_bytes=2 << 20) for w in (2, 4, 8)}
    yield made


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("algorithm", ["oneshot", "twoshot"])
@pytest.mark.parametrize("nbytes", [16, 10 * 1024, 60 * 1024, 480 * 1024, 2 * 1024 * 1024])
def test_all_reduce_bit_exact(groups, device, world, dtype, algorithm, nbytes):
    g = groups[world]
    numel = nbytes // torch.tensor([], dtype=dtype).element_size()
    xs = inputs(world, numel, dtype, device, seed=nbytes % 97)
    outs = g.all_reduce(xs, algorithm)
    torch.cuda.synchronize()
    g.check()
    want = rank_order_sum(xs)
    for r in range(world):
        assert torch.equal(outs[r].view(torch.int8), want.view(torch.int8)), f"rank {r} differs"


def test_all_reduce_repeated_mixed_sizes(groups, device):
    """Sequences of different sizes and algorithms: parity slots and sentinels stay clean."""
    g = groups[4]
    for step in range(40):
        nbytes = [16, 4096, 65536, 1 << 20][step % 4]
        algo = "oneshot" if step % 3 else "twoshot"
        xs = inputs(4, nbytes // 2, torch.bfloat16, device, seed=step)
        outs = g.all_reduce(xs, algo)
        torch.cuda.synchronize()
        g.check()
        want = rank_order_sum(xs)
        assert all(torch.equal(o, want) for o in outs), f"step {step}"


def test_special_values_survive_sentinel(groups, device):
    """NaN payloads equal to the sentinel, -0 and infinities are carried correctly."""
    g = groups[2]
    a = torch.zeros(64, dtype=torch.bfloat16, device=device)
    b = torch.zeros(64, dtype=torch.bfloat16, device=device)
    a.view(torch.int16)[0] = -1           # 0xFFFF: a NaN with the sentinel's bits
    a[1] = float("inf")
    b[1] = 1.0
    a[2] = -0.0
    b[2] = -0.0
    a[3] = 3.0
    b[3] = -3.0
    outs = g.all_reduce([a, b], "oneshot")
    torch.cuda.synchronize()
    g.check()
    o = outs[0].float()
    assert torch.isnan(o[0]) and o[1] == float("inf") and o[2] == 0 and o[3] == 0
    assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16))


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("dtype", DTYPES)
def test_reduce_scatter_bit_exact(groups, device, world, dtype):
    g = groups[world]
    rows, cols = 3 * world, 256
    xs = [x.view(rows, cols) for x in inputs(world, rows * cols, dtype, device, seed=world)]
    outs = g.reduce_scatter(xs)
    torch.cuda.synchronize()
    g.check()
    total = rank_order_sum(xs)
    per = rows // world
    for r in range(world):
        assert torch.equal(outs[r], total[r * per:(r + 1) * per])


@pytest.mark.parametrize("world", [2, 8])
@pytest.mark.parametrize("algorithm", ["ll", "push"])
@pytest.mark.parametrize("dim", [0, -1])
@pytest.mark.parametrize("shape", [(1, 64), (6, 5120), (96, 256)])
def test_all_gather(groups, device, world, algorithm, dim, shape):
    g = groups[world]
    xs = [torch.randn(shape, device=device).to(torch.bfloat16) + r for r in range(world)]
    outs = g.all_gather(xs, dim=dim, algorithm=algorithm)
    torch.cuda.synchronize()
    g.check()
    want = torch.cat(xs, dim=dim)
    for r in range(world):
        assert torch.equal(outs[r], want)


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("copy_self", [False, True])
def test_exchange(groups, device, world, copy_self):
    g = groups[world]
    chunks = [torch.randn(world, 16, 512, device=device).to(torch.bfloat16) for _ in range(world)]
    parts = g.exchange(chunks, copy_self=copy_self, fill=-7.0)
    torch.cuda.synchronize()
    g.check()
    for r in range(world):
        for p in range(world):
            if p == r and not copy_self:
                assert torch.all(parts[r][p] == -7.0)
            else:
                assert torch.equal(parts[r][p], chunks[p][r])


def fused_reference(xs, residual, gamma, eps):
    s = rank_order_sum(xs)
    res = (s.float() + residual.float()).to(s.dtype)
    var = res.float().pow(2).mean(dim=-1, keepdim=True)
    out = (res.float() * torch.rsqrt(var + eps) * gamma.float()).to(s.dtype)
    return out, res


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("tokens", [1, 8, 32, 128, 256])
@pytest.mark.parametrize("algorithm", ["oneshot", "twoshot"])
def test_fused_allreduce_rmsnorm(groups, device, world, tokens, algorithm):
    g = groups[world]
    hidden = 8192
    xs = [x.view(tokens, hidden) for x in inputs(world, tokens * hidden, torch.bfloat16, device, seed=tokens)]
    gen = torch.Generator(device=device).manual_seed(7)
    residual = torch.randn(tokens, hidden, generator=gen, device=device).to(torch.bfloat16)
    gamma = (1.0 + 0.02 * torch.randn(hidden, generator=gen, device=device)).to(torch.bfloat16)
    outs, res_outs = g.fused_norm(xs, [residual] * world, gamma, 1e-5, algorithm)
    torch.cuda.synchronize()
    g.check()
    want_out, want_res = fused_reference(xs, residual, gamma, 1e-5)
    for r in range(world):
        assert torch.equal(res_outs[r], want_res), "residual must equal all_reduce + residual exactly"
        assert torch.equal(outs[r].view(torch.int16), outs[0].view(torch.int16)), "ranks must agree bit for bit"
    torch.testing.assert_close(outs[0].float(), want_out.float(), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("cluster,threads", [(8, 0), (2, 0), (1, 0), (1, 32), (2, 32)])
@pytest.mark.parametrize("max_clusters", [1, 2, 0])
@pytest.mark.parametrize("algorithm", ["oneshot", "twoshot"])
def test_fused_norm_launch_shapes(groups, device, cluster, threads, max_clusters, algorithm):
    """The smoke's shape (2 ranks, 2 tokens, hidden 1024, one residual tensor for both
    ranks) under every launch shape the kernel may meet: clusters of 1, 2 or 8 CTAs per
    row, 1 or 2 clusters per rank looping over rows, and blocks of 32 threads that hold
    several packs each (a cluster of 1 with 32 threads is the launch a profiler issues
    when it drops the cluster attribute).  Repeated, each result checked exactly."""
    g = groups[2]
    hidden, tokens = 1024, 2
    gen = torch.Generator(device=device).manual_seed(11 + cluster + threads + max_clusters)
    gamma = (1.0 + 0.02 * torch.randn(hidden, generator=gen, device=device)).to(torch.bfloat16)
    for _ in range(10):
        xs = [torch.randn(tokens, hidden, generator=gen, device=device).to(torch.bfloat16) for _ in range(2)]
        residual = torch.randn(tokens, hidden, generator=gen, device=device).to(torch.bfloat16)
        outs, res_outs = g.fused_norm(xs, [residual] * 2, gamma, 1e-5, algorithm, cluster,
                                      max_clusters=max_clusters, threads=threads)
        torch.cuda.synchronize()
        g.check()
        want_out, want_res = fused_reference(xs, residual, gamma, 1e-5)
        for r in range(2):
            assert torch.equal(res_outs[r], want_res), f"rank {r}: residual differs"
            assert torch.equal(outs[r].view(torch.int16), outs[0].view(torch.int16)), "ranks must agree"
        torch.testing.assert_close(outs[0].float(), want_out.float(), rtol=1e-2, atol=1e-2)


def test_fused_norm_wide_rows_one_cta(groups, device):
    """hidden 8192 with one CTA per row: 1024 packs over a 512-thread block, two per thread."""
    g = groups[4]
    hidden, tokens = 8192, 8
    xs = [x.view(tokens, hidden) for x in inputs(4, tokens * hidden, torch.bfloat16, device, seed=3)]
    gen = torch.Generator(device=device).manual_seed(5)
    residual = torch.randn(tokens, hidden, generator=gen, device=device).to(torch.bfloat16)
    gamma = (1.0 + 0.02 * torch.randn(hidden, generator=gen, device=device)).to(torch.bfloat16)
    outs, res_outs = g.fused_norm(xs, [residual] * 4, gamma, 1e-5, "oneshot", 1)
    torch.cuda.synchronize()
    g.check()
    want_out, want_res = fused_reference(xs, residual, gamma, 1e-5)
    for r in range(4):
        assert torch.equal(res_outs[r], want_res)
        assert torch.equal(outs[r].view(torch.int16), outs[0].view(torch.int16))
    torch.testing.assert_close(outs[0].float(), want_out.float(), rtol=1e-2, atol=1e-2)


def test_graph_replay(groups, device):
    """Collectives captured once replay with a device-resident epoch."""
    g = groups[4]
    sizes = [5120, 30720, 245760]
    xs = {n: inputs(4, n, torch.bfloat16, device, seed=n % 11) for n in sizes}
    outs = {n: [torch.empty_like(x) for x in xs[n]] for n in sizes}
    for n in sizes:
        g.all_reduce(xs[n], "oneshot", outs=outs[n])
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for n in sizes:
            g.all_reduce(xs[n], "oneshot" if n < 100000 else "twoshot", outs=outs[n])
    for step in range(5):
        for n in sizes:
            for x in xs[n]:
                x.add_(1.0)
        graph.replay()
        torch.cuda.synchronize()
        g.check()
        for n in sizes:
            want = rank_order_sum(xs[n])
            assert all(torch.equal(o, want) for o in outs[n]), f"replay {step} size {n}"


def test_missing_rank_times_out_without_faulting(device, native):
    """A rank that never launches: its peers give up after the timeout, record who they
    waited for, and the context stays usable (no trap); reset() re-arms the group."""
    from sparknet.oneshot.emulate import EmulatedGroup

    g = EmulatedGroup(2, device, max_size=1 << 20, max_gather_bytes=1 << 20, timeout_ms=200)
    xs = inputs(2, 4096, torch.bfloat16, device)
    g.comm.set_skip_rank(1)
    import time

    t0 = time.perf_counter()
    g.all_reduce(xs, "oneshot")
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    fails = g.failures()
    assert len(fails) == 1 and fails[0]["peer"] == 1 and fails[0]["kind"] == 1
    assert 0.15 < waited < 5.0
    # poisoned: later launches exit at entry
    g.all_reduce(xs, "oneshot")
    torch.cuda.synchronize()
    assert g.comm.ctrl(0)["poison"] == 1
    # the GPU still works, and a reset group is healthy again
    assert torch.ones(4, device=device).sum().item() == 4
    g.comm.set_skip_rank(-1)
    g.reset()
    outs = g.all_reduce(xs, "oneshot")
    torch.cuda.synchronize()
    g.check()
    assert torch.equal(outs[0], rank_order_sum(xs))
