"""A Llama-3-shaped tensor-parallel decoder for decode benchmarks and examples.

Megatron-style sharding over ``world`` GPUs of one box: the fused QKV and gate/up
projections are column-parallel (heads and FFN columns split), the O and down
projections are row-parallel (partial sums), so each layer needs two all-reduces.
Each all-reduce is followed by the residual add and the next RMSNorm; with
``comm="sparknet"`` the three run as one fused NVLink kernel
(``AllReduce.all_reduce_residual_rmsnorm``); with ``comm="nccl"`` (the control arm)
the all-reduce is ``torch.distributed.all_reduce`` on NCCL followed by a local
add+RMSNorm kernel with the same rounding points.  The vocabulary projection is
column-parallel; each rank takes the argmax of its shard and the (value, index)
pairs are all-gathered (greedy sampling).

Weights are random (N(0, 0.02)); there are no checkpoints.  They are stored in
``nn.Linear`` layout ``[out, in]``; the gate/up weight interleaves 64-row blocks of gate
and up (``sparknet.ops.interleave_gate_up``).  With ``gemm="sparknet"`` (the default
with ``comm="sparknet"``) every projection is this package's tcgen05 decode GEMM and
SwiGLU runs in the gate/up GEMM's epilogue; ``gemm="cublas"`` (the default of the
NCCL control arm) uses ``torch.mm`` and a separate SwiGLU kernel.  Attention, RoPE +
KV-cache writes, the norms and the argmax are this package's kernels.  A decode step
is one CUDA graph replay.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist

from .. import _native
from ..ops.attention import VARIANTS as ATTENTION_VARIANTS
from ..ops.decode_gemm import INTERLEAVE_ROWS, DecodeGemm


@dataclass(frozen=True)
class LlamaConfig:
    hidden: int = 8192
    layers: int = 80
    heads: int = 64
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 28672
    vocab: int = 128256
    rope_theta: float = 500000.0
    eps: float = 1e-5

    @staticmethod
    def llama3_70b() -> "LlamaConfig":
        return LlamaConfig()

    @staticmethod
    def tiny(layers: int = 2) -> "LlamaConfig":
        return LlamaConfig(hidden=1024, layers=layers, heads=8, kv_heads=8, head_dim=128, ffn=2048, vocab=4096)

    def params(self) -> int:
        per_layer = self.hidden * (self.heads + 2 * self.kv_heads) * self.head_dim + \
            self.heads * self.head_dim * self.hidden + 3 * self.hidden * self.ffn + 2 * self.hidden
        return self.layers * per_layer + 2 * self.vocab * self.hidden + self.hidden


def _normal(shape, device, std=0.02, generator=None):
    t = torch.empty(shape, dtype=torch.bfloat16, device=device)
    t.normal_(0.0, std, generator=generator)
    return t


class TPLlama:
    """One rank's shard of the model plus its KV cache and decode buffers."""

    def __init__(self, cfg: LlamaConfig, *, rank: int, world: int, device, batch: int, max_len: int,
                 comm: str = "sparknet", runtime=None, group=None, seed: int = 0, gemm: str | None = None,
                 pdl: bool = True, attention: str = "auto"):
        if cfg.heads % world or cfg.kv_heads % world or cfg.ffn % world or cfg.vocab % world:
            raise ValueError(f"model does not shard evenly over {world} GPUs")
        if comm not in ("sparknet", "nccl"):
            raise ValueError("comm must be 'sparknet' or 'nccl'")
        if comm == "sparknet" and world > 1 and runtime is None:
            raise ValueError("comm='sparknet' needs the NVLink runtime")
        gemm = gemm or ("sparknet" if comm == "sparknet" else "cublas")
        if gemm not in ("sparknet", "cublas"):
            raise ValueError("gemm must be 'sparknet' or 'cublas'")
        if (cfg.ffn // world) % INTERLEAVE_ROWS:
            raise ValueError("the FFN shard must be a multiple of 64 features")
        if attention not in ATTENTION_VARIANTS:
            raise ValueError(f"attention must be one of {sorted(ATTENTION_VARIANTS)}")
        self.gemm = gemm
        self.attention = attention
        self.cfg, self.rank, self.world, self.device = cfg, rank, world, torch.device(device)
        self.batch, self.max_len, self.comm, self.runtime, self.group = batch, max_len, comm, runtime, group
        self.C = _native.load()
        self.hq = cfg.heads // world
        self.hkv = cfg.kv_heads // world
        self.f = cfg.ffn // world
        self.v = cfg.vocab // world
        gen = torch.Generator(device=self.device)
        gen.manual_seed(seed * 1000 + rank)
        H, D = cfg.hidden, cfg.head_dim
        dev = self.device
        self.embed = _normal((cfg.vocab, H), dev, generator=torch.Generator(device=dev).manual_seed(seed))
        self.layers = []
        for _ in range(cfg.layers):
            self.layers.append({
                "ln1": torch.ones(H, dtype=torch.bfloat16, device=dev),
                "wqkv": _normal(((self.hq + 2 * self.hkv) * D, H), dev, generator=gen),
                "wo": _normal((H, self.hq * D), dev, generator=gen),
                "ln2": torch.ones(H, dtype=torch.bfloat16, device=dev),
                "wgu": _normal((2 * self.f, H), dev, generator=gen),   # [64 gate; 64 up] row blocks
                "wdown": _normal((H, self.f), dev, generator=gen),
                "k": torch.zeros((batch, max_len, self.hkv, D), dtype=torch.bfloat16, device=dev),
                "v": torch.zeros((batch, max_len, self.hkv, D), dtype=torch.bfloat16, device=dev),
            })
        self.norm = torch.ones(H, dtype=torch.bfloat16, device=dev)
        self.lm_head = _normal((self.v, H), dev, generator=gen)
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, D // 2, dtype=torch.float64) * 2 / D))
        ang = torch.arange(max_len, dtype=torch.float64)[:, None] * inv[None, :]
        self.cos = ang.cos().float().to(dev).contiguous()
        self.sin = ang.sin().float().to(dev).contiguous()
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        # zeroed: the attention kernel's split counters sit at its front
        self.workspace = torch.zeros(int(self.C.attention_workspace_floats(batch, self.hq, self.hkv, max_len, sms)),
                                     dtype=torch.float32, device=dev)
        self.pdl = bool(pdl)
        self.mm = DecodeGemm(dev, pdl=pdl)
        # static decode buffers (graph inputs/outputs)
        self.tokens = torch.zeros(batch, dtype=torch.int64, device=dev)
        self.positions = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.lengths = torch.ones(batch, dtype=torch.int32, device=dev)
        self._bufs()
        self.graph = None

    def _bufs(self):
        B, H, D, dev = self.batch, self.cfg.hidden, self.cfg.head_dim, self.device
        e = lambda *s: torch.empty(s, dtype=torch.bfloat16, device=dev)  # noqa: E731
        self.x, self.res, self.partial = e(B, H), e(B, H), e(B, H)
        self.qkv, self.q, self.attn = e(B, (self.hq + 2 * self.hkv) * D), e(B, self.hq, D), e(B, self.hq, D)
        self.gu, self.act, self.logits = e(B, 2 * self.f), e(B, self.f), e(B, self.v)
        self.best = torch.empty((B, 2), dtype=torch.float32, device=dev)
        self.best_all = torch.empty((self.world * B, 2), dtype=torch.float32, device=dev)

    def fill_prompt_cache(self, prompt_len: int, seed: int = 1) -> None:
        """Random KV entries for ``prompt_len`` positions (a prefill stand-in) and the
        decode position right after them."""
        gen = torch.Generator(device=self.device).manual_seed(seed * 7 + self.rank)
        for layer in self.layers:
            layer["k"][:, :prompt_len].normal_(0, 1, generator=gen)
            layer["v"][:, :prompt_len].normal_(0, 1, generator=gen)
        self.positions.fill_(prompt_len)
        self.lengths.fill_(prompt_len + 1)

    # -- the two collectives of a layer ------------------------------------------------
    def _add_norm(self, partial, gamma):
        """residual += all_reduce(partial); x = rms_norm(residual) * gamma."""
        eps = self.cfg.eps
        if self.world == 1:
            self.C.add_rmsnorm(partial, self.res, self.res, gamma, self.x, eps)
        elif self.comm == "sparknet":
            self.runtime.all_reduce_residual_rmsnorm(partial, self.res, gamma, eps, out=self.x,
                                                     residual_out=self.res)
        else:
            dist.all_reduce(partial, group=self.group)
            self.C.add_rmsnorm(partial, self.res, self.res, gamma, self.x, eps)

    def _gather_best(self):
        if self.world == 1:
            return self.best
        if self.comm == "sparknet":
            return self.runtime.all_gather(self.best, dim=0, out=self.best_all)
        dist.all_gather_into_tensor(self.best_all, self.best, group=self.group)
        return self.best_all

    def _linear(self, x, w, out):
        if self.gemm == "sparknet":
            self.mm(x, w, out)
        else:
            torch.mm(x, w.t(), out=out)

    def _swiglu(self, x, w, out):
        if self.gemm == "sparknet":
            self.mm(x, w, out, swiglu=True)
        else:
            torch.mm(x, w.t(), out=self.gu)
            self.C.silu_mul(self.gu, out, INTERLEAVE_ROWS)

    def step_kernels(self) -> None:
        """One decode step on the current stream: tokens -> next tokens (in place)."""
        C, cfg = self.C, self.cfg
        torch.index_select(self.embed, 0, self.tokens, out=self.res)
        C.add_rmsnorm(self.res, None, None, self.layers[0]["ln1"], self.x, cfg.eps)
        scale = 1.0 / math.sqrt(cfg.head_dim)
        for i, L in enumerate(self.layers):
            if self.gemm == "sparknet":  # RoPE and the KV-cache write in the GEMM epilogue
                self.mm.qkv_rope(self.x, L["wqkv"], self.cos, self.sin, self.positions, self.q, L["k"], L["v"],
                                 self.hq, self.hkv)
            else:
                self._linear(self.x, L["wqkv"], self.qkv)
                C.rope_qkv_cache(self.qkv, self.cos, self.sin, self.positions, self.q, L["k"], L["v"], self.hq,
                                 self.hkv)
            C.decode_attention(self.q, L["k"], L["v"], self.lengths, self.attn, self.workspace, self.max_len,
                               scale, self.pdl, ATTENTION_VARIANTS[self.attention])
            last = i + 1 == len(self.layers)
            nxt = self.norm if last else self.layers[i + 1]["ln1"]
            self._linear(self.attn.view(self.batch, -1), L["wo"], self.partial)
            self._add_norm(self.partial, L["ln2"])
            self._swiglu(self.x, L["wgu"], self.act)
            self._linear(self.act, L["wdown"], self.partial)
            self._add_norm(self.partial, nxt)
        self._linear(self.x, self.lm_head, self.logits)
        C.row_argmax(self.logits, self.rank * self.v, self.best)
        allb = self._gather_best().view(self.world, self.batch, 2)
        winner = allb[:, :, 0].argmax(dim=0)                                     # first maximal rank
        idx = allb[:, :, 1].gather(0, winner[None, :])[0]
        self.tokens.copy_(idx.to(torch.int64))
        self.positions.add_(1)
        self.lengths.add_(1)

    def capture(self) -> None:
        """Capture one decode step into a CUDA graph (after one eager warm-up step)."""
        stream = torch.cuda.Stream(device=self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        snap = (self.positions.clone(), self.lengths.clone(), self.tokens.clone())
        with torch.cuda.stream(stream):
            self.step_kernels()
        torch.cuda.current_stream(self.device).wait_stream(stream)
        torch.cuda.synchronize(self.device)
        self.positions.copy_(snap[0])
        self.lengths.copy_(snap[1])
        self.tokens.copy_(snap[2])
        g = torch.cuda.CUDAGraph()
        ctx = self.runtime.capture(stream=stream) if self.runtime is not None else _null()
        with torch.cuda.graph(g, stream=stream), ctx:
            self.step_kernels()
        self.graph = g

    def replay(self) -> None:
        self.graph.replay()

    def release(self) -> None:
        self.graph = None

    def launches_per_step(self) -> int:
        """This package's kernel launches in one step (torch index/copy ops and cuBLAS
        GEMMs excluded): per layer attention and two norms (fused with the all-reduce on
        the NVLink arm), plus four GEMMs with RoPE and SwiGLU fused (``gemm="sparknet"``)
        or the RoPE and SwiGLU kernels (cuBLAS arm)."""
        # sparknet: QKV+RoPE, O, gate/up+SwiGLU, down GEMMs; cuBLAS arm: RoPE and SwiGLU kernels
        per_layer = 1 + 2 + (4 if self.gemm == "sparknet" else 2)
        own_gather = 1 if (self.world > 1 and self.comm == "sparknet") else 0
        lm_head = 1 if self.gemm == "sparknet" else 0
        return 1 + self.cfg.layers * per_layer + lm_head + 1 + own_gather


class _null:
    def __enter__(self):
        return None

    def __exit__(self, *a):
        return False


__all__ = ["LlamaConfig", "TPLlama"]
