"""dgx-spark-networking-b200: NVLink collectives for tensor-parallel inference on B200.

Import name: ``sparknet`` (the reference's public API is kept).  Subpackages:

- ``sparknet.topology``: the GPU map of one NVSwitch box, validation, subsets, NVML discovery.
- ``sparknet.nccl``: the NCCL control profiles (NCCL-only baseline arms).
- ``sparknet.policy``: which backend (one-shot, two-shot, NVLS, NCCL) carries which collective.
- ``sparknet.oneshot``: the NVLink collective runtime (needs torch and the built extension).
- ``sparknet.transport``: the transport seam (NVLink P2P, NVLS, a host-staged test double).
- ``sparknet.ops``: fused kernels (all-reduce + RMSNorm; all-gather->GEMM, GEMM->reduce-scatter).
- ``sparknet.models``: a Llama-3-shaped tensor-parallel decoder for decode benchmarks.
- ``sparknet.parallel``: tensor-parallel layers and process-group helpers.
- ``sparknet.probe``: fabric doctor, collective probe, fail-stop qualification, NVLink counters.
- ``sparknet.integration.vllm``: the vLLM device-communicator adapter.
- ``sparknet.utils``: device timing, clock sampling, environment helpers.

The CPU-only subpackages (topology, nccl, policy, probe planning, CLI) import
nothing from torch.
"""

__version__ = "0.1.0"

# Bumped when the runtime surface used by integrations changes incompatibly.
API_VERSION = 3

__all__ = ["API_VERSION", "__version__"]
