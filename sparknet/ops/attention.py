"""Decode attention (grouped-query, one query token per sequence, head_dim 128, bf16).

``decode_attention(q, k_cache, v_cache, lengths, max_len)`` splits each (sequence, KV
head) into spans of keys that CTAs stream, and merges the spans with their log-sum-exp
weights in span order (the last CTA of a (sequence, KV head) merges the partials it
finds in a workspace).  Two kernels share the workspace layout:

* ``variant="simt"``: CUDA cores, 32-key tiles double-buffered with ``cp.async``
  (``csrc/include/sparknet/attention_kernels.cuh``);
* ``variant="tcgen05"``: tensor cores, 128-key K/V tiles by TMA, ``Q K^T`` and
  ``P V`` by ``tcgen05.mma`` with scores and output in TMEM
  (``csrc/include/sparknet/attention_tc.cuh``);
* ``variant="auto"`` (default): the tensor-core kernel where its spans can merge in one
  thread-block cluster (sequences up to 2048 keys, the whole grid in one wave of one
  CTA per SM) or from 32 (sequence, KV head) pairs up, where it was measured faster;
  else the CUDA-core kernel.

The workspace is held per device here (its counters must start at zero; every completed
call leaves them so), or passed in.  ``q`` is ``[B, Hq, 128]``, the caches
``[B, Lmax, Hkv, 128]``, ``lengths`` ``[B]`` int32 (keys to attend, the new token
included, at most ``max_len``).  ``pdl=True`` launches with programmatic dependent
launch: the kernel may start while its predecessor runs.  It reads ``lengths`` and the
K/V rows below the newest key (``lengths[b] - 1``) before it waits for the predecessor,
q and the newest key / value row after; so the immediately preceding kernel may write q
and the newest cache row (as the decode step's QKV GEMM does), not ``lengths`` or older
rows.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from .. import _native

VARIANTS = {"auto": 0, "simt": 1, "tcgen05": 2}
_workspaces: dict = {}


def split_workspace(q: torch.Tensor, hkv: int, max_len: int) -> torch.Tensor:
    """The split-KV workspace for these shapes on q's device, zeroed (grown as needed)."""
    C = _native.load()
    sms = torch.cuda.get_device_properties(q.device).multi_processor_count
    need = int(C.attention_workspace_floats(q.shape[0], q.shape[1], hkv, max_len, sms))
    ws = _workspaces.get(q.device.index)
    if ws is None or ws.numel() < need:
        ws = _workspaces[q.device.index] = torch.zeros(need, dtype=torch.float32, device=q.device)
    return ws


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, lengths: torch.Tensor,
                     max_len: int, *, scale: Optional[float] = None, out: Optional[torch.Tensor] = None,
                     variant: str = "auto", workspace: Optional[torch.Tensor] = None,
                     pdl: bool = False) -> torch.Tensor:
    """softmax(q k^T * scale) v over each sequence's first ``lengths[b]`` keys."""
    if variant not in VARIANTS:
        raise ValueError(f"variant must be one of {sorted(VARIANTS)}, got {variant!r}")
    C = _native.load()
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else float(scale)
    if out is None:
        out = torch.empty_like(q)
    ws = workspace if workspace is not None else split_workspace(q, k_cache.shape[2], int(max_len))
    C.decode_attention(q, k_cache, v_cache, lengths, out, ws, int(max_len), scale, bool(pdl), VARIANTS[variant])
    return out


__all__ = ["VARIANTS", "decode_attention", "split_workspace"]
