"""Decode attention (grouped-query, one query token per sequence, head_dim 128, bf16).

``decode_attention(q, k_cache, v_cache, lengths, max_len)`` runs the split-KV kernel
(``csrc/include/sparknet/attention_kernels.cuh``): each (sequence, KV head) is cut into
spans of keys that CTAs stream with K/V tiles in flight, and the spans are merged with
their log-sum-exp weights in span order.

* ``variant="split"`` (default, measured): the spans leave their partials in a
  workspace and the last CTA of a (sequence, KV head) merges them.  The workspace is
  held per device here (its counters must start at zero; every completed call leaves
  them so), or passed in.
* ``variant="cluster"`` (opt-in): the spans of one (sequence, KV head) form a
  thread-block cluster and merge through distributed shared memory; no workspace.

``q`` is ``[B, Hq, 128]``, the caches ``[B, Lmax, Hkv, 128]``, ``lengths`` ``[B]``
int32 (keys to attend, the new token included, at most ``max_len``).  ``pdl=True``
launches with programmatic dependent launch: keys below ``lengths - 1`` may be read
while the previous kernel on the stream still runs, so that kernel must not write them.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from .. import _native

_workspaces: dict = {}


def split_workspace(q: torch.Tensor, hkv: int, max_len: int) -> torch.Tensor:
    """The split-KV kernel's zeroed workspace for these shapes on q's device (grown as needed)."""
    C = _native.load()
    sms = torch.cuda.get_device_properties(q.device).multi_processor_count
    need = int(C.attention_workspace_floats(q.shape[0], q.shape[1], hkv, max_len, sms))
    ws = _workspaces.get(q.device.index)
    if ws is None or ws.numel() < need:
        ws = _workspaces[q.device.index] = torch.zeros(need, dtype=torch.float32, device=q.device)
    return ws


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, lengths: torch.Tensor,
                     max_len: int, *, scale: Optional[float] = None, out: Optional[torch.Tensor] = None,
                     variant: str = "split", workspace: Optional[torch.Tensor] = None,
                     pdl: bool = False) -> torch.Tensor:
    """softmax(q k^T * scale) v over each sequence's first ``lengths[b]`` keys."""
    if variant not in ("split", "cluster"):
        raise ValueError("variant must be 'split' or 'cluster'")
    C = _native.load()
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else float(scale)
    if out is None:
        out = torch.empty_like(q)
    if variant == "cluster":
        C.decode_attention_cluster(q, k_cache, v_cache, lengths, out, int(max_len), scale, bool(pdl))
    else:
        ws = workspace if workspace is not None else split_workspace(q, k_cache.shape[2], int(max_len))
        C.decode_attention(q, k_cache, v_cache, lengths, out, ws, int(max_len), scale, bool(pdl))
    return out


__all__ = ["decode_attention", "split_workspace"]
