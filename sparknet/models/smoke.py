"""A tiny single-GPU decode step through the model's kernels (driver smoke test)."""

from __future__ import annotations

import torch

from .llama import LlamaConfig, TPLlama


def tiny_decode_step(device) -> None:
    cfg = LlamaConfig.tiny(layers=2)
    model = TPLlama(cfg, rank=0, world=1, device=device, batch=2, max_len=64)
    model.fill_prompt_cache(8)
    model.tokens.copy_(torch.tensor([1, 2], device=device))
    model.step_kernels()
    torch.cuda.synchronize(device)
    assert int(model.positions[0]) == 9 and bool(((model.tokens >= 0) & (model.tokens < cfg.vocab)).all())
