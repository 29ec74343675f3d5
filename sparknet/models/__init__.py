"""Model code used to measure the collectives inside real decode steps."""

from .llama import LlamaConfig, TPLlama

__all__ = ["LlamaConfig", "TPLlama"]
