"""Tensor-parallel building blocks over the NVLink runtime: process-group setup and
column/row-parallel linear layers whose collectives are the fused kernels."""

from .groups import TPGroup, init_tp
from .linear import ColumnParallelLinear, RowParallelLinear

__all__ = ["ColumnParallelLinear", "RowParallelLinear", "TPGroup", "init_tp"]
