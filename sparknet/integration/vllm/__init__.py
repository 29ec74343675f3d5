"""vLLM device-communicator adapter for the NVLink collectives."""

from .nvlink_all_reduce import SparknetOneShotAllReduce, parse_byte_size

__all__ = ["SparknetOneShotAllReduce", "parse_byte_size"]
