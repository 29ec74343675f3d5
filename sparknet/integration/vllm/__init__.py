"""vLLM device-communicator adapter for the NVLink collectives."""

from .nvlink_all_reduce import REQUIRED_API_VERSION, SparknetOneShotAllReduce, parse_byte_size

__all__ = ["REQUIRED_API_VERSION", "SparknetOneShotAllReduce", "parse_byte_size"]
