"""eosllm_b200: the Q4_K / Q8_0 quantized matmul path of eosllm, rebuilt for
NVIDIA B200 (sm_100a).

The product is the C-ABI shared library eosllm_b200/lib/libeosllm_cuda.so
(interface: include/eosllm_cuda.h) and the C99 backend-registration glue in
eosllm_b200/host/.  `eosllm_b200.backend` binds the library for Python
callers, tests and benchmarks.
"""
from . import backend  # noqa: F401

__all__ = ["backend"]
