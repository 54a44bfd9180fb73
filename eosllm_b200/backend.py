"""Python view of libeosllm_cuda.so (the C ABI in include/eosllm_cuda.h).

The shared library is the product; this module only binds it with ctypes so
tests and benchmarks can drive the same entry points a C host (the reference
engine's backend registry) calls.  There is no fallback: if the library is
missing, or a call fails, an exception says so.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libeosllm_cuda.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "eosllm_cuda.h")

# eos_status_t (reference include/eosllm/eosllm.h:66-77)
EOS_OK = 0
EOS_E_INVALID_ARG = 1
EOS_E_OUT_OF_MEMORY = 2
EOS_E_UNSUPPORTED = 3
EOS_E_FORMAT = 4
EOS_E_NOT_FOUND = 6
EOS_E_IO = 8
EOS_E_INTERNAL = 9
STATUS_NAMES = {0: "EOS_OK", 1: "EOS_E_INVALID_ARG", 2: "EOS_E_OUT_OF_MEMORY", 3: "EOS_E_UNSUPPORTED",
                4: "EOS_E_FORMAT", 5: "EOS_E_VERSION_MISMATCH", 6: "EOS_E_NOT_FOUND", 7: "EOS_E_DEADLINE",
                8: "EOS_E_IO", 9: "EOS_E_INTERNAL"}

# eos_dtype_t (reference include/eosllm/tensor.h:32-33)
DT_Q8_0 = 32
DT_Q4_K = 33


class CudaBackendError(RuntimeError):
    def __init__(self, status: int, where: str, message: str):
        super().__init__(f"{where}: {STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


def build() -> str:
    """Compile libeosllm_cuda.so in-tree for sm_100a (nvcc, no GPU needed)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_vp = C.c_void_p
_u32 = C.c_uint32
_u64 = C.c_uint64
_sz = C.c_size_t

_SIGNATURES = {
    "eosi_cuda_probe": (C.c_int, []),
    "eosi_cuda_device_count": (C.c_int, []),
    "eosi_cuda_set_devices": (C.c_int, [C.POINTER(C.c_int), C.c_int]),
    "eosi_cuda_shutdown": (None, []),
    "eosi_cuda_last_error": (C.c_char_p, []),
    "eosi_cuda_matmul_q": (C.c_int, [_vp, _vp, C.c_int, _vp, _u32, _u32, _u32]),
    "eosi_cuda_matmul_q4_k": (C.c_int, [_vp, _vp, _vp, _u32, _u32, _u32]),
    "eosi_cuda_matmul_q8_0": (C.c_int, [_vp, _vp, _vp, _u32, _u32, _u32]),
    "eosi_cuda_cache_evict": (C.c_int, [_vp]),
    "eosi_cuda_cache_clear": (C.c_int, []),
    "eosi_cuda_cache_preload": (C.c_int, [_vp, C.c_int, _u32, _u32]),
    "eosi_cuda_host_stats": (C.c_int, [_vp, _vp, _vp]),
    "eosi_cuda_q4_k_scratch_bytes": (_sz, [_u32, _u32]),
    "eosi_cuda_matmul_q4_k_dev": (C.c_int, [_vp, _vp, _vp, _u32, _u32, _u32, _vp, _vp]),
    "eosi_cuda_q4_k_pack_act_dev": (C.c_int, [_vp, _u32, _u32, _vp, _vp]),
    "eosi_cuda_q4_k_gemv_dev": (C.c_int, [_vp, _vp, _vp, _u32, _u32, _vp]),
    "eosi_cuda_matmul_q8_0_dev": (C.c_int, [_vp, _vp, _vp, _u32, _u32, _u32, _vp]),
    "eosi_cuda_quantize_act_dev": (C.c_int, [_vp, _u32, _u32, _vp, _vp, _vp, _vp]),
    "eosi_cuda_unpack_scale_min_dev": (C.c_int, [_vp, _u32, _vp, _vp, _vp]),
    "eosi_cuda_q8_0_quantize_dev": (C.c_int, [_vp, _vp, _sz, _vp]),
    "eosi_cuda_q4_k_quantize_dev": (C.c_int, [_vp, _vp, _sz, _vp]),
    "eosi_cuda_fill_gauss_dev": (C.c_int, [_vp, _sz, _u64, _u64, C.c_float, _vp]),
    "eosi_cuda_q4_k_from_gauss_dev": (C.c_int, [_vp, _sz, _u64, C.c_float, _vp]),
    "eosi_cuda_take_device_errors": (C.c_int, [C.POINTER(C.c_uint32)]),
    "eosi_cuda_set_kernel_variant": (C.c_int, [C.c_int, C.c_int]),
    "eosi_cuda_matmul_q4_k_noalloc": (C.c_int, [_vp, _vp, _vp, _u32, _u32, _u32, _vp]),
    "eosi_cuda_q4_k_prefill_weight_bytes": (_sz, [_u32, _u32]),
    "eosi_cuda_q4_k_prefill_scratch_bytes": (_sz, [_u32, _u32]),
    "eosi_cuda_q4_k_prefill_prepare_weights_dev": (C.c_int, [_vp, _u32, _u32, _vp, _vp]),
    "eosi_cuda_q4_k_prefill_dev": (C.c_int, [_vp, _vp, _vp, _u32, _u32, _u32, _vp, _vp]),
    "eosi_cuda_text_open": (C.c_int, [_vp, C.c_int, C.c_int, C.c_int, C.POINTER(_vp)]),
    "eosi_cuda_text_step": (C.c_int, [_vp, _u32, _vp]),
    "eosi_cuda_text_generate": (C.c_int, [_vp, _vp, _u32, _u32, _vp]),
    "eosi_cuda_text_reset": (C.c_int, [_vp]),
    "eosi_cuda_text_prefill": (C.c_int, [_vp, _vp, _u32]),
    "eosi_cuda_gguf_map": (C.c_int, [C.c_char_p, _u32, _vp, _vp]),
    "eosi_cuda_gguf_unmap": (None, [_vp]),
    "eosi_cuda_text_open_gguf": (C.c_int, [C.c_char_p, _u32, C.c_int, C.c_int, C.c_int, _vp]),
    "eosi_cuda_text_set_prefill_min": (C.c_int, [_vp, _u32]),
    "eosi_cuda_text_set_prefill_resident": (C.c_int, [_vp, C.c_int]),
    "eosi_cuda_text_pos": (_u32, [_vp]),
    "eosi_cuda_text_stream": (_vp, [_vp]),
    "eosi_cuda_text_step_kernels": (_u32, [_vp]),
    "eosi_cuda_text_set_step_mode": (C.c_int, [_vp, C.c_int]),
    "eosi_cuda_text_step_mode": (C.c_int, [_vp]),
    "eosi_cuda_text_ipc_handle": (C.c_int, [_vp, _vp, _sz]),
    "eosi_cuda_text_attach_peers": (C.c_int, [_vp, _vp, _sz]),
    "eosi_cuda_text_attach_local": (C.c_int, [_vp, C.c_int]),
    "eosi_cuda_text_set_wait_limit": (C.c_int, [_vp, _u32]),
    "eosi_cuda_text_partition": (C.c_int, [_vp, C.c_int, C.c_int, _vp]),
    "eosi_cuda_text_close": (None, [_vp]),
}

_lib = None


def load(path: str = LIB_PATH):
    """Load the library (once).  Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise FileNotFoundError(
            f"{path} is missing: build it with `make -C {HERE}` (the CUDA path has no fallback)")
    lib = C.CDLL(path)
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def declared_symbols(header: str = HEADER) -> list[str]:
    """Every eosi_cuda_* entry point declared in include/eosllm_cuda.h."""
    import re
    with open(header) as f:
        return sorted(set(re.findall(r"EOSLLM_CUDA_API\s+[\w\s\*]*?\b(eosi_cuda_\w+)\s*\(", f.read())))


def last_error() -> str:
    msg = load().eosi_cuda_last_error()
    return msg.decode() if msg else ""


def check(status: int, where: str) -> None:
    if status != EOS_OK:
        raise CudaBackendError(status, where, last_error())


def available() -> bool:
    """True when the library loads and finds an sm_100 GPU."""
    try:
        return load().eosi_cuda_probe() == EOS_OK
    except OSError:
        return False


def _ptr(x) -> int:
    if isinstance(x, np.ndarray):
        return x.ctypes.data
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    return int(x)


# ---------------------------------------------------------------------------
# Host-pointer layer: the backend slot eos_backend_ops_t.matmul_q
# ---------------------------------------------------------------------------
def matmul_q(a: np.ndarray, b_quant: np.ndarray, dtype: int, m: int, n: int, k: int,
             out: np.ndarray | None = None) -> np.ndarray:
    """C[m,n] = A[m,k] . deq(B)^T through eosi_cuda_matmul_q (host buffers)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    b_quant = np.ascontiguousarray(b_quant, dtype=np.uint8)
    c = out if out is not None else np.empty((m, n), dtype=np.float32)
    check(load().eosi_cuda_matmul_q(_ptr(a), _ptr(b_quant), dtype, _ptr(c), m, n, k), "eosi_cuda_matmul_q")
    return c


def matmul_q_status(a, b_quant, dtype, c, m, n, k) -> int:
    """Raw status of eosi_cuda_matmul_q (pointers may be 0 to probe errors)."""
    return load().eosi_cuda_matmul_q(_ptr(a) if a is not None else None,
                                     _ptr(b_quant) if b_quant is not None else None, dtype,
                                     _ptr(c) if c is not None else None, m, n, k)


def set_devices(ids: list[int] | None) -> None:
    lib = load()
    if not ids:
        check(lib.eosi_cuda_set_devices(None, 0), "eosi_cuda_set_devices")
    else:
        arr = (C.c_int * len(ids))(*ids)
        check(lib.eosi_cuda_set_devices(arr, len(ids)), "eosi_cuda_set_devices")


def shutdown() -> None:
    load().eosi_cuda_shutdown()


def cache_clear() -> None:
    check(load().eosi_cuda_cache_clear(), "eosi_cuda_cache_clear")


def cache_preload(b_quant: np.ndarray, dtype: int, n: int, k: int) -> None:
    check(load().eosi_cuda_cache_preload(_ptr(b_quant), dtype, n, k), "eosi_cuda_cache_preload")


# ---------------------------------------------------------------------------
# Device-pointer layer (pointers are ints or objects with data_ptr())
# ---------------------------------------------------------------------------
def q4_k_scratch_bytes(m: int, k: int) -> int:
    return int(load().eosi_cuda_q4_k_scratch_bytes(m, k))


def matmul_q4_k_dev(a, w, c, m, n, k, scratch, stream=0) -> None:
    check(load().eosi_cuda_matmul_q4_k_dev(_ptr(a), _ptr(w), _ptr(c), m, n, k, _ptr(scratch), stream or None),
          "eosi_cuda_matmul_q4_k_dev")


def q4_k_pack_act_dev(a, m, k, act, stream=0) -> None:
    check(load().eosi_cuda_q4_k_pack_act_dev(_ptr(a), m, k, _ptr(act), stream or None), "eosi_cuda_q4_k_pack_act_dev")


def q4_k_gemv_dev(act, w, c, n, k, stream=0) -> None:
    check(load().eosi_cuda_q4_k_gemv_dev(_ptr(act), _ptr(w), _ptr(c), n, k, stream or None), "eosi_cuda_q4_k_gemv_dev")


def matmul_q8_0_dev(a, w, c, m, n, k, stream=0) -> None:
    check(load().eosi_cuda_matmul_q8_0_dev(_ptr(a), _ptr(w), _ptr(c), m, n, k, stream or None),
          "eosi_cuda_matmul_q8_0_dev")


def quantize_act_dev(a, m, k, aq, scales, sums, stream=0) -> None:
    check(load().eosi_cuda_quantize_act_dev(_ptr(a), m, k, _ptr(aq), _ptr(scales), _ptr(sums), stream or None),
          "eosi_cuda_quantize_act_dev")


def unpack_scale_min_dev(scales12, count, sc, m, stream=0) -> None:
    check(load().eosi_cuda_unpack_scale_min_dev(_ptr(scales12), count, _ptr(sc), _ptr(m), stream or None),
          "eosi_cuda_unpack_scale_min_dev")


def q8_0_quantize_dev(src, dst, n_elements, stream=0) -> None:
    check(load().eosi_cuda_q8_0_quantize_dev(_ptr(src), _ptr(dst), n_elements, stream or None),
          "eosi_cuda_q8_0_quantize_dev")


def q4_k_quantize_dev(src, dst, n_elements, stream=0) -> None:
    check(load().eosi_cuda_q4_k_quantize_dev(_ptr(src), _ptr(dst), n_elements, stream or None),
          "eosi_cuda_q4_k_quantize_dev")


def fill_gauss_dev(dst, n, seed, offset, sigma, stream=0) -> None:
    check(load().eosi_cuda_fill_gauss_dev(_ptr(dst), n, seed, offset, sigma, stream or None),
          "eosi_cuda_fill_gauss_dev")


def q4_k_from_gauss_dev(dst, n_elements, seed, sigma, stream=0) -> None:
    check(load().eosi_cuda_q4_k_from_gauss_dev(_ptr(dst), n_elements, seed, sigma, stream or None),
          "eosi_cuda_q4_k_from_gauss_dev")


def take_device_errors() -> int:
    v = C.c_uint32(0)
    check(load().eosi_cuda_take_device_errors(C.byref(v)), "eosi_cuda_take_device_errors")
    return v.value


def set_kernel_variant(dtype: int, variant: int) -> None:
    check(load().eosi_cuda_set_kernel_variant(dtype, variant), "eosi_cuda_set_kernel_variant")


# ---------------------------------------------------------------------------
# Sizes of the GGUF blocks (reference src/kernels/scalar/scalar.h:239-243)
# ---------------------------------------------------------------------------
def weight_bytes(dtype: int, n: int, k: int) -> int:
    if dtype == DT_Q4_K:
        return n * (k // 256) * 144
    if dtype == DT_Q8_0:
        return n * (k // 32) * 34
    raise ValueError(dtype)


# ---------------------------------------------------------------------------
# Tensor-core prefill
# ---------------------------------------------------------------------------
def prefill_weight_bytes(n: int, k: int) -> int:
    return int(load().eosi_cuda_q4_k_prefill_weight_bytes(n, k))


def prefill_scratch_bytes(m: int, k: int) -> int:
    return int(load().eosi_cuda_q4_k_prefill_scratch_bytes(m, k))


def prefill_prepare_weights_dev(w, n, k, w_prep, stream=0) -> None:
    """Q4_K [n][k] -> the prefill GEMM's weight layout (prefill_weight_bytes)."""
    check(load().eosi_cuda_q4_k_prefill_prepare_weights_dev(_ptr(w), n, k, _ptr(w_prep), stream or None),
          "eosi_cuda_q4_k_prefill_prepare_weights_dev")


def prefill_dev(a, w_prep, c, m, n, k, scratch, stream=0) -> None:
    check(load().eosi_cuda_q4_k_prefill_dev(_ptr(a), _ptr(w_prep), _ptr(c), m, n, k, _ptr(scratch),
                                            stream or None), "eosi_cuda_q4_k_prefill_dev")
