"""ctypes view of the CPU checker -- TEST INFRASTRUCTURE ONLY.

`Oracle` wraps liboracle.so (this project's C restatement of the reference
algorithm, oracle/eos_oracle.c).  `RefKernels` wraps oracle/_ref/, the
unmodified reference sources compiled by `make -C oracle ref` in the build
container.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg use this module; the product package never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")
REF_KERNELS = os.path.join(REF_DIR, "libref_kernels.so")
REF_ENGINE = os.path.join(REF_DIR, "libeosllm_ref.so")

DT_Q8_0 = 32
DT_Q4_K = 33

_fp = C.POINTER(C.c_float)
_vp = C.c_void_p
_u32 = C.c_uint32


def build(ref: bool = False) -> None:
    """Compile liboracle.so (and, with ref, oracle/_ref: the recipe builds it
    where the reference tree exists and leaves it alone elsewhere)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    if ref:
        subprocess.run(["make", "-s", "-C", HERE, "ref"], check=True)


def reference_dir() -> str:
    """Where the recipe (oracle/Makefile) looks for the reference tree."""
    return subprocess.run(["make", "-s", "-C", HERE, "print-ref"], check=True, capture_output=True,
                          text=True).stdout.strip()


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_vp)


def q4k_row_bytes(k: int) -> int:
    return (k // 256) * 144


def q80_row_bytes(k: int) -> int:
    return (k // 32) * 34


class _Matmuls:
    """Shared calling convention: C[m,n] = A[m,k] . deq(B)[n,k]^T."""

    def _mm(self, fn, a: np.ndarray, b: np.ndarray, m: int, n: int, k: int):
        a = np.ascontiguousarray(a, dtype=np.float32)
        b = np.ascontiguousarray(b, dtype=np.uint8)
        c = np.empty((m, n), dtype=np.float32)
        rc = fn(_ptr(a), _ptr(b), _ptr(c), m, n, k)
        return rc, c


class Oracle(_Matmuls):
    def __init__(self, path: str = LIB):
        if not os.path.exists(path):
            build()
        L = self.lib = C.CDLL(path)
        for name in ("orc_matmul_q4_k_int8", "orc_matmul_q4_k_avx2_f32",
                     "orc_matmul_q4_k_scalar", "orc_matmul_q8_0"):
            f = getattr(L, name)
            f.argtypes = [_vp, _vp, _vp, _u32, _u32, _u32]
            f.restype = C.c_int
        L.orc_matmul_q.argtypes = [_vp, _vp, C.c_int, _vp, _u32, _u32, _u32]
        L.orc_matmul_q.restype = C.c_int
        L.orc_matmul_q_threads.argtypes = [_vp, _vp, C.c_int, _vp, _u32, _u32, _u32, C.c_int]
        L.orc_matmul_q_threads.restype = C.c_int
        L.orc_quantize_sub32.argtypes = [_vp, _vp, _vp, _vp]
        L.orc_quantize_act.argtypes = [_vp, _u32, _vp, _vp, _vp]
        L.orc_quantize_act.restype = C.c_int
        L.orc_get_scale_min.argtypes = [C.c_int, _vp, _vp, _vp]
        L.orc_pack_q4k_scales.argtypes = [_vp, _vp, _vp]
        L.orc_unpack_scale_min_batch.argtypes = [_vp, C.c_size_t, _vp, _vp]
        for name in ("orc_q4_k_quantize", "orc_q8_0_quantize"):
            getattr(L, name).argtypes = [_vp, _vp, C.c_size_t]
            getattr(L, name).restype = C.c_int
        for name in ("orc_q4_k_dequantize", "orc_q8_0_dequantize"):
            getattr(L, name).argtypes = [_vp, _vp, C.c_size_t]
            getattr(L, name).restype = C.c_int
        L.orc_f16_to_f32.argtypes = [C.c_uint16]
        L.orc_f16_to_f32.restype = C.c_float
        L.orc_f32_to_f16.argtypes = [C.c_float]
        L.orc_f32_to_f16.restype = C.c_uint16
        L.orc_gauss.argtypes = [C.c_uint64, C.c_uint64, C.c_float]
        L.orc_gauss.restype = C.c_float
        L.orc_fill_gauss.argtypes = [_vp, C.c_size_t, C.c_uint64, C.c_uint64, C.c_float]
        L.orc_xs_rand_unit.argtypes = [C.POINTER(C.c_uint32)]
        L.orc_xs_rand_unit.restype = C.c_float
        L.orc_rmsnorm.argtypes = [_vp, _vp, C.c_float, _vp, _u32, _u32]
        L.orc_rope.argtypes = [_vp, _u32, _u32, _u32, C.c_float]
        L.orc_silu.argtypes = [_vp, _vp, C.c_size_t]

    # --- matmuls -------------------------------------------------------
    def matmul_q4_k_int8(self, a, b, m, n, k):
        return self._mm(self.lib.orc_matmul_q4_k_int8, a, b, m, n, k)

    def matmul_q4_k_avx2_f32(self, a, b, m, n, k):
        return self._mm(self.lib.orc_matmul_q4_k_avx2_f32, a, b, m, n, k)

    def matmul_q4_k_scalar(self, a, b, m, n, k):
        return self._mm(self.lib.orc_matmul_q4_k_scalar, a, b, m, n, k)

    def matmul_q8_0(self, a, b, m, n, k):
        return self._mm(self.lib.orc_matmul_q8_0, a, b, m, n, k)

    def matmul_q(self, a, b, dtype, m, n, k, threads: int | None = None):
        a = np.ascontiguousarray(a, dtype=np.float32)
        b = np.ascontiguousarray(b, dtype=np.uint8)
        c = np.empty((m, n), dtype=np.float32)
        if threads is None:
            rc = self.lib.orc_matmul_q(_ptr(a), _ptr(b), dtype, _ptr(c), m, n, k)
        else:
            rc = self.lib.orc_matmul_q_threads(_ptr(a), _ptr(b), dtype, _ptr(c), m, n, k, threads)
        return rc, c

    # --- activation packing ------------------------------------------
    def quantize_sub32(self, a32: np.ndarray):
        a32 = np.ascontiguousarray(a32, dtype=np.float32)
        aq = np.empty(32, dtype=np.int8)
        s = np.empty(1, dtype=np.float32)
        t = np.empty(1, dtype=np.int32)
        self.lib.orc_quantize_sub32(_ptr(a32), _ptr(aq), _ptr(s), _ptr(t))
        return aq, s[0], t[0]

    def quantize_act(self, a: np.ndarray):
        a = np.ascontiguousarray(a, dtype=np.float32).ravel()
        k = a.size
        aq = np.empty(k, dtype=np.int8)
        s = np.empty(k // 32, dtype=np.float32)
        t = np.empty(k // 32, dtype=np.int32)
        rc = self.lib.orc_quantize_act(_ptr(a), k, _ptr(aq), _ptr(s), _ptr(t))
        assert rc == 0
        return aq, s, t

    def get_scale_min(self, j: int, scales12: np.ndarray):
        q = np.ascontiguousarray(scales12, dtype=np.uint8)
        sc = np.zeros(1, np.uint8)
        m = np.zeros(1, np.uint8)
        self.lib.orc_get_scale_min(j, _ptr(q), _ptr(sc), _ptr(m))
        return int(sc[0]), int(m[0])

    def unpack_scale_min_batch(self, scales12: np.ndarray):
        q = np.ascontiguousarray(scales12, dtype=np.uint8).reshape(-1, 12)
        sc = np.empty((q.shape[0], 8), np.uint8)
        m = np.empty((q.shape[0], 8), np.uint8)
        self.lib.orc_unpack_scale_min_batch(_ptr(q), q.shape[0], _ptr(sc), _ptr(m))
        return sc, m

    def pack_q4k_scales(self, sc, m) -> np.ndarray:
        sc = np.ascontiguousarray(sc, dtype=np.uint8)
        m = np.ascontiguousarray(m, dtype=np.uint8)
        out = np.zeros(12, np.uint8)
        self.lib.orc_pack_q4k_scales(_ptr(sc), _ptr(m), _ptr(out))
        return out

    # --- quant schemes -------------------------------------------------
    def q4_k_quantize(self, w: np.ndarray) -> np.ndarray:
        w = np.ascontiguousarray(w, dtype=np.float32)
        out = np.empty(w.size // 256 * 144, dtype=np.uint8)
        assert self.lib.orc_q4_k_quantize(_ptr(w), _ptr(out), w.size) == 0
        return out

    def q8_0_quantize(self, w: np.ndarray) -> np.ndarray:
        w = np.ascontiguousarray(w, dtype=np.float32)
        out = np.empty(w.size // 32 * 34, dtype=np.uint8)
        assert self.lib.orc_q8_0_quantize(_ptr(w), _ptr(out), w.size) == 0
        return out

    def q4_k_dequantize(self, b: np.ndarray, n_el: int) -> np.ndarray:
        b = np.ascontiguousarray(b, dtype=np.uint8)
        out = np.empty(n_el, dtype=np.float32)
        assert self.lib.orc_q4_k_dequantize(_ptr(b), _ptr(out), n_el) == 0
        return out

    def q8_0_dequantize(self, b: np.ndarray, n_el: int) -> np.ndarray:
        b = np.ascontiguousarray(b, dtype=np.uint8)
        out = np.empty(n_el, dtype=np.float32)
        assert self.lib.orc_q8_0_dequantize(_ptr(b), _ptr(out), n_el) == 0
        return out

    def f16_to_f32(self, h: int) -> float:
        return self.lib.orc_f16_to_f32(h)

    def f32_to_f16(self, f: float) -> int:
        return self.lib.orc_f32_to_f16(f)

    # --- synthetic inputs ---------------------------------------------
    def gauss(self, n: int, seed: int, sigma: float, offset: int = 0) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        self.lib.orc_fill_gauss(_ptr(out), n, seed, offset, sigma)
        return out

    def xs_rand_unit(self, n: int, state: int) -> tuple[np.ndarray, int]:
        st = C.c_uint32(state)
        out = np.array([self.lib.orc_xs_rand_unit(C.byref(st)) for _ in range(n)], np.float32)
        return out, st.value


class RefKernels(_Matmuls):
    """The reference's own kernels, compiled unmodified into oracle/_ref/."""

    def __init__(self, path: str = REF_KERNELS):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = self.lib = C.CDLL(path)
        for name in ("eosi_avx2_matmul_q4_k_int8", "eosi_avx2_matmul_q4_k",
                     "eosi_scalar_matmul_q4_k", "eosi_scalar_matmul_q8_0"):
            f = getattr(L, name)
            f.argtypes = [_vp, _vp, _vp, _u32, _u32, _u32]
            f.restype = C.c_int
        L.eosi_avx2_matmul_q.argtypes = [_vp, _vp, C.c_int, _vp, _u32, _u32, _u32]
        L.eosi_avx2_matmul_q.restype = C.c_int
        L.ref_quantize_sub32.argtypes = [_vp, _vp, _vp, _vp]
        L.ref_get_scale_min.argtypes = [C.c_int, _vp, _vp, _vp]
        L.ref_q4_k_dequantize.argtypes = [_vp, _vp, C.c_size_t]
        L.ref_q8_0_quantize.argtypes = [_vp, _vp, C.c_size_t]
        L.ref_q8_0_dequantize.argtypes = [_vp, _vp, C.c_size_t]

    @staticmethod
    def available() -> bool:
        return os.path.exists(REF_KERNELS)

    def matmul_q4_k_int8(self, a, b, m, n, k):
        return self._mm(self.lib.eosi_avx2_matmul_q4_k_int8, a, b, m, n, k)

    def matmul_q4_k_avx2_f32(self, a, b, m, n, k):
        return self._mm(self.lib.eosi_avx2_matmul_q4_k, a, b, m, n, k)

    def matmul_q4_k_scalar(self, a, b, m, n, k):
        return self._mm(self.lib.eosi_scalar_matmul_q4_k, a, b, m, n, k)

    def matmul_q8_0(self, a, b, m, n, k):
        return self._mm(self.lib.eosi_scalar_matmul_q8_0, a, b, m, n, k)

    def matmul_q(self, a, b, dtype, m, n, k):
        a = np.ascontiguousarray(a, dtype=np.float32)
        b = np.ascontiguousarray(b, dtype=np.uint8)
        c = np.empty((m, n), dtype=np.float32)
        rc = self.lib.eosi_avx2_matmul_q(_ptr(a), _ptr(b), dtype, _ptr(c), m, n, k)
        return rc, c

    def quantize_sub32(self, a32):
        a32 = np.ascontiguousarray(a32, dtype=np.float32)
        aq = np.empty(32, dtype=np.int8)
        s = np.empty(1, dtype=np.float32)
        t = np.empty(1, dtype=np.int32)
        self.lib.ref_quantize_sub32(_ptr(a32), _ptr(aq), _ptr(s), _ptr(t))
        return aq, s[0], t[0]

    def get_scale_min(self, j, scales12):
        q = np.ascontiguousarray(scales12, dtype=np.uint8)
        sc = np.zeros(1, np.uint8)
        m = np.zeros(1, np.uint8)
        self.lib.ref_get_scale_min(j, _ptr(q), _ptr(sc), _ptr(m))
        return int(sc[0]), int(m[0])

    def q4_k_dequantize(self, b, n_el):
        b = np.ascontiguousarray(b, dtype=np.uint8)
        out = np.empty(n_el, dtype=np.float32)
        assert self.lib.ref_q4_k_dequantize(_ptr(b), _ptr(out), n_el) == 0
        return out

    def q8_0_quantize(self, w):
        w = np.ascontiguousarray(w, dtype=np.float32)
        out = np.empty(w.size // 32 * 34, dtype=np.uint8)
        assert self.lib.ref_q8_0_quantize(_ptr(w), _ptr(out), w.size) == 0
        return out

    def q8_0_dequantize(self, b, n_el):
        b = np.ascontiguousarray(b, dtype=np.uint8)
        out = np.empty(n_el, dtype=np.float32)
        assert self.lib.ref_q8_0_dequantize(_ptr(b), _ptr(out), n_el) == 0
        return out
