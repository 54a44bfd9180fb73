"""Synthetic Llama models and two CPU decoders -- TEST INFRASTRUCTURE ONLY.

  make_llama()   a random-init Llama-architecture model (numpy arrays):
                 F16 token embeddings, F32 norms, Q4_K (or Q8_0) linears from
                 the seeded generator and quantizers of oracle/eos_oracle.c.
  OracleDecoder  the C restatement of eosi_text_step (orc_text_*).
  RefDecoder     the reference engine itself (oracle/_ref/libeosllm_ref.so,
                 compiled from its sources): eos_model_open on a GGUF written
                 by oracle/gguf_writer.py, then eosi_text_open/eosi_text_step
                 with the op table the engine's dispatch selects on an AVX2
                 host (x86_avx2 matmul_q, scalar rmsnorm/rope/silu).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from .oracle import REF_ENGINE, Oracle

DT_Q8_0, DT_Q4_K = 32, 33


def make_llama(o: Oracle, n_embd=256, n_layer=2, n_head=4, n_kv_head=4, n_ff=512, n_vocab=320, max_ctx=64,
               seed=3, wdtype=DT_Q4_K, out_dtype=DT_Q4_K, rms_eps=1e-5, rope_base=10000.0, sigma=0.02):
    hd = n_embd // n_head
    kvd = n_kv_head * hd
    stream = [seed * 1000]

    def gauss(n, s=sigma):
        stream[0] += 1
        return o.gauss(n, stream[0], s)

    def quant(rows, k, dt):
        w = gauss(rows * k)
        return o.q4_k_quantize(w) if dt == DT_Q4_K else o.q8_0_quantize(w)

    def norm(n):
        return (1.0 + gauss(n, 0.1)).astype(np.float32)

    layers = []
    for _ in range(n_layer):
        layers.append(dict(attn_norm=norm(n_embd), ffn_norm=norm(n_embd),
                           wq=quant(n_embd, n_embd, wdtype), wk=quant(kvd, n_embd, wdtype),
                           wv=quant(kvd, n_embd, wdtype), wo=quant(n_embd, n_embd, wdtype),
                           wg=quant(n_ff, n_embd, wdtype), wu=quant(n_ff, n_embd, wdtype),
                           wd=quant(n_embd, n_ff, wdtype)))
    tok = gauss(n_vocab * n_embd, 1.0).astype(np.float16).view(np.uint16)
    cfg = dict(n_embd=n_embd, n_layer=n_layer, n_head=n_head, n_kv_head=n_kv_head, n_ff=n_ff, n_vocab=n_vocab,
               max_ctx=max_ctx, rms_eps=rms_eps, rope_base=rope_base, wdtype=wdtype, out_dtype=out_dtype)
    return dict(config=cfg, tok_embd=tok, output_norm=norm(n_embd), output=quant(n_vocab, n_embd, out_dtype),
                layers=layers)


class _OrcLlama(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("n_embd", "n_layer", "n_head", "n_kv_head", "n_ff", "n_vocab", "max_ctx")] + \
               [("rms_eps", C.c_float), ("rope_base", C.c_float), ("wdtype", C.c_int), ("out_dtype", C.c_int),
                ("tok_embd", C.c_void_p), ("output_norm", C.c_void_p), ("output_w", C.c_void_p)] + \
               [(n, C.POINTER(C.c_void_p)) for n in ("attn_norm", "ffn_norm", "wq", "wk", "wv", "wo", "wg", "wu", "wd")]


class OracleDecoder:
    """orc_text_step on `model`.  sum_order (orc_set_sum_order, a bit mask)
    measures the reference algorithm's own sensitivity to summation order:
    1 runs rmsnorm's mean square in a 256-wide strided order, 2 accumulates
    the quantized matmuls' blocks last to first; 0 is the reference's order."""

    def __init__(self, o: Oracle, model: dict, sum_order: int = 0):
        self.o, self.model, self.sum_order = o, model, sum_order
        o.lib.orc_set_sum_order.argtypes = [C.c_int]
        c = model["config"]
        L = o.lib
        L.orc_text_open.argtypes = [C.POINTER(_OrcLlama), C.POINTER(C.c_void_p)]
        L.orc_text_step.argtypes = [C.c_void_p, C.c_uint32, C.c_void_p]
        L.orc_text_close.argtypes = [C.c_void_p]
        d = _OrcLlama()
        for k in ("n_embd", "n_layer", "n_head", "n_kv_head", "n_ff", "n_vocab", "max_ctx", "wdtype", "out_dtype"):
            setattr(d, k, c[k])
        d.rms_eps, d.rope_base = c["rms_eps"], c["rope_base"]
        d.tok_embd = model["tok_embd"].ctypes.data
        d.output_norm = model["output_norm"].ctypes.data
        d.output_w = model["output"].ctypes.data
        self._tables = {}
        for key in ("attn_norm", "ffn_norm", "wq", "wk", "wv", "wo", "wg", "wu", "wd"):
            arr = (C.c_void_p * c["n_layer"])(*[lay[key].ctypes.data for lay in model["layers"]])
            self._tables[key] = arr
            setattr(d, key, arr)
        self._desc = d
        self.st = C.c_void_p()
        rc = L.orc_text_open(C.byref(d), C.byref(self.st))
        assert rc == 0, rc

    def step(self, token: int) -> np.ndarray:
        out = np.empty(self.model["config"]["n_vocab"], np.float32)
        self.o.lib.orc_set_sum_order(self.sum_order)
        try:
            rc = self.o.lib.orc_text_step(self.st, token, out.ctypes.data)
        finally:
            self.o.lib.orc_set_sum_order(0)
        assert rc == 0, rc
        return out

    def close(self):
        if self.st:
            self.o.lib.orc_text_close(self.st)
            self.st = C.c_void_p()

    def __del__(self):
        self.close()


class RefDecoder:
    """The reference's eosi_text_step on a GGUF file."""

    def __init__(self, gguf_path: str, max_ctx: int, n_vocab: int, lib_path: str = REF_ENGINE):
        if not os.path.exists(lib_path):
            raise FileNotFoundError(lib_path)
        L = self.lib = C.CDLL(lib_path)
        L.eos_init_defaults.restype = C.c_int
        assert L.eos_init_defaults() == 0
        L.eos_model_open.argtypes = [C.c_char_p, C.POINTER(C.c_void_p)]
        L.eos_model_open.restype = C.c_int
        L.eosi_text_open.argtypes = [C.c_void_p, C.c_void_p, C.c_uint32, C.POINTER(C.c_void_p)]
        L.eosi_text_open.restype = C.c_int
        L.eosi_text_step.argtypes = [C.c_void_p, C.c_uint32, C.c_void_p]
        L.eosi_text_step.restype = C.c_int
        L.eosi_text_close.argtypes = [C.c_void_p]
        L.eos_model_close.argtypes = [C.c_void_p]
        self.n_vocab = n_vocab
        self.model = C.c_void_p()
        rc = L.eos_model_open(gguf_path.encode(), C.byref(self.model))
        assert rc == 0, rc
        # eos_backend_ops_t (include/eosllm/backend.h:32-64) as the AVX2 host's
        # dispatch resolves it (src/core/session.c:53-81)
        names = ("eosi_scalar_matmul_f32", "eosi_avx2_matmul_q", "eosi_scalar_rmsnorm", "eosi_scalar_softmax",
                 "eosi_scalar_rope", "eosi_scalar_silu", "eosi_scalar_gelu")
        self.ops = (C.c_void_p * 7)(*[C.cast(getattr(L, n), C.c_void_p).value for n in names])
        self.st = C.c_void_p()
        rc = L.eosi_text_open(self.model, C.cast(self.ops, C.c_void_p), max_ctx, C.byref(self.st))
        assert rc == 0, rc

    def step(self, token: int) -> np.ndarray:
        out = np.empty(self.n_vocab, np.float32)
        rc = self.lib.eosi_text_step(self.st, token, out.ctypes.data)
        assert rc == 0, rc
        return out

    def close(self):
        if self.st:
            self.lib.eosi_text_close(self.st)
            self.st = C.c_void_p()
        if self.model:
            self.lib.eos_model_close(self.model)
            self.model = C.c_void_p()

    def __del__(self):
        self.close()
