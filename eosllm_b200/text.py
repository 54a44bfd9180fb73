"""Device-resident Llama text decoder: Python view of eosi_cuda_text_*.

Mirrors the reference's text-modality interface (src/modality/text/text.h:
eosi_text_open / eosi_text_step / eosi_text_close) and the greedy scheduler
(src/sched/greedy.c): `TextDecoder.step(token)` returns the logits of one
step, `TextDecoder.generate(prompt, n_gen)` runs prefill plus greedy decoding
on the GPU without a host round trip per token.

Models are dicts in the layout of a GGUF Llama file:
    {"config": {n_embd, n_layer, n_head, n_kv_head, n_ff, n_vocab, max_ctx,
                rms_eps, rope_base, wdtype, out_dtype},
     "tok_embd": F16 bits [n_vocab * n_embd], "output_norm": F32 [n_embd],
     "output": quantized [n_vocab rows],
     "layers": [{"attn_norm", "ffn_norm", "wq", "wk", "wv", "wo", "wg", "wu",
                 "wd"}, ...]}
with numpy arrays (host memory, uploaded at open) or CUDA tensors on the
decoder's device (copied device to device).

`synthetic_llama()` builds a random-init model of any shape straight on the
device with this library's seeded generator and quantizers.  Stream
numbering (shared with the CPU test models): stream s = seed * 1000 + 1,
+2, ... in the order, per layer, attn_norm, ffn_norm, wq, wk, wv, wo, wg, wu,
wd; then tok_embd, output_norm, output.  Linear weights are N(0, sigma)
(sigma = 0.02), norms 1 + N(0, 0.1), embeddings N(0, 1) rounded to F16.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import backend as B

_LAYER_KEYS = ("attn_norm", "ffn_norm", "wq", "wk", "wv", "wo", "wg", "wu", "wd")


class LlamaDesc(C.Structure):
    """eosi_cuda_llama_t (include/eosllm_cuda.h)."""
    _fields_ = [(n, C.c_uint32) for n in ("n_embd", "n_layer", "n_head", "n_kv_head", "n_ff", "n_vocab",
                                          "max_ctx")] + \
               [("rms_eps", C.c_float), ("rope_base", C.c_float), ("wdtype", C.c_int32),
                ("out_dtype", C.c_int32), ("weights_on_device", C.c_int32),
                ("tok_embd", C.c_void_p), ("output_norm", C.c_void_p), ("output_w", C.c_void_p)] + \
               [(n, C.POINTER(C.c_void_p)) for n in _LAYER_KEYS]


def _addr(x) -> int:
    return x.ctypes.data if isinstance(x, np.ndarray) else x.data_ptr()


class TextDecoder:
    """One rank's decoder (world == 1: the whole model on `device`)."""

    def __init__(self, model: dict, device: int = 0, rank: int = 0, world: int = 1):
        self.lib = B.load()
        c = model["config"]
        self.config = dict(c)
        self.n_vocab = c["n_vocab"]
        d = LlamaDesc()
        for k in ("n_embd", "n_layer", "n_head", "n_kv_head", "n_ff", "n_vocab", "max_ctx"):
            setattr(d, k, int(c[k]))
        d.rms_eps, d.rope_base = float(c["rms_eps"]), float(c["rope_base"])
        d.wdtype, d.out_dtype = int(c["wdtype"]), int(c["out_dtype"])
        on_dev = not isinstance(model["tok_embd"], np.ndarray)
        d.weights_on_device = 1 if on_dev else 0
        self._keep = [model]  # the arrays must outlive the open call
        d.tok_embd = _addr(model["tok_embd"])
        d.output_norm = _addr(model["output_norm"])
        d.output_w = _addr(model["output"])
        for key in _LAYER_KEYS:
            arr = (C.c_void_p * max(1, c["n_layer"]))(*[_addr(lay[key]) for lay in model["layers"]])
            self._keep.append(arr)
            setattr(d, key, arr)
        self.handle = C.c_void_p()
        B.check(self.lib.eosi_cuda_text_open(C.byref(d), device, rank, world, C.byref(self.handle)),
                "eosi_cuda_text_open")
        self._keep = None  # weights are resident on the device now

    @classmethod
    def from_gguf(cls, path: str, max_ctx: int = 0, device: int = 0, rank: int = 0, world: int = 1):
        """eosi_cuda_text_open_gguf: a GGUF v3 Llama file straight to this
        rank's GPU (only its own slices are read from the mapped file)."""
        desc, g = gguf_map(path, max_ctx)
        self = cls.__new__(cls)
        self.lib = B.load()
        self.config = {k: getattr(desc, k) for k in ("n_embd", "n_layer", "n_head", "n_kv_head", "n_ff", "n_vocab",
                                                    "max_ctx", "rms_eps", "rope_base", "wdtype", "out_dtype")}
        self.lib.eosi_cuda_gguf_unmap(g)
        self.n_vocab = self.config["n_vocab"]
        self._keep = None
        self.handle = C.c_void_p()
        B.check(self.lib.eosi_cuda_text_open_gguf(path.encode(), max_ctx, device, rank, world,
                                                  C.byref(self.handle)), "eosi_cuda_text_open_gguf")
        return self

    def ipc_handle(self) -> bytes:
        """This rank's exchange-buffer IPC handle (tensor parallel)."""
        buf = (C.c_ubyte * 64)()
        B.check(self.lib.eosi_cuda_text_ipc_handle(self.handle, buf, 64), "eosi_cuda_text_ipc_handle")
        return bytes(buf)

    def attach_peers(self, handles: list) -> None:
        """Map every rank's exchange buffer (handles in rank order) and build
        the step (tensor parallel)."""
        blob = b"".join(handles)
        buf = (C.c_ubyte * len(blob)).from_buffer_copy(blob)
        B.check(self.lib.eosi_cuda_text_attach_peers(self.handle, buf, len(blob)), "eosi_cuda_text_attach_peers")

    @staticmethod
    def attach_local(ranks: list) -> None:
        """eosi_cuda_text_attach_local: tensor-parallel ranks opened in this
        one process (ranks[q] is rank q's decoder)."""
        arr = (C.c_void_p * len(ranks))(*[r.handle.value for r in ranks])
        B.check(B.load().eosi_cuda_text_attach_local(arr, len(ranks)), "eosi_cuda_text_attach_local")

    def set_wait_limit(self, limit_us: int) -> None:
        """Bound on every tensor-parallel flag wait, in microseconds."""
        B.check(self.lib.eosi_cuda_text_set_wait_limit(self.handle, int(limit_us)), "eosi_cuda_text_set_wait_limit")

    def connect(self, group=None) -> None:
        """attach_peers with the handles all-gathered over a torch.distributed
        process group (any backend)."""
        import torch.distributed as dist
        handles = [None] * dist.get_world_size(group)
        dist.all_gather_object(handles, self.ipc_handle(), group=group)
        self.attach_peers(handles)

    def step(self, token: int) -> np.ndarray:
        """eosi_text_step: logits of the next position for `token`."""
        out = np.empty(self.n_vocab, np.float32)
        B.check(self.lib.eosi_cuda_text_step(self.handle, int(token), out.ctypes.data), "eosi_cuda_text_step")
        return out

    def step_status(self, token: int) -> int:
        out = np.empty(self.n_vocab, np.float32)
        return self.lib.eosi_cuda_text_step(self.handle, int(token), out.ctypes.data)

    def generate(self, prompt, n_gen: int) -> np.ndarray:
        """Prefill `prompt`, then n_gen greedy picks (the first follows the
        last prompt token)."""
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.empty(max(1, n_gen), np.uint32)
        B.check(self.lib.eosi_cuda_text_generate(self.handle, p.ctypes.data, p.size, n_gen, out.ctypes.data),
                "eosi_cuda_text_generate")
        return out[:n_gen]

    def prefill(self, tokens) -> None:
        """Feed `tokens` in one batched pass on the tensor cores (KV cache
        rows, no logits); Q4_K linears (EOS_E_UNSUPPORTED otherwise), on one
        GPU or tensor parallel."""
        p = np.ascontiguousarray(tokens, dtype=np.uint32)
        B.check(self.lib.eosi_cuda_text_prefill(self.handle, p.ctypes.data if p.size else None, p.size),
                "eosi_cuda_text_prefill")

    def set_prefill_min(self, min_tokens: int) -> None:
        """generate() prefills in batch when at least `min_tokens` prompt
        tokens precede the last one (0: always token by token)."""
        B.check(self.lib.eosi_cuda_text_set_prefill_min(self.handle, int(min_tokens)),
                "eosi_cuda_text_set_prefill_min")

    def set_prefill_resident(self, resident: bool) -> None:
        """Keep every layer's weights prepared for the prefill GEMM (default,
        when they fit in half of the free memory) or prepare each matrix just
        before its GEMM."""
        B.check(self.lib.eosi_cuda_text_set_prefill_resident(self.handle, int(bool(resident))),
                "eosi_cuda_text_set_prefill_resident")

    def reset(self) -> None:
        B.check(self.lib.eosi_cuda_text_reset(self.handle), "eosi_cuda_text_reset")

    @property
    def pos(self) -> int:
        return int(self.lib.eosi_cuda_text_pos(self.handle))

    # eosi_cuda_text_set_step_mode: how a step runs
    STEP_AUTO, STEP_PERSISTENT, STEP_PER_OP = 0, 1, 2

    def set_step_mode(self, mode: int) -> None:
        """STEP_PER_OP: a graph of one kernel per operation; STEP_PERSISTENT:
        one cooperative kernel per token (Q4_K, head_dim 64/128, n_embd <=
        4096); STEP_AUTO (default): per-op, the faster on a B200.  Both give
        bit-identical logits.  Tensor parallel: every rank, no step running."""
        B.check(self.lib.eosi_cuda_text_set_step_mode(self.handle, int(mode)), "eosi_cuda_text_set_step_mode")

    @property
    def step_mode(self) -> int:
        """The mode in use (STEP_PERSISTENT or STEP_PER_OP)."""
        return int(self.lib.eosi_cuda_text_step_mode(self.handle))

    @property
    def step_kernels(self) -> int:
        """Kernels one step launches (nodes of the step's CUDA graph)."""
        return int(self.lib.eosi_cuda_text_step_kernels(self.handle))

    @property
    def stream(self) -> int:
        return int(self.lib.eosi_cuda_text_stream(self.handle) or 0)

    def close(self) -> None:
        if self.handle:
            self.lib.eosi_cuda_text_close(self.handle)
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def gguf_map(path: str, max_ctx: int = 0):
    """eosi_cuda_gguf_map (no GPU needed): (LlamaDesc with pointers into the
    read-only mapping, mapping handle for eosi_cuda_gguf_unmap)."""
    lib = B.load()
    desc, g = LlamaDesc(), C.c_void_p()
    B.check(lib.eosi_cuda_gguf_map(path.encode(), max_ctx, C.byref(g), C.byref(desc)), "eosi_cuda_gguf_map")
    return desc, g


def partition(config: dict, rank: int, world: int) -> dict:
    """The slice of the model rank `rank` of `world` owns (host only)."""
    d = LlamaDesc()
    for k in ("n_embd", "n_layer", "n_head", "n_kv_head", "n_ff", "n_vocab", "max_ctx"):
        setattr(d, k, int(config[k]))
    d.wdtype, d.out_dtype = int(config["wdtype"]), int(config["out_dtype"])
    out = (C.c_uint32 * 11)()
    B.check(B.load().eosi_cuda_text_partition(C.byref(d), rank, world, out), "eosi_cuda_text_partition")
    keys = ("head_dim", "head0", "heads", "kv_head0", "kv_heads", "ff0", "ff_len", "vocab0", "vocab_len",
            "out_row0", "out_rows")
    return dict(zip(keys, list(out)))


def synthetic_llama(n_embd=256, n_layer=2, n_head=4, n_kv_head=4, n_ff=512, n_vocab=320, max_ctx=64, seed=3,
                    wdtype=B.DT_Q4_K, out_dtype=B.DT_Q4_K, rms_eps=1e-5, rope_base=10000.0, sigma=0.02,
                    device: int = 0) -> dict:
    """A random-init Llama-architecture model generated on `device` (CUDA
    tensors), stream numbering as in the module docstring."""
    import torch
    dev = torch.device("cuda", device)
    hd = n_embd // n_head
    kvd = n_kv_head * hd
    stream = [seed * 1000]

    def next_stream() -> int:
        stream[0] += 1
        return stream[0]

    def gauss(n: int, s: float):
        t = torch.empty(n, dtype=torch.float32, device=dev)
        B.fill_gauss_dev(t, n, next_stream(), 0, s)
        return t

    def quant(rows: int, k: int, dt: int):
        n = rows * k
        out = torch.empty(B.weight_bytes(dt, rows, k), dtype=torch.uint8, device=dev)
        if dt == B.DT_Q4_K:
            B.q4_k_from_gauss_dev(out, n, next_stream(), sigma)
        else:
            src = gauss(n, sigma)
            B.q8_0_quantize_dev(src, out, n)
            del src
        return out

    def norm(n: int):
        return gauss(n, 0.1) + 1.0

    with torch.cuda.device(dev):
        layers = []
        for _ in range(n_layer):
            lay = {}
            lay["attn_norm"] = norm(n_embd)
            lay["ffn_norm"] = norm(n_embd)
            lay["wq"] = quant(n_embd, n_embd, wdtype)
            lay["wk"] = quant(kvd, n_embd, wdtype)
            lay["wv"] = quant(kvd, n_embd, wdtype)
            lay["wo"] = quant(n_embd, n_embd, wdtype)
            lay["wg"] = quant(n_ff, n_embd, wdtype)
            lay["wu"] = quant(n_ff, n_embd, wdtype)
            lay["wd"] = quant(n_embd, n_ff, wdtype)
            layers.append(lay)
        tok = gauss(n_vocab * n_embd, 1.0).to(torch.float16).view(torch.int16)
        output_norm = norm(n_embd)
        output = quant(n_vocab, n_embd, out_dtype)
        torch.cuda.synchronize(dev)
    cfg = dict(n_embd=n_embd, n_layer=n_layer, n_head=n_head, n_kv_head=n_kv_head, n_ff=n_ff, n_vocab=n_vocab,
               max_ctx=max_ctx, rms_eps=rms_eps, rope_base=rope_base, wdtype=wdtype, out_dtype=out_dtype)
    return dict(config=cfg, tok_embd=tok, output_norm=output_norm, output=output, layers=layers)


def weight_bytes_per_token(config: dict) -> int:
    """Quantized weight bytes one decode step reads: every block linear and
    the LM head (the embedding row and norms are negligible)."""
    E, F, V = config["n_embd"], config["n_ff"], config["n_vocab"]
    kvd = config["n_kv_head"] * (E // config["n_head"])
    wdt, odt = config["wdtype"], config["out_dtype"]
    per_layer = (B.weight_bytes(wdt, E + 2 * kvd, E) + B.weight_bytes(wdt, E, E) + B.weight_bytes(wdt, 2 * F, E)
                 + B.weight_bytes(wdt, E, F))
    return config["n_layer"] * per_layer + B.weight_bytes(odt, V, E)
