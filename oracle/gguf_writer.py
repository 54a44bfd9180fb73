"""Minimal GGUF v3 writer for synthetic Llama models -- TEST INFRASTRUCTURE.

Writes the subset of the GGUF container the reference engine reads
(src/format/gguf/gguf.c): metadata of the types used below, tensor infos
(dims in GGUF order, innermost first), 32-byte aligned tensor data.
GGML type codes: F32 = 0, F16 = 1, Q8_0 = 8, Q4_K = 12 (gguf.c:40-45).
"""
from __future__ import annotations

import struct

import numpy as np

GGUF_U32, GGUF_F32, GGUF_STRING, GGUF_ARRAY = 4, 6, 8, 9
GGML_F32, GGML_F16, GGML_Q8_0, GGML_Q4_K = 0, 1, 8, 12
ALIGN = 32


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, value) -> bytes:
    out = _str(key)
    if isinstance(value, str):
        return out + struct.pack("<I", GGUF_STRING) + _str(value)
    if isinstance(value, float):
        return out + struct.pack("<If", GGUF_F32, value)
    if isinstance(value, int):
        return out + struct.pack("<II", GGUF_U32, value)
    if isinstance(value, list):  # array of strings
        body = b"".join(_str(v) for v in value)
        return out + struct.pack("<IIQ", GGUF_ARRAY, GGUF_STRING, len(value)) + body
    raise TypeError(type(value))


def write_gguf(path: str, metadata: list[tuple[str, object]], tensors: list[tuple[str, list[int], int, bytes]]):
    """tensors: (name, dims innermost-first, ggml type, raw bytes)."""
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(metadata))
    head += b"".join(_kv(k, v) for k, v in metadata)
    infos, blobs, off = b"", [], 0
    for name, dims, gtype, raw in tensors:
        infos += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        infos += struct.pack("<IQ", gtype, off)
        pad = (-len(raw)) % ALIGN
        blobs.append(raw + b"\0" * pad)
        off += len(raw) + pad
    pre = head + infos
    pre += b"\0" * ((-len(pre)) % ALIGN)
    with open(path, "wb") as f:
        f.write(pre)
        for b in blobs:
            f.write(b)


def llama_tokens(n_vocab: int) -> list[str]:
    """A byte-level-looking vocabulary of n_vocab distinct strings."""
    return ["<s>", "</s>"] + [f"t{i}" for i in range(n_vocab - 2)]


def byte_fallback_tokens(n_vocab: int) -> list[str]:
    """A vocabulary the engine's BPE tokenizer can encode any text with: the
    256 byte tokens <0xNN> (its fallback set) after <s>, </s>, then fillers."""
    assert n_vocab >= 258
    return ["<s>", "</s>"] + [f"<0x{b:02X}>" for b in range(256)] + [f"t{i}" for i in range(n_vocab - 258)]


def write_llama(path: str, model: dict, tokens: list[str] | None = None) -> None:
    """model: dict from oracle.llama.make_llama (numpy arrays + config);
    tokens: the vocabulary strings (default llama_tokens)."""
    write_gguf(path, *llama_parts(model, tokens))


def llama_parts(model: dict, tokens: list[str] | None = None):
    """(metadata, tensors) of write_llama, for tests that alter single items."""
    c = model["config"]
    meta = [("general.architecture", "llama"), ("general.alignment", ALIGN),
            ("llama.embedding_length", c["n_embd"]), ("llama.block_count", c["n_layer"]),
            ("llama.attention.head_count", c["n_head"]), ("llama.attention.head_count_kv", c["n_kv_head"]),
            ("llama.feed_forward_length", c["n_ff"]), ("llama.context_length", c["max_ctx"]),
            ("llama.rope.freq_base", float(c["rope_base"])),
            ("llama.attention.layer_norm_rms_epsilon", float(c["rms_eps"])),
            ("tokenizer.ggml.model", "llama"),
            ("tokenizer.ggml.tokens", tokens if tokens is not None else llama_tokens(c["n_vocab"]))]
    wt = GGML_Q4_K if c["wdtype"] == 33 else GGML_Q8_0
    ot = GGML_Q4_K if c["out_dtype"] == 33 else GGML_Q8_0
    E, V, F, H = c["n_embd"], c["n_vocab"], c["n_ff"], c["n_embd"] // c["n_head"] * c["n_kv_head"]
    t = [("token_embd.weight", [E, V], GGML_F16, model["tok_embd"].tobytes()),
         ("output_norm.weight", [E], GGML_F32, model["output_norm"].tobytes()),
         ("output.weight", [E, V], ot, model["output"].tobytes())]
    for L in range(c["n_layer"]):
        lay = model["layers"][L]
        t += [(f"blk.{L}.attn_norm.weight", [E], GGML_F32, lay["attn_norm"].tobytes()),
              (f"blk.{L}.attn_q.weight", [E, E], wt, lay["wq"].tobytes()),
              (f"blk.{L}.attn_k.weight", [E, H], wt, lay["wk"].tobytes()),
              (f"blk.{L}.attn_v.weight", [E, H], wt, lay["wv"].tobytes()),
              (f"blk.{L}.attn_output.weight", [E, E], wt, lay["wo"].tobytes()),
              (f"blk.{L}.ffn_norm.weight", [E], GGML_F32, lay["ffn_norm"].tobytes()),
              (f"blk.{L}.ffn_gate.weight", [E, F], wt, lay["wg"].tobytes()),
              (f"blk.{L}.ffn_up.weight", [E, F], wt, lay["wu"].tobytes()),
              (f"blk.{L}.ffn_down.weight", [F, E], wt, lay["wd"].tobytes())]
    return meta, t
