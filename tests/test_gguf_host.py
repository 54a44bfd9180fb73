"""GGUF straight to the device (eosllm_b200/csrc/gguf_open.cu): the parser
and model description, on the CPU (no GPU needed).  Files are written by the
test-infrastructure GGUF writer in the layout the reference engine reads
(oracle/gguf_writer.py); the rules checked are the reference's
(src/format/gguf/gguf.c, src/modality/text/text.c:104-215)."""
from __future__ import annotations

import ctypes as C
import struct

import numpy as np
import pytest

from oracle.gguf_writer import GGML_F32, llama_parts, write_gguf, write_llama
from oracle.llama import make_llama
from oracle.oracle import DT_Q4_K, DT_Q8_0


def _map(path, max_ctx=0):
    from eosllm_b200.text import gguf_map
    return gguf_map(str(path), max_ctx)


def _status(path, max_ctx=0):
    from eosllm_b200 import backend as B
    try:
        _, g = _map(path, max_ctx)
    except B.CudaBackendError as e:
        return e.status
    B.load().eosi_cuda_gguf_unmap(g)
    return B.EOS_OK


@pytest.mark.parametrize("kw", [dict(), dict(n_kv_head=2, wdtype=DT_Q8_0, out_dtype=DT_Q8_0),
                                dict(out_dtype=DT_Q8_0, n_layer=3), dict(n_embd=256, n_head=2, n_kv_head=1)])
def test_map_describes_the_model(oracle, tmp_path, kw):
    from eosllm_b200 import backend as B
    model = make_llama(oracle, **kw)
    c = model["config"]
    path = tmp_path / "m.gguf"
    write_llama(str(path), model)
    d, g = _map(path)
    try:
        for k in ("n_embd", "n_layer", "n_head", "n_kv_head", "n_ff", "n_vocab", "max_ctx", "wdtype", "out_dtype"):
            assert getattr(d, k) == c[k], k
        assert d.rms_eps == np.float32(c["rms_eps"]) and d.rope_base == np.float32(c["rope_base"])
        assert d.weights_on_device == 0
        for ptr, arr in ((d.tok_embd, model["tok_embd"]), (d.output_norm, model["output_norm"]),
                         (d.output_w, model["output"])):
            assert C.string_at(ptr, arr.nbytes) == arr.tobytes()
        for key in ("attn_norm", "ffn_norm", "wq", "wk", "wv", "wo", "wg", "wu", "wd"):
            for L in range(c["n_layer"]):
                arr = model["layers"][L][key]
                assert C.string_at(getattr(d, key)[L], arr.nbytes) == arr.tobytes(), (key, L)
    finally:
        B.load().eosi_cuda_gguf_unmap(g)


def test_context_bound(oracle, tmp_path):
    model = make_llama(oracle, max_ctx=64)
    path = tmp_path / "m.gguf"
    write_llama(str(path), model)
    from eosllm_b200 import backend as B
    for req, want in ((0, 64), (16, 16), (10 ** 6, 64)):
        d, g = _map(path, req)
        assert d.max_ctx == want
        B.load().eosi_cuda_gguf_unmap(g)


def _write(path, meta, tensors):
    write_gguf(str(path), meta, tensors)
    return path


def test_defaults_for_optional_keys(oracle, tmp_path):
    """head_count_kv defaults to head_count, rope.freq_base to 10000 and the
    rms epsilon to 1e-5 (text.c:136-153)."""
    from eosllm_b200 import backend as B
    meta, t = llama_parts(make_llama(oracle))
    drop = ("llama.attention.head_count_kv", "llama.rope.freq_base", "llama.attention.layer_norm_rms_epsilon")
    d, g = _map(_write(tmp_path / "m.gguf", [(k, v) for k, v in meta if k not in drop], t))
    assert d.n_kv_head == d.n_head and d.rope_base == 10000.0 and d.rms_eps == np.float32(1e-5)
    B.load().eosi_cuda_gguf_unmap(g)


def test_errors_follow_the_reference(oracle, tmp_path):
    from eosllm_b200 import backend as B
    model = make_llama(oracle, n_layer=2)
    meta, t = llama_parts(model)
    good = _write(tmp_path / "good.gguf", meta, t)
    raw = good.read_bytes()
    assert _status(good) == B.EOS_OK
    assert _status(tmp_path / "absent.gguf") == B.EOS_E_IO
    (tmp_path / "magic.gguf").write_bytes(b"GGUX" + raw[4:])
    assert _status(tmp_path / "magic.gguf") == B.EOS_E_FORMAT
    (tmp_path / "v2.gguf").write_bytes(raw[:4] + struct.pack("<I", 2) + raw[8:])
    assert _status(tmp_path / "v2.gguf") == B.EOS_E_FORMAT
    (tmp_path / "cut.gguf").write_bytes(raw[:len(raw) - 1000])  # last tensor past EOF
    assert _status(tmp_path / "cut.gguf") == B.EOS_E_FORMAT
    (tmp_path / "head.gguf").write_bytes(raw[:40])  # truncated metadata
    assert _status(tmp_path / "head.gguf") == B.EOS_E_FORMAT
    no_down = [x for x in t if x[0] != "blk.1.ffn_down.weight"]
    assert _status(_write(tmp_path / "nodown.gguf", meta, no_down)) == B.EOS_E_FORMAT
    no_key = [(k, v) for k, v in meta if k != "llama.feed_forward_length"]
    assert _status(_write(tmp_path / "nokey.gguf", no_key, t)) == B.EOS_E_NOT_FOUND
    no_arch = [(k, v) for k, v in meta if k != "general.architecture"]
    assert _status(_write(tmp_path / "noarch.gguf", no_arch, t)) == B.EOS_E_FORMAT
    bad_align = [(k, 48 if k == "general.alignment" else v) for k, v in meta]
    assert _status(_write(tmp_path / "align.gguf", bad_align, t)) == B.EOS_E_FORMAT
    q40 = [(n, d, 2 if n == "blk.0.attn_q.weight" else g, b) for n, d, g, b in t]  # GGML Q4_0
    assert _status(_write(tmp_path / "q40.gguf", meta, q40)) == B.EOS_E_UNSUPPORTED
    E, V = model["config"]["n_embd"], model["config"]["n_vocab"]
    f32_emb = [(n, d, GGML_F32, np.zeros(E * V, np.float32).tobytes()) if n == "token_embd.weight" else (n, d, g, b)
               for n, d, g, b in t]
    assert _status(_write(tmp_path / "f32emb.gguf", meta, f32_emb)) == B.EOS_E_UNSUPPORTED
    tied = [x for x in t if x[0] != "output.weight"]
    assert _status(_write(tmp_path / "tied.gguf", meta, tied)) == B.EOS_E_UNSUPPORTED
    wrong = [(n, [E, 3 * E] if n == "blk.0.attn_q.weight" else d, g, b) for n, d, g, b in t]
    assert _status(_write(tmp_path / "shape.gguf", meta, wrong)) == B.EOS_E_FORMAT
