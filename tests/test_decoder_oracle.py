"""The decoder oracle (orc_text_step, a C restatement of eosi_text_step,
src/modality/text/text.c:267-436) pinned against the reference engine:
logits committed from the engine itself (tests/golden/decoder_tiny.npz) and,
where oracle/_ref is built, a live comparison on further shapes."""
from __future__ import annotations

import os
import tempfile

import numpy as np
import pytest

from oracle.gguf_writer import write_llama
from oracle.llama import OracleDecoder, RefDecoder, make_llama
from oracle.oracle import DT_Q8_0, REF_ENGINE

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "decoder_tiny.npz")
CASES = {"mha_q4k": dict(), "gqa_q4k": dict(n_kv_head=2),
         "mha_q80": dict(wdtype=DT_Q8_0, out_dtype=DT_Q8_0)}


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_decoder_matches_reference_logits(oracle, name):
    g = np.load(GOLDEN)
    model = make_llama(oracle, **CASES[name])
    dec = OracleDecoder(oracle, model)
    got = np.stack([dec.step(int(t)) for t in g["tokens"]])
    dec.close()
    np.testing.assert_array_equal(got.view(np.uint32), g[f"{name}_logits"].view(np.uint32))


def test_oracle_decoder_errors(oracle):
    """text.c:277-278: out-of-vocab token -> INVALID_ARG, full context ->
    OUT_OF_MEMORY; neither advances the position."""
    model = make_llama(oracle, n_layer=1, max_ctx=3)
    dec = OracleDecoder(oracle, model)
    out = np.empty(model["config"]["n_vocab"], np.float32)
    assert oracle.lib.orc_text_step(dec.st, model["config"]["n_vocab"], out.ctypes.data) == 1
    for t in (1, 2, 3):
        dec.step(t)
    assert oracle.lib.orc_text_step(dec.st, 4, out.ctypes.data) == 2
    dec.close()


@pytest.mark.skipif(not os.path.exists(REF_ENGINE), reason="oracle/_ref engine not built (needs the reference tree)")
@pytest.mark.parametrize("kw", [dict(n_layer=3, n_head=8, n_kv_head=2, n_ff=768, n_vocab=257, max_ctx=16),
                                dict(n_embd=512, n_head=4, n_kv_head=1, n_ff=256, n_vocab=33, max_ctx=9,
                                     wdtype=DT_Q8_0),
                                dict(rope_base=500000.0, rms_eps=1e-6, max_ctx=12, seed=11)])
def test_oracle_decoder_live_vs_reference_engine(oracle, kw):
    model = make_llama(oracle, **kw)
    c = model["config"]
    rng = np.random.default_rng(7)
    tokens = rng.integers(0, c["n_vocab"], c["max_ctx"])
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "m.gguf")
        write_llama(path, model)
        rd = RefDecoder(path, c["max_ctx"], c["n_vocab"])
        od = OracleDecoder(oracle, model)
        for t in tokens:
            a, b = od.step(int(t)), rd.step(int(t))
            np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
        od.close()
        rd.close()
