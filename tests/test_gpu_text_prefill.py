"""Batched prefill of the device decoder (eosllm_b200/csrc/prefill_text.cu +
the tcgen05 GEMM) against the decoder oracle.

The reference feeds a prompt one token at a time (src/core/session.c:231-236
-> eosi_text_step).  The batched pass computes the same KV-cache rows with
the linears on the tensor cores (activations packed exactly as the reference
packs them, products carried to ~2^-16 relative, f32 sums in another order)
and a streaming softmax, so the logits of the steps that follow it agree
with the oracle stepping every token to the same tolerance as the step path
itself: LOGIT_TOL * rms on tiny models, ENVELOPE_FACTOR times the reference's
own envelope (see test_gpu_decoder.py), here measured with both rmsnorm's
and the matmuls' sums reordered, since the batched pass reorders both.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle.llama import OracleDecoder, make_llama
from oracle.oracle import DT_Q4_K, DT_Q8_0
from test_gpu_decoder import ENVELOPE_FACTOR, LOGIT_TOL, _teacher_forced_check, logit_err, pick_agrees

pytestmark = pytest.mark.gpu


ENVELOPE_ORDERS = (1, 2, 3)  # rmsnorm strided, matmul blocks reversed, both


def prefill_check(oracle, model, tokens, splits, resident=True):
    """Oracle: every token stepped, in the reference's order and with its
    sums reordered (orc_set_sum_order 1, 2, 3: rmsnorm strided, matmul blocks
    and products reversed, both -- the kinds of rounding-level change the
    batched pass makes).  The envelope is the largest deviation of any
    reordered run from the reference's order over all steps.  GPU:
    prefill(tokens[a:b]) for each (a, b) in `splits`, then step() for the
    rest; the logits of those steps must stay within ENVELOPE_FACTOR times
    the envelope (floor LOGIT_TOL), and the picks inside that band."""
    from eosllm_b200.text import TextDecoder
    n_pre = splits[-1][1]
    ref = OracleDecoder(oracle, model)
    alts = [OracleDecoder(oracle, model, sum_order=o) for o in ENVELOPE_ORDERS]
    want, env = [], []
    for j, t in enumerate(tokens):
        r = ref.step(int(t))
        env.extend(logit_err(a.step(int(t)), r) for a in alts)
        if j >= n_pre:
            want.append(r)
    ref.close()
    for a in alts:
        a.close()
    dec = TextDecoder(model)
    dec.set_prefill_resident(resident)
    for a, b in splits:
        dec.prefill(tokens[a:b])
    assert dec.pos == n_pre
    errs, picks = [], []
    for j, t in enumerate(tokens[n_pre:]):
        got = dec.step(int(t))
        errs.append(logit_err(got, want[j]))
        picks.append(int(np.argmax(got)))
    assert dec.pos == len(tokens)
    dec.close()
    bound = max(LOGIT_TOL, ENVELOPE_FACTOR * max(env))
    print("prefill %s: max logit err / rms %.2e, reordered-oracle envelope %.2e" % (splits, max(errs), max(env)))
    assert max(errs) <= bound, (errs, env)
    for j, r in enumerate(want):
        assert pick_agrees(r, picks[j], bound), (j, picks[j], int(np.argmax(r)))
    return errs


@pytest.mark.parametrize("kw", [dict(), dict(n_kv_head=2), dict(n_kv_head=1, n_layer=3),
                                dict(n_embd=256, n_head=2, n_kv_head=1),            # head_dim 128
                                dict(n_embd=512, n_head=4, n_kv_head=2, n_ff=768, n_vocab=1000),
                                dict(n_embd=256, n_head=1, n_kv_head=1, n_ff=512),  # head_dim 256
                                dict(wdtype=DT_Q4_K, out_dtype=DT_Q8_0)])
def test_prefill_then_steps_match_oracle(gpu, oracle, kw):
    model = make_llama(oracle, max_ctx=128, **kw)
    tokens = np.random.default_rng(21).integers(0, model["config"]["n_vocab"], 100).astype(np.uint32)
    prefill_check(oracle, model, tokens, [(0, 93)])


def test_prefill_in_pieces_and_odd_sizes(gpu, oracle):
    """Several prefill calls (later ones attend to the cache rows of earlier
    ones), sizes that are not multiples of the 16-query and 128-row tiles,
    and a one-token prefill."""
    model = make_llama(oracle, max_ctx=160)
    tokens = np.random.default_rng(22).integers(0, model["config"]["n_vocab"], 150).astype(np.uint32)
    prefill_check(oracle, model, tokens, [(0, 1), (1, 18), (18, 53), (53, 141)])


def test_prefill_weights_prepared_per_layer(gpu, oracle):
    """The same pass with each matrix prepared just before its GEMM (the
    path taken when the prepared weights do not fit)."""
    model = make_llama(oracle, max_ctx=128, n_kv_head=2, n_layer=3)
    tokens = np.random.default_rng(25).integers(0, model["config"]["n_vocab"], 100).astype(np.uint32)
    prefill_check(oracle, model, tokens, [(0, 60), (60, 95)], resident=False)


def test_prefill_longer_than_one_block(gpu, oracle):
    """More tokens than one batched block (1024 rows): the second block
    attends to the first block's cache rows."""
    model = make_llama(oracle, n_layer=2, max_ctx=1100)
    tokens = np.random.default_rng(23).integers(0, model["config"]["n_vocab"], 1090).astype(np.uint32)
    prefill_check(oracle, model, tokens, [(0, 1084)])


def test_prefill_model_shape_layer(gpu, oracle):
    """One layer at the 7B layer shape (dim 4096, 32 heads of 128, FFN 11008):
    64 tokens in batch, then 6 steps, against the reference's envelope."""
    model = make_llama(oracle, n_embd=4096, n_layer=1, n_head=32, n_kv_head=32, n_ff=11008, n_vocab=512,
                       max_ctx=80, seed=9)
    tokens = np.random.default_rng(9).integers(0, 512, 70).astype(np.uint32)
    prefill_check(oracle, model, tokens, [(0, 64)])


def test_generate_prefill_on_and_off(gpu, oracle):
    """generate() with the batched prefill (default) and token by token
    (set_prefill_min(0)): both greedy runs agree with the oracle."""
    from eosllm_b200.text import TextDecoder
    model = make_llama(oracle, max_ctx=200, n_kv_head=2)
    prompt = np.random.default_rng(24).integers(0, model["config"]["n_vocab"], 120)
    runs = []
    for pmin in (16, 0):
        dec = TextDecoder(model)
        dec.set_prefill_min(pmin)
        runs.append(dec.generate(prompt, 30))
        assert dec.pos == 120 + 29
        dec.close()
    for picks in runs:
        _teacher_forced_check(oracle, model, prompt, picks)


def test_prefill_errors(gpu, oracle):
    from eosllm_b200 import backend as B
    from eosllm_b200.text import TextDecoder
    model = make_llama(oracle, n_layer=1, max_ctx=8)
    dec = TextDecoder(model)
    with pytest.raises(RuntimeError):
        dec.prefill(np.array([model["config"]["n_vocab"]], np.uint32))  # token out of range
    assert dec.pos == 0
    with pytest.raises(RuntimeError):
        dec.prefill(np.arange(9, dtype=np.uint32))  # beyond the context
    assert dec.pos == 0
    dec.prefill(np.arange(0, dtype=np.uint32))  # nothing to do
    dec.prefill(np.arange(8, dtype=np.uint32))
    assert dec.pos == 8
    assert dec.step_status(1) == B.EOS_E_OUT_OF_MEMORY  # context full
    dec.close()
    q8 = TextDecoder(make_llama(oracle, n_layer=1, max_ctx=8, wdtype=DT_Q8_0, out_dtype=DT_Q8_0))
    with pytest.raises(RuntimeError, match="prefill"):
        q8.prefill(np.arange(4, dtype=np.uint32))  # Q8_0 linears: feed token by token
    assert q8.pos == 0
    q8.close()


def test_decoder_layer_at_position_1024(gpu, oracle):
    """The one-decoder-layer configuration (dim 4096, 32 heads of 128, FFN
    11008, f32 KV, ctx 2048, decode at position 1024): the cache filled by a
    1024-token batched prefill, then steps at positions 1024..1031, against
    the same steps after feeding all 1024 tokens one by one (the step path
    is itself checked against the oracle at model width).  The bound is the
    reference's envelope measured at this layer shape."""
    from eosllm_b200.text import TextDecoder
    model = make_llama(oracle, n_embd=4096, n_layer=1, n_head=32, n_kv_head=32, n_ff=11008, n_vocab=512,
                       max_ctx=2048, seed=3)
    tokens = np.random.default_rng(3).integers(0, 512, 1032).astype(np.uint32)
    a, b = TextDecoder(model), TextDecoder(model)
    a.set_prefill_min(0)
    a.generate(tokens[:1024], 0)  # token by token
    b.prefill(tokens[:1024])
    assert a.pos == b.pos == 1024
    errs = []
    for t in tokens[1024:]:
        la, lb = a.step(int(t)), b.step(int(t))
        errs.append(float(np.max(np.abs(la.astype(np.float64) - lb)) / np.sqrt(np.mean(la.astype(np.float64) ** 2))))
    a.close()
    b.close()
    # 3x the 7B-layer envelope measured on the oracle (3.23e-2, test_gpu_decoder.py)
    print("position 1024: max logit diff / rms %.2e" % max(errs))
    assert max(errs) <= ENVELOPE_FACTOR * 3.23e-2, errs
