"""The persistent step (one cooperative kernel per token, decoder_persistent.cu)
against the per-op step graph (decoder.cu) on the same model: every phase
runs the per-op kernel's arithmetic in the same order, so the logits of
every step must be BIT-IDENTICAL, and so must the greedy generation --
stepped from position 0, after a batched prefill that leaves many
32-position attention chunks to merge, and across switches of the mode on
one decoder.  Each step's pick must be the first index of the largest logit
(src/sched/greedy.c:66-69)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CASES = {
    # head_dim 128, MHA
    "mha_hd128": dict(n_embd=512, n_layer=2, n_head=4, n_kv_head=4, n_ff=1024, n_vocab=320, max_ctx=100),
    # head_dim 64, grouped-query attention
    "gqa_hd64": dict(n_embd=256, n_layer=2, n_head=4, n_kv_head=2, n_ff=768, n_vocab=300, max_ctx=80),
    # one layer of the 7B shape, full vocabulary
    "layer7b": dict(n_embd=4096, n_layer=1, n_head=32, n_kv_head=32, n_ff=11008, n_vocab=32000, max_ctx=48),
}


def _same(a, b) -> bool:
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


def _pair(name, seed=3):
    from eosllm_b200.text import TextDecoder, synthetic_llama
    model = synthetic_llama(**CASES[name], seed=seed)
    per = TextDecoder(model)
    assert per.step_mode == TextDecoder.STEP_PER_OP  # the default (AUTO)
    pst = TextDecoder(model)
    pst.set_step_mode(TextDecoder.STEP_PERSISTENT)
    return model, pst, per


@pytest.mark.parametrize("name", sorted(CASES))
def test_persistent_step_is_bit_identical_to_per_op(gpu, name):
    from eosllm_b200.text import TextDecoder
    model, pst, per = _pair(name)
    try:
        assert pst.step_mode == TextDecoder.STEP_PERSISTENT and pst.step_kernels == 1
        assert per.step_mode == TextDecoder.STEP_PER_OP and per.step_kernels > 1
        cfg = CASES[name]
        rng = np.random.default_rng(11)
        tokens = rng.integers(0, cfg["n_vocab"], min(40, cfg["max_ctx"] - 4))
        for i, t in enumerate(tokens):
            a, b = pst.step(int(t)), per.step(int(t))
            assert _same(a, b), f"step {i}: logits differ (max |d| {np.max(np.abs(a - b))})"
        # greedy generation through the step's own argmax
        pst.reset()
        per.reset()
        prompt = rng.integers(0, cfg["n_vocab"], 6)
        ga, gb = pst.generate(prompt, 12), per.generate(prompt, 12)
        assert ga.tolist() == gb.tolist()
        # the first pick is the first index of the largest logit after the prompt
        pst.reset()
        for t in prompt[:-1]:
            pst.step(int(t))
        lg = pst.step(int(prompt[-1]))
        assert int(np.argmax(lg)) == int(ga[0])
    finally:
        pst.close()
        per.close()
        del model


def test_persistent_step_after_long_prefill_merges_many_chunks(gpu):
    """A 600-token context: the batched prefill writes the cache (the same
    path for both modes), then steps attend over 19+ chunks of 32 positions
    (more than one merge batch of 16)."""
    from eosllm_b200.text import TextDecoder, synthetic_llama
    cfg = dict(n_embd=512, n_layer=2, n_head=4, n_kv_head=2, n_ff=768, n_vocab=500, max_ctx=640)
    model = synthetic_llama(**cfg, seed=7)
    pst, per = TextDecoder(model), TextDecoder(model)
    pst.set_step_mode(TextDecoder.STEP_PERSISTENT)
    try:
        rng = np.random.default_rng(5)
        ctx = rng.integers(0, cfg["n_vocab"], 600).astype(np.uint32)
        pst.prefill(ctx)
        per.prefill(ctx)
        for i, t in enumerate(rng.integers(0, cfg["n_vocab"], 20)):
            a, b = pst.step(int(t)), per.step(int(t))
            assert _same(a, b), f"step {600 + i}: logits differ"
    finally:
        pst.close()
        per.close()


def test_step_mode_switches_on_one_decoder(gpu):
    """Switching re-records the step (and clears the exchange words): the
    logits stay those of the per-op decoder at every position."""
    from eosllm_b200.text import TextDecoder
    model, pst, per = _pair("mha_hd128", seed=4)
    try:
        rng = np.random.default_rng(3)
        for i, t in enumerate(rng.integers(0, 320, 30)):
            if i in (5, 15):  # to per-op (AUTO), back to persistent
                pst.set_step_mode(TextDecoder.STEP_AUTO if pst.step_mode == TextDecoder.STEP_PERSISTENT
                                  else TextDecoder.STEP_PERSISTENT)
            assert _same(pst.step(int(t)), per.step(int(t))), f"step {i}"
        assert pst.step_mode == TextDecoder.STEP_PERSISTENT
    finally:
        pst.close()
        per.close()


def test_persistent_mode_refused_where_unsupported(gpu):
    """Q8_0 linears run the per-op step only: asking for the persistent step
    is EOS_E_UNSUPPORTED and the decoder stays per-op."""
    from eosllm_b200 import backend as B
    from eosllm_b200.text import TextDecoder, synthetic_llama
    model = synthetic_llama(n_embd=256, n_layer=1, n_head=4, n_kv_head=4, n_ff=512, n_vocab=300, max_ctx=32,
                            wdtype=B.DT_Q8_0, out_dtype=B.DT_Q8_0)
    dec = TextDecoder(model)
    try:
        assert dec.step_mode == TextDecoder.STEP_PER_OP
        with pytest.raises(B.CudaBackendError) as e:
            dec.set_step_mode(TextDecoder.STEP_PERSISTENT)
        assert e.value.status == B.EOS_E_UNSUPPORTED
        assert dec.step_mode == TextDecoder.STEP_PER_OP
    finally:
        dec.close()
