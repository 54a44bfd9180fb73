"""Generate tests/golden/greedy_7b.npz from the REFERENCE ENGINE ITSELF.

The full synthetic 7B-shape Llama model (32 layers, dim 4096, 32 heads, FFN
11008, vocabulary 32000, Q4_K linears and LM head, F16 embeddings, F32 norms;
random-init from stream seed 4 of this project's generator, the same bytes as
`eosllm_b200.text.synthetic_llama(seed=4)` builds on a GPU) is written to a
GGUF file and run through the unmodified reference engine compiled from its
sources (oracle/_ref/libeosllm_ref.so: eos_model_open, eosi_text_open,
eosi_text_step with the x86 AVX2 backend's op table).  The prompt is 512 ids
uniform in [0, 32000) from numpy's default_rng(4); after it the engine picks
257 tokens greedily (src/sched/greedy.c:60-72: the first index of the largest
logit), feeding each pick back (src/core/session.c:228-262).

Stored per pick: the token, the eight largest logits and their indices (in
descending order, ties by index) and the rms of the logits, so a GPU run can
be checked teacher-forced: at every step it is fed the reference's previous
pick and its own pick must be the reference's, or tie with it within a stated
band.  Takes about 15 minutes on one core:

    make -C oracle && make -C oracle ref && python tests/golden/make_greedy_7b.py
"""
from __future__ import annotations

import os
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle.gguf_writer import write_llama  # noqa: E402
from oracle.llama import RefDecoder, make_llama  # noqa: E402
from oracle.oracle import Oracle  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "greedy_7b.npz")
MODEL = dict(n_embd=4096, n_layer=32, n_head=32, n_kv_head=32, n_ff=11008, n_vocab=32000)
PROMPT, PICKS, SEED, TOPK = 512, 257, 4, 8


def topk(logits: np.ndarray, k: int):
    """The k largest logits, descending; equal values by ascending index
    (the greedy rule's strict > from index 0)."""
    idx = np.lexsort((np.arange(logits.size), -logits.astype(np.float64)))[:k]
    return idx.astype(np.int32), logits[idx].astype(np.float32)


def main() -> None:
    t0 = time.time()
    max_ctx = PROMPT + PICKS - 1
    model = make_llama(Oracle(), **MODEL, max_ctx=max_ctx, seed=SEED)
    print(f"model generated in {time.time() - t0:.0f} s", flush=True)
    prompt = np.random.default_rng(SEED).integers(0, MODEL["n_vocab"], PROMPT).astype(np.uint32)
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "llama7b.gguf")
        write_llama(path, model)
        del model
        ref = RefDecoder(path, max_ctx, MODEL["n_vocab"])
        print(f"gguf written and opened at {time.time() - t0:.0f} s", flush=True)
        logits = None
        for i, t in enumerate(prompt):
            logits = ref.step(int(t))
            if i % 64 == 63:
                print(f"prompt {i + 1}/{PROMPT} at {time.time() - t0:.0f} s", flush=True)
        toks = np.zeros(PICKS, np.int32)
        top_i = np.zeros((PICKS, TOPK), np.int32)
        top_v = np.zeros((PICKS, TOPK), np.float32)
        rms = np.zeros(PICKS, np.float32)
        for j in range(PICKS):
            ti, tv = topk(logits, TOPK)
            toks[j], top_i[j], top_v[j] = ti[0], ti, tv
            rms[j] = np.sqrt(np.mean(logits.astype(np.float64) ** 2))
            if j + 1 < PICKS:
                logits = ref.step(int(toks[j]))
            if j % 32 == 31:
                print(f"pick {j + 1}/{PICKS} at {time.time() - t0:.0f} s", flush=True)
        ref.close()
    np.savez_compressed(OUT, prompt=prompt, tokens=toks, top_idx=top_i, top_val=top_v, logit_rms=rms,
                        seed=np.int32(SEED), config=np.array([MODEL[k] for k in
                                                              ("n_embd", "n_layer", "n_head", "n_kv_head", "n_ff",
                                                               "n_vocab")], np.int32))
    print(f"wrote {OUT} in {time.time() - t0:.0f} s; margins top1-top2: min "
          f"{float(np.min(top_v[:, 0] - top_v[:, 1])):.4g}, median {float(np.median(top_v[:, 0] - top_v[:, 1])):.4g}")


if __name__ == "__main__":
    main()
