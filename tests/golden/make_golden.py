"""Generate tests/golden/*.npz from the REFERENCE ITSELF.

Runs the unmodified reference kernels compiled from their own sources by
`make -C oracle ref` (oracle/_ref/libref_kernels.so) -- only possible in the
build container, where the reference tree exists.  The fixtures then pin the
oracle (oracle/eos_oracle.c) and the CUDA kernels on machines without the
reference.  Inputs are seeded (the reference's own xorshift32 seeds where its
tests define them, else this project's generator), so the script is
reproducible:

    make -C oracle && make -C oracle ref && python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle.oracle import DT_Q4_K, DT_Q8_0, Oracle, RefKernels  # noqa: E402
from oracle.llama import RefDecoder, make_llama  # noqa: E402
from oracle.gguf_writer import write_llama  # noqa: E402

# tiny Llama decoders whose logits the reference engine produces below
DECODER_CASES = {"mha_q4k": dict(), "gqa_q4k": dict(n_kv_head=2),
                 "mha_q80": dict(wdtype=DT_Q8_0, out_dtype=DT_Q8_0)}
DECODER_TOKENS = [5, 17, 200, 3, 99, 42, 7, 250, 1, 319, 0, 128]

OUT = os.path.dirname(os.path.abspath(__file__))


def known_answer_block(o: Oracle) -> np.ndarray:
    """The all-sub-blocks super-block of tests/unit/test_runner.c:727-803:
    d=0.25, dmin=0.0625, sc={3,12,7,21,15,9,30,4}, m={1..8}, qs low nibble
    i&15, high nibble 15-(i&15)."""
    blk = np.zeros(144, np.uint8)
    blk[0:2] = np.frombuffer(np.uint16(o.f32_to_f16(0.25)).tobytes(), np.uint8)
    blk[2:4] = np.frombuffer(np.uint16(o.f32_to_f16(0.0625)).tobytes(), np.uint8)
    blk[4:16] = o.pack_q4k_scales(np.array([3, 12, 7, 21, 15, 9, 30, 4], np.uint8),
                                  np.array([1, 2, 3, 4, 5, 6, 7, 8], np.uint8))
    i = np.arange(128)
    blk[16:] = ((i & 15) | ((15 - (i & 15)) << 4)).astype(np.uint8)
    return blk


def act_edge_cases(rng: np.random.Generator) -> np.ndarray:
    """Groups of 32 activations that exercise every branch of quantize_sub32."""
    groups = []
    groups.append(np.zeros(32, np.float32))                           # max_abs == 0
    groups.append(-np.zeros(32, np.float32))                          # negative zeros
    g = np.zeros(32, np.float32); g[5] = 1e-40; groups.append(g)      # subnormal max -> inv = inf
    g = rng.standard_normal(32).astype(np.float32) * 1e-39; groups.append(g)
    g = rng.standard_normal(32).astype(np.float32); g[3] = np.nan; groups.append(g)
    g = rng.standard_normal(32).astype(np.float32); g[0] = np.nan; groups.append(g)
    g = rng.standard_normal(32).astype(np.float32); g[31] = np.nan; groups.append(g)
    g = rng.standard_normal(32).astype(np.float32); g[7] = np.inf; groups.append(g)
    g = rng.standard_normal(32).astype(np.float32); g[9] = -np.inf; groups.append(g)
    g = np.full(32, np.nan, np.float32); groups.append(g)
    g = (np.round(rng.standard_normal(32) * 8) / 2).astype(np.float32); g[0] = 127.0; groups.append(g)  # .5 ties
    g = np.linspace(-127, 127, 32).astype(np.float32); groups.append(g)
    g = (rng.uniform(-1, 1, 32) * 3e38).astype(np.float32); groups.append(g)
    g = np.full(32, 1.0, np.float32); groups.append(g)
    g = np.full(32, -2.5, np.float32); groups.append(g)
    for e in (-30, -10, -3, 0, 3, 10, 30):
        groups.append((rng.standard_normal(32) * 10.0 ** e).astype(np.float32))
    for _ in range(40):
        groups.append(rng.standard_normal(32).astype(np.float32))
    return np.concatenate(groups)


def decoder_fixture(o: Oracle) -> None:
    """Logits of the reference engine's own eosi_text_step
    (src/modality/text/text.c:267-436) for seeded synthetic models."""
    import tempfile
    out = {"tokens": np.array(DECODER_TOKENS, np.int64)}
    for name, kw in DECODER_CASES.items():
        m = make_llama(o, **kw)
        with tempfile.TemporaryDirectory() as td:
            path = os.path.join(td, "model.gguf")
            write_llama(path, m)
            rd = RefDecoder(path, m["config"]["max_ctx"], m["config"]["n_vocab"])
            out[f"{name}_logits"] = np.stack([rd.step(t) for t in DECODER_TOKENS])
            rd.close()
    np.savez_compressed(os.path.join(OUT, "decoder_tiny.npz"), **out)


def main() -> None:
    if not RefKernels.available():
        raise SystemExit("oracle/_ref is not built: run `make -C oracle ref` where the reference exists")
    o, r = Oracle(), RefKernels()
    if "--decoder-only" in sys.argv:
        decoder_fixture(o)
        return
    rng = np.random.default_rng(20240601)

    # 1. the reference's own known-answer block (test_runner.c:727-803)
    blk = known_answer_block(o)
    ones = np.ones(256, np.float32)
    ka_scalar = r.matmul_q4_k_scalar(ones, blk, 1, 1, 256)[1]
    # int8 parity fixture (test_runner.c:1075-1150): N=4 copies, xorshift32 seed 0x42424242
    a_xs, _ = o.xs_rand_unit(256, 0x42424242)
    w4 = np.tile(blk, 4)
    xs_int8 = r.matmul_q4_k_int8(a_xs, w4, 1, 4, 256)[1]
    xs_scalar = r.matmul_q4_k_scalar(a_xs, w4, 1, 4, 256)[1]
    xs_avx2_f32 = r.matmul_q4_k_avx2_f32(a_xs, blk, 1, 1, 256)[1]
    np.savez_compressed(os.path.join(OUT, "q4k_known_answers.npz"), block=blk, ka_scalar=ka_scalar, a_xs=a_xs,
                        xs_int8=xs_int8, xs_scalar=xs_scalar, xs_avx2_f32=xs_avx2_f32)

    # 2. activation packing edge cases (quantize_sub32, matmul_q4_k_int8.c:98-154)
    a = act_edge_cases(rng)
    aq, sc, sm = [], [], []
    for g in range(a.size // 32):
        q, s, t = r.quantize_sub32(a[32 * g:32 * g + 32])
        aq.append(q); sc.append(s); sm.append(t)
    np.savez_compressed(os.path.join(OUT, "act_pack.npz"), a=a, aq=np.concatenate(aq),
                        scales=np.array(sc, np.float32), sums=np.array(sm, np.int32))

    # 3. Q4_K matmuls on small shapes (own quantizer output; reference kernels)
    cases = {}
    for idx, (m, n, k) in enumerate([(1, 1, 256), (1, 2, 512), (1, 3, 256), (1, 4, 256), (1, 5, 512),
                                     (1, 37, 1024), (2, 16, 768), (3, 9, 2048), (1, 16, 4096), (1, 4, 11008)]):
        w = o.gauss(n * k, 100 + idx, 0.02)
        bq = o.q4_k_quantize(w)
        x = o.gauss(m * k, 200 + idx, 1.0)
        cases[f"c{idx}_shape"] = np.array([m, n, k], np.int64)
        cases[f"c{idx}_w"] = bq
        cases[f"c{idx}_a"] = x
        cases[f"c{idx}_matmul_q"] = r.matmul_q(x, bq, DT_Q4_K, m, n, k)[1]
        cases[f"c{idx}_scalar"] = r.matmul_q4_k_scalar(x, bq, m, n, k)[1]
        if n * k <= 8192:
            cases[f"c{idx}_deq"] = r.q4_k_dequantize(bq, n * k)
    np.savez_compressed(os.path.join(OUT, "q4k_matmul.npz"), **cases)

    # 4. Q8_0: reference quantizer + scalar matmul; the stress grid of
    #    test_runner.c:648-709 (k 32..128, m 1,2,4) plus model-like rows
    cases = {}
    for idx, (m, n, k) in enumerate([(1, 1, 32), (2, 1, 64), (4, 1, 96), (1, 1, 128), (1, 7, 288),
                                     (2, 33, 1024), (1, 8, 4096), (1, 3, 11008)]):
        w = o.gauss(n * k, 300 + idx, 0.02)
        q8 = r.q8_0_quantize(w)
        x = o.gauss(m * k, 400 + idx, 1.0)
        cases[f"c{idx}_shape"] = np.array([m, n, k], np.int64)
        if n * k <= 8192:
            cases[f"c{idx}_src"] = w
        cases[f"c{idx}_w"] = q8
        cases[f"c{idx}_a"] = x
        cases[f"c{idx}_matmul_q"] = r.matmul_q(x, q8, DT_Q8_0, m, n, k)[1]
    np.savez_compressed(os.path.join(OUT, "q8_0_matmul.npz"), **cases)

    # 5. tiny decoders run by the reference engine itself
    decoder_fixture(o)
    print("golden fixtures written to", OUT)


if __name__ == "__main__":
    main()
