/*
 * oracle/eos_oracle.h -- CPU restatement of eosllm's quantized matmul path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the checker the CUDA kernels are
 * compared against; it is never linked into, loaded by, or called from the
 * product library (eosllm_b200/).  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg may use it.
 *
 * Every function restates one function of the reference (embeddedos-org/
 * eosllm) and cites the file:line it follows.  Pinning: the restatement is
 * checked against the reference's own golden vectors and known answers
 * (tests/unit/test_runner.c) and, in the build container, bit-for-bit
 * against the reference sources compiled by oracle/Makefile into
 * oracle/_ref/ (tests/golden/ holds fixtures generated that way).
 *
 * Build with -std=c99 -ffp-contract=off: the reference is compiled as ISO
 * C99, where GCC does not contract a*b+c into an FMA, so neither may we.
 */
#ifndef EOS_ORACLE_H
#define EOS_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* eos_status_t values (include/eosllm/eosllm.h:66-77 in the reference). */
enum {
    ORC_OK = 0,
    ORC_E_INVALID_ARG = 1,
    ORC_E_OUT_OF_MEMORY = 2,
    ORC_E_UNSUPPORTED = 3,
    ORC_E_INTERNAL = 9
};

/* eos_dtype_t values used on this path (include/eosllm/tensor.h:22-37). */
enum { ORC_DT_F32 = 0, ORC_DT_F16 = 1, ORC_DT_Q8_0 = 32, ORC_DT_Q4_K = 33 };

#define ORC_Q4K_BLOCK_ELEMS 256
#define ORC_Q4K_BLOCK_BYTES 144
#define ORC_Q80_BLOCK_ELEMS 32
#define ORC_Q80_BLOCK_BYTES 34

/* --- binary16 (src/util/f16.h:17-82) ---------------------------------- */
float    orc_f16_to_f32(uint16_t h);
uint16_t orc_f32_to_f16(float f);

/* --- Q4_K block helpers ------------------------------------------------- */
/* 6-bit scale/min unpack: src/kernels/avx2/matmul_q4_k_int8.c:58-67. */
void orc_get_scale_min(int j, const uint8_t *scales12, uint8_t *sc, uint8_t *m);
/* All 8 (sc, m) pairs of `count` 12-byte fields: sc[8i+j], m[8i+j]. */
void orc_unpack_scale_min_batch(const uint8_t *scales12, size_t count, uint8_t *sc, uint8_t *m);
/* Inverse packing: tests/unit/test_runner.c:716-725. */
void orc_pack_q4k_scales(const uint8_t sc[8], const uint8_t m[8], uint8_t out[12]);

/* --- activation packing (src/kernels/avx2/matmul_q4_k_int8.c:98-154) ---
 * 32 floats -> 32 int8 (source order), f32 scale, i32 sum of the
 * pre-saturation lanes, with x86 MAXPS / CVTPS2DQ / PACKSS semantics. */
void orc_quantize_sub32(const float *a32, int8_t *aq32, float *scale, int32_t *sum_aq);
/* Whole vector: k % 32 == 0; writes k int8, k/32 scales, k/32 sums. */
int  orc_quantize_act(const float *a, uint32_t k, int8_t *aq, float *scales, int32_t *sums);

/* --- matmuls: C[m,n] = A[m,k] . deq(B)[n,k]^T ---------------------------- */
/* Production x86 Q4_K path: src/kernels/avx2/matmul_q4_k_int8.c:164-269
 * (n < 4 routes to the f32 path exactly as :182-184 does). */
int orc_matmul_q4_k_int8(const float *a, const void *b, float *c,
                         uint32_t m, uint32_t n, uint32_t k);
/* AVX2 f32-dequant path: src/kernels/avx2/matmul_q4_k.c:70-153 (8-lane FMA
 * accumulators, SSE horizontal sum). */
int orc_matmul_q4_k_avx2_f32(const float *a, const void *b, float *c,
                             uint32_t m, uint32_t n, uint32_t k);
/* Scalar f32 oracle: src/kernels/scalar/matmul_q4_k.c:43-104. */
int orc_matmul_q4_k_scalar(const float *a, const void *b, float *c,
                           uint32_t m, uint32_t n, uint32_t k);
/* Scalar Q8_0 (production on every backend): src/kernels/scalar/matmul_q8.c:21-58. */
int orc_matmul_q8_0(const float *a, const void *b, float *c,
                    uint32_t m, uint32_t n, uint32_t k);
/* Scalar f32: src/kernels/scalar/matmul_f32.c:14-32. */
int orc_matmul_f32(const float *a, const float *b, float *c,
                   uint32_t m, uint32_t n, uint32_t k);
/* The x86_avx2 backend's matmul_q slot: src/kernels/avx2/matmul_q4_k.c:155-171. */
int orc_matmul_q(const float *a, const void *b, int dtype, float *c,
                 uint32_t m, uint32_t n, uint32_t k);

/* Row-sharded multithreaded driver around orc_matmul_q (rows are
 * independent, matmul_q4_k_int8.c:215-265): threads <= 0 means all cores.
 * Used only for the all-cores CPU baseline. */
int orc_matmul_q_threads(const float *a, const void *b, int dtype, float *c,
                         uint32_t m, uint32_t n, uint32_t k, int threads);

/* --- quant schemes (src/quant/q4_k.c:42-81, src/quant/q8_0.c:33-93) ----- */
int orc_q4_k_dequantize(const void *src, float *dst, size_t n_elements);
int orc_q8_0_dequantize(const void *src, float *dst, size_t n_elements);
int orc_q8_0_quantize(const float *src, void *dst, size_t n_elements);

/* Q4_K quantizer.  The reference has none (src/quant/q4_k.c:83-93 returns
 * UNSUPPORTED), so this is this project's own affine min/max fit; the
 * device quantizer in the product reproduces it bit-for-bit. */
int orc_q4_k_quantize(const float *src, void *dst, size_t n_elements);

/* --- synthetic inputs ---------------------------------------------------- */
/* Counter-based normal-ish generator shared bit-for-bit with the device:
 * x = sigma * (sum of 12 uniform 24-bit draws - 6), Irwin-Hall(12), from
 * splitmix64(seed, index).  Only integer ops, one int->float conversion and
 * one multiply, so CPU and GPU produce identical floats. */
float orc_gauss(uint64_t seed, uint64_t index, float sigma);
void  orc_fill_gauss(float *dst, size_t n, uint64_t seed, uint64_t offset, float sigma);

/* xorshift32 as used by the reference's unit tests (test_runner.c:633-646). */
uint32_t orc_xorshift32(uint32_t *state);
float    orc_xs_rand_unit(uint32_t *state);

/* --- decoder ops (src/kernels/scalar/{rmsnorm,rope,silu}.c) -------------- */
/* Summation orders, a bit mask; 0 (default) = the reference's order
 * everywhere.  Bit 1: rmsnorm's mean square as a 256-wide strided reduction
 * (per-thread partials, warp butterfly, warps in order) instead of the
 * sequential loop.  Bit 2: the quantized matmuls (orc_matmul_q4_k_int8,
 * orc_matmul_q8_0) accumulate their blocks last to first.  The non-zero
 * orders exist only to MEASURE how much the reference algorithm itself moves
 * under a rounding-level reordering of its sums: decoder tests bound the
 * GPU's deviation by that envelope.  Parity results always use order 0. */
void orc_set_sum_order(int order);
int orc_rmsnorm(const float *x, const float *w, float eps, float *y,
                uint32_t rows, uint32_t cols);
int orc_rope(float *x, uint32_t n_heads, uint32_t head_dim, uint32_t pos, float base);
int orc_silu(const float *x, float *y, size_t n);

/* --- Llama decoder step: restates eosi_text_step ------------------------
 * (src/modality/text/text.c:267-436) with the x86 dispatch the engine builds
 * on an AVX2 host: matmul_q -> orc_matmul_q (int8 Q4_K, scalar Q8_0),
 * rmsnorm / rope / silu -> the scalar ops.  Weights are caller-owned: per
 * layer pointer tables (GGUF row-major, one row per output), F16 token
 * embeddings [n_vocab][n_embd], F32 norms. */
typedef struct {
    uint32_t n_embd, n_layer, n_head, n_kv_head, n_ff, n_vocab, max_ctx;
    float rms_eps, rope_base;
    int wdtype;                     /* ORC_DT_Q4_K or ORC_DT_Q8_0 for all linears */
    int out_dtype;                  /* dtype of output.weight */
    const uint16_t *tok_embd;       /* F16 */
    const float *output_norm;
    const void *output_w;
    const float *const *attn_norm;  /* [n_layer] */
    const float *const *ffn_norm;
    const void *const *wq, *const *wk, *const *wv, *const *wo;
    const void *const *wg, *const *wu, *const *wd;
} orc_llama_t;

typedef struct orc_text orc_text_t;
int  orc_text_open(const orc_llama_t *m, orc_text_t **out);
int  orc_text_step(orc_text_t *st, uint32_t token, float *logits);
uint32_t orc_text_pos(const orc_text_t *st);
void orc_text_close(orc_text_t *st);

#ifdef __cplusplus
}
#endif
#endif /* EOS_ORACLE_H */
