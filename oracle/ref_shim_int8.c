/*
 * oracle/ref_shim_int8.c -- exposes the reference's static activation
 * packer and scale unpacker for bit-exact checks.
 *
 * TEST INFRASTRUCTURE ONLY.  Compiled by oracle/Makefile in the build
 * container, where the reference tree exists; the #include below pulls the
 * UNMODIFIED reference source file src/kernels/avx2/matmul_q4_k_int8.c into
 * this translation unit so its `static` helpers quantize_sub32 (:98-154)
 * and get_scale_min (:58-67) become reachable.  Output goes to oracle/_ref/
 * only (git-ignored).
 */
#include "src/kernels/avx2/matmul_q4_k_int8.c"

void ref_quantize_sub32(const float *a32, int8_t *aq32, float *scale, int32_t *sum) {
    __m256i v;
    quantize_sub32(a32, &v, scale, sum);
    _mm256_storeu_si256((__m256i *)aq32, v);
}

void ref_get_scale_min(int j, const uint8_t *q, uint8_t *sc, uint8_t *m) {
    get_scale_min(j, q, sc, m);
}
