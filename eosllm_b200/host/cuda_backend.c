/*
 * cuda_backend.c -- eosllm's "cuda" kernel backend (ISO C99).
 *
 * The C half of the B200 backend: it registers a backend vtable with the
 * engine's registry exactly like the x86_avx2 backend does
 * (src/kernels/avx2/avx2.c:59-85 of the reference) and forwards the one op
 * it accelerates, matmul_q, to libeosllm_cuda.so through the extern "C"
 * entry points of include/eosllm_cuda.h.  Written to drop into the engine as
 * src/kernels/cuda/cuda.c and to be called from eosi_backend_register_all
 * (src/kernels/register_all.c:3-15) under EOSLLM_HAVE_KERNEL_CUDA.
 *
 * Only matmul_q is filled in: every other slot stays NULL so the engine's
 * per-op priority merge (src/core/session.c:43-81) keeps taking rmsnorm,
 * rope, softmax, silu, gelu and matmul_f32 from the CPU backends.  The
 * backend accepts Q4_K and Q8_0 and returns EOS_E_UNSUPPORTED for any other
 * dtype, as eosi_avx2_matmul_q does (src/kernels/avx2/matmul_q4_k.c:155-171);
 * it never falls back to a CPU kernel itself.
 */
#include <stddef.h>
#include <stdint.h>

#include "eosllm/backend.h"
#include "eosllm/eosllm.h"
#include "eosllm_cuda.h"

eos_status_t eosi_backend_cuda_register(void);

#if defined(EOSLLM_HAVE_KERNEL_CUDA) && EOSLLM_HAVE_KERNEL_CUDA

/* The registry calls probe at every session open and every
 * eos_backend_available (src/core/registry.c:103-114); the library caches
 * the answer after the first device query. */
static eos_status_t cuda_probe(void) { return (eos_status_t)eosi_cuda_probe(); }

static eos_status_t cuda_matmul_q(const float *a, const void *b_quant, eos_dtype_t b_dtype, float *c,
                                  uint32_t m, uint32_t n, uint32_t k) {
    return (eos_status_t)eosi_cuda_matmul_q(a, b_quant, (int)b_dtype, c, m, n, k);
}

/* Priority 90: above x86_avx2 (50) and arm_neon (40), so matmul_q resolves
 * here whenever a B200 is present. */
static const eos_backend_vt_t k_cuda = {
    "cuda", 90, cuda_probe,
    {
        NULL,          /* matmul_f32 -- CPU backends */
        cuda_matmul_q, /* Q4_K / Q8_0 on the GPU */
        NULL, NULL, NULL, NULL, NULL
    }
};

eos_status_t eosi_backend_cuda_register(void) { return eos_backend_register(&k_cuda); }

#else

eos_status_t eosi_backend_cuda_register(void) { return EOS_E_UNSUPPORTED; }

#endif
