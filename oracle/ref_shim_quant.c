/*
 * oracle/ref_shim_quant.c -- exposes the reference's static Q4_K
 * dequantizer (src/quant/q4_k.c:42-81) through its registered vtable.
 *
 * TEST INFRASTRUCTURE ONLY, compiled by oracle/Makefile from the
 * UNMODIFIED reference sources; output into oracle/_ref/ only.  The
 * registry call inside the included file is satisfied by the capture
 * function below instead of the engine's registry.
 */
#include "src/quant/q4_k.c"

static const eos_quant_vt_t *g_captured;

eos_status_t eos_quant_register(const eos_quant_vt_t *vt) {
    g_captured = vt;
    return EOS_OK;
}

int ref_q4_k_dequantize(const void *src, float *dst, size_t n) {
    g_captured = NULL;
    if (eosi_quant_q4_k_register() != EOS_OK || g_captured == NULL) return EOS_E_UNSUPPORTED;
    return (int)g_captured->dequantize(src, dst, n);
}
