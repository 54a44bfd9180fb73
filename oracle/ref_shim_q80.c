/*
 * oracle/ref_shim_q80.c -- exposes the reference's static Q8_0 quantizer
 * and dequantizer (src/quant/q8_0.c:33-93) through its registered vtable.
 *
 * TEST INFRASTRUCTURE ONLY, compiled by oracle/Makefile from the
 * UNMODIFIED reference sources; output into oracle/_ref/ only.
 */
#define eos_quant_register ref_q80_capture_register
#include "src/quant/q8_0.c"
#undef eos_quant_register

static const eos_quant_vt_t *g_captured;

eos_status_t ref_q80_capture_register(const eos_quant_vt_t *vt) {
    g_captured = vt;
    return EOS_OK;
}

static const eos_quant_vt_t *q80_vt(void) {
    g_captured = NULL;
    if (eosi_quant_q8_0_register() != EOS_OK) return NULL;
    return g_captured;
}

int ref_q8_0_quantize(const float *src, void *dst, size_t n) {
    const eos_quant_vt_t *vt = q80_vt();
    return vt ? (int)vt->quantize(src, dst, n) : EOS_E_UNSUPPORTED;
}

int ref_q8_0_dequantize(const void *src, float *dst, size_t n) {
    const eos_quant_vt_t *vt = q80_vt();
    return vt ? (int)vt->dequantize(src, dst, n) : EOS_E_UNSUPPORTED;
}
