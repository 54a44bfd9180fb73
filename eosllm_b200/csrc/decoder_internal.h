// decoder_internal.h -- structures of the device-resident decoder
// (decoder.cu).  Internal: the public boundary is include/eosllm_cuda.h.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "eos_common.cuh"

namespace eos {

// Words the step kernels share in device memory.
struct DecState {
  uint32_t pos;         // position of the next step == tokens consumed
  uint32_t n_prompt;    // steps at pos < n_prompt read their token from prompt[pos]
  uint32_t next_token;  // greedy pick of the previous step
  uint32_t arg_count;   // argmax CTA arrivals (reset by the last CTA)
  uint32_t err;         // EOS_DEVERR_* bits
  uint32_t epoch;       // completed steps (never reset): tensor-parallel exchange epochs
  uint32_t wait_limit_us;  // bound on every tensor-parallel flag wait
  uint32_t pad;
};

// Tensor-parallel exchanges of one decode step, in order, per layer: the
// attention output (packed for the O projection), the O projection's output
// rows, the SiLU output (packed for the down projection), the down
// projection's output rows; after the last layer the greedy pick.
enum : uint32_t { kXAttn = 0, kXORows = 1, kXSilu = 2, kXDRows = 3, kXArgmax = 4, kXTypes = 5 };

// Tensor-parallel receive words of one rank, in its exchange buffer; the
// other ranks write them through CUDA IPC mappings (push).  Flag values are
// epochs: step_epoch * (4 n_layer + 1) + exchange + 1.
struct XRecv {
  uint32_t flag[kXTypes][8];  // [type][q]: written by rank q
  float arg_v[8];       // rank q's best logit
  uint32_t arg_i[8];    // its global vocabulary index
  uint32_t first_nan;   // from rank 0: logits[0] is NaN
  uint32_t pad[7];
  // batched prefill, same four exchange types per layer; values are the
  // prefill's own exchange counter (1, 2, ...)
  uint32_t pf_flag[4][8];
};

// One layer's resident weights (this rank's slices; tensor parallel shards
// every matrix by output rows).
struct DecLayer {
  uint8_t* wqkv;  // [q rows; k rows; v rows] of this rank's heads x n_embd
  uint8_t* wo;    // this rank's n_embd output rows x n_embd
  uint8_t* wgu;   // [gate rows; up rows] of this rank's FFN slice x n_embd
  uint8_t* wd;    // this rank's n_embd output rows x n_ff
  float* attn_norm;
  float* ffn_norm;
};

// RoPE of the pair (x0, x1) at dims (i, i+1) of a head of size HD
// (rope.c:25-33): th = pos * base^(-i/HD), then the rotation with separately
// rounded products.  Shared by the step attention and the batched prefill so
// both rotate identically.
// The rotation's sine and cosine depend only on (i, pos), so callers that
// know the position early compute them first (rope_factors) and rotate later
// (rope_apply); rope_pair does both.
template <int HD>
__device__ __forceinline__ void rope_factors(uint32_t i, uint32_t pos, float base, float& sn, float& cs) {
  const float th = __fmul_rn((float)pos, powf(base, __fdiv_rn(-(float)i, (float)HD)));
  sincosf(th, &sn, &cs);
}
__device__ __forceinline__ void rope_apply(float& x0, float& x1, float sn, float cs) {
  const float p0 = x0, p1 = x1;
  x0 = __fsub_rn(__fmul_rn(p0, cs), __fmul_rn(p1, sn));
  x1 = __fadd_rn(__fmul_rn(p0, sn), __fmul_rn(p1, cs));
}
template <int HD>
__device__ __forceinline__ void rope_pair(float& x0, float& x1, uint32_t i, uint32_t pos, float base) {
  float sn, cs;
  rope_factors<HD>(i, pos, base, sn, cs);
  rope_apply(x0, x1, sn, cs);
}

// Batched prefill kernels (prefill_text.cu).  `act`: the prefill GEMM's
// activation buffer for m rows of k (int8 values, then the per-32 scale
// pairs; prefill_operand_bytes(m, k) bytes).
// x[m][n] = embedding(tokens) when tokens != nullptr; then rmsnorm * w and the
// Q8 packing per 32.
cudaError_t launch_pf_norm_pack(float* x, const uint32_t* tokens, const uint16_t* tok_embd, const float* w, float eps,
                                uint32_t m, uint32_t n, void* act, cudaStream_t st);
// RoPE on q (in place) and k at positions pos0 + row; k and v rows into the
// layer's caches.
cudaError_t launch_pf_rope_kv(float* qkv, float* kc, float* vc, uint32_t m, uint32_t hl, uint32_t kvl, uint32_t hd,
                              uint32_t pos0, float base, cudaStream_t st);
// Causal attention of query rows [0, m) (positions pos0 + row) over cache
// positions [0, pos0 + row] of this rank's hl heads, packed into the O GEMM's
// operand of k = k_total columns (head h0 + h at columns (h0 + h) * hd; one
// GPU: k_total = hl * hd, h0 = 0) and into the n_extra further operands of
// the same layout (tensor parallel: the other ranks' copies).
cudaError_t launch_pf_attn(const float* qkv, const float* kc, const float* vc, void* act, uint32_t m, uint32_t hl,
                           uint32_t kvl, uint32_t h0, uint32_t kv0, uint32_t n_head, uint32_t n_kv_head,
                           uint32_t hd, uint32_t pos0, float scale, uint32_t k_total, void* const* act_extra,
                           uint32_t n_extra, cudaStream_t st);
// silu(gate) * up of gu[m][2 ffl] (gate | up) -- FFN units [f0, f0 + ffl) --
// packed into the down GEMM's operand of k = k_total columns at column f0,
// and into the n_extra further operands of the same layout.
cudaError_t launch_pf_silu_pack(const float* gu, uint32_t m, uint32_t ffl, void* act, uint32_t f0, uint32_t k_total,
                                void* const* act_extra, uint32_t n_extra, cudaStream_t st);
// Tensor-parallel exchange of the prefill: raise this rank's flag in every
// rank's words and wait -- bounded -- for every other rank's flag in this
// rank's words (xs: epoch in xs.add); then, when src != nullptr,
// x[i] += src[i] over m rows of n (the rows every rank pushed into src).
cudaError_t launch_pf_xchg(const XchgSync& xs, float* x, const float* src, uint32_t m, uint32_t n, cudaStream_t st);

}  // namespace eos
