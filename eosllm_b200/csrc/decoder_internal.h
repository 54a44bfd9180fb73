// decoder_internal.h -- structures of the device-resident decoder
// (decoder.cu).  Internal: the public boundary is include/eosllm_cuda.h.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "eos_common.cuh"

namespace eos {

constexpr uint32_t kMaxParts = 8;  // tensor-parallel ranks
// Attention splits a head's context into chunks of 32 positions (one CTA of
// the per-op step, one 4-warp group of the persistent step; both reduce in
// the same order).  32 positions are 32 KB of K/V staging, small enough for
// an attention CTA to share an SM with the two CTAs of the QKV GEMV before
// it and start its K/V copies early (programmatic dependent launch).
constexpr uint32_t kAttnChunk = 32;       // positions per attention chunk
constexpr uint32_t kMaxAttnChunks = 512;  // max_ctx <= 16384
constexpr uint32_t kMergeBatch = 16;      // chunks whose o[d] the merge loads in one batch

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

// ---------------------------------------------------------------------------
// Persistent step (decoder_persistent.cu): one cooperative kernel per token
// ---------------------------------------------------------------------------
struct PLayer {
  const uint8_t* w[4];  // this rank's rows of [q; k; v], O, [gate; up], down
  const float* attn_norm;
  const float* ffn_norm;
};

struct PStepParams {
  const PLayer* layers;  // [n_layer], device memory
  const uint8_t* wout;   // this rank's LM-head rows
  const float* out_norm;
  const uint16_t* tok_embd;
  const uint32_t* prompt;
  DecState* state;
  uint32_t* out_tokens;
  float* kc;  // [n_layer][max_ctx][kvl * hd]
  float* vc;
  float* attn_part;  // [hl][max_chunks][hd + 4]
  uint32_t* attn_count;
  float* logits;     // this rank's vocabulary slice
  float* arg_v;      // [gridDim.x]
  uint32_t* arg_i;
  uint64_t* qkv_x;   // this rank's q/k/v rows as pairs
  uint64_t* gu_x;    // this rank's gate/up rows as pairs
  // exchanged: this rank's buffer (in) and every rank's (out, own included)
  const uint64_t* ao_in;  // attention output, Q4_K records of all heads (word pairs)
  const uint64_t* o_in;   // O rows, all n_embd
  const uint64_t* ad_in;  // SiLU output records, all n_ff
  const uint64_t* d_in;   // down rows, all n_embd
  uint64_t* ao_out[kMaxParts];
  uint64_t* o_out[kMaxParts];
  uint64_t* ad_out[kMaxParts];
  uint64_t* d_out[kMaxParts];
  XRecv* recv[kMaxParts];  // the greedy pick's words, as in argmax_kernel
  XRecv* own;
  XchgSync xs;
  uint32_t world, rank;
  uint32_t n_layer, E, F, hl, h0, kvl, kv0, n_head, n_kv_head, ffl, ff0, el, e0, vl, v0, max_ctx, max_chunks;
  float eps, rope_base, attn_scale;
};

// Shared memory of the persistent step for the geometry (bytes).
uint32_t persistent_step_smem(uint32_t E, uint32_t F, uint32_t hd, uint32_t max_chunks, uint32_t n_layer);
// Whether this device runs it (one 384-thread CTA per SM, every CTA resident;
// sets the kernel's shared-memory attribute): Q4_K geometry, head_dim 64 or
// 128, n_embd <= 4096.
bool persistent_step_supported(uint32_t E, uint32_t F, uint32_t hd, uint32_t max_chunks, uint32_t n_layer,
                               int max_smem);
// One step on `grid` CTAs (the SM count), a cooperative launch.
cudaError_t launch_persistent_step(const PStepParams& p, uint32_t hd, uint32_t grid, cudaStream_t st);

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
