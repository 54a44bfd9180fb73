// decoder.cu -- device-resident Llama decoder step for sm_100a: the work of
// eosi_text_step (src/modality/text/text.c:267-436) with every tensor in HBM
// and the greedy pick of the next token (src/sched/greedy.c:48-73) on the
// device, so a whole generation runs without a host round trip per token.
//
// One token = one CUDA graph replay.  The position, the token fed in and the
// greedy pick live in a DecState word block in device memory, so the same
// graph serves every step.  Kernels of a step are chained with programmatic
// dependent launch (PDL): each kernel triggers its dependent early and waits
// (griddepcontrol.wait) before it touches any buffer an earlier kernel
// writes or reads, so the GEMVs stream their weights while the small
// kernels before them run.
//
// Per layer (tensor-parallel rank r of G; G == 1 is the whole model; every
// matrix is sharded by output rows, so every output element is computed
// whole on one rank, exactly as on one GPU):
//   norm_pack    x = x_prev + t (residual, text.c:404-406 and :420-421),
//                rmsnorm (src/kernels/scalar/rmsnorm.c:14-37), then the Q8
//                activation packing of the next GEMV; every rank normalises
//                the whole vector
//   GEMV         [q; k; v] rows of this rank's heads          (text.c:349-352)
//   attention    RoPE on q and k (src/kernels/scalar/rope.c:16-38), K/V append
//                at `pos` (text.c:359-362), softmax attention with the GQA
//                head map (text.c:364-401), split over positions; the last
//                CTA of a head merges the pieces and packs the head's output
//                (tensor parallel: into every rank's copy of the O input)
//   GEMV         O projection, this rank's output rows (of all n_embd) -> t
//   norm_pack    ffn_norm
//   GEMV         [gate; up] rows of this rank's FFN slice     (text.c:413-415)
//   silu_pack    silu(gate) * up (src/kernels/scalar/silu.c:12-23), packed
//                (tensor parallel: into every rank's copy of the down input)
//   GEMV         down projection, this rank's output rows -> t
// then norm_pack(output_norm), the LM-head GEMV (this rank's vocabulary rows)
// and argmax_kernel.  A tensor-parallel step makes 4 exchanges per layer plus
// the pick.  The per-layer ones are low-latency pushes (LLExchange): every
// 32-bit word goes to every rank together with the exchange's epoch in one
// 64-bit store, written while the producer runs, and the consumer (the O and
// down GEMVs, norm_pack) polls the words in its own memory -- bounded --
// until all carry the epoch.  The pick uses a flag handshake
// (xchg_handshake) on the (value, index) words.
//
// Numerics: every GEMV is the bit-exact reference kernel (q4k_gemv.cu) or
// (Q8_0) agrees with it to fp32 rounding.  The glue ops use IEEE
// round-to-nearest arithmetic in the reference's operation order where that
// is cheap (rmsnorm scaling, RoPE products, SiLU), but sums over a vector
// (rmsnorm's mean square, attention dot products and softmax sums) are
// parallel reductions, and expf / powf / sinf / cosf are CUDA's, so logits
// agree with the CPU engine to a tolerance, not bit for bit.  Those
// reductions run in the same order on any number of GPUs, so a
// tensor-parallel run picks exactly the one-GPU tokens.
#include <cmath>
#include <cstddef>
#include <cstdlib>
#include <cstring>
#include <new>
#include <utility>
#include <vector>

#include "decoder_internal.h"
#include "eos_common.cuh"
#include "eos_kernels.h"
#include "eosllm_cuda.h"

namespace eos {

constexpr uint32_t kArgmaxBlocks = 64;  // CTAs of the argmax kernel (upper bound)
constexpr uint32_t kPrefillRows = 1024;  // tokens per batched-prefill block


// ---------------------------------------------------------------------------
// Residual + rmsnorm + activation packing
// ---------------------------------------------------------------------------
struct NormPackParams {
  const float* x_in;         // residual stream; nullptr: embedding lookup
  const float* part;         // t added to x_in (nullptr: none)
  const uint16_t* tok_embd;  // F16 [n_vocab][n]      (embedding mode)
  const uint32_t* prompt;    // token of step pos when pos < n_prompt
  const DecState* state;
  float* x_out;     // updated residual stream (may be nullptr)
  const float* w;   // norm weight
  float eps;
  uint32_t n;
  uint8_t* act;     // Q4_K consumers: packed records for k = n
  float* act_f32;   // Q8_0 consumers: the normalised vector
  // tensor parallel (ll.epoch_word != nullptr): t comes as the (epoch, word)
  // pairs every rank's GEMV pushed into ll.in instead of from `part`
  LLExchange ll;
};

constexpr uint32_t kNormMaxChunks = 16;  // float4 chunks per thread: n <= 16384

__device__ __forceinline__ float4 ld4(const float* p, uint32_t c) { return reinterpret_cast<const float4*>(p)[c]; }
__device__ __forceinline__ float4 add4(float4 a, float4 b) {
  return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}

// Grid: n / 256 CTAs of 256 threads; thread t holds the float4 chunks
// t, t + 256, ... of the vector, all loaded in one batch.  Every CTA reduces
// the mean square of the whole vector (the same fixed order in every CTA, so
// all agree bit for bit) and then normalises and packs its own 256 elements
// (CTA b: chunks [64 b, 64 b + 64), held by threads 64 (b % 4) + q at
// iteration b / 4).  Residual element i is x_in[i] + t[i], the reference's
// x[i] += t[i] (text.c:406).
template <uint32_t NCH>  // float4 chunks per thread: n <= 1024 NCH
__global__ void __launch_bounds__(256) norm_pack_kernel(const NormPackParams p) {
  __shared__ float red[8];
  __shared__ __align__(16) float ys[256];
  pdl_trigger();
  pdl_wait();
  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  const uint32_t nch = p.n >> 2, b = blockIdx.x;
  const uint32_t jown = b >> 2;
  const bool owner = (tid >> 6) == (b & 3u);
  float4 v[NCH];
  if (p.x_in == nullptr) {
    const uint32_t pos = p.state->pos;
    const uint32_t tok = pos < p.state->n_prompt ? p.prompt[pos] : p.state->next_token;
    const uint2* emb = reinterpret_cast<const uint2*>(p.tok_embd + (size_t)tok * p.n);
#pragma unroll
    for (uint32_t j = 0; j < NCH; ++j) {
      const uint32_t c = tid + 256u * j;
      if (c < nch) {
        const uint2 h = emb[c];  // F16 -> F32 is exact (src/util/f16.h)
        v[j] = make_float4(f16_bits_to_f32(h.x), f16_bits_to_f32(h.x >> 16), f16_bits_to_f32(h.y),
                           f16_bits_to_f32(h.y >> 16));
      }
    }
  } else {
#pragma unroll
    for (uint32_t j = 0; j < NCH; ++j) {
      const uint32_t c = tid + 256u * j;
      if (c < nch) v[j] = ld4(p.x_in, c);
    }
    if (p.ll.epoch_word != nullptr) {
      // tensor parallel: every chunk's four (epoch, word) pairs, all loads in
      // flight at once, the round reloaded until every pair is there
      const uint32_t epoch = ll_epoch(p.ll, p.ll.in_add);
      float4 t[NCH];
      uint64_t t0 = 0;
      bool ready, ok = true;
      do {
        ready = true;
#pragma unroll
        for (uint32_t j = 0; j < NCH; ++j) {
          const uint32_t c = tid + 256u * j;
          if (c < nch) {
            uint64_t q0, q1, q2, q3;
            ll_load2(p.ll.in + 4u * c, q0, q1);
            ll_load2(p.ll.in + 4u * c + 2u, q2, q3);
            t[j] = make_float4(__uint_as_float((uint32_t)q0), __uint_as_float((uint32_t)q1),
                               __uint_as_float((uint32_t)q2), __uint_as_float((uint32_t)q3));
            if ((uint32_t)(q0 >> 32) != epoch || (uint32_t)(q1 >> 32) != epoch || (uint32_t)(q2 >> 32) != epoch ||
                (uint32_t)(q3 >> 32) != epoch)
              ready = false;
          }
        }
        if (!ready && !ll_keep_waiting(p.ll, t0)) {
          ok = false;
          break;
        }
      } while (!ready);
      if (!__syncthreads_and(ok)) {
        if (tid == 0) report(p.ll.err, EOS_DEVERR_PEER);
        return;  // a peer never arrived: the error bit is set, outputs are invalid
      }
#pragma unroll
      for (uint32_t j = 0; j < NCH; ++j)
        if (tid + 256u * j < nch) v[j] = add4(v[j], t[j]);
    } else if (p.part != nullptr) {
#pragma unroll
      for (uint32_t j = 0; j < NCH; ++j) {
        const uint32_t c = tid + 256u * j;
        if (c < nch) v[j] = add4(v[j], __ldcg(reinterpret_cast<const float4*>(p.part) + c));
      }
    }
  }
  const float4 w4 = owner ? ld4(p.w, (b << 6) + (tid & 63u)) : make_float4(0.f, 0.f, 0.f, 0.f);
  float ss = 0.0f;
#pragma unroll
  for (uint32_t j = 0; j < NCH; ++j) {
    if (tid + 256u * j < nch) {
      ss = __fadd_rn(ss, __fmul_rn(v[j].x, v[j].x));
      ss = __fadd_rn(ss, __fmul_rn(v[j].y, v[j].y));
      ss = __fadd_rn(ss, __fmul_rn(v[j].z, v[j].z));
      ss = __fadd_rn(ss, __fmul_rn(v[j].w, v[j].w));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) tot = __fadd_rn(tot, red[w]);
  // ms /= cols; s = 1 / sqrtf(ms + eps); y = x * s * w  (rmsnorm.c:24-33)
  const float ms = __fdiv_rn(tot, (float)p.n);
  const float sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, p.eps)));
  if (owner) {
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (uint32_t j = 0; j < NCH; ++j)
      if (j == jown) x = v[j];
    const uint32_t c = (b << 6) + (tid & 63u);
    if (p.x_out != nullptr) reinterpret_cast<float4*>(p.x_out)[c] = x;
    const uint32_t o = (tid & 63u) << 2;
    ys[o] = __fmul_rn(__fmul_rn(x.x, sc), w4.x);
    ys[o + 1] = __fmul_rn(__fmul_rn(x.y, sc), w4.y);
    ys[o + 2] = __fmul_rn(__fmul_rn(x.z, sc), w4.z);
    ys[o + 3] = __fmul_rn(__fmul_rn(x.w, sc), w4.w);
  }
  __syncthreads();
  const float y = ys[tid];
  if (p.act != nullptr)
    pack_group_to_record(y, (b << 3) + warp, lane, p.act);
  else
    p.act_f32[(b << 8) + tid] = y;
}

// ---------------------------------------------------------------------------
// Attention over the KV cache, split over positions
// ---------------------------------------------------------------------------
struct AttnParams {
  const float* qkv;  // [hl*hd q | kvl*hd k | kvl*hd v] of this step
  float* kc;         // this layer's caches: [max_ctx][kvl*hd] f32 (text.c:220-226)
  float* vc;
  float* part;       // [hl][max_chunks][hd + 4]: {max, sum, -, -, o[hd]}
  uint32_t* count;   // [hl] chunk arrivals, reset by the merging CTA
  const DecState* state;
  // the O projection's input, all n_head heads (head h at h * hd): Q4_K packed
  // records, or (Q8_0) the attention output itself; tensor parallel, as
  // (epoch, word) pairs into every rank's buffer (ll.out) instead
  uint8_t* act;
  float* act_f32;
  LLExchange ll;
  uint32_t hl, h0, kvl, kv0, n_head, n_kv_head, max_chunks;
  float base, scale;
};

// The warp's 32-group g (lane i holds element i) packed into records: this
// rank's (rec), or, tensor parallel, as (epoch, word) pairs into every
// rank's buffer (word w of the record layout is pair w; four lanes' int8
// values make one word).
__device__ __forceinline__ void pack_group_out(float v, uint32_t g, uint32_t lane, uint8_t* rec, const LLExchange& ll,
                                               uint32_t epoch) {
  if (ll.epoch_word == nullptr) {
    pack_group_to_record(v, g, lane, rec);
    return;
  }
  float scale;
  int32_t sum;
  const uint32_t b = static_cast<uint8_t>(quant_group32(v, scale, sum));
  const unsigned FULL = 0xffffffffu;
  const uint32_t w = b | (__shfl_down_sync(FULL, b, 1) << 8) | (__shfl_down_sync(FULL, b, 2) << 16) |
                     (__shfl_down_sync(FULL, b, 3) << 24);
  if ((lane & 3u) == 0) ll_put(ll, (rec_aq_offset(g) >> 2) + (lane >> 2), w, epoch);
  if (lane == 0) {
    ll_put(ll, rec_st_offset(g) >> 2, __float_as_uint(scale), epoch);
    ll_put(ll, (rec_st_offset(g) >> 2) + 1u, __float_as_uint((float)sum), epoch);
  }
}

// Dynamic shared memory of attn_kernel<E>: the K and V rows of one chunk.
__host__ __device__ constexpr uint32_t attn_smem_bytes(uint32_t hd) { return 2u * kAttnChunk * hd * 4u; }

// Grid (hl, max_chunks), 128 threads.  E = dims per lane (head_dim = 32 E).
// CTA (h, c) covers positions [32 c, 32 c + 32) up to `pos`: it stages the
// cached K and V rows of the chunk into shared memory with one batch of
// 16-byte cp.async copies -- issued before the PDL wait, since rows < pos
// were written by earlier steps -- then computes the scores (one warp per
// position, lane = E dims), the chunk's softmax pieces (max, sum, sum of
// weighted V) and parks them; the last CTA of the head merges the chunks.
template <int E>
__global__ void __launch_bounds__(128) attn_kernel(const AttnParams p) {
  constexpr uint32_t HD = 32u * E;
  extern __shared__ __align__(16) float kv_s[];  // [kAttnChunk][HD] K, then V
  __shared__ float s_score[kAttnChunk];
  __shared__ __align__(16) float s_o[4][HD];
  __shared__ float s_l[4];
  __shared__ float s_out[HD];
  __shared__ float s_wc[kMaxAttnChunks];  // merge: chunk maxima, then weights
  __shared__ float s_lc[kMaxAttnChunks];  // merge: chunk sums
  __shared__ uint32_t s_last;
  pdl_trigger();
  const uint32_t hloc = blockIdx.x, c = blockIdx.y;
  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  // pos was written by the previous step's argmax_kernel, which completed
  // before this step's first kernel started
  const uint32_t pos = p.state->pos;
  const uint32_t p0 = c * kAttnChunk;
  if (p0 > pos) return;  // chunk beyond the context: no work, not counted
  const uint32_t p1 = (p0 + kAttnChunk) < (pos + 1u) ? (p0 + kAttnChunk) : (pos + 1u);
  const uint32_t np = p1 - p0;
  const uint32_t gh = p.h0 + hloc;
  const uint32_t gkv = (gh * p.n_kv_head) / p.n_head;  // GQA map (text.c:367)
  const uint32_t kvi = gkv - p.kv0;
  const uint32_t row = p.kvl * HD;  // floats per cache position
  const uint32_t d0 = lane * E;
  float* ks = kv_s;
  float* vs = kv_s + kAttnChunk * HD;
  {
    const uint32_t ncached = (p1 < pos ? p1 : pos) - p0;  // rows < pos in this chunk
    const uint32_t per_row = HD / 4u;
    const uint64_t pol = l2_policy_evict_first();
    const float* kg = p.kc + (size_t)p0 * row + kvi * HD;
    const float* vg = p.vc + (size_t)p0 * row + kvi * HD;
    for (uint32_t t = tid; t < ncached * per_row; t += 128u) {
      const uint32_t r = t / per_row, q4 = (t - r * per_row) * 4u;
      cp_async16(ks + r * HD + q4, kg + (size_t)r * row + q4, pol);
    }
    cp_async_commit();
    for (uint32_t t = tid; t < ncached * per_row; t += 128u) {
      const uint32_t r = t / per_row, q4 = (t - r * per_row) * 4u;
      cp_async16(vs + r * HD + q4, vg + (size_t)r * row + q4, pol);
    }
    cp_async_commit();
  }
  // the rotation at `pos` does not depend on this step's q and k: computed
  // while the QKV GEMV still runs
  float rsn[E / 2], rcs[E / 2];
#pragma unroll
  for (int e = 0; e < E; e += 2) rope_factors<HD>(d0 + e, pos, p.base, rsn[e / 2], rcs[e / 2]);
  pdl_wait();  // q, k, v of this step come from the QKV GEMV

  float q[E], kn[E], vn[E];
  const float* qp = p.qkv + hloc * HD + d0;
  const float* kp = p.qkv + p.hl * HD + kvi * HD + d0;
  const float* vp = p.qkv + p.hl * HD + p.kvl * HD + kvi * HD + d0;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    q[e] = qp[e];
    kn[e] = kp[e];
    vn[e] = vp[e];
  }
#pragma unroll
  for (int e = 0; e < E; e += 2) {
    rope_apply(q[e], q[e + 1], rsn[e / 2], rcs[e / 2]);
    rope_apply(kn[e], kn[e + 1], rsn[e / 2], rcs[e / 2]);
  }
  const bool has_pos = p1 == pos + 1u;
  // the first local head of each KV group appends this step's K and V
  if (has_pos && warp == 0 && (hloc == 0 || ((gh - 1u) * p.n_kv_head) / p.n_head != gkv)) {
#pragma unroll
    for (int e = 0; e < E; ++e) {
      p.kc[(size_t)pos * row + kvi * HD + d0 + e] = kn[e];
      p.vc[(size_t)pos * row + kvi * HD + d0 + e] = vn[e];
    }
  }

  cp_async_wait<1>();  // this thread's K copies
  __syncthreads();     // everyone's
  for (uint32_t j = warp; j < np; j += 4u) {
    const float* kr = ks + j * HD + d0;
    float acc = 0.0f;
    if (p0 + j == pos) {
#pragma unroll
      for (int e = 0; e < E; ++e) acc = __fmaf_rn(q[e], kn[e], acc);
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) acc = __fmaf_rn(q[e], kr[e], acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) s_score[j] = __fmul_rn(acc, p.scale);
  }
  cp_async_wait<0>();
  __syncthreads();
  // chunk max: every warp reduces the <= 64 scores itself (no serial loop)
  float mx = fmaxf(lane < np ? s_score[lane] : -INFINITY, lane + 32u < np ? s_score[lane + 32u] : -INFINITY);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  // o = sum_t exp(s_t - mx) v_t over this chunk, one warp per position
  float o[E];
#pragma unroll
  for (int e = 0; e < E; ++e) o[e] = 0.0f;
  float l = 0.0f;
  for (uint32_t j = warp; j < np; j += 4u) {
    const float a = expf(s_score[j] - mx);
    const float* vr = vs + j * HD + d0;
    l += a;
    if (p0 + j == pos) {
#pragma unroll
      for (int e = 0; e < E; ++e) o[e] = __fmaf_rn(a, vn[e], o[e]);
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) o[e] = __fmaf_rn(a, vr[e], o[e]);
    }
  }
#pragma unroll
  for (int e = 0; e < E; ++e) s_o[warp][d0 + e] = o[e];
  if (lane == 0) s_l[warp] = l;
  __syncthreads();
  float* out = p.part + ((size_t)hloc * p.max_chunks + c) * (HD + 4u);
  for (uint32_t d = tid; d < HD; d += 128u) out[4 + d] = ((s_o[0][d] + s_o[1][d]) + s_o[2][d]) + s_o[3][d];
  if (tid == 0) {
    out[0] = mx;
    out[1] = ((s_l[0] + s_l[1]) + s_l[2]) + s_l[3];
  }
  __threadfence();
  __syncthreads();
  const uint32_t nvalid = pos / kAttnChunk + 1u;
  if (tid == 0) s_last = atomicAdd(&p.count[hloc], 1u) == nvalid - 1u;
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  // last CTA of the head: merge the chunks (log-sum-exp), normalise.  The
  // chunk maxima and sums load in parallel, the weights are computed once,
  // and each thread's o[d] of up to kMergeBatch chunks load in one batch.
  const float* base = p.part + (size_t)hloc * p.max_chunks * (HD + 4u);
  for (uint32_t cc = tid; cc < nvalid; cc += 128u) {
    s_wc[cc] = __ldcg(base + cc * (HD + 4u));
    s_lc[cc] = __ldcg(base + cc * (HD + 4u) + 1);
  }
  constexpr int NDT = (HD + 127) / 128;  // dims per thread
  float od[NDT][kMergeBatch];
#pragma unroll
  for (int e = 0; e < NDT; ++e) {
    const uint32_t d = tid + 128u * e;
#pragma unroll
    for (uint32_t cc = 0; cc < kMergeBatch; ++cc)
      od[e][cc] = (d < HD && cc < nvalid) ? __ldcg(base + cc * (HD + 4u) + 4u + d) : 0.0f;
  }
  __syncthreads();
  float gmx = -INFINITY;
  for (uint32_t cc = 0; cc < nvalid; ++cc) gmx = fmaxf(gmx, s_wc[cc]);
  __syncthreads();
  for (uint32_t cc = tid; cc < nvalid; cc += 128u) s_wc[cc] = expf(s_wc[cc] - gmx);
  __syncthreads();
  float L = 0.0f;
  for (uint32_t cc = 0; cc < nvalid; ++cc) L += s_lc[cc] * s_wc[cc];
  const float inv = 1.0f / L;
#pragma unroll
  for (int e = 0; e < NDT; ++e) {
    const uint32_t d = tid + 128u * e;
    if (d < HD) {
      float acc = 0.0f;
#pragma unroll
      for (uint32_t cc = 0; cc < kMergeBatch; ++cc)
        if (cc < nvalid) acc = __fmaf_rn(od[e][cc], s_wc[cc], acc);
      for (uint32_t cc = kMergeBatch; cc < nvalid; ++cc)
        acc = __fmaf_rn(__ldcg(base + cc * (HD + 4u) + 4u + d), s_wc[cc], acc);
      s_out[d] = acc * inv;
    }
  }
  if (tid == 0) p.count[hloc] = 0u;
  __syncthreads();
  const uint32_t epoch = p.ll.epoch_word != nullptr ? ll_epoch(p.ll, p.ll.out_add) : 0u;
  if (p.act != nullptr) {
    for (uint32_t g = warp; g < E; g += 4u) pack_group_out(s_out[g * 32u + lane], gh * E + g, lane, p.act, p.ll, epoch);
  } else {
    for (uint32_t d = tid; d < HD; d += 128u) {
      if (p.ll.epoch_word != nullptr)
        ll_put(p.ll, gh * HD + d, __float_as_uint(s_out[d]), epoch);
      else
        p.act_f32[gh * HD + d] = s_out[d];
    }
  }
}

// ---------------------------------------------------------------------------
// silu(gate) * up, packed for the down projection
// ---------------------------------------------------------------------------
struct SiluParams {
  const float* gu;  // [gate | up] of this rank's FFN slice, ffl each
  uint32_t ffl, ff0;
  // the down projection's input, all n_ff units (unit ff0 + i of this rank's
  // i): Q4_K packed records, or (Q8_0) the values; tensor parallel, as
  // (epoch, word) pairs into every rank's buffer (ll.out) instead
  uint8_t* act;
  float* act_f32;
  LLExchange ll;
};

__global__ void __launch_bounds__(256) silu_pack_kernel(const SiluParams p) {
  pdl_trigger();
  pdl_wait();
  const uint32_t i = blockIdx.x * 256u + threadIdx.x;
  if (i >= p.ffl) return;  // warp-uniform: ffl % 32 == 0
  const float g = p.gu[i], u = p.gu[p.ffl + i];
  // x * (1 / (1 + expf(-x))) (silu.c:17), then gate * up (text.c:417)
  const float h = __fmul_rn(__fmul_rn(g, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)))), u);
  const uint32_t gi = p.ff0 + i;
  const uint32_t epoch = p.ll.epoch_word != nullptr ? ll_epoch(p.ll, p.ll.out_add) : 0u;
  if (p.act != nullptr) {
    pack_group_out(h, gi >> 5, threadIdx.x & 31u, p.act, p.ll, epoch);
  } else if (p.ll.epoch_word != nullptr) {
    ll_put(p.ll, gi, __float_as_uint(h), epoch);
  } else {
    p.act_f32[gi] = h;
  }
}

// ---------------------------------------------------------------------------
// Greedy pick: the first index of the largest logit (greedy.c:66-69: strict >
// from logits[0], so a NaN logits[0] keeps index 0 and other NaNs never win)
// ---------------------------------------------------------------------------
struct ArgmaxParams {
  const float* logits;   // this rank's vocabulary slice
  uint32_t n;
  float* part_v;     // [gridDim.x]
  uint32_t* part_i;
  DecState* state;
  uint32_t* out_tokens;  // [max_ctx]: pick of step pos
  // tensor parallel: every rank's slice result, pushed into every rank's
  // receive words and merged in rank order
  uint32_t world, rank, v0;  // v0: global index of logits[0]
  XRecv* recv[kMaxParts];    // rank q's receive words (IPC-mapped; own local)
  XRecv* own;
  XchgSync xs;               // the pick's handshake (flags kXArgmax)
};

__device__ __forceinline__ bool arg_better(float av, uint32_t ai, float bv, uint32_t bi) {
  if (av != av) return false;
  if (bv != bv) return true;
  return av > bv || (av == bv && ai < bi);
}

__device__ __forceinline__ void arg_reduce_block(float& v, uint32_t& idx, float* sv, uint32_t* si) {
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (arg_better(ov, oi, v, idx)) {
      v = ov;
      idx = oi;
    }
  }
  if (lane == 0) {
    sv[warp] = v;
    si[warp] = idx;
  }
  __syncthreads();
  v = sv[0];
  idx = si[0];
  for (uint32_t w = 1; w < blockDim.x / 32u; ++w)
    if (arg_better(sv[w], si[w], v, idx)) {
      v = sv[w];
      idx = si[w];
    }
}

__global__ void __launch_bounds__(256) argmax_kernel(const ArgmaxParams p) {
  __shared__ float sv[8];
  __shared__ uint32_t si[8];
  __shared__ uint32_t s_last;
  pdl_trigger();
  pdl_wait();
  float v = __int_as_float(0x7fc00000);  // "nothing yet"
  uint32_t idx = 0xffffffffu;
  for (uint32_t i = blockIdx.x * 256u + threadIdx.x; i < p.n; i += gridDim.x * 256u) {
    const float x = p.logits[i];
    if (arg_better(x, i, v, idx)) {
      v = x;
      idx = i;
    }
  }
  arg_reduce_block(v, idx, sv, si);
  if (threadIdx.x == 0) {
    p.part_v[blockIdx.x] = v;
    p.part_i[blockIdx.x] = idx;
    __threadfence();
    s_last = atomicAdd(&p.state->arg_count, 1u) == gridDim.x - 1u;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  __syncthreads();
  v = __int_as_float(0x7fc00000);
  idx = 0xffffffffu;
  for (uint32_t b = threadIdx.x; b < gridDim.x; b += 256u) {
    const float bv = __ldcg(p.part_v + b);
    const uint32_t bi = __ldcg(p.part_i + b);
    if (arg_better(bv, bi, v, idx)) {
      v = bv;
      idx = bi;
    }
  }
  __syncthreads();
  arg_reduce_block(v, idx, sv, si);
  const float first = __ldcg(p.logits);
  uint32_t first_nan = (p.rank == 0 && first != first) ? 1u : 0u;
  uint32_t gidx = idx == 0xffffffffu ? idx : p.v0 + idx;
  if (p.world > 1) {
    if (threadIdx.x == 0) {  // push this slice's result into every rank's words
      for (uint32_t q = 0; q < p.world; ++q) {
        p.recv[q]->arg_v[p.rank] = v;
        p.recv[q]->arg_i[p.rank] = gidx;
        if (p.rank == 0) p.recv[q]->first_nan = first_nan;
      }
    }
    // this CTA published the pushes itself (stores, then the handshake's
    // fence and release), so it waits for its own flag too
    if (!xchg_handshake(p.xs, true, false)) return;
    if (threadIdx.x == 0) {
      v = __int_as_float(0x7fc00000);
      gidx = 0xffffffffu;
      const volatile XRecv* x = p.own;
      for (uint32_t q = 0; q < p.world; ++q) {  // rank order = vocabulary order
        (void)ld_acquire_sys(&p.own->flag[kXArgmax][q]);
        const float qv = x->arg_v[q];
        const uint32_t qi = x->arg_i[q];
        if (arg_better(qv, qi, v, gidx)) {
          v = qv;
          gidx = qi;
        }
      }
      first_nan = x->first_nan;
    }
  }
  if (threadIdx.x == 0) {
    const uint32_t tok = (first_nan || gidx == 0xffffffffu) ? 0u : gidx;
    const uint32_t pos = p.state->pos;
    p.out_tokens[pos] = tok;
    p.state->next_token = tok;
    p.state->arg_count = 0u;
    p.state->pos = pos + 1u;
    p.state->epoch = p.state->epoch + 1u;
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace {

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t lc = {};
  lc.gridDim = grid;
  lc.blockDim = block;
  lc.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  return cudaLaunchKernelEx(&lc, kernel, std::forward<Args>(args)...);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_smem(void (*kernel)(KArgs...), dim3 grid, dim3 block, uint32_t smem, cudaStream_t st,
                            Args&&... args) {
  cudaLaunchConfig_t lc = {};
  lc.gridDim = grid;
  lc.blockDim = block;
  lc.dynamicSmemBytes = smem;
  lc.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  return cudaLaunchKernelEx(&lc, kernel, std::forward<Args>(args)...);
}

size_t wbytes(int dt, uint64_t n, uint64_t k) {
  return dt == EOS_DT_Q4_K ? (size_t)(n * (k / Q4K_ELEMS) * Q4K_BYTES) : (size_t)(n * (k / Q80_ELEMS) * Q80_BYTES);
}
uint32_t blk_elems(int dt) { return dt == EOS_DT_Q4_K ? Q4K_ELEMS : Q80_ELEMS; }

}  // namespace

struct TextDecoder {
  eosi_cuda_llama_t m{};
  int device = 0, rank = 0, world = 1;
  uint32_t hd = 0, hl = 0, h0 = 0, kvl = 0, kv0 = 0, ffl = 0, ff0 = 0, vl = 0, v0 = 0, el = 0, e0 = 0;
  uint32_t max_chunks = 0;
  int num_sms = 0, max_smem = 0;
  cudaStream_t st = nullptr;
  std::vector<void*> allocs;
  std::vector<DecLayer> layers;
  uint16_t* tok_embd = nullptr;
  float* out_norm = nullptr;
  uint8_t* wout = nullptr;
  // activations (local)
  float *x0 = nullptr, *x1 = nullptr, *qkv = nullptr, *gu = nullptr;
  uint8_t* act_e = nullptr;  // normalised residual, Q4_K records
  float* actf_e = nullptr;   // normalised residual for Q8_0 consumers
  float *kc = nullptr, *vc = nullptr;
  float* attn_part = nullptr;
  uint32_t* attn_count = nullptr;
  float* arg_v = nullptr;
  uint32_t* arg_i = nullptr;
  DecState* state = nullptr;
  uint32_t* prompt = nullptr;
  uint32_t* out_tokens = nullptr;
  uint32_t* gemv_err = nullptr;
  uint32_t arg_blocks = 0;
  // Exchange buffer, one per rank; the other ranks write (push) into it
  // through CUDA IPC mappings.  It holds what every rank reads whole (one
  // GPU: plain values; tensor parallel: each 32-bit word as an (epoch, word)
  // pair, see LLExchange, so those regions are sized for twice the bytes):
  //   o_full, d_full    O / down projection outputs, all n_embd rows
  //   logits            this rank's vocabulary slice (read back by the host)
  //   XRecv             flags and the greedy-pick words
  //   act_o / actf_o    O projection input, all heads (Q4_K records / Q8_0 f32)
  //   act_d / actf_d    down projection input, all n_ff units
  // and, tensor parallel with Q4_K, the batched prefill's counterparts for
  // xpf_rows rows: output rows [xpf_rows][n_embd] of O and down, and the
  // GEMM operands of the O and down inputs.
  uint8_t* xbuf = nullptr;
  size_t xoff_o = 0, xoff_d = 0, xoff_lg = 0, xoff_fl = 0, xoff_ao = 0, xoff_ad = 0, xbytes = 0;
  size_t xstep_bytes = 0;  // the step's regions: [0, xstep_bytes)
  size_t xoff_pfo = 0, xoff_pfd = 0, xoff_pfa = 0, xoff_pfs = 0;
  uint32_t xpf_rows = 0, pf_epoch = 0;
  float *o_full = nullptr, *d_full = nullptr, *logits = nullptr;
  uint8_t *act_o = nullptr, *act_d = nullptr;
  float *actf_o = nullptr, *actf_d = nullptr;
  uint8_t* xpeer[kMaxParts] = {};  // every rank's exchange buffer (own included)
  bool peer_opened[kMaxParts] = {};
  // where this rank's pushes land in the other ranks' exchange buffers
  cudaGraphExec_t graph = nullptr;
  uint32_t step_kernels = 0;  // kernel nodes of the step graph
  // persistent step (decoder_persistent.cu): one cooperative kernel per
  // token when the geometry allows (persistent_ok) and the mode asks for it
  int step_mode_req = EOSI_CUDA_STEP_AUTO;
  bool persistent_ok = false, persistent = false;
  PLayer* players = nullptr;                 // device copy of the layer table
  uint64_t *qkv_x = nullptr, *gu_x = nullptr;  // this rank's q/k/v and gate/up rows as pairs
  float* parg_v = nullptr;                   // per-CTA greedy candidates
  uint32_t* parg_i = nullptr;
  uint32_t host_pos = 0;
  bool step_mode = false;  // prompt[] holds every fed token (n_prompt = max_ctx)
  // batched prefill (prefill_text.cu): scratch for pf_rows tokens, allocated
  // at first use; generate() prefills in batch when at least prefill_min
  // prompt tokens precede the last one (0: never)
  uint32_t pf_rows = 0;
  float *pf_x = nullptr, *pf_qkv = nullptr, *pf_gu = nullptr;
  void *pf_act = nullptr, *pf_w = nullptr;  // GEMM operand buffers (activations, prepared weights)
  // every layer's four matrices in the GEMM layout, prepared once at the
  // first prefill when they fit in half of the free device memory (a
  // load-time repack; empty: each matrix is prepared into pf_w before use)
  std::vector<void*> pf_wres;
  bool pf_resident = true;  // allow pf_wres (eosi_cuda_text_set_prefill_resident)
  uint32_t prefill_min = 16;

  template <typename T>
  cudaError_t alloc(T** p, size_t bytes) {
    void* v = nullptr;
    cudaError_t e = cudaMalloc(&v, bytes < 16 ? 16 : bytes);
    if (e != cudaSuccess) return e;
    allocs.push_back(v);
    *p = static_cast<T*>(v);
    return cudaMemsetAsync(v, 0, bytes < 16 ? 16 : bytes, st);
  }

  ~TextDecoder() {
    if (graph) cudaGraphExecDestroy(graph);
    if (st) cudaStreamSynchronize(st);
    for (int q = 0; q < world && q < (int)kMaxParts; ++q)
      if (peer_opened[q]) cudaIpcCloseMemHandle(xpeer[q]);
    for (void* p : allocs) cudaFree(p);
    if (st) cudaStreamDestroy(st);
  }

  cudaMemcpyKind kind() const {
    return m.weights_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  }

  // rows [r0, r0 + rows) of an [n][k] quantized matrix into dst
  cudaError_t copy_rows(uint8_t* dst, const void* src, int dt, uint64_t k, uint64_t r0, uint64_t rows) {
    const size_t rb = wbytes(dt, 1, k);
    return cudaMemcpyAsync(dst, static_cast<const uint8_t*>(src) + r0 * rb, rows * rb, kind(), st);
  }

  int open(const eosi_cuda_llama_t* desc, int dev, int rk, int ws);
  int attach(const uint8_t* handles);
  int attach_buffers(uint8_t* const* bufs);  // every rank's exchange buffer, already mapped
  // the batched path serves Q4_K linears, on one GPU or tensor parallel
  bool prefill_ok() const { return m.wdtype == EOS_DT_Q4_K && m.n_layer > 0 && (world == 1 || xpf_rows > 0); }
  cudaError_t prefill(uint32_t n);  // tokens at prompt[host_pos, host_pos + n)
  XRecv* xrecv(int q) const { return reinterpret_cast<XRecv*>(xpeer[q] + xoff_fl); }
  cudaError_t record_step(cudaStream_t s);
  cudaError_t record_step_persistent(cudaStream_t s);
  int capture();
  int set_step_mode(int mode);
};

// The slice of the model rank rk of ws owns: heads [h0, h0 + hl) (and their
// KV heads) for q/k/v rows and attention, FFN units [ff0, ff0 + ffl) for
// gate/up rows, output rows [e0, e0 + el) of the O and down projections,
// vocabulary rows [v0, v0 + vl) of the LM head.  Every matrix is split by
// output rows, so each output element is computed whole on one rank.  Host
// only; returns an eos_status_t.
struct Geometry {
  uint32_t hd, hl, h0, kvl, kv0, ffl, ff0, vl, v0, el, e0;
};
int model_geometry(const eosi_cuda_llama_t& m, int rk, int ws, Geometry& g) {
  const int wdt = m.wdtype, odt = m.out_dtype;
  if (m.n_head == 0 || m.n_kv_head == 0 || m.n_embd % m.n_head) {
    set_error_message("cuda text: n_embd must be a multiple of n_head");
    return EOS_E_INVALID_ARG;
  }
  g.hd = m.n_embd / m.n_head;
  if (g.hd != 64 && g.hd != 128 && g.hd != 256) {
    set_error_message("cuda text: head_dim must be 64, 128 or 256");
    return EOS_E_UNSUPPORTED;
  }
  if ((wdt != EOS_DT_Q4_K && wdt != EOS_DT_Q8_0) || (odt != EOS_DT_Q4_K && odt != EOS_DT_Q8_0)) {
    set_error_message("cuda text: linears must be Q4_K or Q8_0");
    return EOS_E_UNSUPPORTED;
  }
  if (m.n_embd % 256 || m.n_embd > 256u * 4u * kNormMaxChunks || m.n_ff % blk_elems(wdt) ||
      m.n_embd % blk_elems(odt)) {
    set_error_message("cuda text: n_embd must be a multiple of 256 (at most 16384), n_ff of the block size");
    return EOS_E_UNSUPPORTED;
  }
  if (m.max_ctx > kAttnChunk * kMaxAttnChunks) {
    set_error_message("cuda text: max_ctx above 16384");
    return EOS_E_UNSUPPORTED;
  }
  if (ws < 1 || ws > (int)kMaxParts || rk < 0 || rk >= ws || m.n_head % ws || m.n_kv_head % ws) {
    set_error_message("cuda text: world size must divide the head counts (at most 8 ranks)");
    return EOS_E_INVALID_ARG;
  }
  g.hl = m.n_head / ws;
  g.h0 = g.hl * rk;
  g.kvl = m.n_kv_head / ws;
  g.kv0 = g.kvl * rk;
  g.el = m.n_embd / ws;  // n_head % ws == 0, so n_embd % ws == 0
  g.e0 = g.el * rk;
  // FFN units in whole 32-element groups (the activation packing's unit)
  const uint32_t units = m.n_ff / 32u;
  g.ff0 = (uint32_t)(((uint64_t)units * rk) / ws) * 32u;
  g.ffl = (uint32_t)(((uint64_t)units * (rk + 1)) / ws) * 32u - g.ff0;
  g.v0 = (uint32_t)(((uint64_t)m.n_vocab * rk) / ws);
  g.vl = (uint32_t)(((uint64_t)m.n_vocab * (rk + 1)) / ws) - g.v0;
  if (g.ffl == 0 || g.vl == 0) {
    set_error_message("cuda text: too many ranks for the FFN or the vocabulary");
    return EOS_E_INVALID_ARG;
  }
  return EOS_OK;
}

int TextDecoder::open(const eosi_cuda_llama_t* desc, int dev, int rk, int ws) {
  m = *desc;
  device = dev;
  rank = rk;
  world = ws;
  const int wdt = m.wdtype, odt = m.out_dtype;
  Geometry g{};
  const int gs = model_geometry(m, rk, ws, g);
  if (gs != EOS_OK) return gs;
  hd = g.hd;
  hl = g.hl;
  h0 = g.h0;
  kvl = g.kvl;
  kv0 = g.kv0;
  ffl = g.ffl;
  ff0 = g.ff0;
  vl = g.vl;
  v0 = g.v0;
  el = g.el;
  e0 = g.e0;
  max_chunks = (m.max_ctx + kAttnChunk - 1) / kAttnChunk;

  if (cudaSetDevice(dev) != cudaSuccess) return EOS_E_INTERNAL;
  cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) return EOS_E_INTERNAL;

  const uint32_t E = m.n_embd, F = m.n_ff;
  cudaError_t e = cudaSuccess;
  auto chk = [&](cudaError_t r) {
    if (e == cudaSuccess) e = r;
  };
  // ---- resident weights (this rank's rows) ----
  layers.resize(m.n_layer);
  for (uint32_t L = 0; L < m.n_layer; ++L) {
    DecLayer& d = layers[L];
    const size_t rb = wbytes(wdt, 1, E);
    chk(alloc(&d.wqkv, rb * (hl * hd + 2 * kvl * hd)));
    chk(copy_rows(d.wqkv, m.wq[L], wdt, E, h0 * hd, hl * hd));
    chk(copy_rows(d.wqkv + rb * hl * hd, m.wk[L], wdt, E, kv0 * hd, kvl * hd));
    chk(copy_rows(d.wqkv + rb * (hl * hd + kvl * hd), m.wv[L], wdt, E, kv0 * hd, kvl * hd));
    chk(alloc(&d.wo, wbytes(wdt, el, E)));
    chk(copy_rows(d.wo, m.wo[L], wdt, E, e0, el));
    chk(alloc(&d.wgu, 2 * rb * ffl));
    chk(copy_rows(d.wgu, m.wg[L], wdt, E, ff0, ffl));
    chk(copy_rows(d.wgu + rb * ffl, m.wu[L], wdt, E, ff0, ffl));
    chk(alloc(&d.wd, wbytes(wdt, el, F)));
    chk(copy_rows(d.wd, m.wd[L], wdt, F, e0, el));
    chk(alloc(&d.attn_norm, 4ull * E));
    chk(cudaMemcpyAsync(d.attn_norm, m.attn_norm[L], 4ull * E, kind(), st));
    chk(alloc(&d.ffn_norm, 4ull * E));
    chk(cudaMemcpyAsync(d.ffn_norm, m.ffn_norm[L], 4ull * E, kind(), st));
  }
  chk(alloc(&tok_embd, 2ull * m.n_vocab * E));
  chk(cudaMemcpyAsync(tok_embd, m.tok_embd, 2ull * m.n_vocab * E, kind(), st));
  chk(alloc(&out_norm, 4ull * E));
  chk(cudaMemcpyAsync(out_norm, m.output_norm, 4ull * E, kind(), st));
  chk(alloc(&wout, wbytes(odt, vl, E)));
  chk(copy_rows(wout, m.output_w, odt, E, v0, vl));
  // ---- activations and caches ----
  chk(alloc(&x0, 4ull * E));
  chk(alloc(&x1, 4ull * E));
  chk(alloc(&qkv, 4ull * (hl * hd + 2 * kvl * hd)));
  {
    const uint32_t vmax = (m.n_vocab + ws - 1) / ws + 1;
    auto up = [](size_t x) { return (x + 4095) & ~(size_t)4095; };  // operand bases: 1024-byte aligned TMA
    const bool q4 = wdt == EOS_DT_Q4_K;
    xoff_o = 0;
    xoff_d = up(8ull * E);
    xoff_lg = xoff_d + up(8ull * E);
    xoff_fl = xoff_lg + up(4ull * vmax);
    xoff_ao = xoff_fl + up(sizeof(XRecv));
    xoff_ad = xoff_ao + up(2ull * (q4 ? (size_t)(E / 256) * kActRec : 4ull * E));
    xbytes = xoff_ad + up(2ull * (q4 ? (size_t)(F / 256) * kActRec : 4ull * F));
    xstep_bytes = xbytes;
    if (ws > 1 && q4) {  // batched-prefill exchange (allocated with the handles)
      xpf_rows = m.max_ctx < kPrefillRows ? m.max_ctx : kPrefillRows;
      xoff_pfo = xbytes;
      xoff_pfd = xoff_pfo + up(4ull * xpf_rows * E);
      xoff_pfa = xoff_pfd + up(4ull * xpf_rows * E);
      xoff_pfs = xoff_pfa + up(prefill_operand_bytes(xpf_rows, E));
      xbytes = xoff_pfs + up(prefill_operand_bytes(xpf_rows, F));
    }
    chk(alloc(&xbuf, xbytes));
    o_full = reinterpret_cast<float*>(xbuf + xoff_o);
    d_full = reinterpret_cast<float*>(xbuf + xoff_d);
    logits = reinterpret_cast<float*>(xbuf + xoff_lg);
    if (q4) {
      act_o = xbuf + xoff_ao;
      act_d = xbuf + xoff_ad;
    } else {
      actf_o = reinterpret_cast<float*>(xbuf + xoff_ao);
      actf_d = reinterpret_cast<float*>(xbuf + xoff_ad);
    }
    xpeer[rk] = xbuf;
  }
  chk(alloc(&gu, 8ull * ffl));
  // the normalised residual feeds the block linears (wdtype) and the head (out_dtype)
  if (wdt == EOS_DT_Q4_K || odt == EOS_DT_Q4_K) chk(alloc(&act_e, (size_t)(E / 256) * kActRec));
  if (wdt == EOS_DT_Q8_0 || odt == EOS_DT_Q8_0) chk(alloc(&actf_e, 4ull * E));
  const size_t kv_bytes = 4ull * m.n_layer * m.max_ctx * kvl * hd;
  chk(alloc(&kc, kv_bytes));
  chk(alloc(&vc, kv_bytes));
  const uint32_t chunks32 = (m.max_ctx + 31u) / 32u;
  chk(alloc(&attn_part, 4ull * hl * (chunks32 > max_chunks ? chunks32 : max_chunks) * (hd + 4)));
  chk(alloc(&attn_count, 4ull * hl));
  arg_blocks = (vl + 2047u) / 2048u;
  if (arg_blocks > kArgmaxBlocks) arg_blocks = kArgmaxBlocks;
  if (arg_blocks < 1) arg_blocks = 1;
  chk(alloc(&arg_v, 4ull * kArgmaxBlocks));
  chk(alloc(&arg_i, 4ull * kArgmaxBlocks));
  chk(alloc(&state, sizeof(DecState)));
  {
    const uint32_t limit_us = (uint32_t)(EOS_WAIT_LIMIT_NS / 1000ull);
    chk(cudaMemcpyAsync(&state->wait_limit_us, &limit_us, 4, cudaMemcpyHostToDevice, st));
  }
  chk(alloc(&prompt, 4ull * m.max_ctx));
  chk(alloc(&out_tokens, 4ull * m.max_ctx));
  chk(alloc(&gemv_err, 16));
  if (e == cudaSuccess && wdt == EOS_DT_Q4_K && odt == EOS_DT_Q4_K &&
      persistent_step_supported(E, F, hd, max_chunks, m.n_layer, max_smem)) {
    std::vector<PLayer> tab(m.n_layer);
    for (uint32_t L = 0; L < m.n_layer; ++L)
      tab[L] = PLayer{{layers[L].wqkv, layers[L].wo, layers[L].wgu, layers[L].wd}, layers[L].attn_norm,
                      layers[L].ffn_norm};
    chk(alloc(&players, sizeof(PLayer) * (m.n_layer ? m.n_layer : 1u)));
    if (m.n_layer) chk(cudaMemcpyAsync(players, tab.data(), sizeof(PLayer) * m.n_layer, cudaMemcpyHostToDevice, st));
    chk(alloc(&qkv_x, 8ull * (hl * hd + 2 * kvl * hd)));
    chk(alloc(&gu_x, 16ull * ffl));
    chk(alloc(&parg_v, 4ull * num_sms));
    chk(alloc(&parg_i, 4ull * num_sms));
    persistent_ok = e == cudaSuccess;
    // the table must outlive the copy
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  }
  persistent = persistent_ok && step_mode_req == EOSI_CUDA_STEP_PERSISTENT;
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    set_error_message(cudaGetErrorString(e));
    return e == cudaErrorMemoryAllocation ? EOS_E_OUT_OF_MEMORY : EOS_E_INTERNAL;
  }
  // tensor parallel: the step graph reads the other ranks' exchange buffers,
  // so it is built by attach() once their IPC handles are known
  return ws == 1 ? capture() : EOS_OK;
}

int TextDecoder::attach(const uint8_t* handles) {
  if (world == 1 || graph != nullptr) return graph != nullptr ? EOS_OK : capture();
  if (cudaSetDevice(device) != cudaSuccess) return EOS_E_INTERNAL;
  uint8_t* bufs[kMaxParts] = {};
  for (int q = 0; q < world; ++q) {
    if (q == rank) {
      bufs[q] = xbuf;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, handles + (size_t)q * sizeof(cudaIpcMemHandle_t), sizeof(h));
    void* ptr = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      set_error_message(cudaGetErrorString(e));
      return EOS_E_INTERNAL;
    }
    bufs[q] = static_cast<uint8_t*>(ptr);
    peer_opened[q] = true;
  }
  return attach_buffers(bufs);
}

int TextDecoder::attach_buffers(uint8_t* const* bufs) {
  if (world == 1 || graph != nullptr) return graph != nullptr ? EOS_OK : capture();
  for (int q = 0; q < world; ++q) xpeer[q] = bufs[q];
  return capture();
}

cudaError_t TextDecoder::record_step(cudaStream_t s) {
  if (persistent) return record_step_persistent(s);
  const uint32_t E = m.n_embd, F = m.n_ff;
  const int wdt = m.wdtype, odt = m.out_dtype;
  const uint32_t nqkv = hl * hd + 2 * kvl * hd;
  const uint32_t xps = 4u * m.n_layer + 1u;  // exchanges per step
  cudaError_t e = cudaSuccess;
  int status = EOS_OK;
  // flag handshake of the step's exchange number xk, of kind `type` (the
  // greedy pick's)
  auto xsync = [&](uint32_t type, uint32_t xk) {
    XchgSync x{};
    x.world = (uint32_t)world;
    x.rank = (uint32_t)rank;
    for (int q = 0; q < world; ++q) x.pub[q] = &xrecv(q)->flag[type][rank];
    x.wait = &xrecv(rank)->flag[type][0];
    x.epoch_word = &state->epoch;
    x.mul = xps;
    x.add = xk + 1u;
    x.limit_us = &state->wait_limit_us;
    x.err = &state->err;
    return x;
  };
  // Low-latency exchange of a kernel (tensor parallel only; one GPU: plain
  // buffers): it reads this rank's pairs at xbuf + in_off carrying the
  // epoch of exchange in_xk, and writes pairs of exchange out_xk into every
  // rank's buffer at out_off, word 0 at out_word0 (no_off: none).
  constexpr size_t no_off = ~(size_t)0;
  auto llx = [&](size_t in_off, uint32_t in_xk, size_t out_off, uint32_t out_xk, uint32_t out_word0) {
    LLExchange x{};
    if (world == 1) return x;
    x.epoch_word = &state->epoch;
    x.mul = xps;
    x.in_add = in_xk + 1u;
    x.out_add = out_xk + 1u;
    x.in = in_off == no_off ? nullptr : reinterpret_cast<const uint64_t*>(xbuf + in_off);
    if (out_off != no_off)
      for (int q = 0; q < world; ++q) x.out[x.n_out++] = reinterpret_cast<uint64_t*>(xpeer[q] + out_off) + out_word0;
    x.limit_us = &state->wait_limit_us;
    x.err = &state->err;
    return x;
  };
  auto gemv = [&](int dt, const uint8_t* w, const uint8_t* act, const float* actf, float* c, uint32_t n,
                  uint32_t k, const LLExchange* ll = nullptr) -> cudaError_t {
    if (n == 0) return cudaSuccess;
    if (dt == EOS_DT_Q4_K)
      return launch_q4k_gemv(w, act, nullptr, c, n, k, gemv_err, num_sms, max_smem, true, s, &status, nullptr, 0,
                             ll);
    return launch_q80_gemv(w, actf, c, n, k, gemv_err, num_sms, max_smem, s, &status, nullptr, 0, ll);
  };
  // x_out = x_in + part (part: d_full / o_full, tensor parallel: the pairs
  // every rank pushed into the same region), then rmsnorm and the packing
  // for a consumer of dtype dt_a
  auto norm_pack = [&](const float* x_in, const float* part, float* x_out, const float* w, int dt_a, size_t part_off,
                       uint32_t xk) -> cudaError_t {
    NormPackParams p{};
    p.x_in = x_in;
    p.part = part;
    if (part != nullptr) p.ll = llx(part_off, xk, no_off, 0, 0);
    p.tok_embd = tok_embd;
    p.prompt = prompt;
    p.state = state;
    p.x_out = x_out;
    p.w = w;
    p.eps = m.rms_eps;
    p.n = E;
    p.act = dt_a == EOS_DT_Q4_K ? act_e : nullptr;
    p.act_f32 = dt_a == EOS_DT_Q8_0 ? actf_e : nullptr;
    // chunk registers for the model width only (the sums run in the same order)
    return E <= 4096u ? launch_pdl(norm_pack_kernel<4>, dim3(E / 256u), dim3(256), s, p)
                      : launch_pdl(norm_pack_kernel<kNormMaxChunks>, dim3(E / 256u), dim3(256), s, p);
  };
  for (uint32_t L = 0; L < m.n_layer && e == cudaSuccess; ++L) {
    const DecLayer& d = layers[L];
    // x1 = (L == 0 ? embedding : x0 + down output); act_e = pack(rmsnorm(x1))
    e = norm_pack(L == 0 ? nullptr : x0, L == 0 ? nullptr : d_full, x1, d.attn_norm, wdt, xoff_d,
                  L == 0 ? 0u : 4u * L - 1u);
    if (e == cudaSuccess) e = gemv(wdt, d.wqkv, act_e, actf_e, qkv, nqkv, E);
    if (e == cudaSuccess) {
      AttnParams a{};
      a.qkv = qkv;
      a.kc = kc + (size_t)L * m.max_ctx * kvl * hd;
      a.vc = vc + (size_t)L * m.max_ctx * kvl * hd;
      a.part = attn_part;
      a.count = attn_count;
      a.state = state;
      a.act = act_o;
      a.act_f32 = actf_o;
      a.ll = llx(no_off, 0, xoff_ao, 4u * L, 0);  // exchange 4 L: the attention output
      a.hl = hl;
      a.h0 = h0;
      a.kvl = kvl;
      a.kv0 = kv0;
      a.n_head = m.n_head;
      a.n_kv_head = m.n_kv_head;
      a.max_chunks = max_chunks;
      a.base = m.rope_base;
      a.scale = 1.0f / sqrtf((float)hd);  // text.c:365
      const dim3 grid(hl, max_chunks);
      const uint32_t sm = attn_smem_bytes(hd);
      if (hd == 64) e = launch_pdl_smem(attn_kernel<2>, grid, dim3(128), sm, s, a);
      else if (hd == 128) e = launch_pdl_smem(attn_kernel<4>, grid, dim3(128), sm, s, a);
      else e = launch_pdl_smem(attn_kernel<8>, grid, dim3(128), sm, s, a);
    }
    if (e == cudaSuccess) {  // this rank's O rows of all heads' attention output (exchange 4 L + 1)
      const LLExchange ll = llx(xoff_ao, 4u * L, xoff_o, 4u * L + 1u, e0);
      e = gemv(wdt, d.wo, act_o, actf_o, o_full + e0, el, E, &ll);
    }
    // x0 = x1 + O output; act_e = pack(rmsnorm(x0))
    if (e == cudaSuccess) e = norm_pack(x1, o_full, x0, d.ffn_norm, wdt, xoff_o, 4u * L + 1u);
    if (e == cudaSuccess) e = gemv(wdt, d.wgu, act_e, actf_e, gu, 2 * ffl, E);
    if (e == cudaSuccess) {
      SiluParams sp{};
      sp.gu = gu;
      sp.ffl = ffl;
      sp.ff0 = ff0;
      sp.act = act_d;
      sp.act_f32 = actf_d;
      sp.ll = llx(no_off, 0, xoff_ad, 4u * L + 2u, 0);  // exchange 4 L + 2: the SiLU output
      e = launch_pdl(silu_pack_kernel, dim3((ffl + 255u) / 256u), dim3(256), s, sp);
    }
    if (e == cudaSuccess) {  // this rank's down rows over all FFN units (exchange 4 L + 3)
      const LLExchange ll = llx(xoff_ad, 4u * L + 2u, xoff_d, 4u * L + 3u, e0);
      e = gemv(wdt, d.wd, act_d, actf_d, d_full + e0, el, F, &ll);
    }
  }
  // final norm + LM head + greedy pick (text.c:425-432, greedy.c:66-69)
  if (e == cudaSuccess)
    e = norm_pack(m.n_layer ? x0 : nullptr, m.n_layer ? d_full : nullptr, x1, out_norm, odt, xoff_d,
                  m.n_layer ? 4u * m.n_layer - 1u : 0u);
  if (e == cudaSuccess) e = gemv(odt, wout, act_e, actf_e, logits, vl, E);
  if (e == cudaSuccess) {
    ArgmaxParams a{};
    a.logits = logits;
    a.n = vl;
    a.part_v = arg_v;
    a.part_i = arg_i;
    a.state = state;
    a.out_tokens = out_tokens;
    a.world = (uint32_t)world;
    a.rank = (uint32_t)rank;
    a.v0 = v0;
    a.own = xrecv(rank);
    for (int q = 0; q < world; ++q) a.recv[q] = xrecv(q);
    a.xs = xsync(kXArgmax, 4u * m.n_layer);
    e = launch_pdl(argmax_kernel, dim3(arg_blocks), dim3(256), s, a);
  }
  if (e == cudaSuccess && status != EOS_OK) e = cudaErrorNotSupported;
  return e;
}

// The step as one persistent kernel: every vector that crosses CTAs or ranks
// as (epoch, word) pairs, 6 exchanges per layer plus the pick's handshake.
cudaError_t TextDecoder::record_step_persistent(cudaStream_t s) {
  PStepParams p{};
  p.layers = players;
  p.wout = wout;
  p.out_norm = out_norm;
  p.tok_embd = tok_embd;
  p.prompt = prompt;
  p.state = state;
  p.out_tokens = out_tokens;
  p.kc = kc;
  p.vc = vc;
  p.attn_part = attn_part;
  p.attn_count = attn_count;
  p.logits = logits;
  p.arg_v = parg_v;
  p.arg_i = parg_i;
  p.qkv_x = qkv_x;
  p.gu_x = gu_x;
  p.ao_in = reinterpret_cast<const uint64_t*>(xbuf + xoff_ao);
  p.o_in = reinterpret_cast<const uint64_t*>(xbuf + xoff_o);
  p.ad_in = reinterpret_cast<const uint64_t*>(xbuf + xoff_ad);
  p.d_in = reinterpret_cast<const uint64_t*>(xbuf + xoff_d);
  for (int q = 0; q < world; ++q) {
    p.ao_out[q] = reinterpret_cast<uint64_t*>(xpeer[q] + xoff_ao);
    p.o_out[q] = reinterpret_cast<uint64_t*>(xpeer[q] + xoff_o);
    p.ad_out[q] = reinterpret_cast<uint64_t*>(xpeer[q] + xoff_ad);
    p.d_out[q] = reinterpret_cast<uint64_t*>(xpeer[q] + xoff_d);
    p.recv[q] = xrecv(q);
  }
  p.own = xrecv(rank);
  const uint32_t xps = 6u * m.n_layer + 1u;  // exchanges per step
  p.xs.world = (uint32_t)world;
  p.xs.rank = (uint32_t)rank;
  for (int q = 0; q < world; ++q) p.xs.pub[q] = &xrecv(q)->flag[kXArgmax][rank];
  p.xs.wait = &xrecv(rank)->flag[kXArgmax][0];
  p.xs.epoch_word = &state->epoch;
  p.xs.mul = xps;
  p.xs.add = xps;
  p.xs.limit_us = &state->wait_limit_us;
  p.xs.err = &state->err;
  p.world = (uint32_t)world;
  p.rank = (uint32_t)rank;
  p.n_layer = m.n_layer;
  p.E = m.n_embd;
  p.F = m.n_ff;
  p.hl = hl;
  p.h0 = h0;
  p.kvl = kvl;
  p.kv0 = kv0;
  p.n_head = m.n_head;
  p.n_kv_head = m.n_kv_head;
  p.ffl = ffl;
  p.ff0 = ff0;
  p.el = el;
  p.e0 = e0;
  p.vl = vl;
  p.v0 = v0;
  p.max_ctx = m.max_ctx;
  p.max_chunks = max_chunks;
  p.eps = m.rms_eps;
  p.rope_base = m.rope_base;
  p.attn_scale = 1.0f / sqrtf((float)hd);  // text.c:365
  return launch_persistent_step(p, hd, (uint32_t)num_sms, s);
}

// Switches between the persistent and the per-op step and re-records the
// step graph.  The exchange buffers and the local pair buffers are cleared
// first: the two steps number their exchanges differently, and a word or
// flag left by one must not pass for the other's.  Tensor parallel: every
// rank switches, with no step running.
int TextDecoder::set_step_mode(int mode) {
  if (mode != EOSI_CUDA_STEP_AUTO && mode != EOSI_CUDA_STEP_PERSISTENT && mode != EOSI_CUDA_STEP_PER_OP) {
    set_error_message("cuda text: unknown step mode");
    return EOS_E_INVALID_ARG;
  }
  if (mode == EOSI_CUDA_STEP_PERSISTENT && !persistent_ok) {
    set_error_message("cuda text: the persistent step needs Q4_K linears and LM head, head_dim 64 or 128 and "
                      "n_embd <= 4096, with its shared memory on this device");
    return EOS_E_UNSUPPORTED;
  }
  step_mode_req = mode;
  const bool want = persistent_ok && mode == EOSI_CUDA_STEP_PERSISTENT;
  if (want == persistent) return EOS_OK;
  persistent = want;
  if (graph == nullptr) return EOS_OK;  // tensor parallel, not attached yet: recorded at attach
  if (cudaSetDevice(device) != cudaSuccess) return EOS_E_INTERNAL;
  cudaError_t e = cudaStreamSynchronize(st);
  if (e == cudaSuccess) e = cudaGraphExecDestroy(graph);
  graph = nullptr;
  if (e == cudaSuccess) e = cudaMemsetAsync(xbuf, 0, xstep_bytes, st);
  if (e == cudaSuccess && qkv_x) e = cudaMemsetAsync(qkv_x, 0, 8ull * (hl * hd + 2 * kvl * hd), st);
  if (e == cudaSuccess && gu_x) e = cudaMemsetAsync(gu_x, 0, 16ull * ffl, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    set_error_message(cudaGetErrorString(e));
    return EOS_E_INTERNAL;
  }
  return capture();
}

// Batched prefill of the n tokens at prompt[host_pos ...]: per block of up to
// pf_rows tokens and per layer, the block's rows go through the GEMMs and
// the prefill kernels, which write their K/V rows into the cache; the next
// block attends to them.  Only the cache matters afterwards (the next step
// reads it), so the last layer stops after its K/V rows and no block computes
// logits.  Tensor parallel, the matrices are split by output rows as in the
// step: each rank packs its heads' attention output and its FFN units'
// SiLU output into every rank's copy of the next GEMM's operand, and pushes
// its O / down output rows into every rank's row buffer, which the exchange
// kernel then adds to the residual rows -- so every rank holds the one-GPU
// residual stream bit for bit.  Leaves state->pos = host_pos + n (not
// host_pos itself: the caller commits it after its synchronisation).
cudaError_t TextDecoder::prefill(uint32_t n) {
  const uint32_t E = m.n_embd, F = m.n_ff, nqkv = hl * hd + 2u * kvl * hd;
  cudaError_t e = cudaSuccess;
  if (pf_rows == 0) {
    const uint32_t rows = m.max_ctx < kPrefillRows ? m.max_ctx : kPrefillRows;
    // the operand size grows with the row count: `rows` bounds every block
    size_t amax = 0;
    for (const uint32_t kk : {E, F})
      if (prefill_operand_bytes(rows, kk) > amax) amax = prefill_operand_bytes(rows, kk);
    size_t wmax = prefill_operand_bytes(nqkv, E);
    for (const size_t b : {prefill_operand_bytes(el, E), prefill_operand_bytes(2u * ffl, E),
                           prefill_operand_bytes(el, F)})
      if (b > wmax) wmax = b;
    if (e == cudaSuccess) e = alloc(&pf_x, 4ull * rows * E);
    if (e == cudaSuccess) e = alloc(&pf_qkv, 4ull * rows * nqkv);
    if (e == cudaSuccess) e = alloc(&pf_gu, 8ull * rows * ffl);
    if (e == cudaSuccess) e = alloc(&pf_act, amax);
    if (e == cudaSuccess) e = alloc(&pf_w, wmax);
    if (e != cudaSuccess) return e;
    pf_rows = rows;
  }
  int status = EOS_OK;
  const uint32_t mat_n[4] = {nqkv, el, 2u * ffl, el}, mat_k[4] = {E, E, E, F};  // qkv, o, gate|up, down
  auto mat_w = [&](uint32_t L, int i) -> const uint8_t* {
    const DecLayer& d = layers[L];
    return i == 0 ? d.wqkv : (i == 1 ? d.wo : (i == 2 ? d.wgu : d.wd));
  };
  if (pf_wres.empty() && pf_resident) {
    size_t need = 0;
    for (int i = 0; i < 4; ++i) need += prefill_operand_bytes(mat_n[i], mat_k[i]);
    need *= m.n_layer;
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) == cudaSuccess && need <= free_b / 2) {
      std::vector<void*> res(4u * m.n_layer, nullptr);
      cudaError_t r = cudaSuccess;
      for (uint32_t L = 0; L < m.n_layer && r == cudaSuccess; ++L)
        for (int i = 0; i < 4 && r == cudaSuccess; ++i) {
          r = cudaMalloc(&res[4u * L + i], prefill_operand_bytes(mat_n[i], mat_k[i]));
          if (r == cudaSuccess) r = launch_prefill_w_prep(mat_w(L, i), mat_n[i], mat_k[i], res[4u * L + i], st);
        }
      if (r == cudaSuccess) {
        pf_wres = res;
        for (void* q : res) allocs.push_back(q);
      } else {
        for (void* q : res)
          if (q) cudaFree(q);
        cudaGetLastError();  // not fatal: prepare per layer instead
      }
    }
  }
  // C (+)= act . deq(W)^T with W resident in the GEMM layout, or prepared on
  // the fly; rows of C ldc floats apart, pushed into `extra` too
  auto gemm = [&](uint32_t L, int i, const void* act, float* c, uint32_t mm, bool acc, uint32_t ldc = 0,
                  float* const* extra = nullptr, uint32_t n_extra = 0) {
    const uint32_t nn = mat_n[i], kk = mat_k[i];
    const bool res = pf_resident && !pf_wres.empty();
    const void* wp = res ? pf_wres[4u * L + i] : pf_w;
    if (e == cudaSuccess && !res) e = launch_prefill_w_prep(mat_w(L, i), nn, kk, pf_w, st);
    if (e == cudaSuccess)
      e = launch_prefill_gemm(act, wp, c, mm, nn, kk, gemv_err, st, &status, acc, extra, n_extra, ldc);
    if (e == cudaSuccess && status != EOS_OK) e = cudaErrorNotSupported;
  };
  // tensor parallel: the other ranks' copies of the O / down output rows and
  // of the O / down operands
  float* push_rows[2][kMaxParts] = {};
  void* push_op[2][kMaxParts] = {};
  uint32_t np = 0;
  for (int q = 0; q < world && world > 1; ++q) {
    if (q == rank) continue;
    push_rows[0][np] = reinterpret_cast<float*>(xpeer[q] + xoff_pfo) + e0;
    push_rows[1][np] = reinterpret_cast<float*>(xpeer[q] + xoff_pfd) + e0;
    push_op[0][np] = xpeer[q] + xoff_pfa;
    push_op[1][np] = xpeer[q] + xoff_pfs;
    ++np;
  }
  float* rows_o = world > 1 ? reinterpret_cast<float*>(xbuf + xoff_pfo) : nullptr;
  float* rows_d = world > 1 ? reinterpret_cast<float*>(xbuf + xoff_pfd) : nullptr;
  void* op_o = world > 1 ? static_cast<void*>(xbuf + xoff_pfa) : pf_act;
  void* op_d = world > 1 ? static_cast<void*>(xbuf + xoff_pfs) : pf_act;
  // handshake of one prefill exchange (kind `type`); with src, x += src
  auto exchange = [&](int type, const float* src, uint32_t mm) {
    if (e != cudaSuccess) return;
    XchgSync xs{};
    xs.world = (uint32_t)world;
    xs.rank = (uint32_t)rank;
    for (int q = 0; q < world; ++q) xs.pub[q] = &xrecv(q)->pf_flag[type][rank];
    xs.wait = &xrecv(rank)->pf_flag[type][0];
    xs.epoch_word = nullptr;
    xs.add = ++pf_epoch;
    xs.limit_us = &state->wait_limit_us;
    xs.err = &state->err;
    e = launch_pf_xchg(xs, pf_x, src, mm, E, st);
  };
  const float scale = 1.0f / sqrtf((float)hd);  // text.c:365
  for (uint32_t b0 = 0; b0 < n && e == cudaSuccess; b0 += pf_rows) {
    const uint32_t mm = (n - b0) < pf_rows ? (n - b0) : pf_rows;
    const uint32_t pos0 = host_pos + b0;
    for (uint32_t L = 0; L < m.n_layer && e == cudaSuccess; ++L) {
      const DecLayer& d = layers[L];
      float* kcl = kc + (size_t)L * m.max_ctx * kvl * hd;
      float* vcl = vc + (size_t)L * m.max_ctx * kvl * hd;
      e = launch_pf_norm_pack(pf_x, L == 0 ? prompt + pos0 : nullptr, tok_embd, d.attn_norm, m.rms_eps, mm, E,
                              pf_act, st);
      gemm(L, 0, pf_act, pf_qkv, mm, false);
      if (e == cudaSuccess) e = launch_pf_rope_kv(pf_qkv, kcl, vcl, mm, hl, kvl, hd, pos0, m.rope_base, st);
      if (L + 1u == m.n_layer) break;  // the cache needs nothing more of the last layer
      if (e == cudaSuccess)
        e = launch_pf_attn(pf_qkv, kcl, vcl, op_o, mm, hl, kvl, h0, kv0, m.n_head, m.n_kv_head, hd, pos0, scale,
                           E, push_op[0], np, st);
      if (world == 1) {
        gemm(L, 1, op_o, pf_x, mm, true);
      } else {
        exchange(kXAttn, nullptr, mm);
        gemm(L, 1, op_o, rows_o + e0, mm, false, E, push_rows[0], np);
        exchange(kXORows, rows_o, mm);
      }
      if (e == cudaSuccess)
        e = launch_pf_norm_pack(pf_x, nullptr, tok_embd, d.ffn_norm, m.rms_eps, mm, E, pf_act, st);
      gemm(L, 2, pf_act, pf_gu, mm, false);
      if (e == cudaSuccess) e = launch_pf_silu_pack(pf_gu, mm, ffl, op_d, ff0, F, push_op[1], np, st);
      if (world == 1) {
        gemm(L, 3, op_d, pf_x, mm, true);
      } else {
        exchange(kXSilu, nullptr, mm);
        gemm(L, 3, op_d, rows_d + e0, mm, false, E, push_rows[1], np);
        exchange(kXDRows, rows_d, mm);
      }
    }
  }
  return e;
}

int TextDecoder::capture() {
  cudaGraph_t g = nullptr;
  const int sm = (int)attn_smem_bytes(hd);
  cudaError_t e = hd == 64    ? cudaFuncSetAttribute(attn_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm)
                  : hd == 128 ? cudaFuncSetAttribute(attn_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm)
                              : cudaFuncSetAttribute(attn_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
  // the largest shared-memory carveout, so that a kernel's CTAs can share an
  // SM with the CTAs of the kernel before it (PDL overlap)
  for (const void* f : {(const void*)attn_kernel<2>, (const void*)attn_kernel<4>, (const void*)attn_kernel<8>,
                        (const void*)norm_pack_kernel<4>, (const void*)norm_pack_kernel<kNormMaxChunks>,
                        (const void*)silu_pack_kernel, (const void*)argmax_kernel})
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(f, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (e == cudaSuccess) e = cudaStreamBeginCapture(st, cudaStreamCaptureModeRelaxed);
  if (e == cudaSuccess) {
    const cudaError_t r = record_step(st);
    e = cudaStreamEndCapture(st, &g);
    if (r != cudaSuccess) e = r;
  }
  if (e == cudaSuccess) {
    size_t nodes = 0;
    e = cudaGraphGetNodes(g, nullptr, &nodes);
    step_kernels = (uint32_t)nodes;
  }
  if (e == cudaSuccess) e = cudaGraphInstantiate(&graph, g, 0);
  if (g) cudaGraphDestroy(g);

  if (e != cudaSuccess) {
    set_error_message(cudaGetErrorString(e));
    return EOS_E_INTERNAL;
  }
  return EOS_OK;
}

}  // namespace eos

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
using eos::TextDecoder;

struct eosi_cuda_text {
  TextDecoder d;
};

namespace {
int dec_fail(cudaError_t e) {
  eos::set_error_message(cudaGetErrorString(e));
  return EOS_E_INTERNAL;
}
int dec_check_device_errors(eosi_cuda_text_t* t) {
  uint32_t words[2] = {0, 0};
  cudaError_t e = cudaMemcpyAsync(&words[0], &t->d.state->err, 4, cudaMemcpyDeviceToHost, t->d.st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(&words[1], t->d.gemv_err, 4, cudaMemcpyDeviceToHost, t->d.st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(t->d.st);
  if (e != cudaSuccess) return dec_fail(e);
  if (words[0] & EOS_DEVERR_PEER) {
    eos::set_error_message("cuda text: a tensor-parallel peer did not arrive within the wait limit "
                           "(bounded wait ran out; reset every rank before stepping again)");
    return EOS_E_INTERNAL;
  }
  if (words[0] & EOS_DEVERR_WAIT_ACT) {
    eos::set_error_message("cuda text: a step's activations did not arrive within the wait limit "
                           "(bounded wait ran out)");
    return EOS_E_INTERNAL;
  }
  if (words[0] | words[1]) {
    eos::set_error_message("cuda text: a device-side bounded wait ran out");
    return EOS_E_INTERNAL;
  }
  return EOS_OK;
}
}  // namespace

extern "C" {

EOSLLM_CUDA_API int eosi_cuda_text_open(const eosi_cuda_llama_t* m, int device, int rank, int world,
                                        eosi_cuda_text_t** out) {
  if (m == nullptr || out == nullptr || m->tok_embd == nullptr || m->output_norm == nullptr ||
      m->output_w == nullptr || (m->n_layer > 0 && (m->attn_norm == nullptr || m->ffn_norm == nullptr ||
                                                    m->wq == nullptr || m->wk == nullptr || m->wv == nullptr ||
                                                    m->wo == nullptr || m->wg == nullptr || m->wu == nullptr ||
                                                    m->wd == nullptr)) ||
      m->max_ctx == 0 || m->n_vocab == 0) {
    eos::set_error_message("cuda text: NULL or empty model description");
    return EOS_E_INVALID_ARG;
  }
  *out = nullptr;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
    eos::set_error_message("cuda text: no such CUDA device");
    return EOS_E_UNSUPPORTED;
  }
  eosi_cuda_text_t* t = new (std::nothrow) eosi_cuda_text_t();
  if (t == nullptr) return EOS_E_OUT_OF_MEMORY;
  const int s = t->d.open(m, device, rank, world);
  if (s != EOS_OK) {
    delete t;
    return s;
  }
  *out = t;
  return EOS_OK;
}

EOSLLM_CUDA_API int eosi_cuda_text_step(eosi_cuda_text_t* t, uint32_t token, float* logits) {
  if (t == nullptr || logits == nullptr) return EOS_E_INVALID_ARG;
  TextDecoder& d = t->d;
  if (token >= d.m.n_vocab) {  // text.c:277
    eos::set_error_message("cuda text: token id out of range");
    return EOS_E_INVALID_ARG;
  }
  if (d.host_pos >= d.m.max_ctx) {  // text.c:278
    eos::set_error_message("cuda text: context is full");
    return EOS_E_OUT_OF_MEMORY;
  }
  if (d.graph == nullptr) {
    eos::set_error_message("cuda text: tensor-parallel decoder not attached to its peers");
    return EOS_E_INVALID_ARG;
  }
  if (cudaSetDevice(d.device) != cudaSuccess) return EOS_E_INTERNAL;
  cudaError_t e = cudaSuccess;
  if (!d.step_mode) {  // every later step reads its token from prompt[pos]
    const uint32_t np = d.m.max_ctx;
    e = cudaMemcpyAsync(&d.state->n_prompt, &np, 4, cudaMemcpyHostToDevice, d.st);
    d.step_mode = true;
  }
  if (e == cudaSuccess) e = cudaMemcpyAsync(d.prompt + d.host_pos, &token, 4, cudaMemcpyHostToDevice, d.st);
  if (e == cudaSuccess) e = cudaGraphLaunch(d.graph, d.st);
  // every rank's vocabulary slice (complete: this rank's pick waited for all
  // of them, and no rank writes logits again before this rank's next step)
  for (int q = 0; q < d.world && e == cudaSuccess; ++q) {
    eos::Geometry g{};
    eos::model_geometry(d.m, q, d.world, g);
    e = cudaMemcpyAsync(logits + g.v0, d.xpeer[q] + d.xoff_lg, 4ull * g.vl, cudaMemcpyDeviceToHost, d.st);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(d.st);
  if (e != cudaSuccess) return dec_fail(e);
  d.host_pos++;
  return dec_check_device_errors(t);
}

EOSLLM_CUDA_API int eosi_cuda_text_generate(eosi_cuda_text_t* t, const uint32_t* prompt, uint32_t n_prompt,
                                            uint32_t n_gen, uint32_t* out_tokens) {
  if (t == nullptr || prompt == nullptr || n_prompt == 0 || (n_gen > 0 && out_tokens == nullptr))
    return EOS_E_INVALID_ARG;
  TextDecoder& d = t->d;
  if (d.graph == nullptr) {
    eos::set_error_message("cuda text: tensor-parallel decoder not attached to its peers");
    return EOS_E_INVALID_ARG;
  }
  for (uint32_t i = 0; i < n_prompt; ++i)
    if (prompt[i] >= d.m.n_vocab) {
      eos::set_error_message("cuda text: token id out of range");
      return EOS_E_INVALID_ARG;
    }
  const uint64_t steps = (uint64_t)n_prompt + (n_gen > 0 ? n_gen - 1u : 0u);
  if (d.host_pos + steps > d.m.max_ctx) {
    eos::set_error_message("cuda text: prompt plus generation exceed the context");
    return EOS_E_OUT_OF_MEMORY;
  }
  if (cudaSetDevice(d.device) != cudaSuccess) return EOS_E_INTERNAL;
  const uint32_t np = d.host_pos + n_prompt;
  cudaError_t e = cudaMemcpyAsync(d.prompt + d.host_pos, prompt, 4ull * n_prompt, cudaMemcpyHostToDevice, d.st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(&d.state->n_prompt, &np, 4, cudaMemcpyHostToDevice, d.st);
  d.step_mode = false;
  // all prompt tokens but the last in one batched pass; the last one and the
  // generated ones go through the step graph (logits, pick)
  uint32_t batched = 0;
  if (d.prefill_ok() && d.prefill_min > 0 && n_prompt - 1u >= d.prefill_min) {
    batched = n_prompt - 1u;
    if (e == cudaSuccess) e = d.prefill(batched);
    const uint32_t pos = d.host_pos + batched;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&d.state->pos, &pos, 4, cudaMemcpyHostToDevice, d.st);
  }
  for (uint64_t i = batched; i < steps && e == cudaSuccess; ++i) e = cudaGraphLaunch(d.graph, d.st);
  // the pick of step (n_prompt - 1 + j) is generated token j
  if (e == cudaSuccess && n_gen > 0)
    e = cudaMemcpyAsync(out_tokens, d.out_tokens + np - 1u, 4ull * n_gen, cudaMemcpyDeviceToHost, d.st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(d.st);
  if (e != cudaSuccess) return dec_fail(e);
  d.host_pos += (uint32_t)steps;
  return dec_check_device_errors(t);
}

EOSLLM_CUDA_API int eosi_cuda_text_prefill(eosi_cuda_text_t* t, const uint32_t* tokens, uint32_t n) {
  if (t == nullptr || (tokens == nullptr && n > 0)) return EOS_E_INVALID_ARG;
  TextDecoder& d = t->d;
  if (!d.prefill_ok()) {
    eos::set_error_message("cuda text: batched prefill needs Q4_K linears");
    return EOS_E_UNSUPPORTED;
  }
  if (d.graph == nullptr) {
    eos::set_error_message("cuda text: tensor-parallel decoder not attached to its peers");
    return EOS_E_INVALID_ARG;
  }
  for (uint32_t i = 0; i < n; ++i)
    if (tokens[i] >= d.m.n_vocab) {
      eos::set_error_message("cuda text: token id out of range");
      return EOS_E_INVALID_ARG;
    }
  if ((uint64_t)d.host_pos + n > d.m.max_ctx) {
    eos::set_error_message("cuda text: prompt exceeds the context");
    return EOS_E_OUT_OF_MEMORY;
  }
  if (n == 0) return EOS_OK;
  if (cudaSetDevice(d.device) != cudaSuccess) return EOS_E_INTERNAL;
  cudaError_t e = cudaMemcpyAsync(d.prompt + d.host_pos, tokens, 4ull * n, cudaMemcpyHostToDevice, d.st);
  if (e == cudaSuccess) e = d.prefill(n);
  const uint32_t pos = d.host_pos + n;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&d.state->pos, &pos, 4, cudaMemcpyHostToDevice, d.st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(d.st);
  if (e != cudaSuccess) return dec_fail(e);
  d.host_pos = pos;
  return dec_check_device_errors(t);
}

EOSLLM_CUDA_API int eosi_cuda_text_set_prefill_min(eosi_cuda_text_t* t, uint32_t min_tokens) {
  if (t == nullptr) return EOS_E_INVALID_ARG;
  t->d.prefill_min = min_tokens;
  return EOS_OK;
}

EOSLLM_CUDA_API int eosi_cuda_text_set_prefill_resident(eosi_cuda_text_t* t, int resident) {
  if (t == nullptr) return EOS_E_INVALID_ARG;
  t->d.pf_resident = resident != 0;
  return EOS_OK;
}

EOSLLM_CUDA_API int eosi_cuda_text_reset(eosi_cuda_text_t* t) {
  if (t == nullptr) return EOS_E_INVALID_ARG;
  TextDecoder& d = t->d;
  if (cudaSetDevice(d.device) != cudaSuccess) return EOS_E_INTERNAL;
  // position, prompt length, pick, argmax count and error word; the exchange
  // epoch keeps counting (the peers' flags hold earlier epochs)
  cudaError_t e = cudaMemsetAsync(d.state, 0, offsetof(eos::DecState, epoch), d.st);
  // and the attention chunks' arrival counts (a step that gave up mid-way)
  if (e == cudaSuccess) e = cudaMemsetAsync(d.attn_count, 0, 4ull * d.hl, d.st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(d.st);

  if (e != cudaSuccess) return dec_fail(e);
  d.host_pos = 0;
  d.step_mode = false;
  return EOS_OK;
}

EOSLLM_CUDA_API uint32_t eosi_cuda_text_pos(const eosi_cuda_text_t* t) { return t ? t->d.host_pos : 0u; }

EOSLLM_CUDA_API int eosi_cuda_text_ipc_handle(eosi_cuda_text_t* t, void* out, size_t cap) {
  if (t == nullptr || out == nullptr || cap < sizeof(cudaIpcMemHandle_t)) return EOS_E_INVALID_ARG;
  if (cudaSetDevice(t->d.device) != cudaSuccess) return EOS_E_INTERNAL;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, t->d.xbuf);
  if (e != cudaSuccess) return dec_fail(e);
  memcpy(out, &h, sizeof(h));
  return EOS_OK;
}

EOSLLM_CUDA_API int eosi_cuda_text_attach_peers(eosi_cuda_text_t* t, const void* handles, size_t bytes) {
  if (t == nullptr || handles == nullptr || bytes < (size_t)t->d.world * sizeof(cudaIpcMemHandle_t))
    return EOS_E_INVALID_ARG;
  return t->d.attach(static_cast<const uint8_t*>(handles));
}

EOSLLM_CUDA_API int eosi_cuda_text_attach_local(eosi_cuda_text_t* const* ranks, int world) {
  if (ranks == nullptr || world < 2 || world > (int)eos::kMaxParts) return EOS_E_INVALID_ARG;
  uint8_t* bufs[eos::kMaxParts] = {};
  for (int q = 0; q < world; ++q) {
    if (ranks[q] == nullptr || ranks[q]->d.world != world || ranks[q]->d.rank != q) {
      eos::set_error_message("cuda text: attach_local needs every rank's decoder, in rank order");
      return EOS_E_INVALID_ARG;
    }
    bufs[q] = ranks[q]->d.xbuf;
  }
  for (int r = 0; r < world; ++r) {
    TextDecoder& d = ranks[r]->d;
    if (cudaSetDevice(d.device) != cudaSuccess) return EOS_E_INTERNAL;
    for (int q = 0; q < world; ++q) {  // stores into the other ranks' buffers need peer access
      const int pd = ranks[q]->d.device;
      if (pd == d.device) continue;
      const cudaError_t e = cudaDeviceEnablePeerAccess(pd, 0);
      if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
      } else if (e != cudaSuccess) {
        cudaGetLastError();
        eos::set_error_message("cuda text: attach_local: no peer access between the ranks' devices");
        return EOS_E_UNSUPPORTED;
      }
    }
    const int s = d.attach_buffers(bufs);
    if (s != EOS_OK) return s;
  }
  return EOS_OK;
}

EOSLLM_CUDA_API int eosi_cuda_text_set_wait_limit(eosi_cuda_text_t* t, uint32_t limit_us) {
  if (t == nullptr || limit_us == 0) return EOS_E_INVALID_ARG;
  TextDecoder& d = t->d;
  if (cudaSetDevice(d.device) != cudaSuccess) return EOS_E_INTERNAL;
  cudaError_t e = cudaMemcpyAsync(&d.state->wait_limit_us, &limit_us, 4, cudaMemcpyHostToDevice, d.st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(d.st);
  return e == cudaSuccess ? EOS_OK : dec_fail(e);
}

EOSLLM_CUDA_API int eosi_cuda_text_partition(const eosi_cuda_llama_t* m, int rank, int world, uint32_t* out) {
  if (m == nullptr || out == nullptr) return EOS_E_INVALID_ARG;
  eos::Geometry g{};
  const int s = eos::model_geometry(*m, rank, world, g);
  if (s != EOS_OK) return s;
  const uint32_t v[11] = {g.hd, g.h0, g.hl, g.kv0, g.kvl, g.ff0, g.ffl, g.v0, g.vl, g.e0, g.el};
  memcpy(out, v, sizeof(v));
  return EOS_OK;
}

EOSLLM_CUDA_API void* eosi_cuda_text_stream(eosi_cuda_text_t* t) { return t ? (void*)t->d.st : nullptr; }

EOSLLM_CUDA_API uint32_t eosi_cuda_text_step_kernels(const eosi_cuda_text_t* t) { return t ? t->d.step_kernels : 0u; }

EOSLLM_CUDA_API int eosi_cuda_text_set_step_mode(eosi_cuda_text_t* t, int mode) {
  return t ? t->d.set_step_mode(mode) : EOS_E_INVALID_ARG;
}

EOSLLM_CUDA_API int eosi_cuda_text_step_mode(const eosi_cuda_text_t* t) {
  if (t == nullptr) return 0;
  return t->d.persistent ? EOSI_CUDA_STEP_PERSISTENT : EOSI_CUDA_STEP_PER_OP;
}

EOSLLM_CUDA_API void eosi_cuda_text_close(eosi_cuda_text_t* t) {
  if (t == nullptr) return;
  cudaSetDevice(t->d.device);
  delete t;
}

}  // extern "C"
