// prefill_text.cu -- batched prompt processing for the device-resident
// decoder (decoder.cu): the KV-cache rows of a block of prompt tokens in one
// pass per layer, every linear on the tcgen05 GEMM (prefill_gemm.cu) instead
// of one GEMV step per token.  The reference feeds a prompt one token at a
// time (src/core/session.c:231-236 -> eosi_text_step, text.c:267-436); this
// pass computes the same per-token quantities for m tokens at once:
//
//   pf_norm_pack    embedding (layer 0), rmsnorm (rmsnorm.c:14-37, the step's
//                   own summation order), quantize_sub32 packing per 32
//                   (matmul_q4_k_int8.c:98-154) into the GEMM's int8 layout
//   GEMM            [q; k; v] = A . Wqkv^T                      (text.c:349-352)
//   pf_rope_kv      RoPE on q and k (rope.c:16-38), k/v rows into the cache
//                   at pos0 + row                               (text.c:359-362)
//   pf_attn         causal softmax attention with the GQA head map
//                   (text.c:364-401), packed for the O GEMM
//   GEMM            x += attn . Wo^T                            (text.c:404-406)
//   pf_norm_pack    ffn_norm
//   GEMM            [gate | up] = A . Wgu^T                      (text.c:413-415)
//   pf_silu_pack    silu(gate) * up (silu.c:17, text.c:417), packed
//   GEMM            x += h . Wd^T                                (text.c:420-421)
//
// Numerics: every linear is bit-exact with the reference's int8 kernel (and
// so with the step path's GEMV) given the same input vector; rmsnorm, RoPE
// and SiLU use the step kernels' device arithmetic and order; attention is a
// streaming softmax over 32-position chunks, where the step path merges
// 32-position chunk softmaxes.  K/V rows therefore agree with the step path
// to the rounding of the attention sums, not bit for bit.
#include <cmath>

#include "decoder_internal.h"
#include "eos_common.cuh"
#include "eos_kernels.h"

namespace eos {

constexpr uint32_t kPfNormChunks = 16;  // float4 chunks per thread: n <= 16384
constexpr uint32_t kPfQ = 16;           // query rows per attention CTA (4 per warp)
constexpr uint32_t kPfKC = 32;          // cache positions per staged chunk (one per lane)
constexpr uint32_t kPfMaxDst = 8;       // this rank's operand + up to 7 peers' copies

// Where a packed 32-group goes: this rank's GEMM operand and, tensor
// parallel, the same position in the other ranks' copies (plain stores over
// NVLink through CUDA IPC mappings, performed when the grid completes).
struct PfOperands {
  uint16_t* aq[kPfMaxDst];  // int8 values as bf16, [rows][k]
  float* asc[kPfMaxDst];    // per-32 scale pairs, [2 k/32][pitch]
  uint32_t n;               // destinations
  uint32_t k, pitch;        // operand columns, scale-row pitch (pad4(rows))
};

// pf_pack_group into every destination: the same quantize_sub32 values.
__device__ __forceinline__ void pf_pack_group_to(const PfOperands& d, float v, uint32_t row, uint32_t s,
                                                 uint32_t lane) {
  float scale;
  int32_t sum;
  const int8_t q = quant_group32(v, scale, sum);
  const uint16_t b = __bfloat16_as_ushort(__float2bfloat16_rn((float)q));  // exact
  for (uint32_t j = 0; j < d.n; ++j) {
    d.aq[j][(size_t)row * d.k + s * 32u + lane] = b;
    if (lane == 0) {
      d.asc[j][(size_t)(2u * s) * d.pitch + row] = scale;
      d.asc[j][(size_t)(2u * s + 1u) * d.pitch + row] = (float)sum;
    }
  }
}

// ---------------------------------------------------------------------------
// Residual row -> rmsnorm -> packed activation
// ---------------------------------------------------------------------------
struct PfNormParams {
  float* x;                  // [m][n] residual rows
  const uint32_t* tokens;    // embedding mode: token of each row (else nullptr)
  const uint16_t* tok_embd;  // F16 [n_vocab][n]
  const float* w;            // norm weight
  float eps;
  uint32_t n, pitch;         // pitch: pad4(m), the scale pairs' row pitch
  uint16_t* aq;                // GEMM activation layout (pf_pack_group)
  float* asc;
};

// One CTA (256 threads) per row.  Thread t holds float4 chunks t, t + 256, ...
// and the mean square is reduced in the same order as norm_pack_kernel, so a
// row normalises exactly as the step path normalises the same vector.
__global__ void __launch_bounds__(256) pf_norm_pack_kernel(const PfNormParams p) {
  extern __shared__ __align__(16) float ys[];  // [n]
  __shared__ float red[8];
  const uint32_t row = blockIdx.x, tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  const uint32_t nch = p.n >> 2;
  float4* xr = reinterpret_cast<float4*>(p.x + (size_t)row * p.n);
  float4 v[kPfNormChunks];
  if (p.tokens != nullptr) {
    const uint2* emb = reinterpret_cast<const uint2*>(p.tok_embd + (size_t)p.tokens[row] * p.n);
#pragma unroll
    for (uint32_t j = 0; j < kPfNormChunks; ++j) {
      const uint32_t c = tid + 256u * j;
      if (c < nch) {
        const uint2 h = emb[c];  // F16 -> F32 is exact
        v[j] = make_float4(f16_bits_to_f32(h.x), f16_bits_to_f32(h.x >> 16), f16_bits_to_f32(h.y),
                           f16_bits_to_f32(h.y >> 16));
        xr[c] = v[j];
      }
    }
  } else {
#pragma unroll
    for (uint32_t j = 0; j < kPfNormChunks; ++j) {
      const uint32_t c = tid + 256u * j;
      if (c < nch) v[j] = xr[c];
    }
  }
  float ss = 0.0f;
#pragma unroll
  for (uint32_t j = 0; j < kPfNormChunks; ++j) {
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
  const float ms = __fdiv_rn(tot, (float)p.n);
  const float sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, p.eps)));
  const float4* w4 = reinterpret_cast<const float4*>(p.w);
#pragma unroll
  for (uint32_t j = 0; j < kPfNormChunks; ++j) {
    const uint32_t c = tid + 256u * j;
    if (c < nch) {
      const float4 wv = w4[c];
      ys[4u * c] = __fmul_rn(__fmul_rn(v[j].x, sc), wv.x);
      ys[4u * c + 1u] = __fmul_rn(__fmul_rn(v[j].y, sc), wv.y);
      ys[4u * c + 2u] = __fmul_rn(__fmul_rn(v[j].z, sc), wv.z);
      ys[4u * c + 3u] = __fmul_rn(__fmul_rn(v[j].w, sc), wv.w);
    }
  }
  __syncthreads();
  for (uint32_t g = warp; g < (p.n >> 5); g += 8u)  // warp-uniform
    pf_pack_group(ys[g * 32u + lane], row, g, lane, p.n, p.pitch, p.aq, p.asc);
}

// ---------------------------------------------------------------------------
// RoPE + KV-cache rows
// ---------------------------------------------------------------------------
struct PfRopeParams {
  float* qkv;  // [m][(hl + 2 kvl) HD]: q heads, k heads, v heads
  float* kc;   // this layer's caches [max_ctx][kvl HD]
  float* vc;
  uint32_t hl, kvl, pos0;
  float base;
};

// One CTA per row: thread t rotates pairs t, t + 256, ... of the q and k
// heads (k heads follow the q heads, so pair t of head h sits at h*HD + 2i).
template <int HD>
__global__ void __launch_bounds__(256) pf_rope_kv_kernel(const PfRopeParams p) {
  const uint32_t row = blockIdx.x, pos = p.pos0 + row;
  const uint32_t nqkv = (p.hl + 2u * p.kvl) * HD;
  float* r = p.qkv + (size_t)row * nqkv;
  const size_t crow = (size_t)pos * p.kvl * HD;
  const uint32_t pairs = (p.hl + p.kvl) * (HD / 2u);
  for (uint32_t t = threadIdx.x; t < pairs; t += 256u) {
    const uint32_t head = t / (HD / 2u), i = 2u * (t % (HD / 2u));
    float x0 = r[head * HD + i], x1 = r[head * HD + i + 1u];
    rope_pair<HD>(x0, x1, i, pos, p.base);
    if (head < p.hl) {
      r[head * HD + i] = x0;
      r[head * HD + i + 1u] = x1;
    } else {
      const uint32_t kh = head - p.hl;
      p.kc[crow + kh * HD + i] = x0;
      p.kc[crow + kh * HD + i + 1u] = x1;
    }
  }
  const float* vr = r + (p.hl + p.kvl) * HD;
  for (uint32_t t = threadIdx.x; t < p.kvl * HD; t += 256u) p.vc[crow + t] = vr[t];
}

// ---------------------------------------------------------------------------
// Causal attention over the cache
// ---------------------------------------------------------------------------
struct PfAttnParams {
  const float* qkv;  // q rotated
  const float* kc;
  const float* vc;
  PfOperands out;    // the O GEMM's operand(s); head h0 + h at groups (h0 + h) HD / 32
  uint32_t m, hl, kvl, h0, kv0, n_head, n_kv_head, pos0;
  float scale;
};

template <int E>
__host__ __device__ constexpr uint32_t pf_attn_smem_bytes() {
  // q rows, two buffers of (K chunk -- rows padded by 4 floats: conflict-free
  // 16-byte loads with one row per lane -- and V chunk), per-warp output row
  return 4u * (kPfQ * 32u * E + 2u * (kPfKC * (32u * E + 4u) + kPfKC * 32u * E) + 4u * 32u * E);
}

// Grid (hl, ceil(m / 16)), 128 threads.  CTA (h, y) owns query rows
// [16 b, 16 b + 16) of local head h, b = ceil(m / 16) - 1 - y; warp w owns
// four of them.  Cache
// positions stream through shared memory 32 at a time (K and V rows of the
// head's KV group, double-buffered: the next chunk's copies fly while this
// one is used); lane j scores position c0 + j for the warp's four
// queries (q from shared memory by broadcast, K row per lane), then a
// streaming softmax update (running max, rescaled sum and output) and the
// weighted V rows (lane = E dims).  At the end each query row is normalised
// and packed per 32 dims for the O GEMM.
template <int E>
__global__ void __launch_bounds__(128) pf_attn_kernel(const PfAttnParams p) {
  constexpr uint32_t HD = 32u * E, KP = HD + 4u;
  extern __shared__ __align__(16) float sm[];
  float* qs = sm;                          // [kPfQ][HD]
  float* kv0 = qs + kPfQ * HD;  // buffer b: K [kPfKC][KP] at kv0 + b (KP + HD) kPfKC, then V [kPfKC][HD]
  float* so = kv0 + 2u * kPfKC * (KP + HD);  // [4][HD]
  // query blocks in reverse launch order: the last ones of a head stream the
  // most chunks (causal), so they start first and the short ones fill the tail
  const uint32_t hloc = blockIdx.x, i0 = (gridDim.y - 1u - blockIdx.y) * kPfQ;
  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  const uint32_t gh = p.h0 + hloc;
  const uint32_t gkv = (gh * p.n_kv_head) / p.n_head;  // GQA map (text.c:367)
  const uint32_t kvi = gkv - p.kv0;
  const uint32_t nqkv = (p.hl + 2u * p.kvl) * HD;
  const uint32_t crow = p.kvl * HD;
  const uint32_t nq = (p.m - i0) < kPfQ ? (p.m - i0) : kPfQ;
  for (uint32_t t = tid; t < nq * (HD / 4u); t += 128u) {
    const uint32_t r = t / (HD / 4u), c4 = t % (HD / 4u);
    reinterpret_cast<float4*>(qs + r * HD)[c4] =
        reinterpret_cast<const float4*>(p.qkv + (size_t)(i0 + r) * nqkv + hloc * HD)[c4];
  }
  float o[4][E], mx[4], l[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    mx[r] = -INFINITY;
    l[r] = 0.0f;
#pragma unroll
    for (int e = 0; e < E; ++e) o[r][e] = 0.0f;
  }
  const uint32_t qpos0 = p.pos0 + i0 + warp * 4u;  // position of the warp's first query
  const uint32_t last = p.pos0 + i0 + nq - 1u;      // largest query position of the CTA
  const uint64_t pol = l2_policy_evict_last();      // the layer's cache rows are re-read by every query block
  // K and V rows [c0, c0 + 32) (up to `last`) into buffer b; one commit group
  auto stage = [&](uint32_t c0, int b) {
    const uint32_t np = (last + 1u - c0) < kPfKC ? (last + 1u - c0) : kPfKC;
    const float* kg = p.kc + (size_t)c0 * crow + kvi * HD;
    const float* vg = p.vc + (size_t)c0 * crow + kvi * HD;
    for (uint32_t t = tid; t < np * (HD / 4u); t += 128u) {
      const uint32_t r = t / (HD / 4u), c4 = (t % (HD / 4u)) * 4u;
      float* kb = kv0 + (uint32_t)b * kPfKC * (KP + HD);
      cp_async16(kb + r * KP + c4, kg + (size_t)r * crow + c4, pol);
      cp_async16(kb + kPfKC * KP + r * HD + c4, vg + (size_t)r * crow + c4, pol);
    }
    cp_async_commit();
  };
  stage(0u, 0);
  int cur = 0;
  for (uint32_t c0 = 0; c0 <= last; c0 += kPfKC, cur ^= 1) {
    const uint32_t np = (last + 1u - c0) < kPfKC ? (last + 1u - c0) : kPfKC;
    // the other buffer was last read in the previous iteration, which ended
    // with a barrier: refill it with the next chunk, then wait for this one
    if (c0 + kPfKC <= last) {
      stage(c0 + kPfKC, cur ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // this chunk (and, first time, q staging) visible to all
    const float* ks = kv0 + (uint32_t)cur * kPfKC * (KP + HD);
    const float* vs = ks + kPfKC * KP;
    // scores of position c0 + lane for the warp's four queries (rows >= np
    // of the chunk hold stale values; they are masked)
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const float* kr = ks + lane * KP;
#pragma unroll 4
    for (uint32_t d = 0; d < HD; d += 4u) {
      const float4 k4 = *reinterpret_cast<const float4*>(kr + d);
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const float4 q4 = *reinterpret_cast<const float4*>(qs + (warp * 4u + r) * HD + d);
        acc[r] = __fmaf_rn(q4.x, k4.x, acc[r]);
        acc[r] = __fmaf_rn(q4.y, k4.y, acc[r]);
        acc[r] = __fmaf_rn(q4.z, k4.z, acc[r]);
        acc[r] = __fmaf_rn(q4.w, k4.w, acc[r]);
      }
    }
    float pw[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      pw[r] = 0.0f;
      const uint32_t qi = warp * 4u + r;
      if (qi >= nq || qpos0 + r < c0) continue;  // warp-uniform: no position of this chunk is visible
      const bool valid = lane < np && c0 + lane <= qpos0 + r;
      const float s = valid ? __fmul_rn(acc[r], p.scale) : -INFINITY;
      float cm = s;
#pragma unroll
      for (int sh = 16; sh > 0; sh >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, sh));
      const float nm = fmaxf(mx[r], cm);            // finite: position c0 is visible
      const float alpha = expf(mx[r] - nm);         // 0 on the first chunk
      const float e = valid ? expf(s - nm) : 0.0f;
      float ls = e;
#pragma unroll
      for (int sh = 16; sh > 0; sh >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, sh);
      l[r] = __fmaf_rn(l[r], alpha, ls);
#pragma unroll
      for (int ee = 0; ee < E; ++ee) o[r][ee] *= alpha;
      mx[r] = nm;
      pw[r] = e;
    }
    for (uint32_t j = 0; j < np; ++j) {
      float vv[E];
#pragma unroll
      for (int ee = 0; ee < E; ++ee) vv[ee] = vs[j * HD + lane * E + ee];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const float a = __shfl_sync(0xffffffffu, pw[r], j);
#pragma unroll
        for (int ee = 0; ee < E; ++ee) o[r][ee] = __fmaf_rn(a, vv[ee], o[r][ee]);
      }
    }
    __syncthreads();  // every warp is done with buffer `cur` before it is refilled
  }
  // normalise, pack per 32 dims
  float* sw = so + warp * HD;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const uint32_t qi = warp * 4u + r;
    if (qi >= nq) break;  // warp-uniform
    const float inv = 1.0f / l[r];
#pragma unroll
    for (int ee = 0; ee < E; ++ee) sw[lane * E + ee] = o[r][ee] * inv;
    __syncwarp();
#pragma unroll
    for (int g = 0; g < E; ++g) pf_pack_group_to(p.out, sw[g * 32 + lane], i0 + qi, gh * E + g, lane);
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// silu(gate) * up -> packed
// ---------------------------------------------------------------------------
// Grid (ffl / 256, m), 256 threads; ffl % 32 == 0, so every warp is one group.
// FFN unit f0 + i goes to operand column f0 + i.
__global__ void __launch_bounds__(256) pf_silu_pack_kernel(const float* __restrict__ gu, uint32_t ffl, uint32_t f0,
                                                           const PfOperands out) {
  const uint32_t row = blockIdx.y, i = blockIdx.x * 256u + threadIdx.x;
  if (i >= ffl) return;  // warp-uniform
  const float* r = gu + (size_t)row * 2u * ffl;
  const float g = r[i], u = r[ffl + i];
  // x * (1 / (1 + expf(-x))) (silu.c:17), then gate * up (text.c:417)
  const float h = __fmul_rn(__fmul_rn(g, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)))), u);
  pf_pack_group_to(out, h, row, (f0 + i) >> 5, threadIdx.x & 31u);
}

// ---------------------------------------------------------------------------
// Tensor-parallel exchange (push model, like the decode step's)
// ---------------------------------------------------------------------------
struct PfXchgParams {
  XchgSync xs;
  float* x;         // [m][n] residual rows (identical on every rank)
  const float* src;  // [m][n] rows every rank pushed its slice of, or nullptr
  uint32_t m, n;
};

// The ranks' GEMMs or packing kernels wrote their slices into this rank's
// buffer with plain stores and completed before this kernel started (stream
// order); CTA 0 announces this rank's own push, every CTA waits for the other
// ranks' flags (its own rank's data is local and complete), then, for the
// residual exchanges, x[i] += src[i] -- the reference's x + t, exactly the
// single-GPU epilogue's add.
__global__ void __launch_bounds__(256) pf_xchg_kernel(const PfXchgParams p) {
  if (!xchg_handshake(p.xs, blockIdx.x == 0, true)) return;  // a peer never arrived: error bit set
  if (p.src == nullptr) return;
  const size_t n4 = (size_t)p.m * p.n / 4u;
  float4* x4 = reinterpret_cast<float4*>(p.x);
  for (size_t i = (size_t)blockIdx.x * 256u + threadIdx.x; i < n4; i += (size_t)gridDim.x * 256u) {
    const float4 t = __ldcg(reinterpret_cast<const float4*>(p.src) + i);
    const float4 v = x4[i];
    x4[i] = make_float4(__fadd_rn(v.x, t.x), __fadd_rn(v.y, t.y), __fadd_rn(v.z, t.z), __fadd_rn(v.w, t.w));
  }
}

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------
namespace {
uint16_t* act_q(void* act) { return static_cast<uint16_t*>(act); }
float* act_sc(void* act, uint32_t m, uint32_t k) {
  return reinterpret_cast<float*>(static_cast<uint8_t*>(act) + pf_scale_offset(m, k));
}
}  // namespace

cudaError_t launch_pf_norm_pack(float* x, const uint32_t* tokens, const uint16_t* tok_embd, const float* w, float eps,
                                uint32_t m, uint32_t n, void* act, cudaStream_t st) {
  if (m == 0) return cudaSuccess;
  if (n % 256u || n > 256u * 4u * kPfNormChunks) return cudaErrorInvalidValue;
  const uint32_t smem = 4u * n;
  cudaError_t e = cudaFuncSetAttribute(pf_norm_pack_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  PfNormParams p{x, tokens, tok_embd, w, eps, n, pf_pad4(m), act_q(act), act_sc(act, m, n)};
  pf_norm_pack_kernel<<<m, 256, smem, st>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_pf_rope_kv(float* qkv, float* kc, float* vc, uint32_t m, uint32_t hl, uint32_t kvl, uint32_t hd,
                              uint32_t pos0, float base, cudaStream_t st) {
  if (m == 0) return cudaSuccess;
  PfRopeParams p{qkv, kc, vc, hl, kvl, pos0, base};
  if (hd == 64) pf_rope_kv_kernel<64><<<m, 256, 0, st>>>(p);
  else if (hd == 128) pf_rope_kv_kernel<128><<<m, 256, 0, st>>>(p);
  else if (hd == 256) pf_rope_kv_kernel<256><<<m, 256, 0, st>>>(p);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

namespace {
template <int E>
cudaError_t attn_launch(const PfAttnParams& p, cudaStream_t st) {
  constexpr uint32_t smem = pf_attn_smem_bytes<E>();
  const cudaError_t e = cudaFuncSetAttribute(pf_attn_kernel<E>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
  if (e != cudaSuccess) return e;
  const dim3 grid(p.hl, (p.m + kPfQ - 1u) / kPfQ);
  pf_attn_kernel<E><<<grid, 128, smem, st>>>(p);
  return cudaGetLastError();
}
}  // namespace

namespace {
PfOperands operands(void* act, uint32_t m, uint32_t k, void* const* extra, uint32_t n_extra) {
  PfOperands d{};
  d.n = 1u + n_extra;
  d.k = k;
  d.pitch = pf_pad4(m);
  d.aq[0] = act_q(act);
  d.asc[0] = act_sc(act, m, k);
  for (uint32_t j = 0; j < n_extra; ++j) {
    d.aq[1 + j] = act_q(extra[j]);
    d.asc[1 + j] = act_sc(extra[j], m, k);
  }
  return d;
}
}  // namespace

cudaError_t launch_pf_attn(const float* qkv, const float* kc, const float* vc, void* act, uint32_t m, uint32_t hl,
                           uint32_t kvl, uint32_t h0, uint32_t kv0, uint32_t n_head, uint32_t n_kv_head,
                           uint32_t hd, uint32_t pos0, float scale, uint32_t k_total, void* const* act_extra,
                           uint32_t n_extra, cudaStream_t st) {
  if (m == 0 || hl == 0) return cudaSuccess;
  if (n_extra >= kPfMaxDst || (h0 + hl) * hd > k_total) return cudaErrorInvalidValue;
  PfAttnParams p{qkv, kc, vc, operands(act, m, k_total, act_extra, n_extra), m, hl, kvl, h0, kv0, n_head,
                 n_kv_head, pos0, scale};
  if (hd == 64) return attn_launch<2>(p, st);
  if (hd == 128) return attn_launch<4>(p, st);
  if (hd == 256) return attn_launch<8>(p, st);
  return cudaErrorInvalidValue;
}

cudaError_t launch_pf_xchg(const XchgSync& xs, float* x, const float* src, uint32_t m, uint32_t n, cudaStream_t st) {
  if (xs.world < 2 || xs.world > 8 || n % 4u) return cudaErrorInvalidValue;
  PfXchgParams p{xs, x, src, m, n};
  size_t blocks = 1;
  if (src != nullptr) {
    const size_t n4 = (size_t)m * n / 4u;
    blocks = (n4 + 255u) / 256u;
    if (blocks > 1184u) blocks = 1184u;  // grid-stride beyond 148 SMs x 8
    if (blocks == 0) blocks = 1;
  }
  pf_xchg_kernel<<<(uint32_t)blocks, 256, 0, st>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_pf_silu_pack(const float* gu, uint32_t m, uint32_t ffl, void* act, uint32_t f0, uint32_t k_total,
                                void* const* act_extra, uint32_t n_extra, cudaStream_t st) {
  if (m == 0 || ffl == 0) return cudaSuccess;
  if (ffl % 32u || f0 % 32u || f0 + ffl > k_total || n_extra >= kPfMaxDst) return cudaErrorInvalidValue;
  pf_silu_pack_kernel<<<dim3((ffl + 255u) / 256u, m), 256, 0, st>>>(gu, ffl, f0,
                                                                      operands(act, m, k_total, act_extra, n_extra));
  return cudaGetLastError();
}

}  // namespace eos
