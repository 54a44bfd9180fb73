// q4k_gemv.cu -- Q4_K decode GEMV for sm_100a, bit-exact with the reference's
// production x86 path eosi_avx2_matmul_q4_k_int8
// (src/kernels/avx2/matmul_q4_k_int8.c:164-269).
//
// Two kernels per call:
//   1. act_pack_kernel: one warp per 32 activations, the exact x86 packing of
//      quantize_sub32 (:98-154).  It writes the "GEMV layout" below and lets
//      the dependent GEMV launch early (programmatic dependent launch).
//   2. q4k_gemv_kernel: persistent, one CTA per SM.  A producer warp streams
//      the CTA's contiguous slab of weight rows HBM -> shared memory with 1-D
//      bulk async copies (TMA) into an S-stage mbarrier ring; consumer warps
//      compute integer dp4a dots per 32-element sub-block and the fp32
//      rescale in the reference's evaluation order, so every output is
//      bit-identical to the CPU kernel (the integer dots are exact, and the
//      fp32 operations are issued with explicit round-to-nearest intrinsics
//      in the same order with no FMA contraction).
//
// GEMV activation layout (per activation row, 5k/4 bytes, k % 256 == 0):
//   [0, k)        int8 a_q, super-block b occupies bytes [256b, 256b+256):
//                 bytes 16c..16c+15        = sub-block 2(c/2),   half c%2
//                 bytes 128+16c..128+16c+15 = sub-block 2(c/2)+1, half c%2
//                 for chunk c = 0..7, i.e. exactly the a_q lanes that meet
//                 the 16 qs bytes [16c, 16c+16) of the super-block, so each
//                 quarter-warp reads 128 contiguous bytes (no bank conflict).
//   [k, k + k/4)  per 32-group g: {float scale, int32 sum_aq} (8 bytes).
#include "eos_common.cuh"
#include "eos_kernels.h"

namespace eos {

// ---------------------------------------------------------------------------
// Activation packing
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t gemv_layout_offset(uint32_t e) {
  const uint32_t b = e >> 8, local = e & 255u, sub = local >> 5, pos = local & 31u;
  const uint32_t c = ((sub >> 1) << 1) | (pos >> 4);
  return (b << 8) | ((sub & 1u) << 7) | (c << 4) | (pos & 15u);
}

// grid: ceil(m*k/32 / 8) blocks of 256 threads; warp -> one 32-group.
__global__ void __launch_bounds__(256) act_pack_kernel(const float* __restrict__ a, uint32_t m, uint32_t k,
                                                       uint8_t* __restrict__ out, int layout) {
  pdl_trigger();
  const uint32_t groups_per_row = k >> 5;
  const uint32_t gid = blockIdx.x * 8u + (threadIdx.x >> 5);
  const uint32_t lane = threadIdx.x & 31u;
  if (gid >= m * groups_per_row) return;  // warp-uniform
  const uint32_t row = gid / groups_per_row, g = gid - row * groups_per_row;
  const float v = a[(size_t)row * k + (g << 5) + lane];
  float scale;
  int32_t sum;
  const int8_t q = quant_group32(v, scale, sum);
  if (layout == EOS_ACT_LAYOUT_GEMV) {
    uint8_t* r = out + (size_t)row * (k + (k >> 2));
    r[gemv_layout_offset((g << 5) + lane)] = static_cast<uint8_t>(q);
    if (lane == 0) {
      float2 st;
      st.x = scale;
      st.y = __int_as_float(sum);
      *reinterpret_cast<float2*>(r + k + (g << 3)) = st;
    }
  } else {  // EOS_ACT_LAYOUT_SOURCE: int8[m*k], then float[m*k/32], then int32[m*k/32]
    out[(size_t)row * k + (g << 5) + lane] = static_cast<uint8_t>(q);
    if (lane == 0) {
      float* sc = reinterpret_cast<float*>(out + (size_t)m * k);
      int32_t* sm = reinterpret_cast<int32_t*>(out + (size_t)m * k + (size_t)m * groups_per_row * 4u);
      sc[gid] = scale;
      sm[gid] = sum;
    }
  }
}

// ---------------------------------------------------------------------------
// Q4_K GEMV
// ---------------------------------------------------------------------------
struct Q4kGemvParams {
  const uint8_t* w;    // n rows x row_bytes (GGUF Q4_K super-blocks)
  const uint8_t* act;  // GEMV activation layout, 5k/4 bytes
  float* c;            // n outputs
  uint32_t n, k, nb, row_bytes, stages, act_bytes;
  uint32_t* err;
};

// Dot products of RW weight rows with one packed activation row, computed by
// one warp.  Lane = (g, l8): group g (0..3) takes super-block b0+g of each
// 4-block step, lane l8 its qs bytes [16 l8, 16 l8 + 16).  Row pointers and
// act may point to shared or global memory (16-byte aligned).  Every output
// equals eosi_avx2_matmul_q4_k_int8's bit for bit: exact integer dots, then
//   partial_b = (((0 + t_0) + t_1) + ... + t_7),
//   t_s = ((d*sc_s)*as_s)*dot_s - ((dmin*m_s)*as_s)*sum_s   (no FMA),
//   c = ((0 + partial_0) + partial_1) + ...
// as at src/kernels/avx2/matmul_q4_k_int8.c:194, :254-261, :264.
template <int RW>
__device__ __forceinline__ void q4k_rows_dot(const uint8_t* const (&rowp)[RW], const uint8_t* act, uint32_t nb,
                                             uint32_t k, uint32_t lane, float (&acc)[RW]) {
  const unsigned FULL = 0xffffffffu;
  const uint32_t g = lane >> 3, l8 = lane & 7u, pr = l8 >> 1;
  const uint8_t* st_base = act + k;
#pragma unroll
  for (int r = 0; r < RW; ++r) acc[r] = 0.0f;
  for (uint32_t b0 = 0; b0 < nb; b0 += 4) {
    const uint32_t b = (b0 + g) < nb ? (b0 + g) : (nb - 1);
    // activation lanes + scales for this super-block, shared by the RW rows
    const int4 alo = *reinterpret_cast<const int4*>(act + (b << 8) + (l8 << 4));
    const int4 ahi = *reinterpret_cast<const int4*>(act + (b << 8) + 128 + (l8 << 4));
    const float4 st = *reinterpret_cast<const float4*>(st_base + (((b << 3) + (pr << 1)) << 3));
#pragma unroll
    for (int r = 0; r < RW; ++r) {
      const uint8_t* blk = rowp[r] + b * Q4K_BYTES;
      const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
      const uint4 qs = *reinterpret_cast<const uint4*>(blk + 16 + (l8 << 4));
      int dlo = __dp4a((int)(qs.x & 0x0F0F0F0Fu), alo.x, 0);
      dlo = __dp4a((int)(qs.y & 0x0F0F0F0Fu), alo.y, dlo);
      dlo = __dp4a((int)(qs.z & 0x0F0F0F0Fu), alo.z, dlo);
      dlo = __dp4a((int)(qs.w & 0x0F0F0F0Fu), alo.w, dlo);
      int dhi = __dp4a((int)((qs.x >> 4) & 0x0F0F0F0Fu), ahi.x, 0);
      dhi = __dp4a((int)((qs.y >> 4) & 0x0F0F0F0Fu), ahi.y, dhi);
      dhi = __dp4a((int)((qs.z >> 4) & 0x0F0F0F0Fu), ahi.z, dhi);
      dhi = __dp4a((int)((qs.w >> 4) & 0x0F0F0F0Fu), ahi.w, dhi);
      dlo += __shfl_xor_sync(FULL, dlo, 1);
      dhi += __shfl_xor_sync(FULL, dhi, 1);
      const float d = f16_bits_to_f32(hdr.x), dmin = f16_bits_to_f32(hdr.x >> 16);
      uint32_t sc_lo, m_lo, sc_hi, m_hi;
      q4k_scale_min_w((int)(pr << 1), hdr.y, hdr.z, hdr.w, sc_lo, m_lo);
      q4k_scale_min_w((int)(pr << 1) + 1, hdr.y, hdr.z, hdr.w, sc_hi, m_hi);
      const float t_lo =
          __fsub_rn(__fmul_rn(__fmul_rn(__fmul_rn(d, (float)sc_lo), st.x), (float)dlo),
                    __fmul_rn(__fmul_rn(__fmul_rn(dmin, (float)m_lo), st.x), (float)__float_as_int(st.y)));
      const float t_hi =
          __fsub_rn(__fmul_rn(__fmul_rn(__fmul_rn(d, (float)sc_hi), st.z), (float)dhi),
                    __fmul_rn(__fmul_rn(__fmul_rn(dmin, (float)m_hi), st.z), (float)__float_as_int(st.w)));
      float partial = 0.0f;
#pragma unroll
      for (uint32_t q = 0; q < 4; ++q) {
        const float xl = __shfl_sync(FULL, t_lo, (g << 3) + (q << 1));
        const float xh = __shfl_sync(FULL, t_hi, (g << 3) + (q << 1));
        partial = __fadd_rn(partial, xl);
        partial = __fadd_rn(partial, xh);
      }
#pragma unroll
      for (uint32_t q = 0; q < 4; ++q) {
        const float pq = __shfl_sync(FULL, partial, q << 3);
        if (b0 + q < nb) acc[r] = __fadd_rn(acc[r], pq);
      }
    }
  }
}

// Fallback without staging (rows too long for the shared-memory ring):
// one warp per weight row, straight from global memory.
__global__ void __launch_bounds__(256) q4k_gemv_simple_kernel(const uint8_t* __restrict__ w,
                                                              const uint8_t* __restrict__ act, float* __restrict__ c,
                                                              uint32_t n, uint32_t k) {
  pdl_wait();
  const uint32_t row = blockIdx.x * 8u + (threadIdx.x >> 5);
  if (row >= n) return;  // warp-uniform
  const uint32_t nb = k / Q4K_ELEMS;
  const uint8_t* rowp[1] = {w + (size_t)row * nb * Q4K_BYTES};
  float acc[1];
  q4k_rows_dot<1>(rowp, act, nb, k, threadIdx.x & 31u, acc);
  if ((threadIdx.x & 31u) == 0) c[row] = acc[0];
}

constexpr uint32_t kBarBytes = 256;  // 8 full + 8 empty + 1 act barrier, padded

// CW consumer warps, each owning RW rows of every stage; one producer warp.
template <int CW, int RW>
__global__ void __launch_bounds__((CW + 1) * 32, 1) q4k_gemv_kernel(const Q4kGemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + 8;
  uint64_t* actbar = full + 16;
  uint8_t* act_s = smem + kBarBytes;
  uint8_t* stage0 = act_s + ((p.act_bytes + 127u) & ~127u);
  constexpr uint32_t R = CW * RW;
  const uint32_t stage_bytes = R * p.row_bytes;
  const uint32_t S = p.stages;

  const uint32_t r0 = (uint32_t)(((uint64_t)p.n * blockIdx.x) / gridDim.x);
  const uint32_t r1 = (uint32_t)(((uint64_t)p.n * (blockIdx.x + 1)) / gridDim.x);
  const uint32_t nrows = r1 - r0;
  const uint32_t nst = (nrows + R - 1) / R;
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  if (nrows == 0) return;  // CTA-uniform

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], CW);
    }
    mbar_init(actbar, 1);
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == CW) {  // ---------------- producer warp ----------------
    if (lane == 0) {
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_a = l2_policy_evict_last();
      const uint32_t prime = nst < S ? nst : S;
      uint32_t issued = 0;
      bool ok = true;
      for (uint32_t s = 0; s < nst; ++s) {
        const uint32_t slot = s % S;
        if (s >= S && !mbar_wait(&empty[slot], ((s / S) - 1u) & 1u)) {
          report(p.err, EOS_DEVERR_WAIT_EMPTY);
          ok = false;
          break;
        }
        const uint32_t rows = (nrows - s * R) < R ? (nrows - s * R) : R;
        const uint32_t bytes = rows * p.row_bytes;
        mbar_arrive_expect_tx(&full[slot], bytes);
        bulk_g2s(stage0 + (size_t)slot * stage_bytes, p.w + (size_t)(r0 + s * R) * p.row_bytes, bytes, &full[slot],
                 pol_w);
        ++issued;
        if (s + 1 == prime) {
          // Weights do not depend on the packing kernel; the activations do.
          pdl_wait();
          mbar_arrive_expect_tx(actbar, p.act_bytes);
          bulk_g2s(act_s, p.act, p.act_bytes, actbar, pol_a);
        }
      }
      if (!ok) {
        // Do not leave while our own copies may still land in shared memory.
        for (uint32_t s = (issued > S ? issued - S : 0); s < issued; ++s)
          if (!mbar_wait(&full[s % S], (s / S) & 1u)) report(p.err, EOS_DEVERR_DRAIN);
        if (issued >= 1 && !mbar_wait(actbar, 0)) report(p.err, EOS_DEVERR_DRAIN);
      }
    }
    return;
  }

  // -------------------- consumer warps --------------------
  if (!mbar_wait(actbar, 0)) {
    report(p.err, EOS_DEVERR_WAIT_ACT);
    return;
  }
  const uint32_t nb = p.nb;

  for (uint32_t s = 0; s < nst; ++s) {
    const uint32_t slot = s % S;
    if (!mbar_wait(&full[slot], (s / S) & 1u)) {
      report(p.err, EOS_DEVERR_WAIT_FULL);
      return;
    }
    const uint32_t rows = (nrows - s * R) < R ? (nrows - s * R) : R;
    const uint8_t* stage = stage0 + (size_t)slot * stage_bytes;
    const uint32_t rbase = warp * RW;
    if (rbase < rows) {  // warp-uniform
      const uint8_t* rowp[RW];
#pragma unroll
      for (int r = 0; r < RW; ++r) {
        const uint32_t row = (rbase + r) < rows ? (rbase + r) : (rows - 1);
        rowp[r] = stage + (size_t)row * p.row_bytes;
      }
      float acc[RW];
      q4k_rows_dot<RW>(rowp, act_s, nb, p.k, lane, acc);
      if (lane == 0) {
#pragma unroll
        for (int r = 0; r < RW; ++r)
          if (rbase + r < rows) p.c[r0 + s * R + rbase + r] = acc[r];
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
}

// ---------------------------------------------------------------------------
// Host-side launchers
// ---------------------------------------------------------------------------
size_t act_layout_bytes(uint32_t m, uint32_t k, int layout) {
  if (layout == EOS_ACT_LAYOUT_GEMV) return (size_t)m * (k + (k >> 2));
  return (size_t)m * k + (size_t)m * (k >> 5) * 8u;
}

cudaError_t launch_act_pack(const float* a, uint32_t m, uint32_t k, uint8_t* out, int layout, cudaStream_t st) {
  const uint32_t groups = m * (k >> 5);
  const uint32_t blocks = (groups + 7u) / 8u;
  if (blocks == 0) return cudaSuccess;
  act_pack_kernel<<<blocks, 256, 0, st>>>(a, m, k, out, layout);
  return cudaGetLastError();
}

namespace {
struct GemvConfig {
  void (*fn)(const Q4kGemvParams);
  int cw, rw;
};

template <int CW, int RW>
GemvConfig make_cfg() {
  return GemvConfig{q4k_gemv_kernel<CW, RW>, CW, RW};
}
}  // namespace

static int g_q4k_variant = -1;  // -1: automatic

void set_q4k_gemv_variant(int v) { g_q4k_variant = v; }

cudaError_t launch_q4k_gemv(const uint8_t* w, const uint8_t* act, float* c, uint32_t n, uint32_t k, uint32_t* err,
                            int num_sms, int max_smem, bool pdl, cudaStream_t st, int* out_status) {
  *out_status = EOS_OK;
  if (n == 0) return cudaSuccess;
  static const GemvConfig cfgs[] = {make_cfg<8, 1>(), make_cfg<8, 2>(), make_cfg<16, 1>(), make_cfg<4, 2>()};
  const uint32_t nb = k / Q4K_ELEMS;
  const uint32_t row_bytes = nb * Q4K_BYTES;
  const uint32_t act_bytes = k + (k >> 2);
  const uint32_t act_region = (act_bytes + 127u) & ~127u;
  const uint32_t budget = (uint32_t)max_smem - kBarBytes - act_region;

  int pick = g_q4k_variant;
  if (pick < 0 || pick >= (int)(sizeof(cfgs) / sizeof(cfgs[0]))) {
    // Prefer two rows per warp (activation lanes reused) while >= 3 stages fit.
    pick = (budget / (16u * row_bytes) >= 3u) ? 1 : 0;
  }
  const GemvConfig cfg = cfgs[pick];
  const uint32_t R = (uint32_t)(cfg.cw * cfg.rw);
  uint32_t stages = budget / (R * row_bytes);
  if (stages > 8u) stages = 8u;
  if (stages < 2u) {  // row too long for the staged ring
    q4k_gemv_simple_kernel<<<(n + 7u) / 8u, 256, 0, st>>>(w, act, c, n, k);
    return cudaGetLastError();
  }
  const uint32_t smem = kBarBytes + act_region + stages * R * row_bytes;
  cudaError_t e = cudaFuncSetAttribute(cfg.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;

  Q4kGemvParams prm{w, act, c, n, k, nb, row_bytes, stages, act_bytes, err};
  uint32_t grid = (uint32_t)num_sms;
  if (grid > n) grid = n;
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(grid);
  lc.blockDim = dim3((cfg.cw + 1) * 32);
  lc.dynamicSmemBytes = smem;
  lc.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = pdl ? 1 : 0;
  e = cudaLaunchKernelEx(&lc, cfg.fn, prm);
  return e;
}

}  // namespace eos

// ---------------------------------------------------------------------------
// n < 4: the reference's f32-dequant path, eosi_avx2_matmul_q4_k
// (src/kernels/avx2/matmul_q4_k.c:70-153), bit for bit.  Lane t (0..7) is
// AVX2 lane t: w = fma(d*sc, q, -dmin*m) then acc = fma(a, w, acc) over the
// whole row in the same order, followed by the SSE horizontal sum
// ((l0+l4)+(l2+l6)) + ((l1+l5)+(l3+l7)).  One warp per output; tiny work.
// ---------------------------------------------------------------------------
namespace eos {

__global__ void __launch_bounds__(32) q4k_f32_small_n_kernel(const float* __restrict__ a,
                                                             const uint8_t* __restrict__ w, float* __restrict__ c,
                                                             uint32_t m, uint32_t n, uint32_t k) {
  const uint32_t i = blockIdx.y, j = blockIdx.x, t = threadIdx.x & 7u;
  const uint32_t nb = k / Q4K_ELEMS;
  const float* ar = a + (size_t)i * k;
  const uint8_t* br = w + (size_t)j * nb * Q4K_BYTES;
  float acc = 0.0f;
  for (uint32_t b = 0; b < nb; ++b, br += Q4K_BYTES) {
    const float* aa = ar + (size_t)b * Q4K_ELEMS;
    const float d = f16_bits_to_f32(br[0] | (br[1] << 8));
    const float dmin = f16_bits_to_f32(br[2] | (br[3] << 8));
    const uint8_t* qs = br + 16;
    for (int sub = 0; sub < 8; sub += 2, qs += 32) {
      uint32_t sl, ml, sh, mh;
      q4k_scale_min(sub, br + 4, sl, ml);
      q4k_scale_min(sub + 1, br + 4, sh, mh);
      const float d1 = __fmul_rn(d, (float)sl), m1 = __fmul_rn(dmin, (float)ml);
      const float d2 = __fmul_rn(d, (float)sh), m2 = __fmul_rn(dmin, (float)mh);
      for (uint32_t l = 0; l < 32; l += 8) {
        const uint32_t q = qs[l + t];
        const float wl = __fmaf_rn(d1, (float)(q & 15u), -m1);
        acc = __fmaf_rn(aa[sub * 32 + l + t], wl, acc);
        const float wh = __fmaf_rn(d2, (float)(q >> 4), -m2);
        acc = __fmaf_rn(aa[(sub + 1) * 32 + l + t], wh, acc);
      }
    }
  }
  const unsigned FULL = 0xffffffffu;
  const float p4 = __shfl_down_sync(FULL, acc, 4);  // lane t: acc[t] + acc[t+4]
  const float s = __fadd_rn(acc, p4);
  const float s2 = __shfl_down_sync(FULL, s, 2);  // (s0 + s2), (s1 + s3)
  const float u = __fadd_rn(s, s2);
  const float u1 = __shfl_down_sync(FULL, u, 1);
  if (threadIdx.x == 0) c[(size_t)i * n + j] = __fadd_rn(u, u1);
}

cudaError_t launch_q4k_f32_small_n(const float* a, const uint8_t* w, float* c, uint32_t m, uint32_t n, uint32_t k,
                                   cudaStream_t st) {
  if (m == 0 || n == 0) return cudaSuccess;
  q4k_f32_small_n_kernel<<<dim3(n, m), 32, 0, st>>>(a, w, c, m, n, k);
  return cudaGetLastError();
}

}  // namespace eos
