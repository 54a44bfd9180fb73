// q80_gemv.cu -- Q8_0 decode GEMV for sm_100a (f32 activations x int8 weights
// with an fp16 scale per 32), the production Q8_0 path of every reference
// backend: eosi_scalar_matmul_q8_0 (src/kernels/scalar/matmul_q8.c:21-58).
//
// Same persistent structure as the Q4_K GEMV: one CTA per SM owns a
// contiguous slab of weight rows, a producer warp streams it through an
// S-stage shared-memory ring with 1-D bulk async copies (TMA), consumer warps
// each own RW rows of a stage.  The f32 activation vector is bulk-copied once
// per CTA and each float4 is reused across the RW rows.  Accumulation is
// fp32 in a different association than the reference's sequential loop, so
// results agree to rounding (the parity tests bound it), not bit for bit.
// Block b of a row sits at byte 34b (2-byte aligned): each lane reads the
// aligned word pair around its 4 weights and funnel-shifts.
#include "eos_common.cuh"
#include "eos_kernels.h"

namespace eos {

struct Q80GemvParams {
  const uint8_t* w;  // n rows x row_bytes
  const float* a;    // k floats
  float* c;
  uint32_t n, k, nblk, row_bytes, stages, act_bytes;
  uint32_t* err;
};

constexpr uint32_t kQ80BarBytes = 256;

// int8 byte `sel` (0..3) of x (already biased by 0x80) as an exact float:
// bits 0x4B0000uu are 2^23 + u, minus 2^23 + 128 gives the signed value.
__device__ __forceinline__ float q8_byte(uint32_t xb, uint32_t selector) {
  return __fsub_rn(__int_as_float((int)__byte_perm(xb, 0x4B000000u, selector)), 8388736.0f);
}

// Dot products of RW Q8_0 weight rows with the f32 activation row, one warp.
// Lane = (g, l8): group g takes block j0+g of each 4-block step, lane l8 its
// weights [4 l8, 4 l8 + 4).  Block j of a row starts at byte 34j, so the four
// int8 values are read as the aligned word pair around them (absolute
// address, any row alignment) and funnel-shifted.  `end` (may be null) is
// one past the last readable weight byte: the second word is not read past it.
template <int RW>
__device__ __forceinline__ void q80_rows_dot(const uint8_t* const (&rowp)[RW], const float* act, uint32_t nblk,
                                             uint32_t lane, const uint8_t* end, float (&acc)[RW]) {
  const unsigned FULL = 0xffffffffu;
  const uint32_t g = lane >> 3, l8 = lane & 7u;
#pragma unroll
  for (int r = 0; r < RW; ++r) acc[r] = 0.0f;
  for (uint32_t j0 = 0; j0 < nblk; j0 += 4) {
    const uint32_t j = j0 + g;
    if (j < nblk) {  // no shuffles inside: divergence is safe here
      const float4 av = *reinterpret_cast<const float4*>(act + (j << 5) + (l8 << 2));
#pragma unroll
      for (int r = 0; r < RW; ++r) {
        const uint8_t* src = rowp[r] + j * Q80_BYTES + 2u + (l8 << 2);
        const uintptr_t addr = reinterpret_cast<uintptr_t>(src);
        const uint32_t* wp = reinterpret_cast<const uint32_t*>(addr & ~(uintptr_t)3);
        const uint32_t sh = (uint32_t)(addr & 3u) << 3;
        const uint32_t w0 = wp[0];
        const uint32_t w1 = (sh == 0u || (end != nullptr && reinterpret_cast<const uint8_t*>(wp + 1) >= end)) ? 0u : wp[1];
        const uint32_t x = __funnelshift_r(w0, w1, sh) ^ 0x80808080u;
        const uint8_t* sp = rowp[r] + j * Q80_BYTES;
        const float sc = __half2float(__ushort_as_half((unsigned short)(sp[0] | (sp[1] << 8))));
        float t = av.x * q8_byte(x, 0x7540u);
        t = fmaf(av.y, q8_byte(x, 0x7541u), t);
        t = fmaf(av.z, q8_byte(x, 0x7542u), t);
        t = fmaf(av.w, q8_byte(x, 0x7543u), t);
        acc[r] = fmaf(sc, t, acc[r]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RW; ++r) {
    float v = acc[r];
    v += __shfl_xor_sync(FULL, v, 16);
    v += __shfl_xor_sync(FULL, v, 8);
    v += __shfl_xor_sync(FULL, v, 4);
    v += __shfl_xor_sync(FULL, v, 2);
    v += __shfl_xor_sync(FULL, v, 1);
    acc[r] = v;
  }
}

// Fallback for any k % 32 == 0 and rows without 16-byte alignment: one warp
// per weight row straight from global memory (activations 16-byte aligned).
__global__ void __launch_bounds__(256) q80_gemv_simple_kernel(const uint8_t* __restrict__ w,
                                                              const float* __restrict__ a, float* __restrict__ c,
                                                              uint32_t n, uint32_t k) {
  const uint32_t row = blockIdx.x * 8u + (threadIdx.x >> 5);
  if (row >= n) return;  // warp-uniform
  const uint32_t nblk = k / Q80_ELEMS;
  const size_t row_bytes = (size_t)nblk * Q80_BYTES;
  const uint8_t* rowp[1] = {w + (size_t)row * row_bytes};
  float acc[1];
  q80_rows_dot<1>(rowp, a, nblk, threadIdx.x & 31u, w + (size_t)n * row_bytes, acc);
  if ((threadIdx.x & 31u) == 0) c[row] = acc[0];
}

template <int CW, int RW>
__global__ void __launch_bounds__((CW + 1) * 32, 1) q80_gemv_kernel(const Q80GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + 8;
  uint64_t* actbar = full + 16;
  float* act_s = reinterpret_cast<float*>(smem + kQ80BarBytes);
  uint8_t* stage0 = smem + kQ80BarBytes + ((p.act_bytes + 127u) & ~127u);
  constexpr uint32_t R = CW * RW;
  const uint32_t stage_bytes = R * p.row_bytes;
  const uint32_t S = p.stages;

  const uint32_t r0 = (uint32_t)(((uint64_t)p.n * blockIdx.x) / gridDim.x);
  const uint32_t r1 = (uint32_t)(((uint64_t)p.n * (blockIdx.x + 1)) / gridDim.x);
  const uint32_t nrows = r1 - r0;
  const uint32_t nst = (nrows + R - 1) / R;
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  if (nrows == 0) return;

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], CW);
    }
    mbar_init(actbar, 1);
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == CW) {
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
          pdl_wait();
          mbar_arrive_expect_tx(actbar, p.act_bytes);
          bulk_g2s(act_s, p.a, p.act_bytes, actbar, pol_a);
        }
      }
      if (!ok) {
        for (uint32_t s = (issued > S ? issued - S : 0); s < issued; ++s)
          if (!mbar_wait(&full[s % S], (s / S) & 1u)) report(p.err, EOS_DEVERR_DRAIN);
        if (issued >= 1 && !mbar_wait(actbar, 0)) report(p.err, EOS_DEVERR_DRAIN);
      }
    }
    return;
  }

  if (!mbar_wait(actbar, 0)) {
    report(p.err, EOS_DEVERR_WAIT_ACT);
    return;
  }
  const uint32_t nblk = p.nblk;

  for (uint32_t s = 0; s < nst; ++s) {
    const uint32_t slot = s % S;
    if (!mbar_wait(&full[slot], (s / S) & 1u)) {
      report(p.err, EOS_DEVERR_WAIT_FULL);
      return;
    }
    const uint32_t rows = (nrows - s * R) < R ? (nrows - s * R) : R;
    const uint8_t* stage = stage0 + (size_t)slot * stage_bytes;
    const uint32_t rbase = warp * RW;
    if (rbase < rows) {
      const uint8_t* rowp[RW];
#pragma unroll
      for (int r = 0; r < RW; ++r) {
        const uint32_t row = (rbase + r) < rows ? (rbase + r) : (rows - 1);
        rowp[r] = stage + (size_t)row * p.row_bytes;
      }
      float acc[RW];
      q80_rows_dot<RW>(rowp, act_s, nblk, lane, nullptr, acc);
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

namespace {
struct Q80Config {
  void (*fn)(const Q80GemvParams);
  int cw, rw;
};
template <int CW, int RW>
Q80Config make_q80() {
  return Q80Config{q80_gemv_kernel<CW, RW>, CW, RW};
}
}  // namespace

static int g_q80_variant = -1;
void set_q80_gemv_variant(int v) { g_q80_variant = v; }

cudaError_t launch_q80_gemv(const uint8_t* w, const float* a, float* c, uint32_t n, uint32_t k, uint32_t* err,
                            int num_sms, int max_smem, cudaStream_t st, int* out_status) {
  *out_status = EOS_OK;
  if (n == 0) return cudaSuccess;
  static const Q80Config cfgs[] = {make_q80<8, 2>(), make_q80<8, 1>(), make_q80<8, 4>(), make_q80<16, 2>()};
  const uint32_t nblk = k / Q80_ELEMS;
  const uint32_t row_bytes = nblk * Q80_BYTES;
  const uint32_t act_bytes = k * 4u;
  const uint32_t act_region = (act_bytes + 127u) & ~127u;
  const bool aligned = (k % 256u) == 0 && (reinterpret_cast<uintptr_t>(w) & 15u) == 0 &&
                       (reinterpret_cast<uintptr_t>(a) & 15u) == 0;
  if (!aligned || (uint32_t)max_smem <= kQ80BarBytes + act_region + 16u) {
    q80_gemv_simple_kernel<<<(n + 7u) / 8u, 256, 0, st>>>(w, a, c, n, k);
    return cudaGetLastError();
  }
  const uint32_t budget = (uint32_t)max_smem - kQ80BarBytes - act_region - 16u;
  int pick = g_q80_variant;
  if (pick < 0 || pick >= (int)(sizeof(cfgs) / sizeof(cfgs[0]))) pick = (budget / (16u * row_bytes) >= 3u) ? 0 : 1;
  const Q80Config cfg = cfgs[pick];
  const uint32_t R = (uint32_t)(cfg.cw * cfg.rw);
  uint32_t stages = budget / (R * row_bytes);
  if (stages > 8u) stages = 8u;
  if (stages < 2u) {
    q80_gemv_simple_kernel<<<(n + 7u) / 8u, 256, 0, st>>>(w, a, c, n, k);
    return cudaGetLastError();
  }
  // +16: the last lane's funnel-shift pair may read 4 bytes past the last row.
  const uint32_t smem = kQ80BarBytes + act_region + stages * R * row_bytes + 16u;
  cudaError_t e = cudaFuncSetAttribute(cfg.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  Q80GemvParams prm{w, a, c, n, k, nblk, row_bytes, stages, act_bytes, err};
  uint32_t grid = (uint32_t)num_sms;
  if (grid > n) grid = n;
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(grid);
  lc.blockDim = dim3((cfg.cw + 1) * 32);
  lc.dynamicSmemBytes = smem;
  lc.stream = st;
  return cudaLaunchKernelEx(&lc, cfg.fn, prm);
}

}  // namespace eos
