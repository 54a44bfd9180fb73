// eos_util.cu -- device-side data formats around the matmul path:
//   * Q4_K / Q8_0 weight quantizers (Q8_0 restates src/quant/q8_0.c:58-93;
//     the reference has no Q4_K quantizer -- src/quant/q4_k.c:83-93 -- so
//     this is the project's own affine min/max fit, reproduced bit for bit
//     by the CPU oracle), fed from an f32 tensor or straight from the
//     synthetic generator so multi-GB models never exist in f32;
//   * the seeded synthetic generator (Irwin-Hall(12) normal approximation
//     on splitmix64), identical on host and device;
//   * a scale/min unpack kernel used to check the GEMV's unpack exhaustively.
// Every float operation is an explicit round-to-nearest intrinsic (no FMA
// contraction) so results match the host restatement exactly.
#include "eos_common.cuh"
#include "eos_kernels.h"

namespace eos {

// ---- binary16 encoder of the reference (src/util/f16.h:49-82) ----------
__device__ __forceinline__ uint16_t ref_f32_to_f16(float f) {
  const uint32_t bits = __float_as_uint(f);
  const uint32_t sign = (bits >> 16) & 0x8000u, exp = (bits >> 23) & 0xFFu;
  uint32_t mant = bits & 0x7FFFFFu;
  if (exp == 0xFFu) return (uint16_t)(sign | 0x7C00u | (mant ? ((mant >> 13) | 0x200u) : 0u));
  if (exp == 0) return (uint16_t)sign;
  const int32_t e = (int32_t)exp - 112;
  if (e >= 31) return (uint16_t)(sign | 0x7C00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    mant |= 0x800000u;
    const uint32_t sh = (uint32_t)(14 - e);
    return (uint16_t)(sign | ((mant >> sh) + ((mant >> (sh - 1)) & 1u)));
  }
  return (uint16_t)(sign | ((((uint32_t)e << 10) | (mant >> 13)) + ((mant >> 12) & 1u)));
}

// ---- synthetic generator -------------------------------------------------
// splitmix64 (Steele, Lea & Flood, OOPSLA 2014).
__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__device__ __forceinline__ float gauss(uint64_t key, uint64_t index, float sigma) {
  int32_t s = 0;
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    const uint64_t r = splitmix64(key + 4ull * index + (uint64_t)h);
    s += (int32_t)(r & 0x1FFFFFu) + (int32_t)((r >> 21) & 0x1FFFFFu) + (int32_t)((r >> 42) & 0x1FFFFFu);
  }
  return __fmul_rn(__fmul_rn(__int2float_rn(s - 6 * 2097152), 4.76837158203125e-07f), sigma);
}

__device__ __forceinline__ uint64_t gauss_key(uint64_t seed) { return splitmix64(seed ^ 0x6A09E667F3BCC909ull); }

__global__ void fill_gauss_kernel(float* dst, size_t n, uint64_t seed, uint64_t offset, float sigma) {
  const uint64_t key = gauss_key(seed);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = gauss(key, offset + i, sigma);
}

// ---- Q4_K quantizer ------------------------------------------------------
__device__ __forceinline__ int rint_clamp(float v, int hi) {
  if (!(v > 0.0f)) return 0;
  if (v >= (float)hi) return hi;
  const int q = __float2int_rn(v);
  return q > hi ? hi : q;
}

// Eight lanes per super-block, lane j owning sub-block j: its 32 values stay
// in registers; the super-block maxima are lane-group reductions (order does
// not matter: scales and mins are >= 0 and a NaN is taken as 0, exactly as
// the sequential `if (v > max) max = v` starting from 0 ignores it); lane
// 2p+1 hands its nibbles to lane 2p, which writes the shared qs bytes.
template <bool GEN>
__global__ void __launch_bounds__(256) q4k_quantize_kernel(const float* __restrict__ src, uint8_t* __restrict__ dst,
                                                           size_t nblocks, uint64_t seed, uint64_t offset,
                                                           float sigma) {
  const unsigned FULL = 0xffffffffu;
  const size_t gt = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const size_t b = gt >> 3;
  const uint32_t j = threadIdx.x & 7u;
  const bool live = b < nblocks;
  const uint64_t key = GEN ? gauss_key(seed) : 0;
  float x[32];
#pragma unroll
  for (int l = 0; l < 32; ++l) {
    const size_t e = b * 256u + 32u * j + (uint32_t)l;
    x[l] = !live ? 0.0f : (GEN ? gauss(key, offset + e, sigma) : src[e]);
  }
  float lo = x[0], hi = x[0];
#pragma unroll
  for (int l = 1; l < 32; ++l) {
    if (x[l] < lo) lo = x[l];
    if (x[l] > hi) hi = x[l];
  }
  if (lo > 0.0f) lo = 0.0f;
  const float scale = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
  const float mins = -lo;
  float ms = scale > 0.0f ? scale : 0.0f, mm = mins > 0.0f ? mins : 0.0f;
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) {
    const float a = __shfl_xor_sync(FULL, ms, o), c = __shfl_xor_sync(FULL, mm, o);
    ms = a > ms ? a : ms;
    mm = c > mm ? c : mm;
  }
  const uint16_t dh = ref_f32_to_f16(__fdiv_rn(ms, 63.0f));
  const uint16_t mh = ref_f32_to_f16(__fdiv_rn(mm, 63.0f));
  const float d = f16_bits_to_f32(dh), dmin = f16_bits_to_f32(mh);
  const uint32_t sc = d > 0.0f ? (uint32_t)rint_clamp(__fdiv_rn(scale, d), 63) : 0u;
  const uint32_t mq = dmin > 0.0f ? (uint32_t)rint_clamp(__fdiv_rn(mins, dmin), 63) : 0u;
  const float es = __fmul_rn(d, (float)sc), em = __fmul_rn(dmin, (float)mq);
  // the 32 quants of this sub-block, one per byte: element l in byte l % 4 of word l / 4
  uint32_t nib[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
#pragma unroll
  for (int l = 0; l < 32; ++l) {
    const uint32_t q = es > 0.0f ? (uint32_t)rint_clamp(__fdiv_rn(__fadd_rn(x[l], em), es), 15) : 0u;
    nib[l >> 2] |= q << (8 * (l & 3));
  }
  // qs byte l of pair p = q[2p][l] | q[2p+1][l] << 4: lane 2p+1's quants
  // become the high nibbles of lane 2p's bytes
  uint32_t qs[8];
#pragma unroll
  for (int w = 0; w < 8; ++w) qs[w] = nib[w] | (__shfl_down_sync(FULL, nib[w], 1) << 4);
  // all 8 scales and mins to lane 0 of the group
  uint32_t scs[8], mqs[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    scs[i] = __shfl_sync(FULL, sc, (threadIdx.x & ~7u) | (uint32_t)i);
    mqs[i] = __shfl_sync(FULL, mq, (threadIdx.x & ~7u) | (uint32_t)i);
  }
  if (!live) return;
  uint8_t* blk = dst + b * Q4K_BYTES;  // super-blocks are 16-byte aligned
  if ((j & 1u) == 0) {  // pair p = j / 2 owns qs bytes [32p, 32p + 32) at offset 16 + 32p
    uint4* q4 = reinterpret_cast<uint4*>(blk + 16 + 16 * j);
    q4[0] = make_uint4(qs[0], qs[1], qs[2], qs[3]);
    q4[1] = make_uint4(qs[4], qs[5], qs[6], qs[7]);
  }
  if (j == 0) {
    // packing of tests/unit/test_runner.c:716-725
    uint32_t s0 = 0, s1 = 0, s2 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      s0 |= ((scs[i] & 63u) | ((scs[i + 4] >> 4) << 6)) << (8 * i);
      s1 |= ((mqs[i] & 63u) | ((mqs[i + 4] >> 4) << 6)) << (8 * i);
      s2 |= ((scs[i + 4] & 15u) | ((mqs[i + 4] & 15u) << 4)) << (8 * i);
    }
    *reinterpret_cast<uint4*>(blk) = make_uint4((uint32_t)dh | ((uint32_t)mh << 16), s0, s1, s2);
  }
}

// ---- Q8_0 quantizer: restates src/quant/q8_0.c:58-93 ---------------------
__global__ void q80_quantize_kernel(const float* __restrict__ src, uint8_t* __restrict__ dst, size_t nblocks) {
  const size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const float* bs = src + b * 32u;
  float amax = 0.0f;
  for (int i = 0; i < 32; ++i) {
    const float v = bs[i] < 0.0f ? -bs[i] : bs[i];
    if (v > amax) amax = v;
  }
  const float scale = __fdiv_rn(amax, 127.0f);
  const float inv = scale > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
  uint8_t* p = dst + b * Q80_BYTES;
  for (int i = 0; i < 32; ++i) {
    const float v = __fmul_rn(bs[i], inv);
    int q = __float2int_rz(v < 0.0f ? __fsub_rn(v, 0.5f) : __fadd_rn(v, 0.5f));
    q = q > 127 ? 127 : (q < -128 ? -128 : q);
    p[2 + i] = (uint8_t)(int8_t)q;
  }
  const uint16_t h = ref_f32_to_f16(scale);
  p[0] = (uint8_t)(h & 0xffu);
  p[1] = (uint8_t)(h >> 8);
}

// ---- scale/min unpack check: one thread per 12-byte field ----------------
__global__ void unpack_scale_min_kernel(const uint8_t* __restrict__ s12, uint32_t count, uint8_t* __restrict__ sc,
                                        uint8_t* __restrict__ m) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= count) return;
  const uint8_t* q = s12 + (size_t)i * 12u;
  const uint32_t w0 = q[0] | (q[1] << 8) | (q[2] << 16) | ((uint32_t)q[3] << 24);
  const uint32_t w1 = q[4] | (q[5] << 8) | (q[6] << 16) | ((uint32_t)q[7] << 24);
  const uint32_t w2 = q[8] | (q[9] << 8) | (q[10] << 16) | ((uint32_t)q[11] << 24);
  for (int j = 0; j < 8; ++j) {
    uint32_t a, bm;
    q4k_scale_min_w(j, w0, w1, w2, a, bm);
    sc[(size_t)i * 8u + j] = (uint8_t)a;
    m[(size_t)i * 8u + j] = (uint8_t)bm;
  }
}

// ---- launchers --------------------------------------------------------------
static unsigned grid_for(size_t n, unsigned block) {
  size_t g = (n + block - 1) / block;
  if (g > 65535u * 16u) g = 65535u * 16u;
  return (unsigned)(g ? g : 1);
}

cudaError_t launch_fill_gauss(float* dst, size_t n, uint64_t seed, uint64_t offset, float sigma, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  fill_gauss_kernel<<<grid_for(n, 256), 256, 0, st>>>(dst, n, seed, offset, sigma);
  return cudaGetLastError();
}

cudaError_t launch_q4k_quantize(const float* src, uint8_t* dst, size_t n_el, cudaStream_t st) {
  const size_t nb = n_el / Q4K_ELEMS;
  if (nb == 0) return cudaSuccess;
  q4k_quantize_kernel<false><<<(unsigned)((nb + 31) / 32), 256, 0, st>>>(src, dst, nb, 0, 0, 0.0f);
  return cudaGetLastError();
}

cudaError_t launch_q4k_from_gauss(uint8_t* dst, size_t nblocks, uint64_t seed, uint64_t offset, float sigma,
                                  cudaStream_t st) {
  if (nblocks == 0) return cudaSuccess;
  q4k_quantize_kernel<true><<<(unsigned)((nblocks + 31) / 32), 256, 0, st>>>(nullptr, dst, nblocks, seed, offset,
                                                                             sigma);
  return cudaGetLastError();
}

cudaError_t launch_q80_quantize(const float* src, uint8_t* dst, size_t n_el, cudaStream_t st) {
  const size_t nb = n_el / Q80_ELEMS;
  if (nb == 0) return cudaSuccess;
  q80_quantize_kernel<<<(unsigned)((nb + 127) / 128), 128, 0, st>>>(src, dst, nb);
  return cudaGetLastError();
}

cudaError_t launch_unpack_scale_min(const uint8_t* s12, uint32_t count, uint8_t* sc, uint8_t* m, cudaStream_t st) {
  if (count == 0) return cudaSuccess;
  unpack_scale_min_kernel<<<(count + 255) / 256, 256, 0, st>>>(s12, count, sc, m);
  return cudaGetLastError();
}

}  // namespace eos
