// q80_gemv.cu -- Q8_0 decode GEMV for sm_100a (f32 activations x int8 weights
// with an fp16 scale per 32), the production Q8_0 path of every reference
// backend: eosi_scalar_matmul_q8_0 (src/kernels/scalar/matmul_q8.c:21-58).
//
// The reference multiplies every int8 weight, converted to float, by the f32
// activation.  Converting four bytes at a time to floats costs more integer
// instructions than the dot itself, so the staged kernel moves the
// conversion to the activations, once per CTA: each 32-value activation block
// becomes block-float integers (a power-of-two scale per block, 20-bit signed
// values, exact scaling, rounding error at most 2^-20 of the block's largest
// magnitude) held as three signed base-128 digits of int8, and a weight
// block's dot with it is three exact integer dp4a chains recombined in f32.
// Results agree with the reference's f32 loop to fp32 rounding (the tests
// bound it at 1e-3 relative plus 1e-3 rms), not bit for bit -- the summation
// order differs anyway.
//
// Skeleton as the Q4_K GEMV: each CTA owns a contiguous slab of weight rows,
// which is one contiguous byte range; warp w streams stages w, w + NW, ... of
// 256 blocks (8704 bytes, 32 groups of 8 blocks) HBM -> shared memory, each
// stage one TMA bulk copy (lane 0, completing on the buffer's mbarrier)
// through D private buffers, the first D issued before the PDL wait (17
// cp.async per lane and stage before: sweep 4208 -> 4380 GB/s on a B200).  Lane l of a stage takes group l: 8 consecutive blocks of
// one row, 272 bytes at a 16-byte aligned offset, so block c of every lane's
// group starts at the same position mod 16 and the realignment of its 2-byte
// aligned data is the same compile-time byte permute in every lane (3
// conflict-free 16-byte loads per block).  Group sums go to shared memory;
// at the end one thread per row adds its groups in order (deterministic).
#include "eos_common.cuh"
#include "eos_kernels.h"

namespace eos {


// ---------------------------------------------------------------------------
// Unstaged fallback: any k % 32 == 0 and any alignment of the weights.
// One warp per row; lane = (g, l8): block j0+g, weights [4 l8, 4 l8 + 4).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float q8_byte(uint32_t xb, uint32_t selector) {
  return __fsub_rn(__int_as_float((int)__byte_perm(xb, 0x4B000000u, selector)), 8388736.0f);
}

__global__ void __launch_bounds__(256) q80_gemv_simple_kernel(const uint8_t* __restrict__ w,
                                                              const float* __restrict__ a, float* __restrict__ c,
                                                              uint32_t n, uint32_t k) {
  const uint32_t row = blockIdx.x * 8u + (threadIdx.x >> 5), lane = threadIdx.x & 31u;
  if (row >= n) return;  // warp-uniform
  const uint32_t nblk = k / Q80_ELEMS, g = lane >> 3, l8 = lane & 7u;
  const size_t row_bytes = (size_t)nblk * Q80_BYTES;
  const uint8_t* rp = w + (size_t)row * row_bytes;
  const uint8_t* end = w + (size_t)n * row_bytes;
  float acc = 0.0f;
  for (uint32_t j0 = 0; j0 < nblk; j0 += 4) {
    const uint32_t j = j0 + g;
    if (j < nblk) {
      const float4 av = *reinterpret_cast<const float4*>(a + (j << 5) + (l8 << 2));
      const uint8_t* src = rp + j * Q80_BYTES + 2u + (l8 << 2);
      const uintptr_t addr = reinterpret_cast<uintptr_t>(src);
      const uint32_t* wp = reinterpret_cast<const uint32_t*>(addr & ~(uintptr_t)3);
      const uint32_t sh = (uint32_t)(addr & 3u) << 3;
      const uint32_t w0 = wp[0];
      const uint32_t w1 = (sh == 0u || reinterpret_cast<const uint8_t*>(wp + 1) >= end) ? 0u : wp[1];
      const uint32_t x = __funnelshift_r(w0, w1, sh) ^ 0x80808080u;
      const uint8_t* sp = rp + j * Q80_BYTES;
      const float sc = __half2float(__ushort_as_half((unsigned short)(sp[0] | (sp[1] << 8))));
      float t = av.x * q8_byte(x, 0x7540u);
      t = fmaf(av.y, q8_byte(x, 0x7541u), t);
      t = fmaf(av.z, q8_byte(x, 0x7542u), t);
      t = fmaf(av.w, q8_byte(x, 0x7543u), t);
      acc = fmaf(sc, t, acc);
    }
  }
  acc += __shfl_xor_sync(0xffffffffu, acc, 16);
  acc += __shfl_xor_sync(0xffffffffu, acc, 8);
  acc += __shfl_xor_sync(0xffffffffu, acc, 4);
  acc += __shfl_xor_sync(0xffffffffu, acc, 2);
  acc += __shfl_xor_sync(0xffffffffu, acc, 1);
  if (lane == 0) c[row] = acc;
}

// ---------------------------------------------------------------------------
// Staged kernel
// ---------------------------------------------------------------------------
constexpr uint32_t kQ8Group = 8;                            // blocks per lane and stage
constexpr uint32_t kQ8GroupBytes = kQ8Group * Q80_BYTES;    // 272, a multiple of 16
constexpr uint32_t kQ8StageBytes = 32u * kQ8GroupBytes;     // 8704: 32 groups per warp stage
constexpr uint32_t kQ8DigitStride = 112;                    // shared bytes per block: 3 x 32 digits + pad

struct Q80GemvParams {
  const uint8_t* w;  // n rows x row_bytes
  const float* a;    // k floats
  float* c;
  uint32_t n, k, nblk, row_bytes;
  uint32_t rows_max;  // rows of the largest CTA slab (the group-sum area)
  uint32_t* err;
  float* c_extra[7];  // further copies of every output (tensor-parallel push)
  uint32_t n_extra;
  // tensor parallel (ll.epoch_word != nullptr): the activations arrive as
  // (epoch, word) pairs from every rank (ll.in), and every output goes to
  // every rank as a pair (ll.out) instead of to c
  LLExchange ll;
};

// Shared-memory layout of the staged kernel (offsets in bytes).
struct Q80Smem {
  uint32_t dig, pw2, part, wbuf, bars, total;
};
__host__ __device__ inline Q80Smem q80_smem(uint32_t nblk, uint32_t rows_max, uint32_t nw, uint32_t d) {
  const uint32_t gpr = nblk / kQ8Group;
  Q80Smem m;
  m.dig = 0;
  m.pw2 = (nblk * kQ8DigitStride + 15u) & ~15u;
  m.part = m.pw2 + ((nblk * 4u + 15u) & ~15u);
  m.wbuf = m.part + ((rows_max * (gpr + 1u) * 4u + 127u) & ~127u);
  m.bars = m.wbuf + nw * d * kQ8StageBytes;  // one mbarrier per staging slot
  m.total = m.bars + nw * d * 8u;
  return m;
}

__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

// Eight lanes convert one 32-value activation block, lane i of the eight
// holding values 4 i .. 4 i + 3: with 2^E <= max|a| < 2^(E+1), every value
// becomes the integer A = round(a * 2^(19 - E)) (the scaling by a power of
// two is exact; |A| <= 2^20), written as three signed base-128 digits
// A = d1 * 2^14 + d2 * 2^7 + d3 (d2, d3 in [-64, 63], |d1| <= 64) -- the
// lane stores its four d1 bytes as one word at ds + 4 i, its d2 bytes at
// ds + 32 + 4 i, its d3 bytes at ds + 64 + 4 i; lane 0 of the eight stores the
// block's unit 2^(E - 19) at *pw.  A block whose largest magnitude is below
// 2^-100 (or subnormal) takes the slower exact library scaling; a block
// holding Inf or NaN gets unit NaN.  All 32 lanes of the warp call this.
__device__ __forceinline__ void q8_act_digits4(float4 v, uint32_t sub, uint8_t* ds, float* pw) {
  uint32_t mbits = max(max(__float_as_uint(v.x) & 0x7fffffffu, __float_as_uint(v.y) & 0x7fffffffu),
                       max(__float_as_uint(v.z) & 0x7fffffffu, __float_as_uint(v.w) & 0x7fffffffu));
  mbits = max(mbits, __shfl_xor_sync(0xffffffffu, mbits, 1));
  mbits = max(mbits, __shfl_xor_sync(0xffffffffu, mbits, 2));
  mbits = max(mbits, __shfl_xor_sync(0xffffffffu, mbits, 4));  // the eight lanes of the block
  const float x[4] = {v.x, v.y, v.z, v.w};
  int A[4] = {0, 0, 0, 0};
  float unit = 0.0f;
  if (mbits >= 0x7f800000u) {
    unit = __int_as_float(0x7fc00000);
  } else if (mbits >= 0x0d800000u) {  // max|a| >= 2^-100: both factors are normal floats
    const int E = (int)(mbits >> 23) - 127;
    const float up = __int_as_float((19 - E + 127) << 23);
#pragma unroll
    for (int q = 0; q < 4; ++q)  // round to nearest even through the 1.5 * 2^23 magic (|a * up| < 2^20)
      A[q] = __float_as_int(__fadd_rn(__fmul_rn(x[q], up), 12582912.0f)) - 0x4B400000;
    unit = __int_as_float((E - 19 + 127) << 23);
  } else if (mbits != 0u) {
    int e;
    frexpf(__uint_as_float(mbits), &e);  // max|a| < 2^e
#pragma unroll
    for (int q = 0; q < 4; ++q) A[q] = __float2int_rn(ldexpf(x[q], 20 - e));
    unit = ldexpf(1.0f, e - 20);
  }
  uint32_t w1 = 0, w2 = 0, w3 = 0;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int d3 = ((A[q] + 64) & 127) - 64;
    const int A2 = (A[q] - d3) >> 7;
    const int d2 = ((A2 + 64) & 127) - 64;
    const int d1 = (A2 - d2) >> 7;
    w1 |= ((uint32_t)d1 & 0xffu) << (8 * q);
    w2 |= ((uint32_t)d2 & 0xffu) << (8 * q);
    w3 |= ((uint32_t)d3 & 0xffu) << (8 * q);
  }
  if (ds != nullptr) {
    reinterpret_cast<uint32_t*>(ds)[sub] = w1;
    reinterpret_cast<uint32_t*>(ds + 32)[sub] = w2;
    reinterpret_cast<uint32_t*>(ds + 64)[sub] = w3;
    if (sub == 0) *pw = unit;
  }
}

template <int NW, int D>
__global__ void __launch_bounds__(NW * 32, 1) q80_gemv_kernel(const Q80GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t nblk = p.nblk, gpr = nblk / kQ8Group;
  const Q80Smem L = q80_smem(nblk, p.rows_max, NW, D);
  uint8_t* dig = smem + L.dig;                            // [slot][3][32] int8 digits
  float* pw2 = reinterpret_cast<float*>(smem + L.pw2);    // [slot] the block unit 2^(E - 19)
  float* part = reinterpret_cast<float*>(smem + L.part);  // [row][gpr + 1] group sums
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  uint8_t* wbuf = smem + L.wbuf + warp * D * kQ8StageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars) + warp * D;

  const uint32_t r0 = (uint32_t)(((uint64_t)p.n * blockIdx.x) / gridDim.x);
  const uint32_t r1 = (uint32_t)(((uint64_t)p.n * (blockIdx.x + 1)) / gridDim.x);
  const uint32_t nrows = r1 - r0;
  const uint32_t ngroups = nrows * gpr;  // this CTA's groups, in memory order
  const uint32_t nst = (ngroups + 31u) / 32u;
  const uint8_t* slab = p.w + (size_t)r0 * p.row_bytes;
  const size_t slab_bytes = (size_t)nrows * p.row_bytes;
  const uint64_t pol_w = l2_policy_evict_first();
  if (lane == 0) {
#pragma unroll
    for (uint32_t d = 0; d < (uint32_t)D; ++d) mbar_init(bars + d, 1u);
    fence_barrier_init();
  }
  __syncwarp();
  // lane 0 issues a stage as one TMA bulk copy (a stage is contiguous in the
  // slab; row_bytes = 34 nblk is a multiple of 272, so every size and address
  // is a multiple of 16 bytes) completing on the slot's mbarrier
  uint32_t issued = 0;
  auto issue = [&](uint32_t s, uint32_t slot) {
    if (s < nst) {
      if (lane == 0) {
        const size_t off = (size_t)s * kQ8StageBytes;
        const uint32_t bytes = (uint32_t)((slab_bytes - off) < kQ8StageBytes ? (slab_bytes - off) : kQ8StageBytes);
        mbar_arrive_expect_tx(bars + slot, bytes);
        bulk_g2s(wbuf + slot * kQ8StageBytes, slab + off, bytes, bars + slot, pol_w);
      }
      ++issued;
    }
  };
  // stages issued and not yet consumed, landed before an early exit
  auto drain = [&](uint32_t i) {
    for (; i < issued; ++i)
      if (!mbar_wait(bars + i % D, (i / D) & 1u) && lane == 0) report(p.err, EOS_DEVERR_DRAIN);
  };
#pragma unroll
  for (uint32_t d = 0; d < (uint32_t)D; ++d) issue(warp + d * NW, d);

  pdl_wait();  // the activations may be the previous kernel's output
  const bool ll = p.ll.epoch_word != nullptr;
  const uint32_t in_epoch = ll ? ll_epoch(p.ll, p.ll.in_add) : 0u;
  const uint32_t out_epoch = ll ? ll_epoch(p.ll, p.ll.out_add) : 0u;
  bool ok = true;
  uint64_t t0 = 0;
  // activation blocks -> digits, four blocks per warp and round (lane l: block
  // 4 r + l / 8, values 4 (l % 8) .. 4 (l % 8) + 3).  Block b sits at slot
  // (b % 8) * gpr + b / 8, so the 8 lanes of a shared-memory phase (groups
  // j .. j + 7, same c) read consecutive slots, 112 bytes apart: distinct
  // bank groups.
  const uint32_t sub = lane & 7u;
  for (uint32_t b0 = 4u * warp; b0 < nblk; b0 += 4u * NW) {
    const uint32_t b = b0 + (lane >> 3);
    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (ll) {  // (epoch, word) pairs: reload until all four of the lane's are there
      bool ready;
      do {
        ready = true;
        if (b < nblk) {
          uint64_t q0, q1, q2, q3;
          ll_load2(p.ll.in + (b << 5) + 4u * sub, q0, q1);
          ll_load2(p.ll.in + (b << 5) + 4u * sub + 2u, q2, q3);
          v = make_float4(__uint_as_float((uint32_t)q0), __uint_as_float((uint32_t)q1),
                          __uint_as_float((uint32_t)q2), __uint_as_float((uint32_t)q3));
          ready = (uint32_t)(q0 >> 32) == in_epoch && (uint32_t)(q1 >> 32) == in_epoch &&
                  (uint32_t)(q2 >> 32) == in_epoch && (uint32_t)(q3 >> 32) == in_epoch;
        }
        ready = __all_sync(0xffffffffu, ready);
        if (!ready && !__all_sync(0xffffffffu, ll_keep_waiting(p.ll, t0))) {
          ok = false;
          break;
        }
      } while (!ready);
      if (!ok) break;
    } else if (b < nblk) {
      v = reinterpret_cast<const float4*>(p.a)[(b << 3) + sub];
    }
    // lanes past the last block convert zeros and store nothing (every lane
    // takes part in the block-max shuffles)
    const uint32_t slot = (b % kQ8Group) * gpr + b / kQ8Group;
    q8_act_digits4(v, sub, b < nblk ? dig + slot * kQ8DigitStride : nullptr, pw2 + (b < nblk ? slot : 0u));
  }
  if (!__syncthreads_and(ok)) {  // a peer never arrived: drain, leave the outputs unwritten
    if (threadIdx.x == 0) report(p.ll.err, EOS_DEVERR_PEER);
    drain(0);
    return;
  }
  pdl_trigger();

  uint32_t slot = 0, i = 0;
  bool landed = true;
  for (uint32_t s = warp; s < nst; s += NW, ++i) {
    if (!__all_sync(0xffffffffu, mbar_wait(bars + slot, (i / D) & 1u))) {
      if (lane == 0) report(p.err, EOS_DEVERR_WAIT_FULL);
      drain(i);
      landed = false;
      break;
    }
    const uint32_t G = s * 32u + lane;
    if (G < ngroups) {
      const uint32_t row = G / gpr, j = G - row * gpr;  // group j of the row: blocks 8 j .. 8 j + 7
      const uint8_t* gb = wbuf + slot * kQ8StageBytes + lane * kQ8GroupBytes;
      float acc = 0.0f;
#pragma unroll
      for (uint32_t c = 0; c < kQ8Group; ++c) {
        const uint32_t o = (Q80_BYTES * c) & 15u;           // block start mod 16 (even)
        const uint8_t* wb = gb + ((Q80_BYTES * c) & ~15u);  // 16-byte aligned window of 48 bytes
        const uint4 v0 = lds128(wb), v1 = lds128(wb + 16), v2 = lds128(wb + 32);
        const uint32_t win[12] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w, v2.x, v2.y, v2.z, v2.w};
        const uint32_t hw = win[o >> 2];
        const uint32_t scale_bits = (o & 2u) ? (hw >> 16) : (hw & 0xffffu);
        // the 32 weight bytes start at o + 2: whole words, or halves of two
        const uint32_t ws = (o + 2u) >> 2;
        uint32_t q[8];
#pragma unroll
        for (uint32_t t = 0; t < 8; ++t)
          q[t] = ((o + 2u) & 2u) ? __byte_perm(win[ws + t], win[ws + t + 1], 0x5432) : win[ws + t];
        const uint32_t ds_slot = c * gpr + j;
        const uint8_t* ds = dig + ds_slot * kQ8DigitStride;
        const int4 a10 = *reinterpret_cast<const int4*>(ds), a11 = *reinterpret_cast<const int4*>(ds + 16);
        const int4 a20 = *reinterpret_cast<const int4*>(ds + 32), a21 = *reinterpret_cast<const int4*>(ds + 48);
        const int4 a30 = *reinterpret_cast<const int4*>(ds + 64), a31 = *reinterpret_cast<const int4*>(ds + 80);
        const int av1[8] = {a10.x, a10.y, a10.z, a10.w, a11.x, a11.y, a11.z, a11.w};
        const int av2[8] = {a20.x, a20.y, a20.z, a20.w, a21.x, a21.y, a21.z, a21.w};
        const int av3[8] = {a30.x, a30.y, a30.z, a30.w, a31.x, a31.y, a31.z, a31.w};
        int D1 = 0, D2 = 0, D3 = 0;
#pragma unroll
        for (uint32_t t = 0; t < 8; ++t) {
          D1 = __dp4a((int)q[t], av1[t], D1);
          D2 = __dp4a((int)q[t], av2[t], D2);
          D3 = __dp4a((int)q[t], av3[t], D3);
        }
        // |D1|, |D2|, |D3| <= 32 * 128 * 64 = 2^18: exact; the block's dot in
        // the block's units, then scale_w * dot * unit
        const float dot = __fadd_rn(__fmul_rn((float)D1, 16384.0f), (float)(D2 * 128 + D3));
        acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(f16_bits_to_f32(scale_bits), dot), pw2[ds_slot]));
      }
      part[row * (gpr + 1u) + j] = acc;
    }
    __syncwarp();  // every lane's reads of the stage have returned (their values are stored)
    issue(s + D * NW, slot);
    if (++slot == (uint32_t)D) slot = 0;
  }
  if (!__syncthreads_and(landed)) return;  // a stage never landed: outputs unwritten (error reported)
  // row sums: the row's groups in order
  for (uint32_t row = threadIdx.x; row < nrows; row += NW * 32u) {
    const float* pr = part + row * (gpr + 1u);
    float sum = 0.0f;
    for (uint32_t j = 0; j < gpr; ++j) sum = __fadd_rn(sum, pr[j]);
    if (ll) {
      ll_put(p.ll, r0 + row, __float_as_uint(sum), out_epoch);
    } else {
      p.c[r0 + row] = sum;
      for (uint32_t x = 0; x < p.n_extra; ++x) p.c_extra[x][r0 + row] = sum;
    }
  }
}

namespace {
struct Q80Config {
  void (*fn)(const Q80GemvParams);
  int nw, d;
  SmemAttr attr;  // dynamic shared memory allowed so far, per device
};
Q80Config g_q80_cfgs[] = {{q80_gemv_kernel<8, 2>, 8, 2, {}}, {q80_gemv_kernel<4, 2>, 4, 2, {}},
                          {q80_gemv_kernel<8, 3>, 8, 3, {}}, {q80_gemv_kernel<4, 3>, 4, 3, {}},
                          {q80_gemv_kernel<6, 2>, 6, 2, {}}, {q80_gemv_kernel<12, 2>, 12, 2, {}}};
constexpr int kNumQ80Cfgs = sizeof(g_q80_cfgs) / sizeof(g_q80_cfgs[0]);
int g_q80_variant = -1;
}  // namespace

void set_q80_gemv_variant(int v) { g_q80_variant = v; }

cudaError_t launch_q80_gemv(const uint8_t* w, const float* a, float* c, uint32_t n, uint32_t k, uint32_t* err,
                            int num_sms, int max_smem, cudaStream_t st, int* out_status, float* const* c_extra,
                            uint32_t n_extra, const LLExchange* ll) {
  if (n_extra > 7) {
    *out_status = EOS_E_INVALID_ARG;
    return cudaSuccess;
  }
  *out_status = EOS_OK;
  if (n == 0) return cudaSuccess;
  const uint32_t nblk = k / Q80_ELEMS;
  const uint32_t row_bytes = nblk * Q80_BYTES;
  // the staged kernel: groups of 8 blocks (k % 256 == 0), 16-byte aligned
  // weights and activations
  const bool aligned = (k % 256u) == 0 && k > 0 && (reinterpret_cast<uintptr_t>(w) & 15u) == 0 &&
                       (reinterpret_cast<uintptr_t>(a) & 15u) == 0;
  // CTAs per SM and the configuration: the first (in preference order) whose
  // shared memory fits at the largest CTA count tried
  int pick = -1;
  uint32_t cps = 1, smem = 0, rows_max = 0;
  auto fits = [&](int ci, uint32_t want_cps) -> bool {
    const Q80Config& g = g_q80_cfgs[ci];
    const uint32_t grid = (uint32_t)num_sms * want_cps;
    const uint32_t rmax = (n + grid - 1) / grid + 1u;
    const Q80Smem m = q80_smem(nblk, rmax, (uint32_t)g.nw, (uint32_t)g.d);
    if (m.total > (uint32_t)max_smem || want_cps * (m.total + 1024u) > (uint32_t)max_smem + 1024u) return false;
    pick = ci;
    cps = want_cps;
    smem = m.total;
    rows_max = rmax;
    return true;
  };
  if (aligned) {
    if (g_q80_variant >= 0 && g_q80_variant < kNumQ80Cfgs) {
      for (uint32_t want = 4; want >= 1 && pick < 0; --want) fits(g_q80_variant, want);
    } else {
      // measured on a B200 (sweep shapes): 8 warps x 2 buffers, one CTA per
      // SM, is fastest; smaller configurations for rows too long for it
      const int order[][2] = {{0, 1}, {4, 1}, {1, 2}, {1, 1}, {3, 1}};
      for (const auto& o : order)
        if (fits(o[0], (uint32_t)o[1])) break;
    }
  }
  if (pick < 0) {
    if (n_extra != 0 || (ll != nullptr && ll->epoch_word != nullptr)) {  // unstaged: one destination, no exchange
      *out_status = EOS_E_UNSUPPORTED;
      return cudaSuccess;
    }
    q80_gemv_simple_kernel<<<(n + 7u) / 8u, 256, 0, st>>>(w, a, c, n, k);
    return cudaGetLastError();
  }
  Q80Config& cfg = g_q80_cfgs[pick];
  {
    const cudaError_t e = ensure_smem_attr((const void*)cfg.fn, (int)smem, cfg.attr);  // on this device
    if (e != cudaSuccess) return e;
  }
  uint32_t grid = (uint32_t)num_sms * cps;
  if (grid > n) grid = n;
  Q80GemvParams prm{w, a, c, n, k, nblk, row_bytes, rows_max, err, {}, n_extra, {}};
  for (uint32_t j = 0; j < n_extra; ++j) prm.c_extra[j] = c_extra[j];
  if (ll != nullptr) prm.ll = *ll;
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(grid);
  lc.blockDim = dim3(cfg.nw * 32);
  lc.dynamicSmemBytes = smem;
  lc.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  return cudaLaunchKernelEx(&lc, cfg.fn, prm);
}

}  // namespace eos
