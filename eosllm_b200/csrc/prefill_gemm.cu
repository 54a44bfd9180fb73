// prefill_gemm.cu -- batched (m > 1) Q4_K matmul on the sm_100a tensor cores
// (tcgen05 / TMEM / TMA), bit-exact with the reference's int8 kernel:
// C[m,n] = A[m,k] . deq(W)[n,k]^T for prompt processing, where the decode
// GEMV's one-row-at-a-time form would leave the tensor cores idle.
//
// The reference's arithmetic (src/kernels/avx2/matmul_q4_k_int8.c:164-269):
// activations are packed per 32 by quantize_sub32 (int8 a_q, scale as, sum of
// the a_q), and for row i, output j
//     c = 0;  c += partial_b  for super-blocks b in order            (:194, :264)
//     partial_b = 0;  partial_b += t_s  for sub-blocks s = 0..7      (:254-261)
//     t_s = ((d*sc_s)*as_s)*dot_s - ((dmin*m_s)*as_s)*sum_s
// where dot_s = sum_l q_l a_q,l over the sub-block's 32 elements is an exact
// integer (4-bit weights times int8 activations).  Here every dot_s of a
// 128 x 128 output tile comes from two tcgen05.mma kind::f16 (M128 N128 K16,
// A and B bf16) into an f32 TMEM accumulator: the 4-bit weights (0..15) and
// the int8 activations are exact in bf16, every product and every partial
// sum is an integer of magnitude below 2^16, so the f32 accumulation is exact
// whatever its order -- and the epilogue reads dot_s as a float, with no
// integer conversion.  The epilogue warps then apply t_s, the partial and the
// row sum in exactly the reference's f32 order (IEEE round-to-nearest, no
// FMA contraction).  So C equals the reference bit for bit, like the GEMV.
//
// Operand layouts (prepared by prefill_w_prep_kernel / the packers):
//   weights  wq  bf16 [n][k] (the 4-bit values), then at byte offset
//                pf_scale_offset(n, k) per sub-block s two f32 rows of
//                pad4(n): d*sc_s at [2s][col], -(dmin*m_s) at [2s + 1][col]
//   activ.   aq  bf16 [m][k] (the int8 values), then at pf_scale_offset(m, k)
//                per sub-block s two f32 rows of pad4(m): as_s at [2s][row],
//                sum_s at [2s + 1][row]
// (the min term is stored negated: t = t1 + (-t2) is exactly t1 - t2).
//
// Kernel: one CTA per 128 x 128 output tile, 576 threads.  Warp 0 lane 0 is
// the TMA producer, warp 1 lane 0 the MMA issuer, warps 2..17 the epilogue
// (warp w reads TMEM lanes 32(w % 4) .. +31 = tile rows, columns
// 32((w - 2) / 4) .. +31, as two 16x256b fragments: a thread holds 4 rows x 4
// column pairs, so a column pair's scales are one 8-byte load over 4
// addresses per warp -- a thread per row with 32 columns read every
// column's scales as warp-uniform 16-byte loads, 4 wavefronts each, and ran
// 6 % slower; four epilogue warps per SM sub-partition hide the TMEM-load
// and shared-memory latencies).  A stage holds a 64-element K
// slice (two sub-blocks): the A and B tiles (128B-swizzled, K-major) and the
// two sub-blocks' scale rows of the tile's rows and columns = 36 KB; four
// stages.  TMEM holds four f32 accumulators of 128 columns (512 columns),
// used by sub-blocks in turn: the MMAs of sub-block g wait until the
// epilogue has read accumulator g % 4 for sub-block g - 4, so tensor core
// and epilogue overlap.  A stage is released when its MMAs have completed
// (tcgen05.commit) and all sixteen epilogue warps have read its scales.  The row sums c live
// in shared memory (updated once per super-block), the partials in
// registers; every operation is an IEEE round-to-nearest multiply or add,
// never a fused multiply-add.  The four products of a term and the partial's
// add run on column pairs (mul.rn.f32x2 / add.rn.f32x2, lane-wise exact:
// checked against __fmul_rn / __fadd_rn on 2^21 random pairs); the term's
// own add, t1 + t2, stays two scalar __fadd_rn because ptxas contracts a
// packed add fed by a packed multiply into a packed FMA even with .rn (on
// this toolchain the contracted pair equalled fma.rn.f32x2 in every case and
// differed from multiply-then-add in 27 % of random pairs).  The accumulator
// is read one 16-lane fragment at a time (fewer live registers: 95 a thread).
//
// Waits are bounded (EOS_WAIT_LIMIT_NS): on a timeout the waiting role
// records an error bit and stops; the MMA issuer always commits the "done"
// barrier after its last MMA (MMAs complete on their own), the producer
// drains its copies (bounded), and TMEM is freed only after "done".  TMA
// boxes start at K offsets that are multiples of 128 bytes and at row / column
// offsets that are multiples of 128, so every x coordinate is 16-byte
// aligned; no multicast.
#include <cuda.h>
#include <cuda_bf16.h>

#include "eos_common.cuh"
#include "eos_kernels.h"
#include "eosllm_cuda.h"

namespace eos {

// Packed f32 pairs: lane-wise IEEE round-to-nearest multiply and add (no
// flush-to-zero, no contraction), each lane exactly the scalar operation.
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
  uint32_t lo, hi;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(__float_as_uint(a.x)), "r"(__float_as_uint(a.y)), "r"(__float_as_uint(b.x)), "r"(__float_as_uint(b.y)));
  return make_float2(__uint_as_float(lo), __uint_as_float(hi));
}
__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) {
  uint32_t lo, hi;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(__float_as_uint(a.x)), "r"(__float_as_uint(a.y)), "r"(__float_as_uint(b.x)), "r"(__float_as_uint(b.y)));
  return make_float2(__uint_as_float(lo), __uint_as_float(hi));
}

constexpr uint32_t QG_BM = 128, QG_BN = 128, QG_BK = 64;  // BK in bf16 elements: 128-byte rows
constexpr uint32_t QG_SUBS = QG_BK / 32u;                 // sub-blocks per stage (2)
constexpr uint32_t QG_ACCS = 4;                           // TMEM accumulators of QG_BN f32 columns
constexpr uint32_t QG_STAGES = 4;
constexpr uint32_t QG_A_BYTES = QG_BM * QG_BK * 2u;                              // 16 KB
constexpr uint32_t QG_B_BYTES = QG_BN * QG_BK * 2u;                              // 16 KB
constexpr uint32_t QG_AS_BYTES = 2u * QG_SUBS * QG_BM * 4u;                      // 2 KB
constexpr uint32_t QG_BS_BYTES = 2u * QG_SUBS * QG_BN * 4u;                      // 2 KB
constexpr uint32_t QG_STAGE_BYTES = QG_A_BYTES + QG_B_BYTES + QG_AS_BYTES + QG_BS_BYTES;  // 36 KB
constexpr uint32_t QG_EPI_WARPS = 16;
constexpr uint32_t QG_COLS = QG_BN * 4u / QG_EPI_WARPS;  // columns per epilogue thread (32)
constexpr uint32_t QG_THREADS = 32u * (2u + QG_EPI_WARPS);
constexpr uint32_t QG_ACC_BYTES = QG_EPI_WARPS * 32u * QG_COLS * 4u;  // row sums in shared memory
constexpr uint32_t QG_SMEM = QG_STAGES * QG_STAGE_BYTES + QG_ACC_BYTES + 1024u + 256u;
constexpr uint32_t QG_TMEM_COLS = 512;

// ---------------------------------------------------------------------------
// Operand preparation
// ---------------------------------------------------------------------------
// bf16 bit patterns of the integers 0..15 (exact), two per word.
__device__ __forceinline__ uint32_t bf16_pair(uint32_t lo, uint32_t hi) {
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn((float)lo)) |
         ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn((float)hi)) << 16);
}
// Eight 4-bit values of the word pair (x, y) (bytes b0..b7, nibble `sh`) as
// eight bf16 in a 16-byte vector.
__device__ __forceinline__ uint4 nib8_bf16(uint32_t x, uint32_t y, uint32_t sh) {
  return make_uint4(bf16_pair((x >> sh) & 15u, (x >> (8 + sh)) & 15u), bf16_pair((x >> (16 + sh)) & 15u, (x >> (24 + sh)) & 15u),
                    bf16_pair((y >> sh) & 15u, (y >> (8 + sh)) & 15u), bf16_pair((y >> (16 + sh)) & 15u, (y >> (24 + sh)) & 15u));
}

// One warp per super-block (row-major order: row * k/256 + b).  Lane l writes
// elements 8l .. 8l+7 (sub-block l/4) as bf16 -- the warp's 512 bytes are
// contiguous -- from the 8 bytes of qs that hold them (sub-block pair p =
// s/2 at bytes 32p .. 32p+31: low nibbles = sub-block 2p, high = 2p+1);
// lanes 0..7 write sub-block l's d*sc and -(dmin*m) with the reference's
// rounding (both __fmul_rn).
__global__ void __launch_bounds__(256) prefill_w_prep_kernel(const uint8_t* __restrict__ w, uint32_t n, uint32_t k,
                                                             uint16_t* __restrict__ wq, float* __restrict__ wsc) {
  const uint32_t nb = k / Q4K_ELEMS, lane = threadIdx.x & 31u;
  const uint64_t wi = (uint64_t)blockIdx.x * 8u + (threadIdx.x >> 5);
  if (wi >= (uint64_t)n * nb) return;  // warp-uniform
  const uint32_t row = (uint32_t)(wi / nb), b = (uint32_t)(wi % nb);
  const uint8_t* blk = w + wi * Q4K_BYTES;
  const uint32_t s = lane >> 2, p = s >> 1;
  const uint2 x = *reinterpret_cast<const uint2*>(blk + 16u + 32u * p + 8u * (lane & 3u));
  reinterpret_cast<uint4*>(wq + (size_t)row * k + (size_t)b * Q4K_ELEMS)[lane] = nib8_bf16(x.x, x.y, 4u * (s & 1u));
  if (lane < 8u) {
    const uint32_t h = *reinterpret_cast<const uint32_t*>(blk);
    const float d = f16_bits_to_f32(h), dmin = f16_bits_to_f32(h >> 16);
    uint32_t sc, m;
    q4k_scale_min((int)lane, blk + 4, sc, m);
    const uint32_t npad = pf_pad4(n);
    wsc[(size_t)(2u * (b * 8u + lane)) * npad + row] = __fmul_rn(d, (float)sc);
    wsc[(size_t)(2u * (b * 8u + lane) + 1u) * npad + row] = -__fmul_rn(dmin, (float)m);
  }
}

// quantize_sub32 per 32 activations (matmul_q4_k_int8.c:98-154), one warp
// per group: int8 values, the scale and the sum.
__global__ void __launch_bounds__(256) prefill_act_pack_kernel(const float* __restrict__ a, uint32_t m, uint32_t k,
                                                               uint16_t* __restrict__ aq, float* __restrict__ asc) {
  const uint32_t groups = m * (k / 32u);
  const uint32_t g = blockIdx.x * 8u + (threadIdx.x >> 5), lane = threadIdx.x & 31u;
  if (g >= groups) return;  // warp-uniform
  const uint32_t row = g / (k / 32u), s = g % (k / 32u);
  pf_pack_group(a[(size_t)g * 32u + lane], row, s, lane, k, pf_pad4(m), aq, asc);
}

// ---------------------------------------------------------------------------
// tcgen05 / TMA helpers
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor of a K-major, 128B-swizzled tile whose rows
// are 128 bytes and whose 8-row groups are 1024 bytes apart: start address
// >> 4, LBO 16 B (unused for swizzled K-major), SBO 1024 B, version 1, layout
// type 2 (SWIZZLE_128B).  Advancing K by 32 bytes adds 2 to the start field.
__device__ __forceinline__ uint64_t qg_sw128_desc(uint32_t smem_addr) {
  uint64_t dsc = (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  dsc |= (uint64_t)1u << 16;
  dsc |= (uint64_t)(1024u >> 4) << 32;
  dsc |= (uint64_t)1u << 46;
  dsc |= (uint64_t)2u << 61;
  return dsc;
}

// Instruction descriptor, kind::f16: D f32 (1 << 4), A and B bf16 (1 << 7,
// 1 << 10, the same type), both K-major, N = 128, M = 128.
constexpr uint32_t QG_IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((QG_BN >> 3) << 17) | ((QG_BM >> 4) << 24);

// D (+)= A . B^T over K = 16 (accumulate: enable-input-d)
__device__ __forceinline__ void qg_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(QG_IDESC), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

__device__ __forceinline__ void qg_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void qg_tma_2d(void* dst, const CUtensorMap* map, uint32_t x, uint32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Two 16x256b fragments' worth: 32 accumulator columns of 16 TMEM lanes (the
// address's lane field), four 8-column chunks; thread t gets, per chunk c,
// r[4c .. 4c+1] = row t/4, columns 8c + 2(t%4) + {0, 1}, and r[4c+2 .. 4c+3]
// the same columns of row t/4 + 8.
__device__ __forceinline__ void qg_ld16x256(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x4.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// ---------------------------------------------------------------------------
// GEMM
// ---------------------------------------------------------------------------
struct PrefillParams {
  float* c;          // row r at c + r * ldc (ldc >= n)
  uint32_t m, n, k, ldc;
  uint32_t* err;
  uint32_t accumulate;  // C = C_old + A.W^T (residual add, old value first)
  // tensor parallel: further destinations of C (other GPUs' receive slots,
  // same [m][n] layout), plain stores over NVLink, performed when the grid
  // completes; not combined with `accumulate`
  float* c_extra[7];
  uint32_t n_extra;
};

__global__ void __launch_bounds__(QG_THREADS, 1)
    prefill_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                        const __grid_constant__ CUtensorMap map_as, const __grid_constant__ CUtensorMap map_bs,
                        const PrefillParams p) {
  extern __shared__ uint8_t qg_smem_raw[];
  // 1024-byte aligned stage buffers (128B swizzle atoms)
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(qg_smem_raw) + 1023u) & ~uintptr_t(1023));
  float* acc_s = reinterpret_cast<float*>(smem + QG_STAGES * QG_STAGE_BYTES);  // [warp][column][lane]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + QG_STAGES * QG_STAGE_BYTES + QG_ACC_BYTES);
  uint64_t* empty = full + QG_STAGES;
  uint64_t* tfull = empty + QG_STAGES;
  uint64_t* tempty = tfull + QG_ACCS;
  uint64_t* done = tempty + QG_ACCS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
  // M tiles are the fast grid axis: the CTAs that share a weight tile run
  // together, so the tile is read from HBM once and from L2 by the others
  const uint32_t m0 = blockIdx.x * QG_BM, n0 = blockIdx.y * QG_BN;
  const uint32_t nkb = p.k / QG_BK;

  if (tid == 0) {
    for (uint32_t s = 0; s < QG_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + QG_EPI_WARPS);
    }
    for (uint32_t j = 0; j < QG_ACCS; ++j) {
      mbar_init(&tfull[j], 1);
      mbar_init(&tempty[j], QG_EPI_WARPS);
    }
    mbar_init(done, 1);
    fence_barrier_init();
  }
  if (warp == 0) {  // TMEM: 128 lanes x 512 f32 columns = four 128-column accumulators
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(QG_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer ----
      uint32_t issued = 0;
      for (uint32_t kb = 0; kb < nkb; ++kb) {
        const uint32_t s = kb % QG_STAGES;
        if (kb >= QG_STAGES && !mbar_wait(&empty[s], ((kb / QG_STAGES) - 1u) & 1u)) {
          report(p.err, EOS_DEVERR_WAIT_EMPTY);
          break;
        }
        mbar_arrive_expect_tx(&full[s], QG_STAGE_BYTES);
        uint8_t* base = smem + s * QG_STAGE_BYTES;
        qg_tma_2d(base, &map_a, kb * QG_BK, m0, &full[s]);
        qg_tma_2d(base + QG_A_BYTES, &map_b, kb * QG_BK, n0, &full[s]);
        qg_tma_2d(base + QG_A_BYTES + QG_B_BYTES, &map_as, m0, 2u * kb * QG_SUBS, &full[s]);
        qg_tma_2d(base + QG_A_BYTES + QG_B_BYTES + QG_AS_BYTES, &map_bs, n0, 2u * kb * QG_SUBS, &full[s]);
        issued = kb + 1;
      }
      // never leave copies in flight: the last use of every stage has landed
      for (uint32_t kb = issued > QG_STAGES ? issued - QG_STAGES : 0u; kb < issued; ++kb)
        if (!mbar_wait(&full[kb % QG_STAGES], (kb / QG_STAGES) & 1u)) report(p.err, EOS_DEVERR_DRAIN);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer ----
      bool ok = true;
      for (uint32_t kb = 0; kb < nkb && ok; ++kb) {
        const uint32_t s = kb % QG_STAGES;
        if (!mbar_wait(&full[s], (kb / QG_STAGES) & 1u)) {
          report(p.err, EOS_DEVERR_WAIT_FULL);
          break;
        }
        tc_fence_after();
        uint8_t* base = smem + s * QG_STAGE_BYTES;
        const uint64_t da = qg_sw128_desc(smem_u32(base)), db = qg_sw128_desc(smem_u32(base + QG_A_BYTES));
        for (uint32_t j = 0; j < QG_SUBS; ++j) {
          const uint32_t g = kb * QG_SUBS + j, a = g % QG_ACCS, u = g / QG_ACCS;
          // accumulator a is free once the epilogue has read sub-block g - 4
          if (u > 0 && !mbar_wait(&tempty[a], (u - 1u) & 1u)) {
            report(p.err, EOS_DEVERR_WAIT_EMPTY);
            ok = false;
            break;
          }
          tc_fence_after();
          // elements 32 j .. 32 j + 31 of the 64-element slice: byte offsets
          // 64 j and 64 j + 32 (descriptor start in 16-byte units)
          qg_mma(tmem + a * QG_BN, da + 4u * j, db + 4u * j, 0u);
          qg_mma(tmem + a * QG_BN, da + 4u * j + 2u, db + 4u * j + 2u, 1u);
          qg_commit(&tfull[a]);
        }
        qg_commit(&empty[s]);  // the stage's A/B tiles are consumed once these MMAs complete
      }
      qg_commit(done);  // every MMA issued above has completed
    }
  } else {
    // ---- epilogue: s32 dots -> reference-order f32 terms, partials, row sums ----
    // The warp's 32 TMEM lanes (tile rows quad * 32 ..) and 32 columns (col0
    // ..) are read as two 16x256b fragments of 16 lanes x 32 columns: thread
    // t holds rows quad * 32 + 8 h + t / 4 (h = 0..3; h / 2 is the fragment)
    // and, for c = 0..3, the column pair col0 + 8 c + 2 (t % 4) + {0, 1}.  A
    // column pair's two scales come from one 8-byte load (4 addresses per
    // warp), a row's from 4-byte loads (8 addresses per warp).
    const uint32_t e = warp - 2u, quad = warp & 3u, cg = e >> 2;
    const uint32_t rq = lane >> 2, cq = lane & 3u;
    const uint32_t col0 = cg * QG_COLS;  // first tile column of this warp
    // row sums c (updated once per super-block) in shared memory, this
    // thread's 32 outputs as 8 float4 at acc[32 i]; super-block partials
    // (updated every sub-block) in registers: part[8 h + 2 c + x]
    float4* acc = reinterpret_cast<float4*>(acc_s) + e * (QG_COLS / 4u) * 32u + lane;
    float part[QG_COLS];
#pragma unroll
    for (uint32_t c4 = 0; c4 < QG_COLS / 4; ++c4) acc[32 * c4] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);  // c = 0 (:194)
#pragma unroll
    for (uint32_t c = 0; c < QG_COLS; ++c) part[c] = 0.0f;  // partial = 0
    bool ok = true;
    for (uint32_t kb = 0; kb < nkb && ok; ++kb) {
      const uint32_t s = kb % QG_STAGES;
      ok = __all_sync(0xffffffffu, mbar_wait(&full[s], (kb / QG_STAGES) & 1u)) != 0;  // scales landed
      if (!ok) break;
      const uint8_t* base = smem + s * QG_STAGE_BYTES;
      const float* as_s = reinterpret_cast<const float*>(base + QG_A_BYTES + QG_B_BYTES);  // [2 j + {0,1}][128]
      const float* bs_s = reinterpret_cast<const float*>(base + QG_A_BYTES + QG_B_BYTES + QG_AS_BYTES);
      for (uint32_t j = 0; j < QG_SUBS && ok; ++j) {
        const uint32_t g = kb * QG_SUBS + j, a = g % QG_ACCS;
        ok = __all_sync(0xffffffffu, mbar_wait(&tfull[a], (g / QG_ACCS) & 1u)) != 0;
        if (!ok) break;
        tc_fence_after();
        const float2* dsc = reinterpret_cast<const float2*>(bs_s + (2u * j) * QG_BN + col0) + cq;       // d*sc
        const float2* nmn = reinterpret_cast<const float2*>(bs_s + (2u * j + 1u) * QG_BN + col0) + cq;  // -(dmin*m)
        // the two fragments (16 lanes each) in turn: fewer live registers
#pragma unroll
        for (uint32_t hh = 0; hh < 2; ++hh) {
          uint32_t r[16];
          qg_ld16x256(tmem + ((quad * 32u + 16u * hh) << 16) + a * QG_BN + col0, r);
          if (hh == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[a]);  // accumulator a may be overwritten
          }
          float2 as2[2], sum2[2];
#pragma unroll
          for (uint32_t hl = 0; hl < 2; ++hl) {
            const uint32_t lrow = quad * 32u + 16u * hh + 8u * hl + rq;
            const float as = as_s[(2u * j) * QG_BM + lrow], sum = as_s[(2u * j + 1u) * QG_BM + lrow];
            as2[hl] = make_float2(as, as);
            sum2[hl] = make_float2(sum, sum);
          }
#pragma unroll
          for (uint32_t c = 0; c < 4; ++c) {
            const float2 d2 = dsc[4u * c], n2 = nmn[4u * c];  // columns col0 + 8 c + 2 cq + {0, 1}
#pragma unroll
            for (uint32_t hl = 0; hl < 2; ++hl) {
              const uint32_t pi = 8u * (2u * hh + hl) + 2u * c;  // part index of the pair
              const float2 dot = make_float2(__uint_as_float(r[4u * c + 2u * hl]), __uint_as_float(r[4u * c + 2u * hl + 1u]));
              // t = ((d*sc)*as)*dot - ((dmin*m)*as)*sum   (:254-261), as t1 + (-t2): the four
              // products in pairs, t1 + t2 as two scalar adds (a packed add fed by a
              // packed multiply is contracted into a fused multiply-add by ptxas)
              const float2 t1 = mul2_rn(mul2_rn(d2, as2[hl]), dot), t2 = mul2_rn(mul2_rn(n2, as2[hl]), sum2[hl]);
              const float2 t = make_float2(__fadd_rn(t1.x, t2.x), __fadd_rn(t1.y, t2.y));
              const float2 pc = add2_rn(make_float2(part[pi], part[pi + 1]), t);  // partial += t
              part[pi] = pc.x;
              part[pi + 1] = pc.y;
            }
          }
        }
        if ((g & 7u) == 7u) {  // super-block complete: c += partial (:264), partial = 0
#pragma unroll
          for (uint32_t c4 = 0; c4 < QG_COLS / 4; ++c4) {
            float4 v = acc[32 * c4];
            v.x = __fadd_rn(v.x, part[4 * c4]);
            v.y = __fadd_rn(v.y, part[4 * c4 + 1]);
            v.z = __fadd_rn(v.z, part[4 * c4 + 2]);
            v.w = __fadd_rn(v.w, part[4 * c4 + 3]);
            acc[32 * c4] = v;
          }
#pragma unroll
          for (uint32_t c = 0; c < QG_COLS; ++c) part[c] = 0.0f;
        }
      }
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(&empty[s]);  // this warp has read the stage's scales
    }
    if (!ok) {
      if (lane == 0) report(p.err, EOS_DEVERR_WAIT_FULL);
    } else {
      // output pair (h, c): row m0 + quad * 32 + 8 h + t / 4, columns
      // n0 + col0 + 8 c + 2 (t % 4) + {0, 1} = acc float4 2 h + c / 2, half c % 2;
      // 8-byte stores where every destination allows them
      bool pair_ok = (p.ldc & 1u) == 0 && (reinterpret_cast<uintptr_t>(p.c) & 7u) == 0;
      for (uint32_t x = 0; x < p.n_extra; ++x) pair_ok = pair_ok && (reinterpret_cast<uintptr_t>(p.c_extra[x]) & 7u) == 0;
#pragma unroll
      for (uint32_t h = 0; h < 4; ++h) {
        const uint32_t row = m0 + quad * 32u + 8u * h + rq;
        if (row >= p.m) continue;
#pragma unroll
        for (uint32_t c = 0; c < 4; ++c) {
          const float4 v4 = acc[32 * (2u * h + c / 2u)];
          float2 v = (c & 1u) ? make_float2(v4.z, v4.w) : make_float2(v4.x, v4.y);
          const uint32_t gcol = n0 + col0 + 8u * c + 2u * cq;
          const size_t at = (size_t)row * p.ldc + gcol;
          if (pair_ok && gcol + 2u <= p.n) {
            if (p.accumulate) {
              const float2 o = *reinterpret_cast<const float2*>(p.c + at);
              v = make_float2(__fadd_rn(o.x, v.x), __fadd_rn(o.y, v.y));
            }
            *reinterpret_cast<float2*>(p.c + at) = v;
            for (uint32_t x = 0; x < p.n_extra; ++x) *reinterpret_cast<float2*>(p.c_extra[x] + at) = v;
          } else {
#pragma unroll
            for (uint32_t x2 = 0; x2 < 2; ++x2) {
              if (gcol + x2 < p.n) {
                const float vv = x2 ? v.y : v.x;
                const float w = p.accumulate ? __fadd_rn(p.c[at + x2], vv) : vv;
                p.c[at + x2] = w;
                for (uint32_t x = 0; x < p.n_extra; ++x) p.c_extra[x][at + x2] = vv;
              }
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  // the done barrier follows the last MMA (MMAs wait on nothing, so it always
  // completes); free the accumulators only then
  if (warp == 0) {
    if (!__all_sync(0xffffffffu, mbar_wait(done, 0u)) && lane == 0) report(p.err, EOS_DEVERR_DRAIN);
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(QG_TMEM_COLS) : "memory");
  }
}

// ---------------------------------------------------------------------------
// Host
// ---------------------------------------------------------------------------
namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* q = nullptr;
    cudaDriverEntryPointQueryResult r;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &q, cudaEnableDefault, &r) == cudaSuccess &&
        r == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(q);
  }
  return fn;
}

// rows x k bf16 row-major, boxes of 128 rows x 64 elements (128 bytes) with the 128-byte swizzle
bool make_bf16_map(CUtensorMap* map, const void* base, uint32_t rows, uint32_t k) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {k, rows};
  const cuuint64_t strides[1] = {(cuuint64_t)k * 2u};
  const cuuint32_t box[2] = {QG_BK, 128u};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [2 k/32][pad4(cols)] f32 scale rows, boxes of 128 columns x 8 rows (four sub-blocks)
bool make_scale_map(CUtensorMap* map, const void* base, uint32_t cols, uint32_t k) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {cols, 2u * (k / 32u)};
  const cuuint64_t strides[1] = {(cuuint64_t)pf_pad4(cols) * 4u};
  const cuuint32_t box[2] = {128u, 2u * QG_SUBS};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

size_t prefill_operand_bytes(uint32_t rows, uint32_t k) {
  return pf_scale_offset(rows, k) + (size_t)(k / 32u) * 2u * pf_pad4(rows) * 4u;
}

cudaError_t launch_prefill_act_pack(const float* a, uint32_t m, uint32_t k, void* act, cudaStream_t st) {
  const uint32_t groups = m * (k / 32u);
  if (groups == 0) return cudaSuccess;
  uint16_t* aq = static_cast<uint16_t*>(act);
  float* asc = reinterpret_cast<float*>(static_cast<uint8_t*>(act) + pf_scale_offset(m, k));
  prefill_act_pack_kernel<<<(groups + 7u) / 8u, 256, 0, st>>>(a, m, k, aq, asc);
  return cudaGetLastError();
}

cudaError_t launch_prefill_w_prep(const uint8_t* w, uint32_t n, uint32_t k, void* wprep, cudaStream_t st) {
  const uint64_t warps = (uint64_t)n * (k / Q4K_ELEMS);
  if (warps == 0) return cudaSuccess;
  uint16_t* wq = static_cast<uint16_t*>(wprep);
  float* wsc = reinterpret_cast<float*>(static_cast<uint8_t*>(wprep) + pf_scale_offset(n, k));
  prefill_w_prep_kernel<<<(uint32_t)((warps + 7u) / 8u), 256, 0, st>>>(w, n, k, wq, wsc);
  return cudaGetLastError();
}

// C[m,n] (or C += with `accumulate`) from prepared operands (layouts above;
// k % 256 == 0, base pointers 1024-byte aligned); rows of C (and of every
// extra destination) ldc floats apart (0: n).  out_status:
// EOS_E_UNSUPPORTED when the tensor maps cannot be built.
cudaError_t launch_prefill_gemm(const void* act, const void* wprep, float* c, uint32_t m, uint32_t n, uint32_t k,
                                uint32_t* err, cudaStream_t st, int* out_status, bool accumulate,
                                float* const* c_extra, uint32_t n_extra, uint32_t ldc) {
  *out_status = EOS_OK;
  if (m == 0 || n == 0) return cudaSuccess;
  if (ldc == 0) ldc = n;
  if (n_extra > 7 || (n_extra > 0 && accumulate) || ldc < n) {
    *out_status = EOS_E_INVALID_ARG;
    return cudaSuccess;
  }
  const uint8_t* ab = static_cast<const uint8_t*>(act);
  const uint8_t* wb = static_cast<const uint8_t*>(wprep);
  CUtensorMap ma, mb, mas, mbs;
  if (!make_bf16_map(&ma, ab, m, k) || !make_bf16_map(&mb, wb, n, k) ||
      !make_scale_map(&mas, ab + pf_scale_offset(m, k), m, k) ||
      !make_scale_map(&mbs, wb + pf_scale_offset(n, k), n, k)) {
    *out_status = EOS_E_UNSUPPORTED;
    return cudaSuccess;
  }
  static SmemAttr attr;  // per device
  {
    const cudaError_t e = ensure_smem_attr((const void*)prefill_gemm_kernel, (int)QG_SMEM, attr, false);
    if (e != cudaSuccess) return e;
  }
  const dim3 grid((m + QG_BM - 1) / QG_BM, (n + QG_BN - 1) / QG_BN);
  PrefillParams prm{c, m, n, k, ldc, err, accumulate ? 1u : 0u, {}, n_extra};
  for (uint32_t x = 0; x < n_extra; ++x) prm.c_extra[x] = c_extra[x];
  prefill_gemm_kernel<<<grid, QG_THREADS, QG_SMEM, st>>>(ma, mb, mas, mbs, prm);
  return cudaGetLastError();
}

}  // namespace eos
