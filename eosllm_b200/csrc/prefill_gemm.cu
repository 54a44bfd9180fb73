// prefill_gemm.cu -- batched (m > 1) Q4_K matmul on the sm_100a tensor cores
// (tcgen05 / TMEM / TMA): C[m,n] = A[m,k] . deq(W)[n,k]^T for prompt
// processing, where the decode GEMV's one-row-at-a-time form would leave the
// tensor cores idle.
//
// Numerics.  The reference computes every output with its int8 path
// (src/kernels/avx2/matmul_q4_k_int8.c:164-269): activations quantized per 32
// by quantize_sub32 (a_q, scale as), weights as (d*sc)*q - dmin*m.  In exact
// arithmetic that is sum_p A'_p W'_p with A' = as * a_q and W' = d*sc*q - dmin*m
// (the scalar dequant order, src/kernels/scalar/matmul_q4_k.c:79-98).  Here A'
// and W' are formed exactly as the reference's arithmetic does (same packing
// kernel, same fp32 operations), split into bf16 hi + lo parts, and the
// product is taken as hi*hi + lo*hi + hi*lo: three kind::f16 MMAs per K step,
// f32 accumulation in TMEM.  The dropped lo*lo term and the bf16 rounding of
// lo leave ~2^-16 relative error per product, so outputs agree with the int8
// reference to fp32-summation level (~1e-5 relative); the bound the tests
// state is 1e-3.  Non-finite activations give non-finite outputs (not
// bit-matched).
//
// Kernel: one CTA per 128 x 256 output tile, 128 threads.  Thread 0 is the
// TMA producer, thread 32 the MMA issuer, all four warps the epilogue (warp w
// reads TMEM lanes 32w..32w+31).  Per 64-wide K block a stage holds four
// 128B-swizzled bf16 tiles (A hi/lo 128x64, W hi/lo 256x64) = 96 KB; two
// stages.  Each 16-wide K step issues three tcgen05.mma (M128 N256 K16) into
// a 256-column f32 accumulator; tcgen05.commit frees a stage when its MMAs
// complete.  TMA boxes start at K offsets that are multiples of 64 elements
// (128 bytes), so every x coordinate is 16-byte aligned; no multicast.
//
// Waits are bounded (EOS_WAIT_LIMIT_NS): on a timeout the thread records an
// error bit and stops issuing; the MMA issuer always commits the "done"
// barrier after its last MMA (MMAs complete on their own), the producer waits
// (bounded) for its last copies, and TMEM is freed only after the done
// barrier.
#include <cuda.h>
#include <cuda_bf16.h>

#include "eos_common.cuh"
#include "eos_kernels.h"
#include "eosllm_cuda.h"

namespace eos {

constexpr uint32_t PG_BM = 128, PG_BN = 256, PG_BK = 64, PG_STAGES = 2;
constexpr uint32_t PG_A_BYTES = PG_BM * PG_BK * 2;                    // 16 KB
constexpr uint32_t PG_B_BYTES = PG_BN * PG_BK * 2;                    // 32 KB
constexpr uint32_t PG_STAGE_BYTES = 2 * PG_A_BYTES + 2 * PG_B_BYTES;  // 96 KB
constexpr uint32_t PG_SMEM = PG_STAGES * PG_STAGE_BYTES + 1024 + 256;
constexpr uint32_t PG_TMEM_COLS = 256;

// ---------------------------------------------------------------------------
// Operand preparation
// ---------------------------------------------------------------------------
__device__ __forceinline__ void split_bf16(float x, __nv_bfloat16& hi, __nv_bfloat16& lo) {
  hi = __float2bfloat16_rn(x);
  lo = __float2bfloat16_rn(__fsub_rn(x, __bfloat162float(hi)));
}

// A'[i] = scale * a_q[i] with the exact quantize_sub32 packing
// (matmul_q4_k_int8.c:98-154), one warp per 32-group.
__global__ void __launch_bounds__(256) prefill_act_split_kernel(const float* __restrict__ a, uint32_t groups,
                                                                __nv_bfloat16* __restrict__ hi,
                                                                __nv_bfloat16* __restrict__ lo) {
  const uint32_t g = blockIdx.x * 8u + (threadIdx.x >> 5), lane = threadIdx.x & 31u;
  if (g >= groups) return;  // warp-uniform
  const size_t i = (size_t)g * 32u + lane;
  float scale;
  int32_t sum;
  const int8_t q = quant_group32(a[i], scale, sum);
  split_bf16(__fmul_rn(scale, (float)q), hi[i], lo[i]);
}

// W'[i] = (d*sc)*q - dmin*m (src/kernels/scalar/matmul_q4_k.c:79-98), one
// thread per 32-weight sub-block.
__global__ void __launch_bounds__(256) prefill_w_split_kernel(const uint8_t* __restrict__ w, uint32_t subblocks,
                                                              __nv_bfloat16* __restrict__ hi,
                                                              __nv_bfloat16* __restrict__ lo) {
  const uint32_t t = blockIdx.x * 256u + threadIdx.x;
  if (t >= subblocks) return;
  const uint32_t b = t >> 3, s = t & 7u;  // super-block, sub-block
  const uint8_t* blk = w + (size_t)b * Q4K_BYTES;
  const float d = f16_bits_to_f32(blk[0] | (blk[1] << 8)), dmin = f16_bits_to_f32(blk[2] | (blk[3] << 8));
  uint32_t sc, m;
  q4k_scale_min((int)s, blk + 4, sc, m);
  const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)m);
  // sub-block s: qs bytes 32*(s/2) .. +31, low nibbles for even s, high for odd
  const uint8_t* qs = blk + 16 + 32u * (s >> 1);
  const uint32_t shift = (s & 1u) * 4u;
  const size_t o = (size_t)b * Q4K_ELEMS + s * 32u;
#pragma unroll 4
  for (uint32_t l = 0; l < 32; ++l) {
    const float v = __fsub_rn(__fmul_rn(d1, (float)((qs[l] >> shift) & 15u)), m1);
    split_bf16(v, hi[o + l], lo[o + l]);
  }
}

// ---------------------------------------------------------------------------
// tcgen05 / TMA helpers
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor of a K-major, 128B-swizzled tile whose rows
// are 128 bytes (64 bf16) and whose 8-row groups are 1024 bytes apart: start
// address >> 4, LBO 16 B (unused for swizzled K-major), SBO 1024 B,
// version 1, layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t pg_sw128_desc(uint32_t smem_addr) {
  uint64_t dsc = (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  dsc |= (uint64_t)1u << 16;
  dsc |= (uint64_t)(1024u >> 4) << 32;
  dsc |= (uint64_t)1u << 46;
  dsc |= (uint64_t)2u << 61;
  return dsc;
}

// Instruction descriptor: D f32, A and B bf16, both K-major, M = 128, N = 256.
constexpr uint32_t PG_IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((PG_BN >> 3) << 17) | ((PG_BM >> 4) << 24);

__device__ __forceinline__ void pg_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(PG_IDESC), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

__device__ __forceinline__ void pg_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void pg_tma_2d(void* dst, const CUtensorMap* map, uint32_t x, uint32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ---------------------------------------------------------------------------
// GEMM
// ---------------------------------------------------------------------------
struct PrefillParams {
  float* c;
  uint32_t m, n, k;
  uint32_t* err;
};

__global__ void __launch_bounds__(128, 1)
    prefill_gemm_kernel(const __grid_constant__ CUtensorMap map_ahi, const __grid_constant__ CUtensorMap map_alo,
                        const __grid_constant__ CUtensorMap map_bhi, const __grid_constant__ CUtensorMap map_blo,
                        const PrefillParams p) {
  extern __shared__ uint8_t pg_smem_raw[];
  // 1024-byte aligned stage buffers (128B swizzle atoms)
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(pg_smem_raw) + 1023u) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + PG_STAGES * PG_STAGE_BYTES);
  uint64_t* empty = full + PG_STAGES;
  uint64_t* done = empty + PG_STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
  const uint32_t m0 = blockIdx.y * PG_BM, n0 = blockIdx.x * PG_BN;
  const uint32_t nkb = p.k / PG_BK;

  if (tid == 0) {
    for (uint32_t s = 0; s < PG_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_barrier_init();
  }
  if (warp == 0) {  // TMEM accumulator: 128 lanes x 256 f32 columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(PG_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto sa_hi = [&](uint32_t s) { return smem + s * PG_STAGE_BYTES; };
  auto sa_lo = [&](uint32_t s) { return smem + s * PG_STAGE_BYTES + PG_A_BYTES; };
  auto sb_hi = [&](uint32_t s) { return smem + s * PG_STAGE_BYTES + 2 * PG_A_BYTES; };
  auto sb_lo = [&](uint32_t s) { return smem + s * PG_STAGE_BYTES + 2 * PG_A_BYTES + PG_B_BYTES; };

  if (tid == 0) {
    // ---- TMA producer ----
    uint32_t issued = 0;
    for (uint32_t kb = 0; kb < nkb; ++kb) {
      const uint32_t s = kb % PG_STAGES;
      if (kb >= PG_STAGES && !mbar_wait(&empty[s], ((kb / PG_STAGES) - 1u) & 1u)) {
        report(p.err, EOS_DEVERR_WAIT_EMPTY);
        break;
      }
      mbar_arrive_expect_tx(&full[s], PG_STAGE_BYTES);
      const uint32_t x = kb * PG_BK;
      pg_tma_2d(sa_hi(s), &map_ahi, x, m0, &full[s]);
      pg_tma_2d(sa_lo(s), &map_alo, x, m0, &full[s]);
      pg_tma_2d(sb_hi(s), &map_bhi, x, n0, &full[s]);
      pg_tma_2d(sb_lo(s), &map_blo, x, n0, &full[s]);
      issued = kb + 1;
    }
    // never leave copies in flight: the last use of every stage has landed
    for (uint32_t kb = issued > PG_STAGES ? issued - PG_STAGES : 0u; kb < issued; ++kb)
      if (!mbar_wait(&full[kb % PG_STAGES], (kb / PG_STAGES) & 1u)) report(p.err, EOS_DEVERR_DRAIN);
  } else if (tid == 32) {
    // ---- MMA issuer ----
    for (uint32_t kb = 0; kb < nkb; ++kb) {
      const uint32_t s = kb % PG_STAGES;
      if (!mbar_wait(&full[s], (kb / PG_STAGES) & 1u)) {
        report(p.err, EOS_DEVERR_WAIT_FULL);
        break;
      }
      tc_fence_after();
      const uint64_t ahi = pg_sw128_desc(smem_u32(sa_hi(s))), alo = pg_sw128_desc(smem_u32(sa_lo(s)));
      const uint64_t bhi = pg_sw128_desc(smem_u32(sb_hi(s))), blo = pg_sw128_desc(smem_u32(sb_lo(s)));
#pragma unroll
      for (uint32_t kk = 0; kk < PG_BK / 16u; ++kk) {
        const uint64_t adv = (uint64_t)(kk * 2u);  // 16 bf16 = 32 bytes along K, in 16-byte units
        pg_mma(tmem, ahi + adv, bhi + adv, (kb | kk) != 0u ? 1u : 0u);
        pg_mma(tmem, alo + adv, bhi + adv, 1u);
        pg_mma(tmem, ahi + adv, blo + adv, 1u);
      }
      pg_commit(&empty[s]);  // stage s free once these MMAs have read it
    }
    pg_commit(done);  // every MMA issued above has completed
  }
  __syncwarp();

  // ---- epilogue: TMEM -> registers -> global ----
  // (warp-uniform: tcgen05.ld is .sync.aligned)
  const bool ok = __all_sync(0xffffffffu, mbar_wait(done, 0u)) != 0;
  if (!ok && lane == 0) report(p.err, EOS_DEVERR_WAIT_FULL);
  tc_fence_after();
  const uint32_t row = m0 + warp * 32u + lane;
  if (ok) {
#pragma unroll 1
    for (uint32_t c0 = 0; c0 < PG_BN; c0 += 32u) {
      uint32_t r[32];
      const uint32_t taddr = tmem + ((warp * 32u) << 16) + c0;
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
          "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
          "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
          : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
            "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
            "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
            "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
          : "r"(taddr)
          : "memory");
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      if (row < p.m) {
        float* crow = p.c + (size_t)row * p.n + n0 + c0;
        if (n0 + c0 + 32u <= p.n && (p.n & 3u) == 0) {
#pragma unroll
          for (uint32_t j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(crow + j) = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                                               __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
        } else {
#pragma unroll
          for (uint32_t j = 0; j < 32; ++j)
            if (n0 + c0 + j < p.n) crow[j] = __uint_as_float(r[j]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  // the done barrier follows the last MMA (MMAs wait on nothing, so it always
  // completes); free the accumulator
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(PG_TMEM_COLS) : "memory");
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
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// rows x k bf16 row-major, boxes of box_rows x 64 with the 128-byte swizzle
bool make_map(CUtensorMap* map, const void* base, uint32_t rows, uint32_t k, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {k, rows};
  const cuuint64_t strides[1] = {(cuuint64_t)k * 2u};
  const cuuint32_t box[2] = {PG_BK, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

cudaError_t launch_prefill_act_split(const float* a, uint32_t m, uint32_t k, void* hi, void* lo, cudaStream_t st) {
  const uint32_t groups = m * (k / 32u);
  if (groups == 0) return cudaSuccess;
  prefill_act_split_kernel<<<(groups + 7u) / 8u, 256, 0, st>>>(a, groups, static_cast<__nv_bfloat16*>(hi),
                                                               static_cast<__nv_bfloat16*>(lo));
  return cudaGetLastError();
}

cudaError_t launch_prefill_w_split(const uint8_t* w, uint32_t n, uint32_t k, void* hi, void* lo, cudaStream_t st) {
  const uint32_t sub = n * (k / 32u);
  if (sub == 0) return cudaSuccess;
  prefill_w_split_kernel<<<(sub + 255u) / 256u, 256, 0, st>>>(w, sub, static_cast<__nv_bfloat16*>(hi),
                                                              static_cast<__nv_bfloat16*>(lo));
  return cudaGetLastError();
}

// C[m,n] from split operands (bf16 row-major [m][k] and [n][k], all 16-byte
// aligned, k % 64 == 0).  out_status: EOS_E_UNSUPPORTED when the tensor maps
// cannot be built.
cudaError_t launch_prefill_gemm(const void* a_hi, const void* a_lo, const void* w_hi, const void* w_lo, float* c,
                                uint32_t m, uint32_t n, uint32_t k, uint32_t* err, cudaStream_t st, int* out_status) {
  *out_status = EOS_OK;
  if (m == 0 || n == 0) return cudaSuccess;
  CUtensorMap ma_hi, ma_lo, mb_hi, mb_lo;
  if (!make_map(&ma_hi, a_hi, m, k, PG_BM) || !make_map(&ma_lo, a_lo, m, k, PG_BM) ||
      !make_map(&mb_hi, w_hi, n, k, PG_BN) || !make_map(&mb_lo, w_lo, n, k, PG_BN)) {
    *out_status = EOS_E_UNSUPPORTED;
    return cudaSuccess;
  }
  static bool attr_set = false;
  if (!attr_set) {
    const cudaError_t e = cudaFuncSetAttribute(prefill_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)PG_SMEM);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  const dim3 grid((n + PG_BN - 1) / PG_BN, (m + PG_BM - 1) / PG_BM);
  PrefillParams prm{c, m, n, k, err};
  prefill_gemm_kernel<<<grid, 128, PG_SMEM, st>>>(ma_hi, ma_lo, mb_hi, mb_lo, prm);
  return cudaGetLastError();
}

}  // namespace eos
