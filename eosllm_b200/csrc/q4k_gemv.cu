// q4k_gemv.cu -- Q4_K decode GEMV for sm_100a, bit-exact with the reference's
// production x86 path eosi_avx2_matmul_q4_k_int8
// (src/kernels/avx2/matmul_q4_k_int8.c:164-269).
//
// Activation packing -- the exact x86 arithmetic of quantize_sub32
// (:98-154) -- either runs inside the GEMV (each CTA packs the f32 vector
// into shared memory while its first weight stages stream in) or in
// act_pack_kernel, chained to the GEMV with programmatic dependent launch
// (PDL), when one packed vector feeds several GEMVs or m > 1.
//
// q4k_gemv_kernel: each CTA owns a contiguous slab of weight rows, cut into
// stages of R rows.  Warp w of NW takes stages w, w+NW, ... and streams them
// HBM -> shared memory with coalesced 16-byte cp.async copies through D
// buffers of its own, computing one stage while the next D-1 land.  Weight
// copies are issued before the PDL wait, so they overlap the previous
// kernel's tail.  Two lanes share a super-block: lane h (0/1) takes qs pairs
// 2h, 2h+1, i.e. sub-blocks 4h..4h+3: exact integer dp4a dots, then the
// reference's fp32 rescale terms with round-to-nearest intrinsics (no FMA
// contraction).  Lane 0 adds its four terms to 0, lane 1 continues that
// partial with its four, so the super-block partial is the reference's
// (((0 + t_0) + t_1) + ... + t_7).  Partials are then broadcast in
// super-block order and one lane per row adds them: every output is
// bit-identical to the CPU kernel.
//
// Shared-memory banking: a 16-byte load phase is 8 lanes = 4 super-blocks x
// 2 halves.  With R = 1 the 4 super-blocks are consecutive b (b*144 == 16b
// mod 128, halves at +64); with R >= 2 they are rows at a pitch == 32 (R=2)
// or 16 (R>=4) mod 128.  Activation records are 480 bytes (== 96 mod 128)
// with the second half at +272 (== 16 mod 128).  Every phase therefore hits
// 8 distinct 16-byte bank groups.
//
// Activation record (per super-block b, 480 bytes at 480 b; k % 256 == 0):
//   half h = 0, 1 at offset 272 h:
//     [0, 128)    int8 a_q of sub-blocks 4h .. 4h+3, source order
//     [128, 160)  per sub-block: {f32 scale, f32 (float)sum_aq} (the sum
//                 stored converted, exactly the reference's (float) cast at
//                 :256-261)
//   bytes [160, 272) and [432, 480) are padding.
#include "eos_common.cuh"
#include "eos_kernels.h"
#include "q4k_dot.cuh"

namespace eos {

// ---------------------------------------------------------------------------
// Activation packing kernel: one warp per 32-group.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) act_pack_kernel(const float* __restrict__ a, uint32_t m, uint32_t k,
                                                       uint8_t* __restrict__ out, int layout, uint32_t* zero_word) {
  pdl_trigger();  // let the dependent GEMV start streaming its weights
  pdl_wait();     // `a` may be the previous kernel's output
  // the error word of the GEMVs that follow starts at 0 (they report into it
  // only after their own PDL wait, i.e. after this grid has completed)
  if (zero_word != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *zero_word = 0u;
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
    uint8_t* r = out + (size_t)row * ((k >> 8) * kActRec);
    r[rec_aq_offset(g) + lane] = static_cast<uint8_t>(q);
    if (lane == 0) *reinterpret_cast<float2*>(r + rec_st_offset(g)) = make_float2(scale, (float)sum);
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
// Results to the host: 16-byte stores into mapped pinned memory, coalesced
// per warp into whole 128-byte lines on the PCIe link.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) copy_out_kernel(const uint4* src, uint4* dst, uint32_t n16) {
  pdl_trigger();  // the done-flag kernel may become resident (it waits for this grid)
  pdl_wait();     // src is the previous grid's output
  for (uint32_t i = blockIdx.x * 256u + threadIdx.x; i < n16; i += gridDim.x * 256u) dst[i] = src[i];
}

// One thread raises *flag (mapped host memory) once every kernel before it on
// the stream has completed: the host waits for the word instead of for the
// stream (no synchronisation call on the path of a host-pointer matmul).
// Launched with programmatic dependent launch: resident while the copy runs,
// it waits for the copy grid's completion (its stores performed), then
// fences at system scope before the flag's release store.
__global__ void done_flag_kernel(uint32_t* flag) {
  pdl_wait();
  __threadfence_system();
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(1u) : "memory");
}

cudaError_t launch_done_flag(uint32_t* flag, cudaStream_t st) {
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(1);
  lc.blockDim = dim3(1);
  lc.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  return cudaLaunchKernelEx(&lc, done_flag_kernel, flag);
}

cudaError_t launch_copy_out(const void* src, void* dst, size_t bytes, cudaStream_t st) {
  const uint32_t n16 = (uint32_t)(bytes >> 4);
  if (n16 == 0) return cudaSuccess;
  uint32_t blocks = (n16 + 255u) / 256u;
  if (blocks > 64u) blocks = 64u;
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(blocks);
  lc.blockDim = dim3(256);
  lc.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  return cudaLaunchKernelEx(&lc, copy_out_kernel, reinterpret_cast<const uint4*>(src), reinterpret_cast<uint4*>(dst),
                            n16);
}

// ---------------------------------------------------------------------------
// In-CTA activation packing into shared memory (fused path)
// ---------------------------------------------------------------------------
template <int NW>
__device__ __forceinline__ void pack_into_smem(const float* __restrict__ a, uint32_t k, uint8_t* act_s,
                                               uint32_t warp, uint32_t lane) {
  const uint32_t groups = k >> 5;
  for (uint32_t g0 = warp; g0 < groups; g0 += 4 * NW) {
    float v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t g = g0 + u * NW;
      v[u] = g < groups ? a[(g << 5) + lane] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t g = g0 + u * NW;
      if (g < groups) {  // warp-uniform
        float scale;
        int32_t sum;
        const int8_t q = quant_group32(v[u], scale, sum);
        act_s[rec_aq_offset(g) + lane] = static_cast<uint8_t>(q);
        if (lane == 0) *reinterpret_cast<float2*>(act_s + rec_st_offset(g)) = make_float2(scale, (float)sum);
      }
    }
  }
}

// Packed activation records global -> shared memory with every load of a
// round in flight before the first store: one L2 round trip per 8 x 16
// bytes a thread instead of one per 16 bytes (the records of a k = 11008
// row are 20.6 KB, five 16-byte rounds for 256 threads).
template <int NT>
__device__ __forceinline__ void copy_act_to_smem(const uint8_t* __restrict__ src, uint8_t* dst, uint32_t bytes) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
  uint4* d = reinterpret_cast<uint4*>(dst);
  const uint32_t n16 = bytes >> 4;
  for (uint32_t base = 0; base < n16; base += 8u * NT) {
    uint4 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t t = base + (uint32_t)j * NT + threadIdx.x;
      if (t < n16) v[j] = s[t];  // coherent loads: the previous grid wrote `src`
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t t = base + (uint32_t)j * NT + threadIdx.x;
      if (t < n16) d[t] = v[j];
    }
  }
}

// ---------------------------------------------------------------------------
// Q4_K GEMV
// ---------------------------------------------------------------------------
struct Q4kGemvParams {
  const uint8_t* w;    // n rows x row_bytes (GGUF Q4_K super-blocks)
  const uint8_t* act;  // packed activation records, act_bytes (packed path)
  const float* a;      // f32 activations, k (fused path)
  float* c;            // n outputs
  uint32_t n, k, nb, row_bytes, pitch, R, act_bytes;
  uint32_t cb, nch;  // column-major kernel: super-blocks per staged row chunk, chunks per row
  uint32_t* err;
  // further copies of every output (tensor-parallel push: other GPUs'
  // receive buffers, mapped through CUDA IPC), written after c
  float* c_extra[7];
  uint32_t n_extra;
  // tensor parallel (ll.epoch_word != nullptr): the activation records arrive
  // as (epoch, word) pairs from every rank (ll.in), and every output goes to
  // every rank as a pair (ll.out) instead of to c
  LLExchange ll;
};

// Packed activation records from a buffer of (epoch, word) pairs into shared
// memory (word i of the record layout is pair i), every load of a round in
// flight at once; a round is reloaded until all its pairs carry `epoch`.
// Padding words of the records (bytes [160, 272) and [432, 480) of each
// 480-byte record) are never written by producers and are not waited for.
// Returns false when the wait ran out.
template <int NT>
__device__ __forceinline__ bool copy_act_ll_to_smem(const LLExchange& x, uint32_t epoch, uint8_t* dst,
                                                    uint32_t bytes) {
  const uint32_t n16 = bytes >> 3;  // 16-byte units of the pair buffer (two words of the records each)
  uint64_t t0 = 0;
  for (uint32_t base = 0; base < n16; base += 8u * NT) {
    uint64_t lo[8], hi[8];
    bool ready;
    do {
      ready = true;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t t = base + (uint32_t)j * NT + threadIdx.x;
        if (t < n16) {
          ll_load2(x.in + 2u * t, lo[j], hi[j]);
          const uint32_t rw = (2u * t) % (kActRec / 4u);  // word within its record
          const bool pad = !(rw < 40u || (rw >= kActHalf / 4u && rw < kActHalf / 4u + 40u));
          if (!pad && ((uint32_t)(lo[j] >> 32) != epoch || (uint32_t)(hi[j] >> 32) != epoch)) ready = false;
        }
      }
      if (!ready && !ll_keep_waiting(x, t0)) return false;
    } while (!ready);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t t = base + (uint32_t)j * NT + threadIdx.x;
      if (t < n16) reinterpret_cast<uint2*>(dst)[t] = make_uint2((uint32_t)lo[j], (uint32_t)hi[j]);
    }
  }
  return true;
}

// After the PDL wait: the activations into shared memory -- packed in the CTA
// (fused path), copied from the packed records, or, tensor parallel, polled
// from the (epoch, word) pairs the ranks pushed.  On a timeout the CTA drains
// its weight copies and leaves (outputs unwritten, error bit set).
template <int NW>
__device__ __forceinline__ bool gemv_load_act(const Q4kGemvParams& p, uint8_t* act_s, uint32_t warp, uint32_t lane) {
  bool ok = true;
  if (p.ll.epoch_word != nullptr) {
    ok = copy_act_ll_to_smem<NW * 32>(p.ll, ll_epoch(p.ll, p.ll.in_add), act_s, p.act_bytes);
  } else if (p.a != nullptr) {
    pack_into_smem<NW>(p.a, p.k, act_s, warp, lane);
  } else {
    copy_act_to_smem<NW * 32>(p.act, act_s, p.act_bytes);
  }
  if (__syncthreads_and(ok)) return true;
  if (threadIdx.x == 0) report(p.ll.err, EOS_DEVERR_PEER);
  cp_async_wait<0>();
  return false;
}

// c[r] = v and the same value into every extra destination (other GPUs'
// buffers, plain stores over NVLink), or, tensor parallel, the pair
// (out_epoch, v) into every rank's buffer.
__device__ __forceinline__ void gemv_store(const Q4kGemvParams& p, uint32_t r, float v, uint32_t out_epoch) {
  if (p.ll.epoch_word != nullptr) {
    ll_put(p.ll, r, __float_as_uint(v), out_epoch);
    return;
  }
  p.c[r] = v;
  for (uint32_t j = 0; j < p.n_extra; ++j) p.c_extra[j][r] = v;
}

template <int NW, int D>
__global__ void __launch_bounds__(NW * 32, 1) q4k_gemv_kernel(const Q4kGemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t act_region = (p.act_bytes + 127u) & ~127u;
  uint8_t* act_s = smem;
  const uint32_t R = p.R, nb = p.nb, pitch = p.pitch, row_bytes = p.row_bytes;
  const uint32_t buf_bytes = R * pitch;
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  // per-warp partial buffers [R][nb] floats, then per-warp weight buffers
  const uint32_t pstride = (R * nb + 3u) & ~3u;
  const uint32_t part_region = (NW * pstride * 4u + 127u) & ~127u;
  float* part_w = reinterpret_cast<float*>(smem + act_region) + warp * pstride;
  uint8_t* wbuf = smem + act_region + part_region + warp * D * buf_bytes;

  const uint32_t r0 = (uint32_t)(((uint64_t)p.n * blockIdx.x) / gridDim.x);
  const uint32_t r1 = (uint32_t)(((uint64_t)p.n * (blockIdx.x + 1)) / gridDim.x);
  const uint32_t nrows = r1 - r0;
  const uint32_t nst = (nrows + R - 1) / R;
  const uint32_t cpr = row_bytes >> 4;  // 16-byte chunks per row
  const uint64_t pol_w = l2_policy_evict_first();

  auto issue = [&](uint32_t s, uint32_t slot) {
    if (s < nst) {
      const uint32_t rows = (nrows - s * R) < R ? (nrows - s * R) : R;
      const uint8_t* src = p.w + (size_t)(r0 + s * R) * row_bytes;
      uint8_t* dst = wbuf + slot * buf_bytes;
      for (uint32_t r = 0; r < rows; ++r)
        for (uint32_t t = lane; t < cpr; t += 32)
          cp_async16(dst + r * pitch + (t << 4), src + (size_t)r * row_bytes + (t << 4), pol_w);
    }
    cp_async_commit();  // one group per call, empty or not, keeps the counting uniform
  };

  // Weights do not depend on the previous kernel: start streaming them first.
#pragma unroll
  for (uint32_t d = 0; d < (uint32_t)D; ++d) issue(warp + d * NW, d);

  pdl_wait();  // the activations are the previous kernel's output
  if (!gemv_load_act<NW>(p, act_s, warp, lane)) return;
  const uint32_t out_epoch = p.ll.epoch_word != nullptr ? ll_epoch(p.ll, p.ll.out_add) : 0u;
  pdl_trigger();  // every CTA holds its activations: the next kernel may start

  const uint32_t h = lane & 1u;
  uint32_t i = 0;
  for (uint32_t s = warp; s < nst; s += NW, ++i) {
    const uint32_t slot = i % D;
    cp_async_wait<D - 1>();  // this warp's stage i has landed
    __syncwarp();
    const uint32_t rows = (nrows - s * R) < R ? (nrows - s * R) : R;
    const uint8_t* stage = wbuf + slot * buf_bytes;
    // item q = 2 * (b * rows + row) + h; the odd lane of each pair ends up
    // holding the super-block partial and parks it at part_w[row][b]
    const uint32_t units = rows * nb, items = 2u * units;
    for (uint32_t q0 = 0; q0 < items; q0 += 32) {
      const uint32_t u = (q0 + lane) >> 1;  // (b, row) unit of this lane
      float t[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      uint32_t row = 0, b = 0;
      if (u < units) {
        if (rows == R) {
          row = u & (R - 1u);
          b = u >> (31u - __clz(R));
        } else {
          b = u / rows;
          row = u - b * rows;
        }
        q4k_half_terms(stage + row * pitch + b * Q4K_BYTES, act_s + b * kActRec + h * kActHalf, h, t);
      }
      const float part = pair_partial(t, lane);
      if (u < units && h) part_w[row * nb + b] = part;
    }
    __syncwarp();  // partials parked, stage bytes no longer read
    issue(s + D * NW, slot);
    if (lane < rows) {
      // c[row] = 0; c[row] += partial_b for b in order (:194, :264)
      const float* pr = part_w + lane * nb;
      float acc = 0.0f;
      uint32_t b = 0;
      if ((nb & 3u) == 0) {
        for (; b < nb; b += 4) {
          const float4 v = *reinterpret_cast<const float4*>(pr + b);
          acc = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(acc, v.x), v.y), v.z), v.w);
        }
      }
      for (; b < nb; ++b) acc = __fadd_rn(acc, pr[b]);
      gemv_store(p, r0 + s * R + lane, acc, out_epoch);
    }
    __syncwarp();  // partial buffer free for the next stage
  }
  cp_async_wait<0>();  // never exit with copies still landing in shared memory
}

// Column-major variant: a warp stage is R rows; a lane PAIR owns one
// super-block column b (16 columns per pass) and computes all R rows of it,
// so each activation half-record is read from shared memory once per stage
// instead of once per row.  Long rows are streamed in chunks of p.cb
// super-blocks (p.nch chunks a row; p.nch == 1: whole rows): a warp takes
// row groups warp, warp + NW, ... and runs through the chunks of each in
// order, parking every super-block partial; after the last chunk one lane
// per row adds them in order.  Chunking keeps the staging buffers -- hence
// the CTA's shared memory -- independent of k, so long rows still fit two
// CTAs per SM.  Same terms, partials and ordered row sums as q4k_gemv_kernel,
// so outputs are bit-identical.  CHUNKED = false is the whole-row form
// (nch = 1, cb = nb known at compile time, no chunk bookkeeping).
// Staging is by TMA: lane 0 of a warp issues each stage as bulk copies
// (cp.async.bulk, one for whole rows, else one per row chunk) that complete
// on the slot's mbarrier -- two instructions a stage instead of 16-byte
// cp.async from every lane, which with ~150 KB in flight per SM stalled on
// the load/store unit (the whole sweep measured 4230 vs 3957 GB/s on a B200,
// bit-identical outputs).
template <int NW, int D, int R, bool CHUNKED>
__global__ void __launch_bounds__(NW * 32, 1) q4k_gemv_cols_kernel(const Q4kGemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t act_region = (p.act_bytes + 127u) & ~127u;
  uint8_t* act_s = smem;
  const uint32_t nb = p.nb, pitch = p.pitch, row_bytes = p.row_bytes;
  const uint32_t cb = CHUNKED ? p.cb : nb, nch = CHUNKED ? p.nch : 1u;
  const uint32_t buf_bytes = R * pitch;  // pitch = cb * Q4K_BYTES
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const uint32_t pstride = (R * nb + 3u) & ~3u;
  const uint32_t part_region = (NW * pstride * 4u + 127u) & ~127u;
  float* part_w = reinterpret_cast<float*>(smem + act_region) + warp * pstride;
  uint8_t* wbuf = smem + act_region + part_region + warp * D * buf_bytes;
  // one mbarrier per staging slot, after every warp's buffers
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + act_region + part_region + NW * D * buf_bytes) + warp * D;

  const uint32_t r0 = (uint32_t)(((uint64_t)p.n * blockIdx.x) / gridDim.x);
  const uint32_t r1 = (uint32_t)(((uint64_t)p.n * (blockIdx.x + 1)) / gridDim.x);
  const uint32_t nrows = r1 - r0;
  const uint32_t nst = (nrows + R - 1) / R;  // row groups of this CTA
  const uint64_t pol_w = l2_policy_evict_first();
  if (lane == 0) {
#pragma unroll
    for (uint32_t d = 0; d < (uint32_t)D; ++d) mbar_init(bars + d, 1u);
    fence_barrier_init();
  }
  __syncwarp();
  // this warp's stages in order: row groups warp, warp + NW, ..., each
  // through chunks 0 .. nch - 1.  Cursor (ig, ic) is the next stage to stage;
  // lane 0 issues it as TMA bulk copies (one for whole rows, else one per row)
  // completing on the slot's mbarrier.
  uint32_t ig = warp, ic = 0, issued = 0;
  auto issue = [&](uint32_t slot) {
    if (ig < nst) {
      if (lane == 0) {
        const uint32_t rows = (nrows - ig * R) < R ? (nrows - ig * R) : R;
        const uint32_t b0 = ic * cb, chunk = ((nb - b0) < cb ? (nb - b0) : cb) * Q4K_BYTES;
        const uint8_t* src = p.w + (size_t)(r0 + ig * R) * row_bytes + (size_t)b0 * Q4K_BYTES;
        uint8_t* dst = wbuf + slot * buf_bytes;
        mbar_arrive_expect_tx(bars + slot, rows * chunk);
        if (chunk == row_bytes && pitch == row_bytes) {
          bulk_g2s(dst, src, rows * chunk, bars + slot, pol_w);
        } else {
          for (uint32_t r = 0; r < rows; ++r) bulk_g2s(dst + r * pitch, src + (size_t)r * row_bytes, chunk, bars + slot, pol_w);
        }
      }
      ++issued;
      if (++ic == nch) {
        ic = 0;
        ig += NW;
      }
    }
  };
  // stages issued and not yet consumed, landed before an early exit
  auto drain = [&](uint32_t t) {
    for (; t < issued; ++t)
      if (!mbar_wait(bars + t % D, (t / D) & 1u) && lane == 0) report(p.err, EOS_DEVERR_DRAIN);
  };

#pragma unroll
  for (uint32_t d = 0; d < (uint32_t)D; ++d) issue(d);

  pdl_wait();
  if (!gemv_load_act<NW>(p, act_s, warp, lane)) {
    drain(0);
    return;
  }
  const uint32_t out_epoch = p.ll.epoch_word != nullptr ? ll_epoch(p.ll, p.ll.out_add) : 0u;
  pdl_trigger();

  const uint32_t h = lane & 1u;
  uint32_t g = warp, ch = 0;  // the stage computed now: row group g, chunk ch
  for (uint32_t t = 0; g < nst; ++t) {
    const uint32_t slot = t % D;
    if (!__all_sync(0xffffffffu, mbar_wait(bars + slot, (t / D) & 1u))) {
      if (lane == 0) report(p.err, EOS_DEVERR_WAIT_FULL);
      drain(t);
      return;
    }
    const uint32_t rows = (nrows - g * R) < R ? (nrows - g * R) : R;
    const uint32_t b0 = ch * cb, bn = (nb - b0) < cb ? (nb - b0) : cb;  // super-blocks of this chunk
    const uint8_t* stage = wbuf + slot * buf_bytes;
    for (uint32_t j0 = 0; j0 < bn; j0 += 16u) {
      const uint32_t j = j0 + (lane >> 1);
      const uint32_t jc = j < bn ? j : bn - 1u;
      float tr[R][4];
      q4k_half_terms_rows<R>(stage + jc * Q4K_BYTES, pitch, act_s + (b0 + jc) * kActRec + h * kActHalf, h, tr,
                             rows);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float part = pair_partial(tr[r], lane);
        if (h && j < bn && (uint32_t)r < rows) part_w[r * nb + b0 + j] = part;
      }
    }
    __syncwarp();  // every lane's reads of the slot have returned (their values are stored)
    issue(slot);
    if (ch == nch - 1u && lane < rows) {
      const float* pr = part_w + lane * nb;
      float acc = 0.0f;  // c = 0; c += partial_b in order (:194, :264)
      uint32_t b = 0;
      for (; b + 8u <= nb; b += 8u) {
        float v8[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) v8[q] = pr[b + q];
#pragma unroll
        for (int q = 0; q < 8; ++q) acc = __fadd_rn(acc, v8[q]);
      }
      for (; b < nb; ++b) acc = __fadd_rn(acc, pr[b]);
      gemv_store(p, r0 + g * R + lane, acc, out_epoch);
    }
    __syncwarp();
    if (++ch == nch) {
      ch = 0;
      g += NW;
    }
  }
}

// Fallback without staging (rows too long for shared memory): one warp per
// weight row from global memory, packed activations in global memory.
__global__ void __launch_bounds__(256) q4k_gemv_simple_kernel(const uint8_t* __restrict__ w,
                                                              const uint8_t* __restrict__ act, float* __restrict__ c,
                                                              uint32_t n, uint32_t k) {
  pdl_wait();
  const uint32_t row = blockIdx.x * 8u + (threadIdx.x >> 5), lane = threadIdx.x & 31u;
  if (row >= n) return;  // warp-uniform
  const uint32_t nb = k / Q4K_ELEMS, h = lane & 1u;
  const uint8_t* rp = w + (size_t)row * nb * Q4K_BYTES;
  float acc = 0.0f;
  for (uint32_t b0 = 0; b0 < nb; b0 += 16) {
    const uint32_t b = b0 + (lane >> 1);
    float t[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (b < nb) q4k_half_terms(rp + b * Q4K_BYTES, act + (size_t)b * kActRec + h * kActHalf, h, t);
    const float part = pair_partial(t, lane);
    const uint32_t cnt = (nb - b0) < 16u ? (nb - b0) : 16u;
    for (uint32_t j = 0; j < cnt; ++j) acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, part, 2u * j + 1u));
  }
  if (lane == 0) c[row] = acc;
}

// ---------------------------------------------------------------------------
// Host-side launchers
// ---------------------------------------------------------------------------
size_t act_layout_bytes(uint32_t m, uint32_t k, int layout) {
  if (layout == EOS_ACT_LAYOUT_GEMV) return (size_t)m * (k / Q4K_ELEMS) * kActRec;
  return (size_t)m * k + (size_t)m * (k >> 5) * 8u;
}

cudaError_t launch_act_pack(const float* a, uint32_t m, uint32_t k, uint8_t* out, int layout, cudaStream_t st,
                            uint32_t* zero_word) {
  const uint32_t groups = m * (k >> 5);
  const uint32_t blocks = (groups + 7u) / 8u;
  if (blocks == 0) return zero_word != nullptr ? cudaMemsetAsync(zero_word, 0, 4, st) : cudaSuccess;
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(blocks);
  lc.blockDim = dim3(256);
  lc.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  return cudaLaunchKernelEx(&lc, act_pack_kernel, a, m, k, out, layout, zero_word);
}

namespace {
struct GemvConfig {
  void (*fn)(const Q4kGemvParams);
  int nw, d;
  int cols;      // 0: q4k_gemv_kernel (rows per stage chosen at launch); R: q4k_gemv_cols_kernel<., ., R, .>
  SmemAttr attr;  // dynamic shared memory allowed so far, per device
  void (*fn_chunked)(const Q4kGemvParams);  // column-major: rows staged in chunks
  SmemAttr attr_chunked;
};
#define EOS_COLS_CFG(NW, D, R) \
  { q4k_gemv_cols_kernel<NW, D, R, false>, NW, D, R, {}, q4k_gemv_cols_kernel<NW, D, R, true>, {} }
GemvConfig g_cfgs[] = {
    {q4k_gemv_kernel<16, 4>, 16, 4, 0, {}, nullptr, {}}, {q4k_gemv_kernel<16, 3>, 16, 3, 0, {}, nullptr, {}},
    {q4k_gemv_kernel<16, 2>, 16, 2, 0, {}, nullptr, {}}, {q4k_gemv_kernel<20, 3>, 20, 3, 0, {}, nullptr, {}},
    {q4k_gemv_kernel<8, 4>, 8, 4, 0, {}, nullptr, {}},   {q4k_gemv_kernel<12, 4>, 12, 4, 0, {}, nullptr, {}},
    {q4k_gemv_kernel<24, 2>, 24, 2, 0, {}, nullptr, {}}, {q4k_gemv_kernel<8, 6>, 8, 6, 0, {}, nullptr, {}},
    {q4k_gemv_kernel<20, 2>, 20, 2, 0, {}, nullptr, {}}, {q4k_gemv_kernel<12, 3>, 12, 3, 0, {}, nullptr, {}},
    {q4k_gemv_kernel<16, 2>, 16, 2, 0, {}, nullptr, {}}, {q4k_gemv_kernel<10, 4>, 10, 4, 0, {}, nullptr, {}},
    EOS_COLS_CFG(12, 2, 4), EOS_COLS_CFG(16, 3, 2), EOS_COLS_CFG(8, 3, 4),  EOS_COLS_CFG(16, 2, 2),
    EOS_COLS_CFG(8, 2, 2),  EOS_COLS_CFG(12, 3, 2), EOS_COLS_CFG(16, 2, 1), EOS_COLS_CFG(8, 4, 2)};
#undef EOS_COLS_CFG
constexpr int kNumCfgs = sizeof(g_cfgs) / sizeof(g_cfgs[0]);
int g_q4k_variant = -1;  // kernel config override (-1: automatic)
int g_q4k_rows = 0;      // rows-per-stage override (0: automatic)
int g_q4k_ctas = 0;      // CTAs-per-SM override (0: automatic)
int g_q4k_chunk = 0;     // column-major row chunking override (0: automatic)
}  // namespace

void set_q4k_gemv_variant(int v) {
  // v < 0: automatic.  Else v = cfg + 32 * rows + 512 * ctas_per_sm +
  // 4096 * chunk, each field 0 = automatic (rows applies to the row-major
  // kernels only; chunk to the column-major ones: 1 = whole rows, c >= 2 =
  // chunks of 8 (c - 1) super-blocks).
  g_q4k_variant = v < 0 ? -1 : (v % 32);
  g_q4k_rows = v < 0 ? 0 : ((v / 32) % 16);
  g_q4k_ctas = v < 0 ? 0 : ((v / 512) % 8);
  g_q4k_chunk = v < 0 ? 0 : (v / 4096);
}

cudaError_t launch_q4k_gemv(const uint8_t* w, const uint8_t* act, const float* a, float* c, uint32_t n, uint32_t k,
                            uint32_t* err, int num_sms, int max_smem, bool pdl, cudaStream_t st, int* out_status,
                            float* const* c_extra, uint32_t n_extra, const LLExchange* ll) {
  if (n_extra > 7) {
    *out_status = EOS_E_INVALID_ARG;
    return cudaSuccess;
  }
  *out_status = EOS_OK;
  if (n == 0) return cudaSuccess;
  const uint32_t nb = k / Q4K_ELEMS;
  const uint32_t row_bytes = nb * Q4K_BYTES;
  const uint32_t act_bytes = nb * kActRec;
  const uint32_t act_region = (act_bytes + 127u) & ~127u;
  // row-major kernel: rows per stage give at least 32 half-super-blocks
  // (one per lane) per stage; rows padded to a bank-spreading pitch
  uint32_t R_rm = 1;
  while (R_rm < 16u && 2u * R_rm * nb < 32u) R_rm <<= 1;
  if (g_q4k_rows == 1 || g_q4k_rows == 2 || g_q4k_rows == 4 || g_q4k_rows == 8) R_rm = (uint32_t)g_q4k_rows;
  const uint32_t target = R_rm == 1 ? 0u : (R_rm == 2 ? 32u : 16u);
  const uint32_t pitch_rm = row_bytes + ((target - (row_bytes & 127u)) & 127u);
  // column-major kernels: R rows per stage, unpadded (a load phase spans
  // four columns of one row, always distinct banks), staged whole -- or,
  // when whole rows would leave room for one CTA per SM only, in chunks of
  // 16 super-blocks, so that two CTAs (and the next kernel's) fit an SM
  auto smem_with = [&](const GemvConfig& g, uint32_t R, uint32_t pitch) -> uint32_t {
    const uint32_t part = ((uint32_t)g.nw * ((R * nb + 3u) & ~3u) * 4u + 127u) & ~127u;
    const uint32_t bars = g.cols ? (uint32_t)(g.nw * g.d) * 8u : 0u;  // the column-major kernel's mbarriers
    return act_region + part + (uint32_t)(g.nw * g.d) * R * pitch + bars;
  };
  auto geom = [&](const GemvConfig& g, uint32_t& R, uint32_t& pitch, uint32_t& cb) {
    R = g.cols ? (uint32_t)g.cols : R_rm;
    cb = nb;
    pitch = g.cols ? row_bytes : pitch_rm;
    if (!g.cols) return;
    if (g_q4k_chunk >= 2) {
      cb = 8u * (uint32_t)(g_q4k_chunk - 1);
    } else if (g_q4k_chunk == 0 && nb > 16u &&
               (uint32_t)(max_smem + 1024) / (smem_with(g, R, row_bytes) + 1024u) < 2u) {
      cb = 16u;
    }
    if (cb > nb) cb = nb;
    if (cb == 0) cb = 1;  // k = 0: no super-blocks, every output is c = 0
    pitch = cb * Q4K_BYTES;
  };
  auto smem_of = [&](const GemvConfig& g) -> uint32_t {
    uint32_t R, pitch, cb;
    geom(g, R, pitch, cb);
    return smem_with(g, R, pitch);
  };
  // first configuration that fits: column-major with activation reuse over
  // several rows, then the row-major pipelines
  int pick = -1;
  if (g_q4k_variant >= 0 && g_q4k_variant < kNumCfgs) {
    pick = g_q4k_variant;
  } else {
    const int order[] = {16, 15, 12, 13, 18, 0, 1, 2, 4};
    for (int o : order)
      if (smem_of(g_cfgs[o]) <= (uint32_t)max_smem) {
        pick = o;
        break;
      }
    if (pick < 0) pick = 2;
  }
  GemvConfig& cfg = g_cfgs[pick];
  uint32_t R, pitch, cb;
  geom(cfg, R, pitch, cb);
  const uint32_t smem = smem_of(cfg);
  if (smem > (uint32_t)max_smem) {  // rows too long to stage: unstaged kernel
    // it reads packed activations, writes one destination, exchanges nothing
    if (act == nullptr || n_extra != 0 || (ll != nullptr && ll->epoch_word != nullptr)) {
      *out_status = EOS_E_UNSUPPORTED;
      return cudaSuccess;
    }
    q4k_gemv_simple_kernel<<<(n + 7u) / 8u, 256, 0, st>>>(w, act, c, n, k);
    return cudaGetLastError();
  }
  const uint32_t nch = nb == 0 ? 1u : (nb + cb - 1u) / cb;
  const bool chunked = nch > 1u;  // only column-major configs ever split rows
  void (*fn)(const Q4kGemvParams) = chunked ? cfg.fn_chunked : cfg.fn;
  {
    // on this device; largest carveout so the next kernel's CTAs can share
    // the SM (PDL overlap)
    const cudaError_t e = ensure_smem_attr((const void*)fn, (int)smem, chunked ? cfg.attr_chunked : cfg.attr);
    if (e != cudaSuccess) return e;
  }
  uint32_t cps = (uint32_t)(max_smem + 1024) / (smem + 1024);
  if (cps > 4u) cps = 4u;
  if (cps < 1u) cps = 1u;
  if (g_q4k_ctas > 0) cps = (uint32_t)g_q4k_ctas;
  uint32_t grid = (uint32_t)num_sms * cps;
  const uint32_t max_grid = (n + R - 1) / R;
  if (grid > max_grid) grid = max_grid;
  Q4kGemvParams prm{w, act, a, c, n, k, nb, row_bytes, pitch, R, act_bytes, cb, nch, err, {}, n_extra, {}};
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
  lc.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&lc, fn, prm);
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
