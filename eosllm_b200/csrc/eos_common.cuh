// eos_common.cuh -- shared device helpers for the sm_100a quantized matmul
// kernels: status codes, Q4_K/Q8_0 block constants, mbarrier + bulk-async
// (TMA 1-D) copies, programmatic dependent launch, bounded waits.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

// eos_status_t values of the reference ABI (include/eosllm/eosllm.h:66-77).
enum {
  EOS_OK = 0,
  EOS_E_INVALID_ARG = 1,
  EOS_E_OUT_OF_MEMORY = 2,
  EOS_E_UNSUPPORTED = 3,
  EOS_E_FORMAT = 4,
  EOS_E_NOT_FOUND = 6,
  EOS_E_DEADLINE = 7,
  EOS_E_IO = 8,
  EOS_E_INTERNAL = 9
};

// eos_dtype_t values of the reference ABI (include/eosllm/tensor.h:22-37).
enum { EOS_DT_F32 = 0, EOS_DT_F16 = 1, EOS_DT_Q8_0 = 32, EOS_DT_Q4_K = 33 };

// GGUF block layouts (src/kernels/scalar/scalar.h:239-243).
constexpr uint32_t Q4K_ELEMS = 256, Q4K_BYTES = 144;
constexpr uint32_t Q80_ELEMS = 32, Q80_BYTES = 34;

// Device-side error bits, OR-ed into a host-visible word by kernels whose
// bounded waits ran out.  The host turns a non-zero word into EOS_E_INTERNAL.
enum : uint32_t {
  EOS_DEVERR_WAIT_FULL = 1u << 0,   // consumer gave up waiting for a stage
  EOS_DEVERR_WAIT_EMPTY = 1u << 1,  // producer gave up waiting for a free slot
  EOS_DEVERR_WAIT_ACT = 1u << 2,    // activation tile never arrived
  EOS_DEVERR_DRAIN = 1u << 3,       // in-flight copies did not drain on exit
  EOS_DEVERR_PEER = 1u << 4,        // a peer flag wait ran out
};

// One second: the bound on every spin-wait in this library's kernels.
constexpr uint64_t EOS_WAIT_LIMIT_NS = 1000000000ull;

namespace eos {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarrier ----------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Makes initialised barriers visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on phase `parity`: true when the phase completed, false when
// EOS_WAIT_LIMIT_NS elapsed first (the caller records an error and leaves).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > EOS_WAIT_LIMIT_NS) return false;
  }
  return true;
}

// ---- bulk async copy (TMA, 1-D): global -> this CTA's shared memory ----
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---- 16-byte async copies global -> shared (per-thread groups) ----------
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint64_t policy) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "l"(policy)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---- low-latency exchange (tensor-parallel decode) -----------------------
// Every 32-bit word of an exchanged vector travels together with the epoch
// of the exchange in ONE aligned 64-bit store (epoch in the high half), so a
// consumer needs no separate flag: it polls the words themselves, in its own
// GPU's memory, until each carries the expected epoch.  A 64-bit access is
// single-copy atomic, so a word is never seen without its epoch, and the
// producers' stores leave while the producing kernel still runs -- the
// exchange costs one NVLink trip after the last store instead of a kernel
// completion, a system fence and a flag trip.  Epochs only grow
// (step * exchanges_per_step + exchange + 1), so buffers need no clearing;
// a word is rewritten with the next epoch only after its reader has passed a
// later exchange that the writer waited for.
struct LLExchange {
  const uint32_t* epoch_word;  // completed steps; nullptr: no low-latency exchange (one GPU)
  uint32_t mul;                // exchanges per step
  uint32_t in_add, out_add;    // epoch = *epoch_word * mul + add, of what is read / written
  const uint64_t* in;          // consumer: this rank's buffer of (epoch, word) pairs
  uint64_t* out[8];            // producer: the same buffer of every rank (own included)
  uint32_t n_out;
  const uint32_t* limit_us;    // bound on a consumer's wait, in microseconds
  uint32_t* err;               // EOS_DEVERR_PEER when a wait runs out
};

__device__ __forceinline__ uint32_t ll_epoch(const LLExchange& x, uint32_t add) { return *x.epoch_word * x.mul + add; }

// Word i of the exchanged vector, with `epoch`, into every destination.
__device__ __forceinline__ void ll_put(const LLExchange& x, size_t i, uint32_t word, uint32_t epoch) {
  const uint64_t v = ((uint64_t)epoch << 32) | word;
  for (uint32_t j = 0; j < x.n_out; ++j)
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(x.out[j] + i), "l"(v) : "memory");
}

// Two consecutive pairs (16-byte aligned): each 64-bit half is read atomically.
__device__ __forceinline__ void ll_load2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// A consumer thread's wait budget: false once the limit has passed since its
// first unsuccessful poll (t0), or once an earlier exchange of the step lost
// a peer.
__device__ __forceinline__ bool ll_keep_waiting(const LLExchange& x, uint64_t& t0) {
  const uint64_t now = global_timer_ns();
  if (t0 == 0) {
    t0 = now;
    return true;
  }
  if (now - t0 > (uint64_t)*x.limit_us * 1000ull) return false;
  return !(x.err != nullptr && (*(volatile const uint32_t*)x.err & EOS_DEVERR_PEER) != 0u);
}

// ---- programmatic dependent launch --------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void report(uint32_t* err, uint32_t bits) {
  if (err) atomicOr(err, bits);
}

// ---- tensor-parallel handshakes (device-resident decoder) ---------------
// System-scope release store / acquire load of a flag word that other GPUs
// write through CUDA IPC mappings.
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One exchange of the tensor-parallel decoder: the ranks have pushed data
// into each other's memory (plain stores over NVLink by the kernel before the
// one that runs the handshake), and the consumer must not read its own copy
// before every source's push is visible.  Flag values are epochs,
// *epoch_word * mul + add, that only grow, so flags need no reset.
struct XchgSync {
  uint32_t world;              // > 1: the handshake runs
  uint32_t rank;               // this rank
  uint32_t* pub[8];            // this rank's flag word in every rank's receive words (own included)
  const uint32_t* wait;        // this rank's receive words: [q] is raised by rank q
  const uint32_t* epoch_word;  // completed steps (nullptr: the epoch is `add` itself)
  uint32_t mul, add;
  const uint32_t* limit_us;    // bound on the wait, in microseconds
  uint32_t* err;               // EOS_DEVERR_PEER when a wait runs out
};

// Every thread of the CTA calls this after griddepcontrol.wait (the pushing
// grid has completed, and a grid's stores, remote ones included, are
// performed when it completes).  With `publish`, thread 0 raises this rank's
// flag in every rank's words after a system-scope fence, so a rank that
// acquires the flag sees the pushed data; threads q < world then wait for
// source q's flag in this rank's own memory (local polling, bounded) -- all
// sources, or all but this rank itself when `skip_own` (a CTA of a large
// grid need not wait for its own grid's CTA 0).  Returns false when a wait
// ran out (the error bit is set; the caller leaves its outputs unwritten).
__device__ __forceinline__ bool xchg_handshake(const XchgSync& x, bool publish, bool skip_own) {
  __shared__ uint32_t s_xok;
  const uint32_t epoch = x.epoch_word != nullptr ? *x.epoch_word * x.mul + x.add : x.add;
  if (threadIdx.x == 0) s_xok = 1u;
  if (publish && threadIdx.x == 0) {
    __threadfence_system();
    for (uint32_t q = 0; q < x.world; ++q) st_release_sys(x.pub[q], epoch);
  }
  __syncthreads();
  if (threadIdx.x < x.world && !(skip_own && threadIdx.x == x.rank)) {
    const uint32_t* f = x.wait + threadIdx.x;
    if (ld_acquire_sys(f) < epoch) {
      const uint64_t limit = (uint64_t)*x.limit_us * 1000ull;
      const uint64_t t0 = global_timer_ns();
      while (ld_acquire_sys(f) < epoch) {
        // give up at the limit, or at once when an earlier handshake of
        // this step already lost a peer (the step's outputs are invalid)
        if (global_timer_ns() - t0 > limit ||
            (x.err != nullptr && (*(volatile const uint32_t*)x.err & EOS_DEVERR_PEER) != 0u)) {
          report(x.err, EOS_DEVERR_PEER);
          s_xok = 0u;
          break;
        }
      }
    }
  }
  __syncthreads();
  return s_xok != 0u;
}

// ---- exact activation packing: x86 semantics of quantize_sub32 -----------
// MAXPS/MAXSS: first operand if greater, else second (NaN -> second).
__device__ __forceinline__ float x86_max(float a, float b) { return a > b ? a : b; }

// CVTPS2DQ under the default MXCSR: round to nearest even; NaN and values
// outside the int32 range give 0x80000000.
__device__ __forceinline__ int32_t x86_cvtps(float x) {
  if (!(x == x) || x >= 2147483648.0f || x < -2147483648.0f) return INT32_MIN;
  return __float2int_rn(x);
}

// One warp packs one group of 32 activations, lane i holding element i:
// returns this lane's int8 value; scale and (wrapping) sum are warp-uniform.
// Restates src/kernels/avx2/matmul_q4_k_int8.c:98-154 bit for bit: the max
// tree below is the exact lane pairing of the AVX2 code (two vector maxes,
// then hmax_ps_8's halves / movehl / lane-1 shuffle).
// The AVX2 max tree's exact pick of max |v| over the warp's group (lane i's
// |v| bits in abits) -- needed only when some |v| is a NaN.
__device__ __forceinline__ uint32_t x86_group_absmax_nan(uint32_t abits) {
  const unsigned FULL = 0xffffffffu;
  float t = __uint_as_float(abits);
  t = x86_max(t, __shfl_down_sync(FULL, t, 8));   // max(ma0, ma1) | max(ma2, ma3)
  t = x86_max(t, __shfl_down_sync(FULL, t, 16));  // mx = max(.., ..)
  t = x86_max(t, __shfl_down_sync(FULL, t, 4));   // max_ps(lo, hi)
  t = x86_max(t, __shfl_down_sync(FULL, t, 2));   // max_ps(m, movehl(m))
  t = x86_max(t, __shfl_down_sync(FULL, t, 1));   // max_ss(m, lane 1)
  return __float_as_uint(__shfl_sync(FULL, t, 0));
}

__device__ __forceinline__ int8_t quant_group32(float v, float& scale, int32_t& sum) {
  const unsigned FULL = 0xffffffffu;
  const uint32_t abits = __float_as_uint(v) & 0x7fffffffu;
  // Without NaNs every max order gives the same value, and |x| bit patterns
  // order like the floats, so one integer max reduction is exact.
  uint32_t mbits = __reduce_max_sync(FULL, abits);
  if (mbits > 0x7f800000u) mbits = x86_group_absmax_nan(abits);  // a NaN: the AVX2 tree's exact pick
  const float max_abs = __uint_as_float(mbits);
  float inv;
  if (max_abs > 0.0f) {
    scale = __fdiv_rn(max_abs, 127.0f);
    inv = __fdiv_rn(127.0f, max_abs);
  } else {
    scale = 0.0f;
    inv = 0.0f;
  }
  const int32_t q = x86_cvtps(__fmul_rn(v, inv));
  sum = static_cast<int32_t>(__reduce_add_sync(FULL, static_cast<uint32_t>(q)));
  return static_cast<int8_t>(q < -128 ? -128 : (q > 127 ? 127 : q));
}

// 6-bit sub-block scale/min unpack (src/kernels/avx2/matmul_q4_k_int8.c:58-67).
__device__ __forceinline__ void q4k_scale_min(int j, const uint8_t* q, uint32_t& sc, uint32_t& m) {
  if (j < 4) {
    sc = q[j] & 63u;
    m = q[j + 4] & 63u;
  } else {
    sc = (q[j + 4] & 15u) | ((q[j - 4] >> 6) << 4);
    m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

// Same unpack on the 12 scale bytes held as three little-endian words.
__device__ __forceinline__ void q4k_scale_min_w(int j, uint32_t w0, uint32_t w1, uint32_t w2, uint32_t& sc,
                                                uint32_t& m) {
  // byte(i) of the 12-byte field
  auto byte = [&](int i) -> uint32_t {
    const uint32_t w = i < 4 ? w0 : (i < 8 ? w1 : w2);
    return (w >> (8 * (i & 3))) & 0xffu;
  };
  if (j < 4) {
    sc = byte(j) & 63u;
    m = byte(j + 4) & 63u;
  } else {
    sc = (byte(j + 4) & 15u) | ((byte(j - 4) >> 6) << 4);
    m = (byte(j + 4) >> 4) | ((byte(j) >> 6) << 4);
  }
}

// Packed Q4_K activation record (layout documented in q4k_gemv.cu).
constexpr uint32_t kActRec = 480;   // bytes per super-block of packed activations
constexpr uint32_t kActHalf = 272;  // offset of the second half-record

// Record position of 32-group g (sub-block g % 8 of super-block g / 8).
__device__ __forceinline__ uint32_t rec_aq_offset(uint32_t g) {
  const uint32_t s = g & 7u;
  return (g >> 3) * kActRec + (s >> 2) * kActHalf + ((s & 3u) << 5);
}
__device__ __forceinline__ uint32_t rec_st_offset(uint32_t g) {
  const uint32_t s = g & 7u;
  return (g >> 3) * kActRec + (s >> 2) * kActHalf + 128u + ((s & 3u) << 3);
}

// Packs the warp's 32-group g (lane i holds element i) into a record.
__device__ __forceinline__ void pack_group_to_record(float v, uint32_t g, uint32_t lane, uint8_t* rec) {
  float scale;
  int32_t sum;
  const int8_t q = quant_group32(v, scale, sum);
  rec[rec_aq_offset(g) + lane] = static_cast<uint8_t>(q);
  if (lane == 0) *reinterpret_cast<float2*>(rec + rec_st_offset(g)) = make_float2(scale, (float)sum);
}

__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h & 0xffffu)));
}

// Activation layout of the tensor-core prefill GEMM (prefill_gemm.cu): the
// int8 values as bf16 [rows][k], then at pf_scale_offset per 32-group s two
// f32 rows of pad4(rows): the scales [2s][row] and the sums [2s + 1][row].
__host__ __device__ constexpr uint32_t pf_pad4(uint32_t x) { return (x + 3u) & ~3u; }
__host__ __device__ constexpr size_t pf_scale_offset(uint32_t rows, uint32_t k) {
  return ((size_t)rows * k * 2u + 1023u) & ~(size_t)1023u;
}

// Packs the warp's 32-group s of row `row` (lane i holds element i) into that
// layout: the same quantize_sub32 values as pack_group_to_record.
__device__ __forceinline__ void pf_pack_group(float v, uint32_t row, uint32_t s, uint32_t lane, uint32_t k,
                                              uint32_t pitch, uint16_t* aq, float* asc) {
  float scale;
  int32_t sum;
  const int8_t q = quant_group32(v, scale, sum);
  aq[(size_t)row * k + s * 32u + lane] = __bfloat16_as_ushort(__float2bfloat16_rn((float)q));  // exact
  if (lane == 0) {
    asc[(size_t)(2u * s) * pitch + row] = scale;
    asc[(size_t)(2u * s + 1u) * pitch + row] = (float)sum;
  }
}

// Kernel attributes belong to a device, not to the process: a kernel that
// needs more than 48 KB of dynamic shared memory must be allowed it on every
// device it runs on.  SmemAttr remembers, per device ordinal, the largest
// amount already allowed; ensure_smem_attr sets the attribute (and the
// largest shared-memory carveout) for the current device when needed.
constexpr int kMaxDevices = 64;
struct SmemAttr {
  int set[kMaxDevices] = {};
};
inline cudaError_t ensure_smem_attr(const void* fn, int bytes, SmemAttr& a, bool max_carveout = true) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (bytes <= __atomic_load_n(&a.set[dev], __ATOMIC_ACQUIRE)) return cudaSuccess;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && max_carveout)
    e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (e == cudaSuccess) __atomic_store_n(&a.set[dev], bytes, __ATOMIC_RELEASE);
  return e;
}

}  // namespace eos
