// q80_gemv.cu -- Q8_0 decode GEMV for sm_100a (f32 activations x int8 weights
// with an fp16 scale per 32), the production Q8_0 path of every reference
// backend: eosi_scalar_matmul_q8_0 (src/kernels/scalar/matmul_q8.c:21-58).
//
// Same skeleton as the Q4_K GEMV: each CTA owns a contiguous slab of weight
// rows; warp w of NW streams rows w, w+NW, ... HBM -> shared memory with
// coalesced 16-byte cp.async copies through D private buffers.  The f32
// activation vector is copied once per CTA into shared memory at a 144-byte
// stride per 32 values (== 16 mod 128), so lanes reading different blocks hit
// different banks.  One lane takes a whole 32-weight block: block j of a row
// sits at byte 34j (only 2-byte aligned), so the lane loads the nine aligned
// words around it and realigns the data with one byte permute per word; each
// int8 becomes an exact float through the 2^23 magic (prmt + packed subtract),
// and the products accumulate with packed fp32x2 FMAs.  Per-lane partials
// are reduced across the warp at the end of the row.  The summation order
// differs from the reference's sequential loop, so results agree to fp32
// rounding (the tests bound it), not bit for bit.
#include "eos_common.cuh"
#include "eos_kernels.h"

namespace eos {

constexpr uint32_t kQ8ActStride = 36;  // floats per 32-value block in shared memory

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
struct Q80GemvParams {
  const uint8_t* w;  // n rows x row_bytes
  const float* a;    // k floats
  float* c;
  uint32_t n, k, nblk, row_bytes, pitch;
  uint32_t cb, chunks;  // blocks per chunk (multiple of 8), chunks per row
  uint32_t* err;
  float* c_extra[7];  // further copies of every output (tensor-parallel push)
  uint32_t n_extra;
  XchgSync xs;  // tensor parallel (world > 1): the other ranks pushed parts of `a`
};

// Four signed bytes -> two float2 of exact values: 2^23 + (b + 128) built by
// prmt on the biased word, minus 2^23 + 128 with one packed subtract each.
__device__ __forceinline__ void q8_word_to_f2(uint32_t word, float2& lo, float2& hi) {
  const uint32_t x = word ^ 0x80808080u;
  const float2 bias = make_float2(-8388736.0f, -8388736.0f);
  lo = __fadd2_rn(make_float2(__int_as_float((int)__byte_perm(x, 0x4B000000u, 0x7540u)),
                              __int_as_float((int)__byte_perm(x, 0x4B000000u, 0x7541u))),
                  bias);
  hi = __fadd2_rn(make_float2(__int_as_float((int)__byte_perm(x, 0x4B000000u, 0x7542u)),
                              __int_as_float((int)__byte_perm(x, 0x4B000000u, 0x7543u))),
                  bias);
}

// One 34-byte block at `blk` (2-byte aligned, shared memory) against the 32
// activations at `act` (16-byte aligned): scale * sum(a * w).
__device__ __forceinline__ float q80_block(const uint8_t* blk, const float* act) {
  const uintptr_t addr = reinterpret_cast<uintptr_t>(blk);
  const uint32_t* wp = reinterpret_cast<const uint32_t*>(addr & ~(uintptr_t)3);
  const bool odd = (addr & 2u) != 0;  // block starts in the upper half of its first word
  uint32_t wd[9];
#pragma unroll
  for (int i = 0; i < 9; ++i) wd[i] = wp[i];
  const float scale = f16_bits_to_f32(odd ? (wd[0] >> 16) : wd[0]);
  // data starts 2 bytes after the block: bytes 2..5 of (wd[t], wd[t+1]) when
  // the block is word-aligned, bytes 4..7 (= wd[t+1]) when it is not
  const uint32_t sel = odd ? 0x7654u : 0x5432u;
  float2 acc0 = make_float2(0.0f, 0.0f), acc1 = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const uint32_t word = __byte_perm(wd[t], wd[t + 1], sel);
    float2 lo, hi;
    q8_word_to_f2(word, lo, hi);
    const float4 av = *reinterpret_cast<const float4*>(act + 4 * t);
    acc0 = __ffma2_rn(make_float2(av.x, av.y), lo, acc0);
    acc1 = __ffma2_rn(make_float2(av.z, av.w), hi, acc1);
  }
  return scale * ((acc0.x + acc0.y) + (acc1.x + acc1.y));
}

template <int NW, int D>
__global__ void __launch_bounds__(NW * 32, 1) q80_gemv_kernel(const Q80GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t nblk = p.nblk, row_bytes = p.row_bytes, pitch = p.pitch;
  float* act_s = reinterpret_cast<float*>(smem);
  const uint32_t act_region = (nblk * kQ8ActStride * 4u + 127u) & ~127u;
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  uint8_t* wbuf = smem + act_region + warp * D * pitch;

  const uint32_t r0 = (uint32_t)(((uint64_t)p.n * blockIdx.x) / gridDim.x);
  const uint32_t r1 = (uint32_t)(((uint64_t)p.n * (blockIdx.x + 1)) / gridDim.x);
  const uint32_t nrows = r1 - r0;
  const uint32_t C = p.chunks, cb = p.cb;
  const uint64_t pol_w = l2_policy_evict_first();
  // this warp's stages: rows warp, warp + NW, ..., each as C chunks in order
  const uint32_t my_rows = nrows > warp ? (nrows - warp + NW - 1) / NW : 0u;
  const uint32_t T = my_rows * C;

  // (row, chunk) of the next stage to issue, advanced incrementally
  uint32_t irow = warp, ich = 0;
  auto issue = [&](uint32_t t, uint32_t slot) {
    if (t < T) {
      const uint32_t row = irow, ch = ich;
      if (++ich == C) {
        ich = 0;
        irow += NW;
      }
      const uint32_t b0 = ch * cb, nb = (nblk - b0) < cb ? (nblk - b0) : cb;
      const uint8_t* src = p.w + (size_t)(r0 + row) * row_bytes + b0 * Q80_BYTES;
      uint8_t* dst = wbuf + slot * pitch;
      const uint32_t n16 = (nb * Q80_BYTES) >> 4;  // nb is a multiple of 8: 272-byte units
      for (uint32_t q = lane; q < n16; q += 32) cp_async16(dst + (q << 4), src + (q << 4), pol_w);
    }
    cp_async_commit();
  };
#pragma unroll
  for (uint32_t d = 0; d < (uint32_t)D; ++d) issue(d, d);

  pdl_wait();  // the activations may be the previous kernel's output
  if (p.xs.world > 1 && !xchg_handshake(p.xs, blockIdx.x == 0, true)) {
    cp_async_wait<0>();  // a peer never arrived: drain, leave the outputs unwritten
    return;
  }
  {
    const float4* src = reinterpret_cast<const float4*>(p.a);
    for (uint32_t t = threadIdx.x; t < (p.k >> 2); t += NW * 32) {
      const uint32_t j = t >> 3, v = t & 7u;
      *reinterpret_cast<float4*>(act_s + j * kQ8ActStride + 4u * v) = src[t];
    }
  }
  __syncthreads();
  pdl_trigger();

  float acc = 0.0f;
  uint32_t row = warp, ch = 0, slot = 0;  // stage being consumed
  for (uint32_t t = 0; t < T; ++t) {
    cp_async_wait<D - 1>();
    __syncwarp();
    const uint32_t b0 = ch * cb, nb = (nblk - b0) < cb ? (nblk - b0) : cb;
    const uint8_t* chunk = wbuf + slot * pitch;
    const float* av = act_s + b0 * kQ8ActStride;
    for (uint32_t j = lane; j < nb; j += 32) acc += q80_block(chunk + j * Q80_BYTES, av + j * kQ8ActStride);
    __syncwarp();
    issue(t + D, slot);
    if (++slot == (uint32_t)D) slot = 0;
    if (++ch == C) {  // row complete
      acc += __shfl_xor_sync(0xffffffffu, acc, 16);
      acc += __shfl_xor_sync(0xffffffffu, acc, 8);
      acc += __shfl_xor_sync(0xffffffffu, acc, 4);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      if (lane == 0) {
        p.c[r0 + row] = acc;
        // extra destinations: plain remote stores, ordered before the
        // consumer's flag by grid completion (see gemv_store, q4k_gemv.cu)
        for (uint32_t j = 0; j < p.n_extra; ++j) p.c_extra[j][r0 + row] = acc;
      }
      acc = 0.0f;
      ch = 0;
      row += NW;
    }
  }
  cp_async_wait<0>();
}

namespace {
struct Q80Config {
  void (*fn)(const Q80GemvParams);
  int nw, d;
  SmemAttr attr;  // dynamic shared memory allowed so far, per device
};
Q80Config g_q80_cfgs[] = {{q80_gemv_kernel<16, 4>, 16, 4, {}}, {q80_gemv_kernel<16, 3>, 16, 3, {}},
                          {q80_gemv_kernel<16, 2>, 16, 2, {}}, {q80_gemv_kernel<8, 4>, 8, 4, {}},
                          {q80_gemv_kernel<24, 2>, 24, 2, {}}, {q80_gemv_kernel<12, 3>, 12, 3, {}}};
constexpr int kNumQ80Cfgs = sizeof(g_q80_cfgs) / sizeof(g_q80_cfgs[0]);
int g_q80_variant = -1;
}  // namespace

void set_q80_gemv_variant(int v) { g_q80_variant = v; }

cudaError_t launch_q80_gemv(const uint8_t* w, const float* a, float* c, uint32_t n, uint32_t k, uint32_t* err,
                            int num_sms, int max_smem, cudaStream_t st, int* out_status, float* const* c_extra,
                            uint32_t n_extra, const XchgSync* xs) {
  if (n_extra > 7) {
    *out_status = EOS_E_INVALID_ARG;
    return cudaSuccess;
  }
  *out_status = EOS_OK;
  if (n == 0) return cudaSuccess;
  const uint32_t nblk = k / Q80_ELEMS;
  const uint32_t row_bytes = nblk * Q80_BYTES;
  const uint32_t act_region = (nblk * kQ8ActStride * 4u + 127u) & ~127u;
  // rows stream in chunks of at most 128 blocks (4352 bytes); +16: the last
  // block's nine-word window may reach 2 bytes past the chunk
  const uint32_t cb = nblk < 128u ? nblk : 128u;
  const uint32_t chunks = (nblk + cb - 1) / cb;
  const uint32_t pitch = (cb * Q80_BYTES + 16u + 15u) & ~15u;
  const bool aligned = (k % 256u) == 0 && (reinterpret_cast<uintptr_t>(w) & 15u) == 0 &&
                       (reinterpret_cast<uintptr_t>(a) & 15u) == 0;
  int pick = -1;
  if (g_q80_variant >= 0 && g_q80_variant < kNumQ80Cfgs) {
    pick = g_q80_variant;
  } else {
    const int order[] = {4, 2, 1, 0, 3};
    for (int o : order)
      if (act_region + (uint32_t)(g_q80_cfgs[o].nw * g_q80_cfgs[o].d) * pitch <= (uint32_t)max_smem) {
        pick = o;
        break;
      }
  }
  if (!aligned || pick < 0 ||
      act_region + (uint32_t)(g_q80_cfgs[pick].nw * g_q80_cfgs[pick].d) * pitch > (uint32_t)max_smem) {
    if (n_extra != 0 || (xs != nullptr && xs->world > 1)) {  // the unstaged kernel: one destination, no handshake
      *out_status = EOS_E_UNSUPPORTED;
      return cudaSuccess;
    }
    q80_gemv_simple_kernel<<<(n + 7u) / 8u, 256, 0, st>>>(w, a, c, n, k);
    return cudaGetLastError();
  }
  Q80Config& cfg = g_q80_cfgs[pick];
  const uint32_t smem = act_region + (uint32_t)(cfg.nw * cfg.d) * pitch;
  {
    const cudaError_t e = ensure_smem_attr((const void*)cfg.fn, (int)smem, cfg.attr);  // on this device
    if (e != cudaSuccess) return e;
  }
  uint32_t cps = (uint32_t)(max_smem + 1024) / (smem + 1024);
  if (cps > 4u) cps = 4u;
  if (cps < 1u) cps = 1u;
  uint32_t grid = (uint32_t)num_sms * cps;
  if (grid > n) grid = n;
  Q80GemvParams prm{w, a, c, n, k, nblk, row_bytes, pitch, cb, chunks, err, {}, n_extra, {}};
  for (uint32_t j = 0; j < n_extra; ++j) prm.c_extra[j] = c_extra[j];
  if (xs != nullptr) prm.xs = *xs;
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
