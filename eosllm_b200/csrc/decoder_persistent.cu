// decoder_persistent.cu -- the decoder step of decoder.cu as ONE persistent
// kernel per token (Q4_K linears and LM head, head_dim 64 or 128, n_embd <=
// 4096): the work of eosi_text_step (src/modality/text/text.c:267-436) and
// the greedy pick (src/sched/greedy.c:48-73).
//
// Why one kernel.  A per-op step (decoder.cu) chains 8 kernels per layer;
// measured on a B200 with %globaltimer stamps, every kernel that follows a
// GEMV passes griddepcontrol.wait 2.5-5 us after the GEMV's last CTA exits,
// and each GEMV can prefetch only what two resident CTAs per SM hold, so
// HBM idles through every kernel boundary.  Here one CTA per SM (cooperative
// launch, all resident) runs the whole step, and each warp's weight ring
// streams the step's matrices in order -- layer 0's [q;k;v], O, [gate;up],
// down, layer 1's ..., the LM head -- running ahead of the compute across
// every phase boundary: while a warp waits for the activations of the next
// matrix, its ring already holds that matrix's first stages.
//
// Nothing waits on a kernel or a grid barrier.  Every vector that crosses
// CTAs travels as (epoch, word) pairs (the LLExchange format of
// eos_common.cuh): the QKV and gate/up outputs in this GPU's memory, the
// attention output, O rows, SiLU output and down rows in every rank's
// exchange buffer; a consumer polls the pairs it needs -- bounded -- until
// each carries the exchange's epoch, step * (6 n_layer + 1) + 6 L + k + 1.
// One GPU and tensor parallel are the same code (world destinations).  The
// residual stream never leaves shared memory: every CTA keeps its own copy
// and normalises the whole vector itself.
//
// Numerics: each phase is the arithmetic of its per-op kernel in the same
// order -- the bit-exact Q4_K GEMV (q4k_gemv.cu: the same terms, super-block
// partials and ordered row sums), norm_pack's sum of squares (256 threads x
// 4 float4 chunks, the same shuffle tree), attn_kernel's 32-position chunks
// (4 warps interleaved, the same merge), silu_pack, argmax -- so logits and
// tokens are bit-identical to the per-op step on any number of GPUs.
#include <cstdint>

#include "decoder_internal.h"
#include "eos_common.cuh"
#include "q4k_dot.cuh"

namespace eos {

namespace {

constexpr uint32_t kPW = 12;                    // warps per CTA (167 registers a thread, none spilled)
constexpr uint32_t kPT = kPW * 32u;             // threads per CTA
constexpr uint32_t kPR = 2;                     // weight rows per stage
constexpr uint32_t kPCB = 16;                   // super-blocks per stage (a row chunk; one per lane pair)
constexpr uint32_t kPD = 3;                     // stages in flight per warp (166 KB a CTA)
constexpr uint32_t kPPitch = kPCB * Q4K_BYTES;  // 2304: one staged row chunk
constexpr uint32_t kPStage = kPR * kPPitch;     // 4608
constexpr uint32_t kPPairs = kPW / 2u;          // attention warp pairs per CTA
constexpr uint32_t kPX = 6;                     // exchanges per layer
constexpr uint32_t kAbortBits = EOS_DEVERR_PEER | EOS_DEVERR_WAIT_ACT | EOS_DEVERR_WAIT_FULL;

__host__ __device__ constexpr uint32_t up128(uint32_t x) { return (x + 127u) & ~127u; }

}  // namespace

// Shared-memory layout of the persistent step (host and device agree).
struct PSmem {
  uint32_t xres, act, part, scratch, streams, bars, ring, total;
  uint32_t pstride;      // floats of one warp's super-block partials
  uint32_t grp_floats;   // floats of one attention pair's scratch
  uint32_t layers;       // the layer table
};

// The step's per-CTA context, in shared memory next to a copy of the
// parameters.  Phases read both from there: shared-memory loads the compiler
// does not hoist out of the layer loop, so the ~50 values do not stay live
// in registers across every phase (they would take a third of the 128).
struct PCtx {
  PSmem lay;
  uint32_t pos, tok, ebase, nmat;
  uint64_t limit_ns;
};
constexpr uint32_t kPCtxOff = ((uint32_t)sizeof(PStepParams) + 15u) & ~15u;
constexpr uint32_t kPHead = up128(kPCtxOff + (uint32_t)sizeof(PCtx));

__host__ __device__ inline PSmem psmem_layout(uint32_t E, uint32_t F, uint32_t hd, uint32_t max_chunks,
                                              uint32_t n_layer) {
  PSmem s{};
  const uint32_t nbmax = (E > F ? E : F) / Q4K_ELEMS;
  uint32_t off = kPHead;
  s.xres = off;
  off += up128(4u * E);
  s.act = off;
  off += up128(nbmax * kActRec);
  s.pstride = (kPR * nbmax + 3u) & ~3u;
  s.part = off;
  off += up128(kPW * s.pstride * 4u);
  // attention pair: score[32], o[4][hd], l[4], out[hd], wc/lc[max_chunks], flags[4]
  s.grp_floats = (32u + 4u * hd + 4u + hd + 2u * max_chunks + 4u + 3u) & ~3u;
  uint32_t scr = kPPairs * s.grp_floats * 4u;
  if (scr < 512u) scr = 512u;  // norm / argmax reductions
  s.scratch = off;
  off += up128(scr);
  s.streams = off;  // per-warp stream cursors, parked between GEMV phases
  off += up128(kPW * 128u);
  s.layers = off;
  off += up128(n_layer * (uint32_t)sizeof(PLayer));
  s.bars = off;  // one mbarrier per ring slot
  off += up128(kPW * kPD * 8u);
  s.ring = off;
  off += kPW * kPD * kPStage;
  s.total = off;
  return s;
}

extern __shared__ __align__(128) uint8_t g_psmem[];

namespace {

__device__ __forceinline__ const PStepParams& P() { return *reinterpret_cast<const PStepParams*>(g_psmem); }
__device__ __forceinline__ const PCtx& C() { return *reinterpret_cast<const PCtx*>(g_psmem + kPCtxOff); }
template <class T>
__device__ __forceinline__ T* at(uint32_t off) {
  return reinterpret_cast<T*>(g_psmem + off);
}

// ---------------------------------------------------------------------------
// Pairs
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t pepoch(uint32_t ebase, uint32_t L, uint32_t k) { return ebase + kPX * L + k + 1u; }

// word i of an exchanged vector, with its epoch, into every rank's buffer
__device__ __forceinline__ void put_all(uint64_t* const* outs, uint32_t n_out, size_t i, uint32_t word,
                                        uint32_t epoch) {
  const uint64_t v = ((uint64_t)epoch << 32) | word;
  for (uint32_t j = 0; j < n_out; ++j)
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(outs[j] + i), "l"(v) : "memory");
}
// word i of a vector read only on this GPU
__device__ __forceinline__ void put_local(uint64_t* out, size_t i, uint32_t word, uint32_t epoch) {
  const uint64_t v = ((uint64_t)epoch << 32) | word;
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(out + i), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_pair(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// A polling thread's budget: false once `limit_ns` has passed since its first
// unsuccessful round, or at once when another wait of the step gave up.
__device__ __forceinline__ bool keep_polling(uint64_t& t0, uint64_t limit_ns, const uint32_t* err) {
  const uint64_t now = global_timer_ns();
  if (t0 == 0) {
    t0 = now;
    return true;
  }
  if (now - t0 > limit_ns) return false;
  if ((*(volatile const uint32_t*)err & kAbortBits) != 0u) return false;
  __nanosleep(32);
  return true;
}

// The warp's 32-group g (lane i holds element i), packed, as pairs into every
// rank's record buffer (pack_group_out of decoder.cu).
__device__ __forceinline__ void pack_put(float v, uint32_t g, uint32_t lane, uint64_t* const* outs, uint32_t n_out,
                                         uint32_t epoch) {
  float scale;
  int32_t sum;
  const uint32_t b = static_cast<uint8_t>(quant_group32(v, scale, sum));
  const unsigned FULL = 0xffffffffu;
  const uint32_t w = b | (__shfl_down_sync(FULL, b, 1) << 8) | (__shfl_down_sync(FULL, b, 2) << 16) |
                     (__shfl_down_sync(FULL, b, 3) << 24);
  if ((lane & 3u) == 0) put_all(outs, n_out, (rec_aq_offset(g) >> 2) + (lane >> 2), w, epoch);
  if (lane == 0) {
    put_all(outs, n_out, rec_st_offset(g) >> 2, __float_as_uint(scale), epoch);
    put_all(outs, n_out, (rec_st_offset(g) >> 2) + 1u, __float_as_uint((float)sum), epoch);
  }
}

// N groups of 32 packed into records at once (lane i holds element i of
// each; groups with ok[n] false are skipped): quant_group32's arithmetic
// (eos_common.cuh) for every group, the N reductions and divisions in
// lockstep so their latencies overlap.
template <int N>
__device__ __forceinline__ void pack_groups_to_record(const float (&v)[N], const uint32_t (&g)[N],
                                                      const bool (&ok)[N], uint32_t lane, uint8_t* rec) {
  const unsigned FULL = 0xffffffffu;
  uint32_t mb[N];
#pragma unroll
  for (int n = 0; n < N; ++n) mb[n] = __reduce_max_sync(FULL, __float_as_uint(v[n]) & 0x7fffffffu);
  float scale[N], inv[N];
#pragma unroll
  for (int n = 0; n < N; ++n) {
    if (mb[n] > 0x7f800000u) mb[n] = x86_group_absmax_nan(__float_as_uint(v[n]) & 0x7fffffffu);  // a NaN
    const float max_abs = __uint_as_float(mb[n]);
    if (max_abs > 0.0f) {
      scale[n] = __fdiv_rn(max_abs, 127.0f);
      inv[n] = __fdiv_rn(127.0f, max_abs);
    } else {
      scale[n] = 0.0f;
      inv[n] = 0.0f;
    }
  }
  int32_t q[N];
#pragma unroll
  for (int n = 0; n < N; ++n) q[n] = x86_cvtps(__fmul_rn(v[n], inv[n]));
  int32_t sum[N];
#pragma unroll
  for (int n = 0; n < N; ++n) sum[n] = static_cast<int32_t>(__reduce_add_sync(FULL, static_cast<uint32_t>(q[n])));
#pragma unroll
  for (int n = 0; n < N; ++n) {
    if (!ok[n]) continue;
    const int32_t c = q[n] < -128 ? -128 : (q[n] > 127 ? 127 : q[n]);
    rec[rec_aq_offset(g[n]) + lane] = static_cast<uint8_t>(static_cast<int8_t>(c));
    if (lane == 0) *reinterpret_cast<float2*>(rec + rec_st_offset(g[n])) = make_float2(scale[n], (float)sum[n]);
  }
}

// A lane's AE cached K or V values (16- or 8-byte aligned), through L2.
template <int AE>
__device__ __forceinline__ void ld_row(const float* src, float (&d)[AE]) {
  if constexpr (AE == 4) {
    const float4 v = __ldcg(reinterpret_cast<const float4*>(src));
    d[0] = v.x;
    d[1] = v.y;
    d[2] = v.z;
    d[3] = v.w;
  } else {
    const float2 v = __ldcg(reinterpret_cast<const float2*>(src));
    d[0] = v.x;
    d[1] = v.y;
  }
}

// 64-thread barrier of attention warp pair `pr` (named barrier 1 + pr), and
// the same with an OR over the pair's predicates.
__device__ __forceinline__ void psync(uint32_t pr) {
  asm volatile("bar.sync %0, 64;" ::"r"(pr + 1u) : "memory");
}
__device__ __forceinline__ bool psync_or(uint32_t pr, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, 64, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(pr + 1u)
      : "memory");
  return r != 0u;
}

}  // namespace

namespace {

// ---------------------------------------------------------------------------
// The weight stream: every warp walks the step's matrices in order; in each,
// this CTA's row slice (rows n*b/G .. n*(b+1)/G of CTA b of G) in groups of
// kPR rows, warp w taking groups w, w + kPW, ..., each through its row
// chunks of kPCB super-blocks (the column-major GEMV's schedule).
// ---------------------------------------------------------------------------
struct PCursor {
  uint32_t mi;          // 4 L + {0: qkv, 1: O, 2: gate/up, 3: down}; 4 n_layer: the LM head
  uint32_t g, ch;       // row group of the slice, chunk of the row
  const uint8_t* base;  // first row of the slice
  uint32_t r0, nrows, ngroups, nb, nch, row_bytes;
};

__device__ __forceinline__ void mat_of(const PStepParams& p, uint32_t mi, uint32_t hd, const uint8_t*& w, uint32_t& n,
                                       uint32_t& nb) {
  const uint32_t nbe = p.E / Q4K_ELEMS;
  if (mi >= 4u * p.n_layer) {
    w = p.wout;
    n = p.vl;
    nb = nbe;
    return;
  }
  const uint32_t t = mi & 3u;
  w = at<const PLayer>(C().lay.layers)[mi >> 2].w[t];
  nb = nbe;
  if (t == 0) {
    n = p.hl * hd + 2u * p.kvl * hd;
  } else if (t == 2) {
    n = 2u * p.ffl;
  } else {
    n = p.el;
    if (t == 3) nb = p.F / Q4K_ELEMS;
  }
}

// Positions the cursor on the first matrix at or after c.mi where this warp
// owns a row group (c.mi == nmat: the stream is over).
__device__ void cursor_seek(const PStepParams& p, PCursor& c, uint32_t warp, uint32_t hd, uint32_t nmat) {
  for (; c.mi < nmat; ++c.mi) {
    const uint8_t* w;
    uint32_t n, nb;
    mat_of(p, c.mi, hd, w, n, nb);
    // n * gridDim.x < 2^32 (n <= 2^21 rows per rank, at most 2^11 CTAs)
    c.r0 = (n * blockIdx.x) / gridDim.x;
    c.nrows = (n * (blockIdx.x + 1u)) / gridDim.x - c.r0;
    c.ngroups = (c.nrows + kPR - 1u) / kPR;
    if (warp < c.ngroups) {
      c.nb = nb;
      c.nch = (nb + kPCB - 1u) / kPCB;
      c.row_bytes = nb * Q4K_BYTES;
      c.base = w + (size_t)c.r0 * c.row_bytes;
      c.g = warp;
      c.ch = 0;
      return;
    }
  }
}

__device__ __forceinline__ void cursor_next(const PStepParams& p, PCursor& c, uint32_t warp, uint32_t hd,
                                            uint32_t nmat) {
  if (++c.ch < c.nch) return;
  c.ch = 0;
  c.g += kPW;
  if (c.g < c.ngroups) return;
  ++c.mi;
  cursor_seek(p, c, warp, hd, nmat);
}

// The stage at the issue cursor into ring slot `slot`, then advance: lane 0
// issues TMA bulk copies (cp.async.bulk, this GPU's memory, no multicast) --
// one for two whole 16-super-block rows, else one per row chunk -- that
// complete on the slot's mbarrier with the stage's byte count.  Every lane
// advances the cursor.  Returns whether a stage was issued (false past the
// end of the step's stream).
__device__ __forceinline__ bool issue_stage(const PStepParams& p, PCursor& c, uint8_t* ring_w, uint64_t* bars_w,
                                            uint32_t slot, uint32_t lane, uint32_t warp, uint32_t hd, uint32_t nmat,
                                            uint64_t pol) {
  if (c.mi >= nmat) return false;
  if (lane == 0) {
    const uint32_t rows = (c.nrows - c.g * kPR) < kPR ? (c.nrows - c.g * kPR) : kPR;
    const uint32_t b0 = c.ch * kPCB, bn = (c.nb - b0) < kPCB ? (c.nb - b0) : kPCB;
    const uint32_t chunk = bn * Q4K_BYTES;  // a multiple of 16 bytes, as are both addresses
    const uint8_t* src = c.base + (size_t)(c.g * kPR) * c.row_bytes + (size_t)b0 * Q4K_BYTES;
    uint8_t* dst = ring_w + slot * kPStage;
    uint64_t* bar = bars_w + slot;
    // (the warp's reads of the slot's previous stage have all returned: their
    // values fed the partials stored before the caller's __syncwarp)
    mbar_arrive_expect_tx(bar, rows * chunk);
    if (c.row_bytes == kPPitch) {  // whole rows at the staging pitch: one copy
      bulk_g2s(dst, src, rows * chunk, bar, pol);
    } else {
      for (uint32_t r = 0; r < rows; ++r) bulk_g2s(dst + r * kPPitch, src + (size_t)r * c.row_bytes, chunk, bar, pol);
    }
  }
  cursor_next(p, c, warp, hd, nmat);
  return true;
}

// Waits for ring stage `t` (slot t % kPD, phase (t / kPD) & 1), bounded; gives
// up at once when another wait of the step gave up.
__device__ __forceinline__ bool wait_stage(uint64_t* bars_w, uint32_t t, uint64_t limit_ns, const uint32_t* err) {
  uint64_t* bar = bars_w + t % kPD;
  const uint32_t parity = (t / kPD) & 1u;
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = 0;
  while (!mbar_try_wait(bar, parity))
    if (!keep_polling(t0, limit_ns, err)) return false;
  return true;
}

// Per-warp stream state (parked in 128 bytes of shared memory per warp).
struct PStream {
  PCursor in;       // next stage to issue
  PCursor cur;      // next stage to compute
  uint32_t t;       // stages computed so far (ring slot t % kPD)
  uint32_t issued;  // stages issued so far
};
static_assert(sizeof(PStream) <= 128u, "a warp's parked stream");

// This warp's stages of matrix M: the column-major GEMV's terms, partials and
// ordered row sums (q4k_gemv_cols_kernel), output row r of the CTA's slice
// -> out(r_global_in_matrix, value).
// Before a CTA leaves early: every stage this warp issued and did not consume
// must have landed (bounded; shared memory is not left with copies in flight).
__device__ __noinline__ void drain_stream() {
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  const PStream* parked = at<PStream>(C().lay.streams + warp * 128u);
  uint64_t* bars_w = at<uint64_t>(C().lay.bars) + warp * kPD;
  for (uint32_t t = parked->t; t < parked->issued; ++t)
    if (!mbar_wait(bars_w + t % kPD, (t / kPD) & 1u) && lane == 0) report(&P().state->err, EOS_DEVERR_DRAIN);
  __syncwarp();
}

// Where a GEMV's output row goes (by matrix type; kOutLogits: the LM head).
enum : uint32_t { kOutQkv = 0, kOutO = 1, kOutGu = 2, kOutDown = 3, kOutLogits = 4 };

__device__ __forceinline__ void gemv_out(uint32_t kind, uint32_t L, uint32_t r, float v) {
  const PStepParams& p = P();
  const uint32_t ebase = C().ebase, w = __float_as_uint(v);
  switch (kind) {
    case kOutQkv: put_local(p.qkv_x, r, w, pepoch(ebase, L, 0)); break;
    case kOutO: put_all(p.o_out, p.world, p.e0 + r, w, pepoch(ebase, L, 2)); break;
    case kOutGu: put_local(p.gu_x, r, w, pepoch(ebase, L, 3)); break;
    case kOutDown: put_all(p.d_out, p.world, p.e0 + r, w, pepoch(ebase, L, 5)); break;
    default: p.logits[r] = v; break;
  }
}

// One copy of the GEMV body for every matrix of the step (not inlined: the
// instruction working set of a phase stays small).
__device__ __noinline__ void gemv_phase(uint32_t M, uint32_t hd, uint32_t kind, uint32_t L) {
  const PStepParams& p = P();
  const PSmem& lay = C().lay;
  const uint32_t nmat = C().nmat;
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  const uint8_t* act_s = at<uint8_t>(lay.act);
  float* part_w = at<float>(lay.part) + warp * lay.pstride;
  uint8_t* ring_w = at<uint8_t>(lay.ring) + warp * kPD * kPStage;
  uint64_t* bars_w = at<uint64_t>(lay.bars) + warp * kPD;
  PStream* parked = at<PStream>(lay.streams + warp * 128u);
  const uint64_t limit_ns = C().limit_ns;
  const uint32_t h = lane & 1u;
  const uint64_t pol = l2_policy_evict_first();
  // the compute cursor in registers; the issue cursor stays parked in shared
  // memory (every lane reads the same copy, lane 0 writes it back)
  PCursor cur = parked->cur;
  uint32_t t = parked->t;
  // whole 16-super-block rows (every k = 4096 matrix): lane pair j always
  // takes super-block column j, so its activation half-record stays in
  // registers for the whole phase, and the 16 partials of a row reach its
  // lane by shuffles
  const bool whole = cur.mi == M && cur.nb == kPCB;
  int4 a[2][4];
  float4 st[2];
  if (whole) q4k_load_half(act_s + (lane >> 1) * kActRec + h * kActHalf, a, st);
  while (cur.mi == M) {
    const PCursor& c = cur;
    const uint32_t slot = t % kPD;
    if (!__all_sync(0xffffffffu, wait_stage(bars_w, t, limit_ns, &p.state->err))) {
      // gave up (the step's outputs are invalid; every later wait gives up
      // too): stage t stays unconsumed, so the drain waits for it
      if (lane == 0) report(&p.state->err, EOS_DEVERR_WAIT_FULL);
      break;
    }
    const uint32_t rows = (c.nrows - c.g * kPR) < kPR ? (c.nrows - c.g * kPR) : kPR;
    const uint8_t* stage = ring_w + slot * kPStage;
    if (whole) {
      float tr[kPR][4];
      q4k_half_terms_rows_regs<kPR>(stage + (lane >> 1) * Q4K_BYTES, kPPitch, a, st, h, tr, rows);
      float part[kPR];
#pragma unroll
      for (int r = 0; r < (int)kPR; ++r) part[r] = pair_partial(tr[r], lane);  // super-block lane >> 1, odd lanes
      // row r's partials in super-block order to lane r: c = 0; c += partial_b
      // (matmul_q4_k_int8.c:194, :264)
      float v[kPCB];
#pragma unroll
      for (uint32_t b = 0; b < kPCB; ++b) {
        float x = __shfl_sync(0xffffffffu, part[0], 2u * b + 1u);
#pragma unroll
        for (int r = 1; r < (int)kPR; ++r) {
          const float y = __shfl_sync(0xffffffffu, part[r], 2u * b + 1u);
          if (lane == (uint32_t)r) x = y;
        }
        v[b] = x;
      }
      float acc = 0.0f;
#pragma unroll
      for (uint32_t b = 0; b < kPCB; ++b) acc = __fadd_rn(acc, v[b]);
      {
        PCursor in = parked->in;
        const bool more = issue_stage(p, in, ring_w, bars_w, slot, lane, warp, hd, nmat, pol);
        __syncwarp();
        if (lane == 0) {
          parked->in = in;
          parked->issued += more ? 1u : 0u;
        }
        __syncwarp();
      }
      if (lane < rows) gemv_out(kind, L, c.r0 + c.g * kPR + lane, acc);
    } else {
      const uint32_t b0 = c.ch * kPCB, bn = (c.nb - b0) < kPCB ? (c.nb - b0) : kPCB;
      {
        const uint32_t j = lane >> 1;
        const uint32_t jc = j < bn ? j : bn - 1u;
        float tr[kPR][4];
        q4k_half_terms_rows<kPR>(stage + jc * Q4K_BYTES, kPPitch, act_s + (b0 + jc) * kActRec + h * kActHalf, h,
                                 tr, rows);
#pragma unroll
        for (int r = 0; r < (int)kPR; ++r) {
          const float part = pair_partial(tr[r], lane);
          if (h && j < bn && (uint32_t)r < rows) part_w[r * c.nb + b0 + j] = part;
        }
      }
      __syncwarp();
      {
        PCursor in = parked->in;
        const bool more = issue_stage(p, in, ring_w, bars_w, slot, lane, warp, hd, nmat, pol);
        __syncwarp();
        if (lane == 0) {
          parked->in = in;
          parked->issued += more ? 1u : 0u;
        }
        __syncwarp();
      }
      if (c.ch == c.nch - 1u && lane < rows) {
        const float* pr = part_w + lane * c.nb;
        float acc = 0.0f;  // c = 0; c += partial_b in order (matmul_q4_k_int8.c:194, :264)
        uint32_t b = 0;
        for (; b + 8u <= c.nb; b += 8u) {
          float v8[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) v8[q] = pr[b + q];
#pragma unroll
          for (int q = 0; q < 8; ++q) acc = __fadd_rn(acc, v8[q]);
        }
        for (; b < c.nb; ++b) acc = __fadd_rn(acc, pr[b]);
        gemv_out(kind, L, c.r0 + c.g * kPR + lane, acc);
      }
    }
    __syncwarp();
    cursor_next(p, cur, warp, hd, nmat);
    ++t;
  }
  __syncwarp();
  if (lane == 0) {
    parked->cur = cur;
    parked->t = t;
  }
  __syncwarp();
}

// ---------------------------------------------------------------------------
// Residual + rmsnorm + packing, the whole vector in every CTA: x_res (shared)
// += t (pairs of exchange `epoch` in t_in; t_in == nullptr: x_res = the
// embedding of the step's token), then norm_pack_kernel's arithmetic.
// ---------------------------------------------------------------------------
template <uint32_t NCH>
__device__ __forceinline__ bool norm_phase(const uint64_t* t_in, uint32_t epoch, const float* w) {
  static_assert(kPT >= 256u, "the sum of squares runs on 256 threads");
  const PStepParams& p = P();
  const uint32_t tok = C().tok;
  const uint64_t limit_ns = C().limit_ns;
  float* xres = at<float>(C().lay.xres);
  uint8_t* act_s = at<uint8_t>(C().lay.act);
  float* red = at<float>(C().lay.scratch);
  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  const uint32_t nch = p.E >> 2;
  bool ok = true;
  __syncthreads();  // act_s and red are free
  // x_res chunks c = tid, tid + kPT, ...: every thread polls and adds
  float4* x4 = reinterpret_cast<float4*>(xres);
  if (t_in == nullptr) {
    const uint2* emb = reinterpret_cast<const uint2*>(p.tok_embd + (size_t)tok * p.E);
    for (uint32_t c = tid; c < nch; c += kPT) {
      const uint2 hb = emb[c];  // F16 -> F32 is exact (src/util/f16.h)
      x4[c] = make_float4(f16_bits_to_f32(hb.x), f16_bits_to_f32(hb.x >> 16), f16_bits_to_f32(hb.y),
                          f16_bits_to_f32(hb.y >> 16));
    }
  } else {
    constexpr uint32_t NH = (256u * NCH + kPT - 1u) / kPT;  // chunks per thread
    uint64_t q[NH][4];
    uint64_t t0 = 0;
    bool ready;
    do {
      ready = true;
#pragma unroll
      for (uint32_t j = 0; j < NH; ++j) {
        const uint32_t c = tid + kPT * j;
        if (c < nch) {
          ll_load2(t_in + 4u * c, q[j][0], q[j][1]);
          ll_load2(t_in + 4u * c + 2u, q[j][2], q[j][3]);
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if ((uint32_t)(q[j][e] >> 32) != epoch) ready = false;
        }
      }
      if (!ready && !keep_polling(t0, limit_ns, &p.state->err)) {
        ok = false;
        break;
      }
    } while (!ready);
    if (ok) {
#pragma unroll
      for (uint32_t j = 0; j < NH; ++j) {
        const uint32_t c = tid + kPT * j;
        if (c < nch) {  // x[i] += t[i] (text.c:406)
          const float4 x = x4[c];
          x4[c] = make_float4(__fadd_rn(x.x, __uint_as_float((uint32_t)q[j][0])),
                              __fadd_rn(x.y, __uint_as_float((uint32_t)q[j][1])),
                              __fadd_rn(x.z, __uint_as_float((uint32_t)q[j][2])),
                              __fadd_rn(x.w, __uint_as_float((uint32_t)q[j][3])));
        }
      }
    }
  }
  if (__syncthreads_or(!ok)) {
    if (tid == 0) report(&p.state->err, p.world > 1 ? EOS_DEVERR_PEER : EOS_DEVERR_WAIT_ACT);
    return false;
  }
  // sum of squares in norm_pack_kernel's order: thread t of 256 adds its
  // chunks t, t + 256, ... in turn, then the warps' shuffle tree, then the 8
  // warp sums in order
  if (tid < 256u) {
    float ss = 0.0f;
#pragma unroll
    for (uint32_t j = 0; j < NCH; ++j) {
      const uint32_t c = tid + 256u * j;
      if (c < nch) {
        const float4 v = x4[c];
        ss = __fadd_rn(ss, __fmul_rn(v.x, v.x));
        ss = __fadd_rn(ss, __fmul_rn(v.y, v.y));
        ss = __fadd_rn(ss, __fmul_rn(v.z, v.z));
        ss = __fadd_rn(ss, __fmul_rn(v.w, v.w));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    if (lane == 0) red[warp] = ss;
  }
  __syncthreads();
  float tot = red[0];
#pragma unroll
  for (int w8 = 1; w8 < 8; ++w8) tot = __fadd_rn(tot, red[w8]);
  // ms /= cols; s = 1 / sqrtf(ms + eps); y = x * s * w  (rmsnorm.c:24-33)
  const float ms = __fdiv_rn(tot, (float)p.E);
  const float sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, p.eps)));
  // pack: four groups of a warp at a time
  const uint32_t ng = p.E >> 5;
  for (uint32_t g0 = warp; g0 < ng; g0 += 4u * kPW) {
    float y[4];
    uint32_t g[4];
    bool in[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      g[u] = g0 + (uint32_t)u * kPW;
      in[u] = g[u] < ng;
      const uint32_t i = ((in[u] ? g[u] : g0) << 5) + lane;
      y[u] = __fmul_rn(__fmul_rn(xres[i], sc), w[i]);
    }
    pack_groups_to_record<4>(y, g, in, lane, act_s);
  }
  __syncthreads();
  return true;
}

// Packed activation records (nrec of them) from pairs of exchange `epoch`
// into shared memory; padding words are never written and not waited for.
__device__ __forceinline__ bool load_act_phase(const uint64_t* in, uint32_t nrec, uint32_t epoch) {
  const PStepParams& p = P();
  const uint64_t limit_ns = C().limit_ns;
  uint8_t* act_s = at<uint8_t>(C().lay.act);
  __syncthreads();  // act_s is no longer read
  const uint32_t n16 = nrec * (kActRec / 8u);  // 16-byte units of the pair buffer (two record words each)
  uint64_t t0 = 0;
  bool ok = true;
  for (uint32_t base = 0; base < n16 && ok; base += 4u * kPT) {
    uint64_t lo[4], hi[4];
    bool ready;
    do {
      ready = true;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t t = base + (uint32_t)j * kPT + threadIdx.x;
        if (t < n16) {
          ll_load2(in + 2u * t, lo[j], hi[j]);
          const uint32_t rw = (2u * t) % (kActRec / 4u);  // word within its record
          const bool pad = !(rw < 40u || (rw >= kActHalf / 4u && rw < kActHalf / 4u + 40u));
          if (!pad && ((uint32_t)(lo[j] >> 32) != epoch || (uint32_t)(hi[j] >> 32) != epoch)) ready = false;
        }
      }
      if (!ready && !keep_polling(t0, limit_ns, &p.state->err)) {
        ok = false;
        break;
      }
    } while (!ready);
    if (ok) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t t = base + (uint32_t)j * kPT + threadIdx.x;
        if (t < n16) reinterpret_cast<uint2*>(act_s)[t] = make_uint2((uint32_t)lo[j], (uint32_t)hi[j]);
      }
    }
  }
  if (__syncthreads_or(!ok)) {
    if (threadIdx.x == 0) report(&p.state->err, p.world > 1 ? EOS_DEVERR_PEER : EOS_DEVERR_WAIT_ACT);
    return false;
  }
  return true;
}

// ---------------------------------------------------------------------------
// Attention: work item (head, 32-position chunk) per PAIR of warps, with
// attn_kernel<AE>'s arithmetic (decoder.cu): there four warps w take the
// positions j == w (mod 4) and keep one partial o_w each, summed as
// ((o_0 + o_1) + o_2) + o_3; here warp h of the pair keeps o_{2h} and
// o_{2h+1} for its 16 positions, each summed in the same position order, so
// every value is the same.  The last pair of a head merges the chunks and
// pushes the packed head output to every rank.
// ---------------------------------------------------------------------------
template <int AE>
__device__ __forceinline__ bool attn_phase(uint32_t L) {
  constexpr uint32_t HD = 32u * AE;
  const PStepParams& p = P();
  const uint32_t pos = C().pos, ebase = C().ebase, grp_floats = C().lay.grp_floats;
  const uint64_t limit_ns = C().limit_ns;
  float* scratch = at<float>(C().lay.scratch);
  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  const uint32_t pr = warp >> 1, pw = warp & 1u, pt = tid & 63u;
  float* s_score = scratch + pr * grp_floats;  // [32]
  float* s_o = s_score + 32;                   // [4][HD]
  float* s_l = s_o + 4u * HD;                  // [4]
  float* s_out = s_l + 4;                      // [HD]
  float* s_wc = s_out + HD;                    // [max_chunks]
  float* s_lc = s_wc + p.max_chunks;           // [max_chunks]
  uint32_t* s_last = reinterpret_cast<uint32_t*>(s_lc + p.max_chunks);
  const uint32_t nvalid = pos / kAttnChunk + 1u;
  const uint32_t items = p.hl * nvalid;
  const uint32_t row = p.kvl * HD;  // floats per cache position
  const float* kc = p.kc + (size_t)L * p.max_ctx * row;
  const float* vcr = p.vc + (size_t)L * p.max_ctx * row;
  const uint32_t eq = pepoch(ebase, L, 0), eo = pepoch(ebase, L, 1);
  const uint32_t d0 = lane * AE;
  // the rotation at `pos` (the same for every item of the step)
  float rsn[AE / 2], rcs[AE / 2];
#pragma unroll
  for (int e = 0; e < AE; e += 2) rope_factors<HD>(d0 + e, pos, p.rope_base, rsn[e / 2], rcs[e / 2]);
  bool ok = true;
  __syncthreads();  // the scratch is free
  for (uint32_t it = blockIdx.x * kPPairs + pr; it < items; it += gridDim.x * kPPairs) {
    const uint32_t hloc = it / nvalid, c = it - hloc * nvalid;
    const uint32_t p0 = c * kAttnChunk;
    const uint32_t p1 = (p0 + kAttnChunk) < (pos + 1u) ? (p0 + kAttnChunk) : (pos + 1u);
    const uint32_t np = p1 - p0;
    const uint32_t gh = p.h0 + hloc;
    const uint32_t gkv = (gh * p.n_kv_head) / p.n_head;  // GQA map (text.c:367)
    const uint32_t kvi = gkv - p.kv0;
    // this warp's positions: j = 4 i + r for its residues r = 2 pw + s (s = 0, 1)
    // -- the cached rows of residue 2 pw, which do not depend on this step,
    // load first
    float kr[8][AE];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t j = 4u * i + 2u * pw;
      if (j < np && p0 + j != pos) ld_row<AE>(kc + (size_t)(p0 + j) * row + kvi * HD + d0, kr[i]);
    }
    // this step's q, k, v of the head: the QKV GEMV's pairs
    float q[AE], kn[AE], vn[AE];
    {
      const uint64_t* qp = p.qkv_x + hloc * HD + d0;
      const uint64_t* kp = p.qkv_x + p.hl * HD + kvi * HD + d0;
      const uint64_t* vp = p.qkv_x + p.hl * HD + p.kvl * HD + kvi * HD + d0;
      uint64_t t0 = 0;
      bool ready;
      do {
        ready = true;
#pragma unroll
        for (int e = 0; e < AE; e += 2) {
          uint64_t a0, a1, b0, b1, c0, c1;
          ll_load2(qp + e, a0, a1);
          ll_load2(kp + e, b0, b1);
          ll_load2(vp + e, c0, c1);
          q[e] = __uint_as_float((uint32_t)a0);
          q[e + 1] = __uint_as_float((uint32_t)a1);
          kn[e] = __uint_as_float((uint32_t)b0);
          kn[e + 1] = __uint_as_float((uint32_t)b1);
          vn[e] = __uint_as_float((uint32_t)c0);
          vn[e + 1] = __uint_as_float((uint32_t)c1);
          if ((uint32_t)(a0 >> 32) != eq || (uint32_t)(a1 >> 32) != eq || (uint32_t)(b0 >> 32) != eq ||
              (uint32_t)(b1 >> 32) != eq || (uint32_t)(c0 >> 32) != eq || (uint32_t)(c1 >> 32) != eq)
            ready = false;
        }
        if (!ready && !keep_polling(t0, limit_ns, &p.state->err)) {
          ok = false;
          break;
        }
      } while (!ready);
    }
    if (psync_or(pr, !ok)) {
      ok = false;
      break;
    }
#pragma unroll
    for (int e = 0; e < AE; e += 2) {
      rope_apply(q[e], q[e + 1], rsn[e / 2], rcs[e / 2]);
      rope_apply(kn[e], kn[e + 1], rsn[e / 2], rcs[e / 2]);
    }
    const bool has_pos = p1 == pos + 1u;
    // the first local head of each KV group appends this step's K and V
    if (has_pos && pw == 0 && (hloc == 0 || ((gh - 1u) * p.n_kv_head) / p.n_head != gkv)) {
#pragma unroll
      for (int e = 0; e < AE; ++e) {
        p.kc[(size_t)L * p.max_ctx * row + (size_t)pos * row + kvi * HD + d0 + e] = kn[e];
        p.vc[(size_t)L * p.max_ctx * row + (size_t)pos * row + kvi * HD + d0 + e] = vn[e];
      }
    }
#pragma unroll
    for (int sr = 0; sr < 2; ++sr) {
      if (sr == 1) {  // residue 2 pw + 1
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t j = 4u * i + 2u * pw + 1u;
          if (j < np && p0 + j != pos) ld_row<AE>(kc + (size_t)(p0 + j) * row + kvi * HD + d0, kr[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t j = 4u * i + 2u * pw + sr;
        if (j < np) {  // warp-uniform
          float acc = 0.0f;
          if (p0 + j == pos) {
#pragma unroll
            for (int e = 0; e < AE; ++e) acc = __fmaf_rn(q[e], kn[e], acc);
          } else {
#pragma unroll
            for (int e = 0; e < AE; ++e) acc = __fmaf_rn(q[e], kr[i][e], acc);
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
          if (lane == 0) s_score[j] = __fmul_rn(acc, p.attn_scale);
        }
      }
    }
    // residue 2 pw's V rows load while the pair syncs
    float (&vr)[8][AE] = kr;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t j = 4u * i + 2u * pw;
      if (j < np && p0 + j != pos) ld_row<AE>(vcr + (size_t)(p0 + j) * row + kvi * HD + d0, vr[i]);
    }
    psync(pr);
    float mx = fmaxf(lane < np ? s_score[lane] : -INFINITY, lane + 32u < np ? s_score[lane + 32u] : -INFINITY);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
#pragma unroll
    for (int sr = 0; sr < 2; ++sr) {
      if (sr == 1) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t j = 4u * i + 2u * pw + 1u;
          if (j < np && p0 + j != pos) ld_row<AE>(vcr + (size_t)(p0 + j) * row + kvi * HD + d0, vr[i]);
        }
      }
      float o[AE];
#pragma unroll
      for (int e = 0; e < AE; ++e) o[e] = 0.0f;
      float l = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t j = 4u * i + 2u * pw + sr;
        if (j < np) {
          const float a = expf(s_score[j] - mx);
          l += a;
          if (p0 + j == pos) {
#pragma unroll
            for (int e = 0; e < AE; ++e) o[e] = __fmaf_rn(a, vn[e], o[e]);
          } else {
#pragma unroll
            for (int e = 0; e < AE; ++e) o[e] = __fmaf_rn(a, vr[i][e], o[e]);
          }
        }
      }
      const uint32_t r = 2u * pw + sr;
#pragma unroll
      for (int e = 0; e < AE; ++e) s_o[r * HD + d0 + e] = o[e];
      if (lane == 0) s_l[r] = l;
    }
    psync(pr);
    float* out = p.attn_part + ((size_t)hloc * p.max_chunks + c) * (HD + 4u);
    for (uint32_t d = pt; d < HD; d += 64u)
      out[4 + d] = ((s_o[d] + s_o[HD + d]) + s_o[2u * HD + d]) + s_o[3u * HD + d];
    if (pt == 0) {
      out[0] = mx;
      out[1] = ((s_l[0] + s_l[1]) + s_l[2]) + s_l[3];
    }
    __threadfence();
    psync(pr);
    if (pt == 0) s_last[0] = atomicAdd(&p.attn_count[hloc], 1u) == nvalid - 1u;
    psync(pr);
    if (s_last[0]) {
      __threadfence();
      // the last pair of the head: merge the chunks (log-sum-exp), normalise
      const float* base = p.attn_part + (size_t)hloc * p.max_chunks * (HD + 4u);
      for (uint32_t cc = pt; cc < nvalid; cc += 64u) {
        s_wc[cc] = __ldcg(base + cc * (HD + 4u));
        s_lc[cc] = __ldcg(base + cc * (HD + 4u) + 1);
      }
      constexpr int NDT = (HD + 63) / 64;  // dims per thread
      float od[NDT][kMergeBatch];
#pragma unroll
      for (int e = 0; e < NDT; ++e) {
        const uint32_t d = pt + 64u * e;
#pragma unroll
        for (uint32_t cc = 0; cc < kMergeBatch; ++cc)
          od[e][cc] = (d < HD && cc < nvalid) ? __ldcg(base + cc * (HD + 4u) + 4u + d) : 0.0f;
      }
      psync(pr);
      float gmx = -INFINITY;
      for (uint32_t cc = 0; cc < nvalid; ++cc) gmx = fmaxf(gmx, s_wc[cc]);
      psync(pr);
      for (uint32_t cc = pt; cc < nvalid; cc += 64u) s_wc[cc] = expf(s_wc[cc] - gmx);
      psync(pr);
      float Ls = 0.0f;
      for (uint32_t cc = 0; cc < nvalid; ++cc) Ls += s_lc[cc] * s_wc[cc];
      const float inv = 1.0f / Ls;
#pragma unroll
      for (int e = 0; e < NDT; ++e) {
        const uint32_t d = pt + 64u * e;
        if (d < HD) {
          float acc = 0.0f;
#pragma unroll
          for (uint32_t cc = 0; cc < kMergeBatch; ++cc)
            if (cc < nvalid) acc = __fmaf_rn(od[e][cc], s_wc[cc], acc);
          for (uint32_t cc = kMergeBatch; cc < nvalid; ++cc)
            acc = __fmaf_rn(__ldcg(base + cc * (HD + 4u) + 4u + d), s_wc[cc], acc);
          s_out[d] = acc * inv;
        }
      }
      if (pt == 0) p.attn_count[hloc] = 0u;
      psync(pr);
      for (uint32_t g = pw; g < (uint32_t)AE; g += 2u)
        pack_put(s_out[g * 32u + lane], gh * AE + g, lane, p.ao_out, p.world, eo);
    }
    psync(pr);  // the pair's scratch is free for its next item
  }
  if (__syncthreads_or(!ok)) {
    if (tid == 0) report(&p.state->err, EOS_DEVERR_WAIT_ACT);
    return false;
  }
  return true;
}

// Before the QKV GEMV: each warp pair asks L2 for the cached K and V rows of
// the chunk it will attend to (they do not depend on this step), one
// 4·AE·32-byte head slice per lane, so the attention's loads hit L2 instead
// of queueing behind the weight stream in HBM.
template <int AE>
__device__ __forceinline__ void attn_prefetch(uint32_t L) {
  constexpr uint32_t HD = 32u * AE;
  const PStepParams& p = P();
  const uint32_t pos = C().pos;
  const uint32_t tid = threadIdx.x, pr = tid >> 6, pt = tid & 63u;
  const uint32_t nvalid = pos / kAttnChunk + 1u;
  const uint32_t it = blockIdx.x * kPPairs + pr;
  if (it >= p.hl * nvalid) return;
  const uint32_t hloc = it / nvalid, c = it - hloc * nvalid;
  const uint32_t gkv = ((p.h0 + hloc) * p.n_kv_head) / p.n_head, kvi = gkv - p.kv0;
  const uint32_t j = pt & 31u, p0 = c * kAttnChunk;
  if (p0 + j >= pos) return;  // rows < pos only (the row at pos is this step's)
  const uint32_t row = p.kvl * HD;
  const float* base = (pt < 32u ? p.kc : p.vc) + ((size_t)L * p.max_ctx + p0 + j) * row + kvi * HD;
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base), "r"(HD * 4u) : "memory");
}

// silu(gate) * up of this rank's FFN units, one warp per 32-group, packed and
// pushed to every rank (silu_pack_kernel).
__device__ __forceinline__ bool silu_phase(uint32_t L) {
  const PStepParams& p = P();
  const uint32_t ebase = C().ebase;
  const uint64_t limit_ns = C().limit_ns;
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  const uint32_t groups = p.ffl >> 5;
  const uint32_t eg = pepoch(ebase, L, 3), ea = pepoch(ebase, L, 4);
  bool ok = true;
  for (uint32_t g = blockIdx.x * kPW + warp; g < groups; g += gridDim.x * kPW) {
    const uint32_t i = (g << 5) + lane;
    uint64_t a, b, t0 = 0;
    bool ready;
    do {
      a = ld_pair(p.gu_x + i);
      b = ld_pair(p.gu_x + p.ffl + i);
      ready = (uint32_t)(a >> 32) == eg && (uint32_t)(b >> 32) == eg;
      if (!ready && !keep_polling(t0, limit_ns, &p.state->err)) {
        ok = false;
        break;
      }
    } while (!ready);
    if (!__all_sync(0xffffffffu, ok)) {
      ok = false;
      break;
    }
    const float gv = __uint_as_float((uint32_t)a), uv = __uint_as_float((uint32_t)b);
    // x * (1 / (1 + expf(-x))) (silu.c:17), then gate * up (text.c:417)
    const float hv = __fmul_rn(__fmul_rn(gv, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gv)))), uv);
    pack_put(hv, (p.ff0 >> 5) + g, lane, p.ad_out, p.world, ea);
  }
  if (__syncthreads_or(!ok)) {
    if (threadIdx.x == 0) report(&p.state->err, EOS_DEVERR_WAIT_ACT);
    return false;
  }
  return true;
}

// ---------------------------------------------------------------------------
// Greedy pick (argmax_kernel): first index of the largest logit
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool pbetter(float av, uint32_t ai, float bv, uint32_t bi) {
  if (av != av) return false;
  if (bv != bv) return true;
  return av > bv || (av == bv && ai < bi);
}

__device__ __forceinline__ void preduce_block(float& v, uint32_t& idx, float* sv, uint32_t* si) {
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (pbetter(ov, oi, v, idx)) {
      v = ov;
      idx = oi;
    }
  }
  __syncthreads();
  if (lane == 0) {
    sv[warp] = v;
    si[warp] = idx;
  }
  __syncthreads();
  v = sv[0];
  idx = si[0];
  for (uint32_t w = 1; w < kPW; ++w)
    if (pbetter(sv[w], si[w], v, idx)) {
      v = sv[w];
      idx = si[w];
    }
}

}  // namespace

// ---------------------------------------------------------------------------
// The step
// ---------------------------------------------------------------------------
template <int AE>
__global__ void __launch_bounds__(kPT, 1) text_step_persistent_kernel(const __grid_constant__ PStepParams prm) {
  constexpr uint32_t HD = 32u * AE;
  const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
  {  // the parameters and the step's context into shared memory
    const uint32_t* src = reinterpret_cast<const uint32_t*>(&prm);
    uint32_t* dst = reinterpret_cast<uint32_t*>(g_psmem);
    for (uint32_t i = tid; i < sizeof(PStepParams) / 4u; i += kPT) dst[i] = src[i];
    // and the layer table (read at every matrix a warp's stream enters)
    const PSmem lay = psmem_layout(prm.E, prm.F, HD, prm.max_chunks, prm.n_layer);
    const uint32_t* ls = reinterpret_cast<const uint32_t*>(prm.layers);
    uint32_t* ld = reinterpret_cast<uint32_t*>(g_psmem + lay.layers);
    for (uint32_t i = tid; i < prm.n_layer * (uint32_t)sizeof(PLayer) / 4u; i += kPT) ld[i] = ls[i];
    if (tid == 0) {
      PCtx c;
      c.lay = psmem_layout(prm.E, prm.F, HD, prm.max_chunks, prm.n_layer);
      // the step's words (written by the previous step or the host)
      c.pos = prm.state->pos;
      c.tok = c.pos < prm.state->n_prompt ? prm.prompt[c.pos] : prm.state->next_token;
      c.ebase = prm.state->epoch * (kPX * prm.n_layer + 1u);
      c.nmat = 4u * prm.n_layer + 1u;
      c.limit_ns = (uint64_t)prm.state->wait_limit_us * 1000ull;
      *reinterpret_cast<PCtx*>(g_psmem + kPCtxOff) = c;
    }
    __syncthreads();
  }
  const PStepParams& p = P();
  {  // every warp's ring barriers, and its stream's first kPD stages
    uint64_t* bars_w = at<uint64_t>(C().lay.bars) + warp * kPD;
    if (lane == 0) {
      for (uint32_t d = 0; d < kPD; ++d) mbar_init(bars_w + d, 1u);
      fence_barrier_init();
    }
    __syncwarp();
    PStream s;
    s.in.mi = 0;
    cursor_seek(p, s.in, warp, HD, C().nmat);
    s.cur = s.in;
    s.t = 0;
    s.issued = 0;
    uint8_t* ring_w = at<uint8_t>(C().lay.ring) + warp * kPD * kPStage;
#pragma unroll
    for (uint32_t d = 0; d < kPD; ++d)
      s.issued += issue_stage(p, s.in, ring_w, bars_w, d, lane, warp, HD, C().nmat, l2_policy_evict_first());
    if (lane == 0) *at<PStream>(C().lay.streams + warp * 128u) = s;
    __syncwarp();
  }

  bool ok = true;
  for (uint32_t L = 0; L < p.n_layer && ok; ++L) {
    const uint32_t eb = C().ebase;
    // x1 = (L == 0 ? embedding : x0 + down output); act = pack(rmsnorm(x1))
    ok = norm_phase<4>(L == 0 ? nullptr : p.d_in, L == 0 ? 0u : pepoch(eb, L - 1u, 5),
                       at<const PLayer>(C().lay.layers)[L].attn_norm);
    if (!ok) break;
    attn_prefetch<AE>(L);
    gemv_phase(4u * L, HD, kOutQkv, L);
    ok = attn_phase<AE>(L);
    if (!ok) break;
    ok = load_act_phase(P().ao_in, P().E / Q4K_ELEMS, pepoch(C().ebase, L, 1));
    if (!ok) break;
    gemv_phase(4u * L + 1u, HD, kOutO, L);
    // x0 = x1 + O output; act = pack(rmsnorm(x0))
    ok = norm_phase<4>(P().o_in, pepoch(C().ebase, L, 2), at<const PLayer>(C().lay.layers)[L].ffn_norm);
    if (!ok) break;
    gemv_phase(4u * L + 2u, HD, kOutGu, L);
    ok = silu_phase(L);
    if (!ok) break;
    ok = load_act_phase(P().ad_in, P().F / Q4K_ELEMS, pepoch(C().ebase, L, 4));
    if (!ok) break;
    gemv_phase(4u * L + 3u, HD, kOutDown, L);
  }
  if (ok)  // final norm (text.c:425-427)
    ok = norm_phase<4>(P().n_layer ? P().d_in : nullptr, P().n_layer ? pepoch(C().ebase, P().n_layer - 1u, 5) : 0u,
                       P().out_norm);
  if (!ok) {
    drain_stream();  // never exit with copies still landing in shared memory
    return;
  }
  // LM head (text.c:428-432), then this CTA's best (value, row) of its rows
  gemv_phase(4u * P().n_layer, HD, kOutLogits, 0u);
  drain_stream();   // nothing in flight (a no-op unless a stage wait gave up)
  __syncthreads();  // the CTA's logits are written (through L2)
  float bv = __int_as_float(0x7fc00000);  // "nothing yet"
  uint32_t bi = 0xffffffffu;
  {
    const uint32_t n = P().vl;
    const uint32_t r0 = (n * blockIdx.x) / gridDim.x, r1 = (n * (blockIdx.x + 1u)) / gridDim.x;
    for (uint32_t r = r0 + tid; r < r1; r += kPT) {
      const float v = __ldcg(P().logits + r);
      if (pbetter(v, r, bv, bi)) {
        bv = v;
        bi = r;
      }
    }
  }
  const uint32_t pos = C().pos;
  float* scratch = at<float>(C().lay.scratch);
  float* sv = scratch;
  uint32_t* si = reinterpret_cast<uint32_t*>(scratch + kPW);
  uint32_t* s_last = si + kPW;
  preduce_block(bv, bi, sv, si);
  if (tid == 0) {
    p.arg_v[blockIdx.x] = bv;
    p.arg_i[blockIdx.x] = bi;
    __threadfence();
    s_last[0] = atomicAdd(&p.state->arg_count, 1u) == gridDim.x - 1u;
  }
  __syncthreads();
  if (!s_last[0]) return;
  __threadfence();
  float v = __int_as_float(0x7fc00000);
  uint32_t idx = 0xffffffffu;
  for (uint32_t b = tid; b < gridDim.x; b += kPT) {
    const float qv = __ldcg(p.arg_v + b);
    const uint32_t qi = __ldcg(p.arg_i + b);
    if (pbetter(qv, qi, v, idx)) {
      v = qv;
      idx = qi;
    }
  }
  preduce_block(v, idx, sv, si);
  const float first = __ldcg(p.logits);
  uint32_t first_nan = (p.rank == 0 && first != first) ? 1u : 0u;
  uint32_t gidx = idx == 0xffffffffu ? idx : p.v0 + idx;
  if (p.world > 1) {
    if (tid == 0) {  // this slice's result into every rank's words (argmax_kernel)
      for (uint32_t q = 0; q < p.world; ++q) {
        p.recv[q]->arg_v[p.rank] = v;
        p.recv[q]->arg_i[p.rank] = gidx;
        if (p.rank == 0) p.recv[q]->first_nan = first_nan;
      }
    }
    if (!xchg_handshake(p.xs, true, false)) return;
    if (tid == 0) {
      v = __int_as_float(0x7fc00000);
      gidx = 0xffffffffu;
      const volatile XRecv* x = p.own;
      for (uint32_t q = 0; q < p.world; ++q) {  // rank order = vocabulary order
        (void)ld_acquire_sys(&p.own->flag[kXArgmax][q]);
        const float qv = x->arg_v[q];
        const uint32_t qi = x->arg_i[q];
        if (pbetter(qv, qi, v, gidx)) {
          v = qv;
          gidx = qi;
        }
      }
      first_nan = x->first_nan;
    }
  }
  if (tid == 0) {
    const uint32_t t = (first_nan || gidx == 0xffffffffu) ? 0u : gidx;
    p.out_tokens[pos] = t;
    p.state->next_token = t;
    p.state->arg_count = 0u;
    p.state->pos = pos + 1u;
    p.state->epoch = p.state->epoch + 1u;
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace {
SmemAttr g_pattr[2];
void (*pkernel(uint32_t hd))(const PStepParams) {
  return hd == 64 ? text_step_persistent_kernel<2> : text_step_persistent_kernel<4>;
}
}  // namespace

uint32_t persistent_step_smem(uint32_t E, uint32_t F, uint32_t hd, uint32_t max_chunks, uint32_t n_layer) {
  return psmem_layout(E, F, hd, max_chunks, n_layer).total;
}

// Can this device run the persistent step for the geometry (one CTA per SM,
// all resident)?  Sets the kernel's shared-memory attribute.
bool persistent_step_supported(uint32_t E, uint32_t F, uint32_t hd, uint32_t max_chunks, uint32_t n_layer,
                               int max_smem) {
  if ((hd != 64 && hd != 128) || E % Q4K_ELEMS || F % Q4K_ELEMS || E > 4096u || E == 0 || F == 0) return false;
  const uint32_t smem = persistent_step_smem(E, F, hd, max_chunks, n_layer);
  if (smem > (uint32_t)max_smem) return false;
  void (*fn)(const PStepParams) = pkernel(hd);
  if (ensure_smem_attr((const void*)fn, (int)smem, g_pattr[hd == 64 ? 0 : 1]) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, (int)kPT, smem) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return per_sm >= 1;
}

cudaError_t launch_persistent_step(const PStepParams& p, uint32_t hd, uint32_t grid, cudaStream_t st) {
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(grid);
  lc.blockDim = dim3(kPT);
  lc.dynamicSmemBytes = persistent_step_smem(p.E, p.F, hd, p.max_chunks, p.n_layer);
  lc.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the CTAs wait on one another
  attr[0].val.cooperative = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  return cudaLaunchKernelEx(&lc, pkernel(hd), p);
}

}  // namespace eos
