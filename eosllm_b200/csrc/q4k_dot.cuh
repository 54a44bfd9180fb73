// q4k_dot.cuh -- the exact Q4_K super-block dot of the reference's x86
// int8 path (src/kernels/avx2/matmul_q4_k_int8.c:216-264), used by the GEMV
// kernels (q4k_gemv.cu).
#pragma once

#include "eos_common.cuh"

namespace eos {

// ---------------------------------------------------------------------------
// Half a super-block, one lane
// ---------------------------------------------------------------------------
// dp4a with the first operand's bytes unsigned (the high nibbles kept in
// place, i.e. 16 * q_hi <= 240) and the second's signed (activations).
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Exact integer dots of one qs pair (32 bytes as two uint4) with the
// activation lanes of its two sub-blocks: lo nibbles x sub 2p, hi nibbles x
// sub 2p+1 (src/kernels/avx2/matmul_q4_k_int8.c:234-249).  The high-nibble
// dot is taken on the nibble in place (x16, exact) and shifted back.
__device__ __forceinline__ void pair_dots(uint4 q0, uint4 q1, int4 a0, int4 a1, int4 a2, int4 a3, int& dl, int& dh) {
  constexpr uint32_t LO = 0x0F0F0F0Fu, HI = 0xF0F0F0F0u;
  int l = __dp4a((int)(q0.x & LO), a0.x, 0);
  int h = dp4a_us(q0.x & HI, a2.x, 0);
  l = __dp4a((int)(q0.y & LO), a0.y, l);
  h = dp4a_us(q0.y & HI, a2.y, h);
  l = __dp4a((int)(q0.z & LO), a0.z, l);
  h = dp4a_us(q0.z & HI, a2.z, h);
  l = __dp4a((int)(q0.w & LO), a0.w, l);
  h = dp4a_us(q0.w & HI, a2.w, h);
  l = __dp4a((int)(q1.x & LO), a1.x, l);
  h = dp4a_us(q1.x & HI, a3.x, h);
  l = __dp4a((int)(q1.y & LO), a1.y, l);
  h = dp4a_us(q1.y & HI, a3.y, h);
  l = __dp4a((int)(q1.z & LO), a1.z, l);
  h = dp4a_us(q1.z & HI, a3.z, h);
  l = __dp4a((int)(q1.w & LO), a1.w, l);
  h = dp4a_us(q1.w & HI, a3.w, h);
  dl = l;
  dh = h >> 4;  // exact: the sum is a multiple of 16
}

// t_s = ((d*sc_s)*as_s)*dot_s - ((dmin*m_s)*as_s)*sum_s, in the reference's
// order (:254-261).
__device__ __forceinline__ float sb_term(float d, float dmin, uint32_t sc, uint32_t m, float as, float sum, int dot) {
  return __fsub_rn(__fmul_rn(__fmul_rn(__fmul_rn(d, (float)sc), as), (float)dot),
                   __fmul_rn(__fmul_rn(__fmul_rn(dmin, (float)m), as), sum));
}

// The four terms of sub-blocks 4h..4h+3.  blk: the 144-byte GGUF super-block,
// half: its 160-byte activation half-record (both 16-byte aligned, shared or
// global memory).  The 6-bit scales/mins come out byte-parallel: get_scale_min
// (:58-67) for all j at once.
__device__ __forceinline__ void q4k_half_terms(const uint8_t* blk, const uint8_t* half, uint32_t h, float (&t)[4]) {
  const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
  const float d = f16_bits_to_f32(hdr.x), dmin = f16_bits_to_f32(hdr.x >> 16);
  // sc[4h .. 4h+3] and m[4h .. 4h+3] as bytes of one word each
  const uint32_t scw = h == 0 ? (hdr.y & 0x3F3F3F3Fu) : ((hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u));
  const uint32_t mw = h == 0 ? (hdr.z & 0x3F3F3F3Fu) : (((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u));
  const uint8_t* qs = blk + 16 + 64 * h;
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const uint4 q0 = *reinterpret_cast<const uint4*>(qs + 32 * p);
    const uint4 q1 = *reinterpret_cast<const uint4*>(qs + 32 * p + 16);
    const int4 a0 = *reinterpret_cast<const int4*>(half + 64 * p);
    const int4 a1 = *reinterpret_cast<const int4*>(half + 64 * p + 16);
    const int4 a2 = *reinterpret_cast<const int4*>(half + 64 * p + 32);
    const int4 a3 = *reinterpret_cast<const int4*>(half + 64 * p + 48);
    const float4 st = *reinterpret_cast<const float4*>(half + 128 + 16 * p);
    int dl, dh;
    pair_dots(q0, q1, a0, a1, a2, a3, dl, dh);
    t[2 * p] = sb_term(d, dmin, (scw >> (16 * p)) & 0xFFu, (mw >> (16 * p)) & 0xFFu, st.x, st.y, dl);
    t[2 * p + 1] = sb_term(d, dmin, (scw >> (16 * p + 8)) & 0xFFu, (mw >> (16 * p + 8)) & 0xFFu, st.z, st.w, dh);
  }
}

// Super-block partial from a lane pair (lane h = lane & 1 holds half h): the
// result is valid on the odd lane.  All 32 lanes must call it.
__device__ __forceinline__ float pair_partial(const float (&t)[4], uint32_t lane) {
  float s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(0.0f, t[0]), t[1]), t[2]), t[3]);
  const float first = __shfl_up_sync(0xffffffffu, s, 1);
  if (lane & 1u) s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(first, t[0]), t[1]), t[2]), t[3]);
  return s;
}

}  // namespace eos

namespace eos {

// The same four terms for R rows of one super-block column: row r's block at
// blk + r * row_stride.  The activation half-record is loaded once and reused
// by every row (the single-row form re-reads it per row).  Terms are
// bit-identical to q4k_half_terms.
// The activation half-record in registers: a[p][j] = int8 values 16 j ..
// 16 j + 15 of qs pair p, st[p] = the pair's {scale, sum} words.
__device__ __forceinline__ void q4k_load_half(const uint8_t* half, int4 (&a)[2][4], float4 (&st)[2]) {
#pragma unroll
  for (int p = 0; p < 2; ++p) {
#pragma unroll
    for (int j = 0; j < 4; ++j) a[p][j] = *reinterpret_cast<const int4*>(half + 64 * p + 16 * j);
    st[p] = *reinterpret_cast<const float4*>(half + 128 + 16 * p);
  }
}

// q4k_half_terms_rows with the half-record already in registers (a caller
// that computes many stages of one super-block column loads it once).
template <int R>
__device__ __forceinline__ void q4k_half_terms_rows_regs(const uint8_t* blk, uint32_t row_stride,
                                                         const int4 (&a)[2][4], const float4 (&st)[2], uint32_t h,
                                                         float (&t)[R][4], uint32_t rows = R) {
#pragma unroll
  for (int r = 0; r < R; ++r) {
    // rows beyond `rows` recompute the last row (the caller drops them)
    const uint8_t* rb = blk + ((uint32_t)r < rows ? (uint32_t)r : rows - 1u) * row_stride;
    const uint4 hdr = *reinterpret_cast<const uint4*>(rb);
    const float d = f16_bits_to_f32(hdr.x), dmin = f16_bits_to_f32(hdr.x >> 16);
    const uint32_t scw = h == 0 ? (hdr.y & 0x3F3F3F3Fu) : ((hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u));
    const uint32_t mw = h == 0 ? (hdr.z & 0x3F3F3F3Fu) : (((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u));
    const uint8_t* qs = rb + 16 + 64 * h;
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const uint4 q0 = *reinterpret_cast<const uint4*>(qs + 32 * p);
      const uint4 q1 = *reinterpret_cast<const uint4*>(qs + 32 * p + 16);
      int dl, dh;
      pair_dots(q0, q1, a[p][0], a[p][1], a[p][2], a[p][3], dl, dh);
      t[r][2 * p] = sb_term(d, dmin, (scw >> (16 * p)) & 0xFFu, (mw >> (16 * p)) & 0xFFu, st[p].x, st[p].y, dl);
      t[r][2 * p + 1] =
          sb_term(d, dmin, (scw >> (16 * p + 8)) & 0xFFu, (mw >> (16 * p + 8)) & 0xFFu, st[p].z, st[p].w, dh);
    }
  }
}

template <int R>
__device__ __forceinline__ void q4k_half_terms_rows(const uint8_t* blk, uint32_t row_stride, const uint8_t* half,
                                                    uint32_t h, float (&t)[R][4], uint32_t rows = R) {
  int4 a[2][4];
  float4 st[2];
  q4k_load_half(half, a, st);
  q4k_half_terms_rows_regs<R>(blk, row_stride, a, st, h, t, rows);
}

}  // namespace eos
