// decode.cuh — HEX index streams to 16-bit MMA operands, in registers.
//
// Per (row, scale block) the decoder builds the expert's level table already
// multiplied by the block's scale and rounded to the operand type:
//     T[l] = rne16(levels[l] * (fp8(code) * expert_scale))        (fp32 products)
// which is exactly the value every weight with index l in that block takes in
// the reference dequantization (blackhole/anatomy/hex.py:196-204), rounded
// once to bf16 / f16.  The table is held as two byte planes (low bytes and high
// bytes of the 8 or 16 entries), so one `prmt` looks up one byte of four weights
// at once; two more `prmt` interleave the planes into packed operand pairs.
//
// The codes arrive one per nibble (the layer's tiled copy of the index
// stream, hexmoe_tile_index), which is what prmt selectors are: a 3-bit code
// (8 levels, bit 3 of its nibble clear) selects its table byte directly; for
// a 4-bit code (16 levels) bit 3 selects between the two 8-entry halves
// through a sign-replicating prmt mask.
#pragma once

#include "ptx.cuh"

namespace hexmoe {

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  uint32_t r;
  if constexpr (BF16) {
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  } else {
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  }
  return r;
}

// fp8 e4m3 code -> float with the HEX rules (hex.py:199-203): exponent field 0
// is m/8 * 2^-6, every other exponent (1 + m/8) * 2^(e-7), including 0x7F/0xFF
// (+-480).  Built once per CTA into a 256-entry shared table.
__device__ __forceinline__ float fp8_hex_value(uint32_t c) {
  const uint32_t e = (c >> 3) & 15u, m = c & 7u;
  float v;
  if (e == 0) {
    v = static_cast<float>(m) * 0.001953125f;                       // m * 2^-9
  } else {
    v = __uint_as_float(((e + 120u) << 23) | (m << 20));             // (1 + m/8) * 2^(e-7)
  }
  return (c & 128u) ? -v : v;
}

struct Table8 {   // byte planes of 8 16-bit entries
  uint32_t l0, l1, h0, h1;
};
struct Table16 {  // entries 0-7 (a) and 8-15 (b)
  uint32_t la0, la1, lb0, lb1, ha0, ha1, hb0, hb1;
};

template <bool BF16>
__device__ __forceinline__ Table8 make_table8(const float* lev, float s) {
  const uint32_t p01 = pack2<BF16>(__fmul_rn(lev[0], s), __fmul_rn(lev[1], s));
  const uint32_t p23 = pack2<BF16>(__fmul_rn(lev[2], s), __fmul_rn(lev[3], s));
  const uint32_t p45 = pack2<BF16>(__fmul_rn(lev[4], s), __fmul_rn(lev[5], s));
  const uint32_t p67 = pack2<BF16>(__fmul_rn(lev[6], s), __fmul_rn(lev[7], s));
  Table8 t;
  t.l0 = prmt(p01, p23, 0x6420);
  t.h0 = prmt(p01, p23, 0x7531);
  t.l1 = prmt(p45, p67, 0x6420);
  t.h1 = prmt(p45, p67, 0x7531);
  return t;
}

template <bool BF16>
__device__ __forceinline__ Table16 make_table16(const float* lev, float s) {
  const Table8 a = make_table8<BF16>(lev, s);
  const Table8 b = make_table8<BF16>(lev + 8, s);
  Table16 t;
  t.la0 = a.l0; t.la1 = a.l1; t.ha0 = a.h0; t.ha1 = a.h1;
  t.lb0 = b.l0; t.lb1 = b.l1; t.hb0 = b.h0; t.hb1 = b.h1;
  return t;
}

__device__ __forceinline__ Table8 table8_from(const uint4& v) {
  Table8 t;
  t.l0 = v.x; t.l1 = v.y; t.h0 = v.z; t.h1 = v.w;
  return t;
}
__device__ __forceinline__ Table16 table16_from(const uint4& lo, const uint4& hi) {
  Table16 t;
  t.la0 = lo.x; t.la1 = lo.y; t.lb0 = lo.z; t.lb1 = lo.w;
  t.ha0 = hi.x; t.ha1 = hi.y; t.hb0 = hi.z; t.hb1 = hi.w;
  return t;
}

// 8 consecutive weights (3-bit codes, nibbles of w with bit 3 clear) -> 4
// packed operand pairs, K order.  prmt reads the low 16 bits of its selector:
// codes 0-3 from w itself, codes 4-7 from w >> 16.
__device__ __forceinline__ uint4 dec8_n3(uint32_t w, const Table8& t) {
  const uint32_t s0 = w;
  const uint32_t s1 = __umulhi(w, 65536u);            // w >> 16 on the FMA pipe
  const uint32_t lo0 = prmt(t.l0, t.l1, s0), hi0 = prmt(t.h0, t.h1, s0);
  const uint32_t lo1 = prmt(t.l0, t.l1, s1), hi1 = prmt(t.h0, t.h1, s1);
  uint4 o;
  o.x = prmt(lo0, hi0, 0x5140);
  o.y = prmt(lo0, hi0, 0x7362);
  o.z = prmt(lo1, hi1, 0x5140);
  o.w = prmt(lo1, hi1, 0x7362);
  return o;
}

// 8 consecutive weights (4-bit codes, nibbles of w) -> 4 packed operand pairs.
__device__ __forceinline__ uint4 dec8_b4(uint32_t w, const Table16& t) {
  const uint32_t s0 = w & 0x77777777u;
  const uint32_t s1 = __umulhi(s0, 65536u);
  const uint32_t w4 = w * 16u;
  const uint32_t m0 = prmt(w4, w, 0xD9C8);   // 0xFF per byte where code bit 3 is set (codes 0-3)
  const uint32_t m1 = prmt(w4, w, 0xFBEA);   // codes 4-7
  const uint32_t lo0 = lop3_sel(prmt(t.lb0, t.lb1, s0), prmt(t.la0, t.la1, s0), m0);
  const uint32_t hi0 = lop3_sel(prmt(t.hb0, t.hb1, s0), prmt(t.ha0, t.ha1, s0), m0);
  const uint32_t lo1 = lop3_sel(prmt(t.lb0, t.lb1, s1), prmt(t.la0, t.la1, s1), m1);
  const uint32_t hi1 = lop3_sel(prmt(t.hb0, t.hb1, s1), prmt(t.ha0, t.ha1, s1), m1);
  uint4 o;
  o.x = prmt(lo0, hi0, 0x5140);
  o.y = prmt(lo0, hi0, 0x7362);
  o.z = prmt(lo1, hi1, 0x5140);
  o.w = prmt(lo1, hi1, 0x7362);
  return o;
}

// One 32-weight block (4 tiled words, 8 codes each) -> 4 chunks of 8.
__device__ __forceinline__ void dec32_n3(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3, const Table8& t,
                                         uint4 (&c)[4]) {
  c[0] = dec8_n3(w0, t);
  c[1] = dec8_n3(w1, t);
  c[2] = dec8_n3(w2, t);
  c[3] = dec8_n3(w3, t);
}

__device__ __forceinline__ void dec32_b4(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3, const Table16& t,
                                         uint4 (&c)[4]) {
  c[0] = dec8_b4(w0, t);
  c[1] = dec8_b4(w1, t);
  c[2] = dec8_b4(w2, t);
  c[3] = dec8_b4(w3, t);
}

// Byte offset of 16-byte chunk `chunk` (0..7) of row `row` in a K-major tile
// of 128-byte rows stored with the 128-byte swizzle (the layout TMA SWIZZLE_128B
// writes and the UMMA SW128 descriptor reads).
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

}  // namespace hexmoe
