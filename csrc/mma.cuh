// Warp-level tensor-core helpers (ldmatrix + mma.sync m16n8k16, fp16 in, fp32 accumulate)
// and the XOR-swizzled layout of a [rows][256] fp16 shared-memory tile.
#pragma once
#include "common.cuh"

namespace oscar {
namespace mma {

constexpr int kRowBytes = 512;  // 256 fp16

OSCAR_DEVICE uint32_t swz(int row, int chunk) {  // byte offset of a 16 B chunk in a 512 B row
  return row * kRowBytes + ((chunk ^ (row & 7)) << 4);
}

OSCAR_DEVICE void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
OSCAR_DEVICE void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
OSCAR_DEVICE void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
OSCAR_DEVICE void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                           uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
OSCAR_DEVICE uint32_t h2_u32(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Two INT2 codes -> exact fp16 pair.  The page layout puts the codes of adjacent
// dims 2m and 2m+1 of a 16-dim group at bits 2m and 16+2m of one 32-bit word, so
// (w >> 2m) & 0x00030003 holds both; OR-ing the exponent of 1024.0 makes the fp16
// values 1024 + c, and subtracting 1024 leaves c exactly.
OSCAR_DEVICE uint32_t codes_to_h2(uint32_t w, int m) {
  uint32_t h;
  const uint32_t x = w >> (2 * m);
  asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(h) : "r"(x), "r"(0x00030003u), "r"(0x64006400u));  // (x & a) | b
  __half2 v = *reinterpret_cast<__half2*>(&h);
  const __half2 bias = __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));
  v = __hsub2(v, bias);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Eight fp16 codes of one 32-bit word (pool bit order) as four fp16 pairs, without
// per-pair shifts: for pair m in 0..3 the two codes sit at bits 2m and 16+2m, so
// OR-ing them into the fp16 1024.0 gives 1024 + c * 4^m exactly (mantissa room up
// to 2^8 * 3), and one fma by 4^-m (power of two, exact) subtracts the 1024 and
// rescales.  Pairs 4..7 use the word shifted right by 8.
OSCAR_DEVICE void codes8_to_h2(uint32_t w, uint32_t (&out)[4]) {
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    uint32_t h;
    const uint32_t mask = 0x00030003u << (2 * m);
    asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(h) : "r"(w), "r"(mask), "r"(0x64006400u));
    const float sc = 1.f / (float)(1 << (2 * m));
    const __half2 s2 = __float2half2_rn(sc);
    const __half2 b2 = __float2half2_rn(-1024.f * sc);
    __half2 v = __hfma2(*reinterpret_cast<__half2*>(&h), s2, b2);
    out[m] = *reinterpret_cast<uint32_t*>(&v);
  }
}

}  // namespace mma
}  // namespace oscar
