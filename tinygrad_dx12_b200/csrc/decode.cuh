// decode.cuh -- register decoders shared by the GEMV and GEMM kernels.
//
// Exact fp16 / bf16 values of packed payloads (tinygrad-dx12
// src/tinygrad_dx12/codegen/decomp/dx12.py:69-100): every INT4/UINT4/FP4/FP6 payload value
// has at most 4 significant bits and a small exponent range, so it is exact in both types.
//   * INT4 / UINT4: fp16 0x6400 | n == 1024 + n (bf16: 0x4300 | n == 128 + n) exactly, minus the
//     bias -- pairs payloads (i, i+4) of a 32-bit word;
//   * FP4 E2M1 / FP6 E2M3 / FP6 E3M2: the sm_100a conversions cvt.rn.f16x2.{e2m1,e2m3,e3m2}x2 --
//     pairs payloads (2i, 2i+1).
#pragma once

#include "common.cuh"

namespace b200 {
namespace gemv {

// ---- decode 8 payloads into 4 fp16 pairs (payload i, payload i+4) --------------------------
// 4-bit: v holds 8 nibbles (payload q at bits 4q). Returns pair i = (payload i, payload i+4).
template <int FMT>
__device__ __forceinline__ void decode8_4bit(uint32_t v, uint32_t (&p)[4]) {
  if constexpr (FMT == B200_FMT_INT4 || FMT == B200_FMT_UINT4) {
    // fp16 0x6400 | n == 1024 + n exactly; INT4 flips bit 3 first ((n ^ 8) - 8 == signed nibble).
    constexpr uint32_t X = FMT == B200_FMT_INT4 ? 0x00080008u : 0u;
    const uint32_t lo = v, hi = v >> 8;
    const uint32_t h0 = ((lo & 0x000F000Fu) ^ X) | 0x64006400u;         // 1024 + n0', 1024 + n4'
    const uint32_t h1 = ((lo & 0x00F000F0u) ^ (X << 4)) | 0x64006400u;  // 1024 + 16 n1'
    const uint32_t h2 = ((hi & 0x000F000Fu) ^ X) | 0x64006400u;
    const uint32_t h3 = ((hi & 0x00F000F0u) ^ (X << 4)) | 0x64006400u;
    // h0 = 1024 + n' -> n' - bias ; h1 = 1024 + 16 n' -> (h1 / 16) - 64 - bias  (bias 8 for INT4)
    const float bias = FMT == B200_FMT_INT4 ? 8.f : 0.f;
    const __half2 c0 = __float2half2_rn(1024.f + bias), c16 = __float2half2_rn(0.0625f),
                  c1 = __float2half2_rn(-(64.f + bias));
    __half2 r0 = __hsub2(*reinterpret_cast<const __half2 *>(&h0), c0);
    __half2 r1 = __hfma2(*reinterpret_cast<const __half2 *>(&h1), c16, c1);
    __half2 r2 = __hsub2(*reinterpret_cast<const __half2 *>(&h2), c0);
    __half2 r3 = __hfma2(*reinterpret_cast<const __half2 *>(&h3), c16, c1);
    p[0] = *reinterpret_cast<uint32_t *>(&r0);
    p[1] = *reinterpret_cast<uint32_t *>(&r1);
    p[2] = *reinterpret_cast<uint32_t *>(&r2);
    p[3] = *reinterpret_cast<uint32_t *>(&r3);
  } else {
    // FP4 E2M1: the sm_100a conversion turns the two payloads of a byte (low nibble first)
    // into their exact fp16 values; pair i = (payload 2i, payload 2i+1).
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
        "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
        "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
        "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
        : "=r"(p[0]), "=r"(p[1]), "=r"(p[2]), "=r"(p[3])
        : "r"(v));
  }
}

// Does the decode of FMT pair payloads (i, i+4) (integer magic) or (2i, 2i+1) (conversions)?
template <int FMT>
__host__ __device__ constexpr bool pairs_04() {
  return FMT == B200_FMT_INT4 || FMT == B200_FMT_UINT4;
}

// 6-bit: 4 payloads in the low 24 bits -> one payload per byte (upper two bits zero).
__device__ __forceinline__ uint32_t spread6(uint32_t w) {
  const uint32_t u = (w & 0xFFFu) | ((w << 4) & 0x0FFF0000u);  // payloads 0,1 | 2,3 in 16-bit halves
  return (u & 0x003F003Fu) | ((u << 2) & 0x3F003F00u);
}
// 6-bit: the 8 payloads of a 48-bit value (payload q at bits 6q) -> pairs (2i, 2i+1) of exact
// fp16 values via the sm_100a FP6 conversions.
template <int FMT>
__device__ __forceinline__ void decode8_6bit(uint64_t v, uint32_t (&p)[4]) {
  const uint32_t s0 = spread6((uint32_t)v), s1 = spread6((uint32_t)(v >> 24));
  if constexpr (FMT == B200_FMT_FP6_E3M2) {
    asm("{\n\t.reg .b16 a, b, c, d;\n\t"
        "mov.b32 {a, b}, %4;\n\tmov.b32 {c, d}, %5;\n\t"
        "cvt.rn.f16x2.e3m2x2 %0, a;\n\tcvt.rn.f16x2.e3m2x2 %1, b;\n\t"
        "cvt.rn.f16x2.e3m2x2 %2, c;\n\tcvt.rn.f16x2.e3m2x2 %3, d;\n\t}"
        : "=r"(p[0]), "=r"(p[1]), "=r"(p[2]), "=r"(p[3])
        : "r"(s0), "r"(s1));
  } else {
    asm("{\n\t.reg .b16 a, b, c, d;\n\t"
        "mov.b32 {a, b}, %4;\n\tmov.b32 {c, d}, %5;\n\t"
        "cvt.rn.f16x2.e2m3x2 %0, a;\n\tcvt.rn.f16x2.e2m3x2 %1, b;\n\t"
        "cvt.rn.f16x2.e2m3x2 %2, c;\n\tcvt.rn.f16x2.e2m3x2 %3, d;\n\t}"
        : "=r"(p[0]), "=r"(p[1]), "=r"(p[2]), "=r"(p[3])
        : "r"(s0), "r"(s1));
  }
}

template <int FMT>
__host__ __device__ constexpr float place_factor() {
  return 1.f;  // every decode above yields exact payload values
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 8 payloads starting at unit c of a row held in words `w` -> 4 pairs in natural order
// (payload 2i, 2i+1) of exact values in fp16 (BF16 = false) or bf16 (BF16 = true).
template <int FMT, bool BF16>
__device__ __forceinline__ void decode8_natural(const uint32_t *w, int c, uint32_t (&out)[4]) {
  uint32_t h[4];
  if constexpr (Fmt<FMT>::bits == 4) {
    decode8_4bit<FMT>(w[c], h);
    if constexpr (pairs_04<FMT>()) {  // (i, i+4) -> (2i, 2i+1)
      const uint32_t q0 = __byte_perm(h[0], h[1], 0x5410), q1 = __byte_perm(h[2], h[3], 0x5410);
      const uint32_t q2 = __byte_perm(h[0], h[1], 0x7632), q3 = __byte_perm(h[2], h[3], 0x7632);
      h[0] = q0, h[1] = q1, h[2] = q2, h[3] = q3;
    }
  } else {
    const int bit = 48 * c, wi = bit >> 5, sh = bit & 31;  // the unit lies in words wi, wi+1
    decode8_6bit<FMT>((((uint64_t)w[wi + 1] << 32) | w[wi]) >> sh, h);
  }
  if constexpr (BF16) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&h[i]));
      const __nv_bfloat162 b = __floats2bfloat162_rn(f.x, f.y);  // exact: values are bf16-representable
      out[i] = *reinterpret_cast<const uint32_t *>(&b);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) out[i] = h[i];
  }
}

}  // namespace gemv
}  // namespace b200
