// mx.cuh -- pieces shared by the block-scaled tcgen05 decode kernels (gemv_mx.cu: x pieces
// staged per stage in a ring, any token count; gemv_mxs.cu: x pieces resident for 1..4 tokens).
#pragma once

#include <cuda_fp4.h>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace b200 {
namespace mx {

constexpr int TM = 128;           // weight rows per tile (the MMA's M)
constexpr int KB = 128;           // K codes per tensor-map box of the packed types
constexpr int KS = 2 * KB;        // K codes per stage

// weight-scale handling, a template parameter of the kernels
enum { SM_E8M0 = 0, SM_ROW = 1, SM_NONE = 2 };

// UMMA formats of the A operand (instruction descriptor bits 7..9)
template <int FMT>
__host__ __device__ constexpr uint32_t a_format() {
  return FMT == B200_FMT_FP4_E2M1 ? 5u : FMT == B200_FMT_FP6_E2M3 ? 3u : 4u;
}

// Work split (stream-K): CTA c of the persistent grid takes units [c * U / G, (c + 1) * U / G).
template <class PP>
__device__ __forceinline__ int64_t unit_start(const PP &p, int64_t c) { return c * p.units / p.grid; }

// CTA whose unit range holds unit u.
template <class PP>
__device__ __forceinline__ int owner(const PP &p, int64_t u) {
  int64_t c = u * p.grid / p.units;
  while (c + 1 < p.grid && unit_start(p, c + 1) <= u) ++c;
  while (c > 0 && unit_start(p, c) > u) --c;
  return (int)c;
}

// D (+)= (A x SFA) * (B x SFB)^T, kind::mxf8f6f4, one E8M0 scale per 32 K per row of A and B.
__device__ __forceinline__ void mma_mx(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc,
                                       uint32_t sfa, uint32_t sfb) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb)
      : "memory");
}

__device__ __forceinline__ void tmem_ld_x8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Split 8 activations (one lane's share of a 32-element block, 4 lanes per block) into P E4M3
// pieces with the block's E8M0 scale; returns the scale byte. `v` holds the values as float.
template <int P>
__device__ __forceinline__ uint32_t split_pieces(float (&v)[8], uint2 (&out)[P]) {
  float amax = 0.f;
  uint32_t nonfinite = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float a = fabsf(v[i]);
    nonfinite |= a <= 3.4e38f ? 0u : 1u;  // Inf or NaN
    amax = fmaxf(amax, a);
  }
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  nonfinite |= __shfl_xor_sync(0xffffffffu, nonfinite, 1);
  nonfinite |= __shfl_xor_sync(0xffffffffu, nonfinite, 2);
  uint32_t byte;
  if (nonfinite) byte = 255u;  // a NaN block scale: the block's products become NaN
  else if (amax == 0.f) byte = 127u;
  else {
    const int b = ilogbf(amax) + 120;  // scale 2^(ilogb-7): the maximum lands in [128, 256)
    byte = (uint32_t)(b < 1 ? 1 : b > 253 ? 253 : b);
  }
  const float inv = byte == 255u ? 0.f : __uint_as_float((254u - byte) << 23);  // 2^(127 - byte)
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] *= inv;
#pragma unroll
  for (int q = 0; q < P; ++q) {
    uint32_t w[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) w[h] = __nv_cvt_float2_to_fp8x2(make_float2(v[2 * h], v[2 * h + 1]), __NV_SATFINITE, __NV_E4M3);
    out[q] = make_uint2(w[0] | (w[1] << 16), w[2] | (w[3] << 16));
    if (q + 1 < P) {
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const __half2_raw b2 = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)w[h], __NV_E4M3);
        v[2 * h] -= __half2float(__ushort_as_half(b2.x));
        v[2 * h + 1] -= __half2float(__ushort_as_half(b2.y));
      }
    }
  }
  return byte;
}

// The NP FP4 E2M1 pieces of 8 values under a given E8M0 scale byte of piece 0 (piece q: byte - 2q):
// piece 0 rounds r / 2^(byte-127) to E2M1, each later piece the remainder at a quarter of the
// previous scale. out[q] holds the 8 codes (low nibble = lower element). With |r| < 4 * 2^(byte-127)
// the error after NP pieces is at most 2^(byte-127-2NP).
template <int NP>
__device__ __forceinline__ void fp4_pieces(float (&r)[8], uint32_t byte, uint32_t (&out)[NP]) {
  float inv = __uint_as_float((254u - byte) << 23), scale = __uint_as_float(byte << 23);
#pragma unroll
  for (int q = 0; q < NP; ++q) {
    uint32_t w = 0;
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const __nv_fp4x2_storage_t c =
          __nv_cvt_float2_to_fp4x2(make_float2(r[2 * h] * inv, r[2 * h + 1] * inv), __NV_E2M1, cudaRoundNearest);
      w |= (uint32_t)c << (8 * h);
      if (q + 1 < NP) {
        const __half2_raw back = __nv_cvt_fp4x2_to_halfraw2(c, __NV_E2M1);
        r[2 * h] -= __half2float(__ushort_as_half(back.x)) * scale;
        r[2 * h + 1] -= __half2float(__ushort_as_half(back.y)) * scale;
      }
    }
    out[q] = w;
    inv *= 4.f;
    scale *= 0.25f;
  }
}

// Split 8 activations (one lane's share of a 32-element block, 4 lanes per block) into NP FP4
// E2M1 pieces. Piece 0 takes the E8M0 block scale 2^e that puts the block maximum in [2, 4),
// where the E2M1 grid step is 1, so its rounding error is at most 2^(e-1); piece q takes scale
// 2^(e-2q), under which the remaining values stay within +-2 and round with an error of at most
// a quarter step: every piece after the first adds two bits, and eight leave an error of at most
// 2^(e-16), below 2^-17 of the block maximum. out[q] holds the 8 codes (low nibble = lower
// element); the scale byte of piece q is byte0 - 2q.
template <int NP>
__device__ __forceinline__ uint32_t split_fp4(float (&r)[8], uint32_t (&out)[NP]) {
  float amax = 0.f;
  uint32_t nonfinite = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float a = fabsf(r[i]);
    nonfinite |= a <= 3.4e38f ? 0u : 1u;  // Inf or NaN
    amax = fmaxf(amax, a);
  }
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  nonfinite |= __shfl_xor_sync(0xffffffffu, nonfinite, 1);
  nonfinite |= __shfl_xor_sync(0xffffffffu, nonfinite, 2);
  if (nonfinite) {  // a NaN block scale on piece 0: the block's products become NaN
#pragma unroll
    for (int q = 0; q < NP; ++q) out[q] = 0u;
    return 255u;
  }
  if (amax == 0.f) {
#pragma unroll
    for (int q = 0; q < NP; ++q) out[q] = 0u;
    return 127u + 2u * (NP - 1);  // every piece's scale byte stays >= 127
  }
  const int b = ilogbf(amax) + 126;  // scale 2^(ilogb-1): the maximum lands in [2, 4)
  const uint32_t byte = (uint32_t)(b < 2 * NP - 1 ? 2 * NP - 1 : b > 253 ? 253 : b);
  fp4_pieces<NP>(r, byte, out);
  return byte;
}

// D (+)= (A x SFA) * (B x SFB)^T, kind::mxf4: E2M1 A and B, K = 64, one E8M0 scale per 32 K.
__device__ __forceinline__ void mma_mxf4(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc,
                                         uint32_t sfa, uint32_t sfb) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb)
      : "memory");
}

// 8 activations (one 16-byte load of bf16 or fp16) as float.
template <bool XBF16>
__device__ __forceinline__ void raw_to_f32(const uint4 raw, float (&v)[8]) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (XBF16) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    } else {
      v[2 * i] = __half2float(__ushort_as_half((unsigned short)(w[i] & 0xFFFFu)));
      v[2 * i + 1] = __half2float(__ushort_as_half((unsigned short)(w[i] >> 16)));
    }
  }
}

template <bool XBF16>
__device__ __forceinline__ void load8(const uint16_t *src, float (&v)[8]) {
  const uint4 raw = *reinterpret_cast<const uint4 *>(src);
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (XBF16) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    } else {
      v[2 * i] = __half2float(__ushort_as_half((unsigned short)(w[i] & 0xFFFFu)));
      v[2 * i + 1] = __half2float(__ushort_as_half((unsigned short)(w[i] >> 16)));
    }
  }
}


inline int scale_mode(const LinearArgs &a) {
  if (a.scales == nullptr) return SM_NONE;
  if (a.nblk == 1) return SM_ROW;
  return SM_E8M0;
}

// The fp32 partials of split tiles ([SMs][2][<= 64 tokens][128 rows]) and one ticket per 128-row
// tile, per (device, stream); allocated on first use outside stream capture (gemv_mx.cu).
struct Workspace {
  float *part = nullptr;
  unsigned int *tickets = nullptr;
  size_t part_bytes = 0, tickets_n = 0;
};
constexpr size_t TICKETS = 16384;  // 128-row tiles: N <= 2M rows
int32_t workspace_for(cudaStream_t stream, bool may_allocate, Workspace *&out);

}  // namespace mx

// the resident-pieces kernel for FP4 weights and 1..4 tokens (gemv_mxs.cu); the caller has
// checked mx_supported
bool mxs_supported(const LinearArgs &a);
int32_t launch_mxs(const LinearArgs &a, const mx::Workspace &w, cudaStream_t stream);
}  // namespace b200
