// dequant.cu -- PackedTensor.unpack on the device (tinygrad-dx12
// src/tinygrad_dx12/codegen/decomp/dx12.py:49-106), bit-exact with the reference.
//
// One thread produces 4 consecutive elements (one reference "word": 2 bytes for 4-bit
// formats, 3 bytes for 6-bit formats, dx12.py:69-77), so every byte is read once and the
// stores of a warp are contiguous. Arbitrary element windows [begin, begin+count) are
// supported so that offsets past 2^31 elements / bits (test_packed.py:147-174) decode in
// 64-bit index arithmetic without materialising the whole tensor.
#include "common.cuh"
#include "kernels.h"

namespace b200 {

// dx12.py:78-92 -- exact FP4/FP6 -> FP8 encoding of an unscaled payload.
template <int FMT>
__device__ __forceinline__ uint8_t fp8_encode(uint32_t p, int target) {
  using F = Fmt<FMT>;
  const int tm = target == B200_DT_F8E4M3 ? 3 : 2, tb = target == B200_DT_F8E4M3 ? 7 : 15;
  const uint32_t fraction = p & ((1u << F::mbits) - 1u);
  const uint32_t exponent = (p >> F::mbits) & ((1u << F::ebits) - 1u);
  uint32_t subnormal = 0;
#pragma unroll
  for (int high = 0; high < F::mbits; ++high) {
    const uint32_t enc = ((uint32_t)(tb + 1 - F::bias - F::mbits + high) << tm) |
                         ((fraction << (tm - high)) & ((1u << tm) - 1u));
    if (fraction >= (1u << high)) subnormal = enc;
  }
  const uint32_t normal = ((exponent + tb - F::bias) << tm) | (fraction << (tm - F::mbits));
  return (uint8_t)(((p >> (F::bits - 1)) << 7) | (exponent == 0 ? subnormal : normal));
}

struct DequantArgs {
  const uint8_t *data;
  int64_t data_bytes;
  const void *scales;
  int sdt;
  int64_t cols, nblk, block;
  int64_t begin, count;
  void *out;
  int odt;
  int mode;  // 0 = numeric, 1 = fp8 exact encoding
};

template <int FMT>
__global__ void __launch_bounds__(256) dequant_kernel(DequantArgs a) {
  constexpr int BITS = Fmt<FMT>::bits;
  constexpr int WB = BITS / 2;  // bytes per 4-element word
  const int64_t w_first = a.begin >> 2;
  const int64_t w_last = (a.begin + a.count - 1) >> 2;
  for (int64_t w = w_first + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; w <= w_last;
       w += (int64_t)gridDim.x * blockDim.x) {
    // word build (dx12.py:72-75); bytes past the storage read as the reference's zero pad
    uint32_t word = 0;
    const int64_t b0 = w * WB;
#pragma unroll
    for (int i = 0; i < WB; ++i)
      if (b0 + i < a.data_bytes) word |= (uint32_t)__ldg(a.data + b0 + i) << (8 * i);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t e = w * 4 + i;
      if (e < a.begin || e >= a.begin + a.count) continue;
      const uint32_t p = (word >> (i * BITS)) & ((1u << BITS) - 1u);
      const int64_t o = e - a.begin;
      if (a.mode == 1) {
        if constexpr (!Fmt<FMT>::is_int) ((uint8_t *)a.out)[o] = fp8_encode<FMT>(p, a.odt);
        continue;
      }
      if (a.scales == nullptr) {
        if constexpr (Fmt<FMT>::is_int) store_i64(a.out, o, a.odt, (int64_t)decode_int<FMT>(p));
        else store_f32(a.out, o, a.odt, decode_fp<FMT>(p));
        continue;
      }
      const int64_t row = e / a.cols, col = e - row * a.cols;
      const int64_t si = row * a.nblk + col / a.block;
      const float v = decode_f32<FMT>(p);  // exact
      // multiply in least_upper(float32, scale dtype, out dtype) (dx12.py:103-105)
      if (a.sdt == B200_DT_F64 || a.odt == B200_DT_F64) {
        store_f64(a.out, o, a.odt, (double)v * load_as_f64(a.scales, si, a.sdt));
      } else {
        store_f32(a.out, o, a.odt, v * load_as_f32(a.scales, si, a.sdt));
      }
    }
  }
}

int32_t launch_dequant(const b200_packed_desc *w, int64_t begin, int64_t count, void *out, int32_t out_dtype,
                       bool fp8_exact, cudaStream_t stream) {
  if (count <= 0) return B200_OK;
  DequantArgs a;
  a.data = (const uint8_t *)w->data;
  a.data_bytes = w->data_bytes;
  a.scales = w->scales;
  a.sdt = w->scale_dtype;
  a.cols = w->cols;
  a.block = w->block_size;
  a.nblk = (w->cols + w->block_size - 1) / w->block_size;
  a.begin = begin;
  a.count = count;
  a.out = out;
  a.odt = out_dtype;
  a.mode = fp8_exact ? 1 : 0;
  const int64_t words = ((begin + count - 1) >> 2) - (begin >> 2) + 1;
  int64_t blocks = (words + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;  // grid-stride beyond 32 CTAs per SM
  switch (w->format) {
    case B200_FMT_INT4: dequant_kernel<B200_FMT_INT4><<<(unsigned)blocks, 256, 0, stream>>>(a); break;
    case B200_FMT_UINT4: dequant_kernel<B200_FMT_UINT4><<<(unsigned)blocks, 256, 0, stream>>>(a); break;
    case B200_FMT_FP4_E2M1: dequant_kernel<B200_FMT_FP4_E2M1><<<(unsigned)blocks, 256, 0, stream>>>(a); break;
    case B200_FMT_FP6_E2M3: dequant_kernel<B200_FMT_FP6_E2M3><<<(unsigned)blocks, 256, 0, stream>>>(a); break;
    case B200_FMT_FP6_E3M2: dequant_kernel<B200_FMT_FP6_E3M2><<<(unsigned)blocks, 256, 0, stream>>>(a); break;
    default: return b200_set_error(B200_ERR_INVALID, "unknown packed format %d", w->format);
  }
  B200_LAUNCH_CHECK();
  return B200_OK;
}

}  // namespace b200
