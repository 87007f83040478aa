// gemv_simt.cu -- fp32 CUDA-core fused decode + dot: y[m, n] = sum_k x[m, k] * W[n, k].
//
// The general-purpose fused path (any M, x in f16/bf16/f32, scales f16/bf16/f32/e8m0 with
// block_size % 32 == 0 or one block per row). It is the fp32-activation path of
// linalg.matmul / linalg.matvec (tinygrad-dx12 src/tinygrad_dx12/codegen/linalg.py:136-298)
// and the fallback for shapes the tensor-core kernels do not take.
//
// Work split: a warp owns R consecutive weight rows; lane l streams 32-element chunks
// l, l+32, ... of those rows (16 bytes per row for 4-bit formats, 24 bytes for 6-bit),
// decodes them in registers (common.cuh, bit-exact with dx12.py:69-100), multiplies by x in
// float32 and accumulates per chunk; the chunk's block scale multiplies the chunk partial
// (sum_k x*c*s == s * sum_k x*c, one rounding later). Lanes reduce with warp shuffles.
#include "common.cuh"
#include "kernels.h"

namespace b200 {

template <typename XT>
__device__ __forceinline__ void load_x8(const XT *p, float (&v)[8]) {
  if constexpr (sizeof(XT) == 2) {
    const uint4 u = __ldg(reinterpret_cast<const uint4 *>(p));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (std::is_same<XT, __half>::value) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
        v[2 * i] = f.x, v[2 * i + 1] = f.y;
      } else {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
      }
    }
  } else {
    const float4 a = __ldg(reinterpret_cast<const float4 *>(p));
    const float4 b = __ldg(reinterpret_cast<const float4 *>(p) + 1);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
  }
}

// payload i (0..31) of a 32-element chunk held in CW 32-bit words
template <int BITS, int CW>
__device__ __forceinline__ uint32_t chunk_code(const uint32_t (&w)[CW], int i) {
  const int bit = i * BITS, wi = bit >> 5, sh = bit & 31;
  uint32_t v = w[wi] >> sh;
  if (sh + BITS > 32) v |= w[wi + 1] << (32 - sh);
  return v & ((1u << BITS) - 1u);
}

template <int FMT, typename XT, int MT, int R>
__global__ void __launch_bounds__(256) gemv_simt_kernel(LinearArgs a) {
  constexpr int BITS = Fmt<FMT>::bits;
  constexpr int CB = 32 * BITS / 8;  // chunk bytes: 16 or 24
  constexpr int CW = CB / 4;         // chunk words: 4 or 6
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row0 = ((int64_t)blockIdx.x * (blockDim.x >> 5) + warp) * R;
  const int64_t m0 = (int64_t)blockIdx.y * MT;
  if (row0 >= a.rows) return;
  const int64_t row_bytes = a.cols * BITS / 8;
  const int64_t nchunks = a.cols >> 5;
  const XT *x = reinterpret_cast<const XT *>(a.x);
  float acc[R][MT];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int i = 0; i < MT; ++i) acc[r][i] = 0.f;

  for (int64_t c = lane; c < nchunks; c += 32) {
    uint32_t w[R][CW];
    float s[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t row = row0 + r;
      const bool ok = row < a.rows;
      const uint8_t *p = a.w + (ok ? row : 0) * row_bytes + c * CB;
      if constexpr (CB == 16) {
        uint4 u = ok ? __ldg(reinterpret_cast<const uint4 *>(p)) : make_uint4(0, 0, 0, 0);
        w[r][0] = u.x, w[r][1] = u.y, w[r][2] = u.z, w[r][3] = u.w;
      } else {
#pragma unroll
        for (int q = 0; q < 3; ++q) {
          uint2 u = ok ? __ldg(reinterpret_cast<const uint2 *>(p) + q) : make_uint2(0, 0);
          w[r][2 * q] = u.x, w[r][2 * q + 1] = u.y;
        }
      }
      s[r] = 1.f;
      if (a.scales != nullptr && ok) s[r] = load_as_f32(a.scales, row * a.nblk + (c * 32) / a.block, a.sdt);
    }
#pragma unroll
    for (int i = 0; i < MT; ++i) {
      if (m0 + i >= a.m) break;
      const XT *xr = x + (m0 + i) * a.ldx + c * 32;
      float part[R];
#pragma unroll
      for (int r = 0; r < R; ++r) part[r] = 0.f;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float xv[8];
        load_x8<XT>(xr + q * 8, xv);
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int j = 0; j < 8; ++j) part[r] = fmaf(xv[j], decode_f32<FMT>(chunk_code<BITS, CW>(w[r], q * 8 + j)), part[r]);
      }
#pragma unroll
      for (int r = 0; r < R; ++r) acc[r][i] = fmaf(part[r], s[r], acc[r][i]);
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
#pragma unroll
    for (int i = 0; i < MT; ++i) {
      float v = acc[r][i];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      const int64_t row = row0 + r;
      if (lane == 0 && row < a.rows && m0 + i < a.m) store_f32(a.y, (m0 + i) * a.ldy_m + row * a.ldy_n, a.ydt, v);
    }
  }
}

bool simt_supported(const LinearArgs &a) {
  if (a.xdt != B200_DT_F16 && a.xdt != B200_DT_BF16 && a.xdt != B200_DT_F32) return false;
  if (a.ydt != B200_DT_F16 && a.ydt != B200_DT_BF16 && a.ydt != B200_DT_F32) return false;
  if (a.cols % 32 != 0 || a.cols <= 0 || a.rows <= 0 || a.m <= 0) return false;
  if (a.scales != nullptr) {
    if (!(a.sdt == B200_DT_F16 || a.sdt == B200_DT_BF16 || a.sdt == B200_DT_F32 || a.sdt == B200_DT_E8M0)) return false;
    if (!(a.block % 32 == 0 || a.block >= a.cols)) return false;
  }
  const int bits = fmt_bits(a.fmt);
  const uintptr_t wa = (uintptr_t)a.w;
  if (wa % (bits == 4 ? 16 : 8) != 0) return false;
  const int xs = a.xdt == B200_DT_F32 ? 4 : 2;
  if ((uintptr_t)a.x % 16 != 0 || (a.ldx * xs) % 16 != 0) return false;
  return true;
}

template <int FMT, typename XT>
static int32_t dispatch_mt(const LinearArgs &a, cudaStream_t stream) {
  const int warps = 8;
  auto grid = [&](int R, int MT) {
    return dim3((unsigned)((a.rows + (int64_t)warps * R - 1) / ((int64_t)warps * R)), (unsigned)((a.m + MT - 1) / MT));
  };
  if (a.m == 1) gemv_simt_kernel<FMT, XT, 1, 4><<<grid(4, 1), warps * 32, 0, stream>>>(a);
  else if (a.m == 2) gemv_simt_kernel<FMT, XT, 2, 4><<<grid(4, 2), warps * 32, 0, stream>>>(a);
  else if (a.m <= 4) gemv_simt_kernel<FMT, XT, 4, 2><<<grid(2, 4), warps * 32, 0, stream>>>(a);
  else gemv_simt_kernel<FMT, XT, 8, 2><<<grid(2, 8), warps * 32, 0, stream>>>(a);
  B200_LAUNCH_CHECK();
  return B200_OK;
}

template <int FMT>
static int32_t dispatch_x(const LinearArgs &a, cudaStream_t stream) {
  if (a.xdt == B200_DT_F16) return dispatch_mt<FMT, __half>(a, stream);
  if (a.xdt == B200_DT_BF16) return dispatch_mt<FMT, __nv_bfloat16>(a, stream);
  return dispatch_mt<FMT, float>(a, stream);
}

int32_t launch_gemv_simt(const LinearArgs &a, cudaStream_t stream) {
  switch (a.fmt) {
    case B200_FMT_INT4: return dispatch_x<B200_FMT_INT4>(a, stream);
    case B200_FMT_UINT4: return dispatch_x<B200_FMT_UINT4>(a, stream);
    case B200_FMT_FP4_E2M1: return dispatch_x<B200_FMT_FP4_E2M1>(a, stream);
    case B200_FMT_FP6_E2M3: return dispatch_x<B200_FMT_FP6_E2M3>(a, stream);
    case B200_FMT_FP6_E3M2: return dispatch_x<B200_FMT_FP6_E3M2>(a, stream);
  }
  return b200_set_error(B200_ERR_INVALID, "unknown packed format %d", a.fmt);
}

}  // namespace b200
