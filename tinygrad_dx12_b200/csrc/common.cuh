// common.cuh -- shared device helpers: packed-format decode, dtype loads/stores, errors.
//
// The decode arithmetic restates PackedTensor.unpack (tinygrad-dx12
// src/tinygrad_dx12/codegen/decomp/dx12.py:69-106) bit for bit:
//   word    = b0 | b1 << 8 [| b2 << 16]            (four elements per bits/2 bytes, LSB first)
//   payload = (word >> (i * bits)) & (2^bits - 1)
//   int4    = (payload ^ 8) - 8,  uint4 = payload
//   fp      = sign ? -(sig * 2^(max(e,1) - bias - m)) : +(...),  sig = e ? f + 2^m : f
// Every FP4/FP6 value is a dyadic rational with at most 4 significant bits, so building
// its float32 bit pattern directly is exactly the reference's fp32 product.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "../../include/b200_packed.h"

namespace b200 {

// (total bits, exponent bits, mantissa bits, bias) -- FORMATS, dx12.py:10
template <int FMT> struct Fmt;
template <> struct Fmt<B200_FMT_INT4> { static constexpr int bits = 4, ebits = 0, mbits = 0, bias = 0; static constexpr bool is_int = true, is_signed = true; };
template <> struct Fmt<B200_FMT_UINT4> { static constexpr int bits = 4, ebits = 0, mbits = 0, bias = 0; static constexpr bool is_int = true, is_signed = false; };
template <> struct Fmt<B200_FMT_FP4_E2M1> { static constexpr int bits = 4, ebits = 2, mbits = 1, bias = 1; static constexpr bool is_int = false, is_signed = true; };
template <> struct Fmt<B200_FMT_FP6_E2M3> { static constexpr int bits = 6, ebits = 2, mbits = 3, bias = 1; static constexpr bool is_int = false, is_signed = true; };
template <> struct Fmt<B200_FMT_FP6_E3M2> { static constexpr int bits = 6, ebits = 3, mbits = 2, bias = 3; static constexpr bool is_int = false, is_signed = true; };

__host__ __device__ inline int fmt_bits(int fmt) { return (fmt == B200_FMT_FP6_E2M3 || fmt == B200_FMT_FP6_E3M2) ? 6 : 4; }

// Exact float32 value of an FP payload (dx12.py:95-100).
template <int FMT>
__device__ __forceinline__ float decode_fp(uint32_t p) {
  using F = Fmt<FMT>;
  const uint32_t f = p & ((1u << F::mbits) - 1u);
  const uint32_t e = (p >> F::mbits) & ((1u << F::ebits) - 1u);
  const uint32_t s = (p >> (F::bits - 1)) & 1u;
  // normal: 2^(e-bias) * (1 + f/2^m) ; subnormal: f * 2^(1-bias-m)
  const float normal = __uint_as_float(((e + 127u - F::bias) << 23) | (f << (23 - F::mbits)));
  const float sub = (float)f * __uint_as_float((uint32_t)(127 + 1 - F::bias - F::mbits) << 23);
  const float mag = e ? normal : sub;
  return __uint_as_float(__float_as_uint(mag) | (s << 31));
}

// Integer value of an INT4/UINT4 payload (dx12.py:93-94).
template <int FMT>
__device__ __forceinline__ int decode_int(uint32_t p) {
  return Fmt<FMT>::is_signed ? (int)((p ^ 8u)) - 8 : (int)p;
}

// Payload value as float32 (exact for every format).
template <int FMT>
__device__ __forceinline__ float decode_f32(uint32_t p) {
  if constexpr (Fmt<FMT>::is_int) return (float)decode_int<FMT>(p);
  else return decode_fp<FMT>(p);
}

// ---- scalar loads/stores by runtime dtype --------------------------------------------
__device__ __forceinline__ float e8m0_to_f32(uint8_t b) {
  if (b == 0xFF) return __uint_as_float(0x7FC00000u);
  if (b == 0) return __uint_as_float(0x00400000u);  // 2^-127 (float32 subnormal)
  return __uint_as_float((uint32_t)b << 23);
}

__device__ __forceinline__ double load_as_f64(const void *p, int64_t i, int dt) {
  switch (dt) {
    case B200_DT_BOOL: return ((const uint8_t *)p)[i] ? 1.0 : 0.0;
    case B200_DT_I8: return ((const int8_t *)p)[i];
    case B200_DT_U8: return ((const uint8_t *)p)[i];
    case B200_DT_I16: return ((const int16_t *)p)[i];
    case B200_DT_U16: return ((const uint16_t *)p)[i];
    case B200_DT_I32: return ((const int32_t *)p)[i];
    case B200_DT_U32: return ((const uint32_t *)p)[i];
    case B200_DT_I64: return (double)((const int64_t *)p)[i];
    case B200_DT_U64: return (double)((const uint64_t *)p)[i];
    case B200_DT_F8E4M3: { __nv_fp8_e4m3 v; v.__x = ((const uint8_t *)p)[i]; return (double)(float)v; }
    case B200_DT_F8E5M2: { __nv_fp8_e5m2 v; v.__x = ((const uint8_t *)p)[i]; return (double)(float)v; }
    case B200_DT_F16: return __half2float(((const __half *)p)[i]);
    case B200_DT_BF16: return __bfloat162float(((const __nv_bfloat16 *)p)[i]);
    case B200_DT_F32: return ((const float *)p)[i];
    case B200_DT_F64: return ((const double *)p)[i];
    case B200_DT_E8M0: return (double)e8m0_to_f32(((const uint8_t *)p)[i]);
  }
  return 0.0;
}

__device__ __forceinline__ float load_as_f32(const void *p, int64_t i, int dt) {
  switch (dt) {
    case B200_DT_F16: return __half2float(((const __half *)p)[i]);
    case B200_DT_BF16: return __bfloat162float(((const __nv_bfloat16 *)p)[i]);
    case B200_DT_F32: return ((const float *)p)[i];
    case B200_DT_E8M0: return e8m0_to_f32(((const uint8_t *)p)[i]);
    default: return (float)load_as_f64(p, i, dt);
  }
}

__device__ __forceinline__ int64_t load_as_i64(const void *p, int64_t i, int dt) {
  switch (dt) {
    case B200_DT_BOOL: return ((const uint8_t *)p)[i] ? 1 : 0;
    case B200_DT_I8: return ((const int8_t *)p)[i];
    case B200_DT_U8: return ((const uint8_t *)p)[i];
    case B200_DT_I16: return ((const int16_t *)p)[i];
    case B200_DT_U16: return ((const uint16_t *)p)[i];
    case B200_DT_I32: return ((const int32_t *)p)[i];
    case B200_DT_U32: return ((const uint32_t *)p)[i];
    case B200_DT_I64: return ((const int64_t *)p)[i];
    case B200_DT_U64: return (int64_t)((const uint64_t *)p)[i];
    default: return (int64_t)load_as_f64(p, i, dt);
  }
}

// float -> fp8 with round-to-nearest-even; overflow saturates to the largest finite value.
__device__ __forceinline__ uint8_t f32_to_fp8(float v, int dt) {
  if (dt == B200_DT_F8E4M3) return (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
  return (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E5M2);
}

__device__ __forceinline__ void store_f64(void *p, int64_t i, int dt, double v) {
  switch (dt) {
    case B200_DT_BOOL: ((uint8_t *)p)[i] = v != 0.0; break;
    case B200_DT_I8: ((int8_t *)p)[i] = (int8_t)(int64_t)v; break;
    case B200_DT_U8: ((uint8_t *)p)[i] = (uint8_t)(int64_t)v; break;
    case B200_DT_I16: ((int16_t *)p)[i] = (int16_t)(int64_t)v; break;
    case B200_DT_U16: ((uint16_t *)p)[i] = (uint16_t)(int64_t)v; break;
    case B200_DT_I32: ((int32_t *)p)[i] = (int32_t)(int64_t)v; break;
    case B200_DT_U32: ((uint32_t *)p)[i] = (uint32_t)(int64_t)v; break;
    case B200_DT_I64: ((int64_t *)p)[i] = (int64_t)v; break;
    case B200_DT_U64: ((uint64_t *)p)[i] = (uint64_t)v; break;
    case B200_DT_F8E4M3:
    case B200_DT_F8E5M2: ((uint8_t *)p)[i] = f32_to_fp8((float)v, dt); break;
    case B200_DT_F16: ((__half *)p)[i] = __double2half(v); break;
    case B200_DT_BF16: ((__nv_bfloat16 *)p)[i] = __double2bfloat16(v); break;
    case B200_DT_F32: ((float *)p)[i] = (float)v; break;
    case B200_DT_F64: ((double *)p)[i] = v; break;
  }
}

__device__ __forceinline__ void store_f32(void *p, int64_t i, int dt, float v) {
  switch (dt) {
    case B200_DT_F16: ((__half *)p)[i] = __float2half_rn(v); break;
    case B200_DT_BF16: ((__nv_bfloat16 *)p)[i] = __float2bfloat16_rn(v); break;
    case B200_DT_F32: ((float *)p)[i] = v; break;
    case B200_DT_F8E4M3:
    case B200_DT_F8E5M2: ((uint8_t *)p)[i] = f32_to_fp8(v, dt); break;
    case B200_DT_I32: ((int32_t *)p)[i] = (int32_t)v; break;
    default: store_f64(p, i, dt, (double)v); break;
  }
}

__device__ __forceinline__ void store_i64(void *p, int64_t i, int dt, int64_t v) {
  switch (dt) {
    case B200_DT_I8: ((int8_t *)p)[i] = (int8_t)v; break;
    case B200_DT_U8: ((uint8_t *)p)[i] = (uint8_t)v; break;
    case B200_DT_I16: ((int16_t *)p)[i] = (int16_t)v; break;
    case B200_DT_U16: ((uint16_t *)p)[i] = (uint16_t)v; break;
    case B200_DT_I32: ((int32_t *)p)[i] = (int32_t)v; break;
    case B200_DT_U32: ((uint32_t *)p)[i] = (uint32_t)v; break;
    case B200_DT_I64: ((int64_t *)p)[i] = v; break;
    case B200_DT_U64: ((uint64_t *)p)[i] = (uint64_t)v; break;
    case B200_DT_BOOL: ((uint8_t *)p)[i] = v != 0; break;
    default: store_f64(p, i, dt, (double)v); break;
  }
}

__host__ __device__ inline bool dt_is_float(int dt) {
  return dt == B200_DT_F8E4M3 || dt == B200_DT_F8E5M2 || dt == B200_DT_F16 || dt == B200_DT_BF16 ||
         dt == B200_DT_F32 || dt == B200_DT_F64 || dt == B200_DT_E8M0;
}
__host__ __device__ inline int dt_size(int dt) {
  switch (dt) {
    case B200_DT_BOOL: case B200_DT_I8: case B200_DT_U8: case B200_DT_F8E4M3: case B200_DT_F8E5M2: case B200_DT_E8M0: return 1;
    case B200_DT_I16: case B200_DT_U16: case B200_DT_F16: case B200_DT_BF16: return 2;
    case B200_DT_I32: case B200_DT_U32: case B200_DT_F32: return 4;
    case B200_DT_I64: case B200_DT_U64: case B200_DT_F64: return 8;
  }
  return 0;
}

}  // namespace b200

// ---- host-side error plumbing (defined in capi.cu) ------------------------------------
int32_t b200_set_error(int32_t code, const char *fmt, ...);
#define B200_CUDA_TRY(expr)                                                                   \
  do {                                                                                        \
    cudaError_t _e = (expr);                                                                  \
    if (_e != cudaSuccess) return b200_set_error(B200_ERR_CUDA, "%s: %s (%s:%d)", #expr,       \
                                                 cudaGetErrorString(_e), __FILE__, __LINE__); \
  } while (0)
#define B200_LAUNCH_CHECK()                                                                   \
  do {                                                                                        \
    cudaError_t _e = cudaGetLastError();                                                      \
    if (_e != cudaSuccess) return b200_set_error(B200_ERR_CUDA, "kernel launch: %s (%s:%d)",   \
                                                 cudaGetErrorString(_e), __FILE__, __LINE__); \
  } while (0)

namespace b200 {

// Number of SMs of the current device (cached per device, thread-safe).
inline cudaError_t device_sms(int *sms) {
  static std::atomic<int> cache[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  int v = cache[dev & 63].load(std::memory_order_relaxed);
  if (v == 0) {
    e = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    cache[dev & 63].store(v, std::memory_order_relaxed);
  }
  *sms = v;
  return cudaSuccess;
}

// Raise kernel K's dynamic shared-memory limit to `bytes` once per device (a per-function,
// per-device setting; thread-safe, repeated calls are no-ops).
template <auto K>
inline cudaError_t ensure_dynamic_smem(int bytes) {
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(K, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_release);
  return e;
}

// Resident CTAs per SM of kernel K (always launched with `threads` threads) at `smem` dynamic
// bytes: the occupancy query costs about a microsecond of host time per launch, so the last
// answer is kept per device (entry = 1 << 63 | smem << 8 | CTAs; thread-safe).
template <auto K>
inline cudaError_t occupancy_cached(int *per_sm, int threads, size_t smem) {
  static std::atomic<uint64_t> cache[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::atomic<uint64_t> &slot = cache[dev & 63];
  const uint64_t v = slot.load(std::memory_order_relaxed);
  if ((v >> 63) && ((v >> 8) & 0xFFFFFFFFull) == smem) {
    *per_sm = (int)(v & 0xFF);
    return cudaSuccess;
  }
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(per_sm, K, threads, smem);
  if (e == cudaSuccess && *per_sm >= 0 && *per_sm < 256 && smem < (1ull << 32))
    slot.store((1ull << 63) | ((uint64_t)smem << 8) | (uint64_t)*per_sm, std::memory_order_relaxed);
  return e;
}

}  // namespace b200

