// generic.cu -- ordinary kernels the packed path still needs around the fused kernels:
//   * matmul_generic: the "tiled" scope (tinygrad-dx12 src/tinygrad_dx12/codegen/linalg.py:188-189,
//     ordinary compute). fp16 / bf16 operands in tensor-core layouts go to the tcgen05 dense GEMM
//     (gemm_dense.cu); everything else -- integer / float64 / mixed cases, e.g. packed integer
//     weights times int32/int64 activations (test_linalg.py:202-218) -- runs the tiled kernel here;
//   * cast: elementwise numeric conversion (the `.cast()` nodes of linalg.py:180-181);
//   * wait_flag: a bounded device-side wait that reports a timeout instead of hanging.
#include "common.cuh"
#include "kernels.h"

namespace b200 {

template <typename Acc>
__device__ __forceinline__ Acc load_acc(const void *p, int64_t i, int dt) {
  if constexpr (std::is_same<Acc, float>::value) return load_as_f32(p, i, dt);
  else if constexpr (std::is_same<Acc, double>::value) return load_as_f64(p, i, dt);
  else return (Acc)load_as_i64(p, i, dt);
}

template <typename Acc>
__device__ __forceinline__ void store_acc(void *p, int64_t i, int dt, Acc v) {
  if constexpr (std::is_same<Acc, float>::value) store_f32(p, i, dt, v);
  else if constexpr (std::is_same<Acc, double>::value) store_f64(p, i, dt, v);
  else store_i64(p, i, dt, (int64_t)v);
}

// 16x16 output tile per CTA, K staged through shared memory 16 at a time.
template <typename Acc>
__global__ void __launch_bounds__(256) matmul_generic_kernel(const void *a, int adt, int64_t sam, int64_t sak,
                                                             const void *b, int bdt, int64_t sbk, int64_t sbn, void *c,
                                                             int cdt, int64_t scm, int64_t scn, int64_t M, int64_t N,
                                                             int64_t K) {
  __shared__ Acc As[16][17];
  __shared__ Acc Bs[16][17];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t row = (int64_t)blockIdx.y * 16 + ty, col = (int64_t)blockIdx.x * 16 + tx;
  Acc acc = Acc(0);
  for (int64_t k0 = 0; k0 < K; k0 += 16) {
    const int64_t ka = k0 + tx, kb = k0 + ty;
    As[ty][tx] = (row < M && ka < K) ? load_acc<Acc>(a, row * sam + ka * sak, adt) : Acc(0);
    Bs[ty][tx] = (kb < K && col < N) ? load_acc<Acc>(b, kb * sbk + col * sbn, bdt) : Acc(0);
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 16; ++k) acc += As[ty][k] * Bs[k][tx];
    __syncthreads();
  }
  if (row < M && col < N) store_acc<Acc>(c, row * scm + col * scn, cdt, acc);
}

int32_t launch_matmul_generic(const void *a, int adt, int64_t sam, int64_t sak, const void *b, int bdt, int64_t sbk,
                              int64_t sbn, void *c, int cdt, int64_t scm, int64_t scn, int64_t M, int64_t N, int64_t K,
                              int accdt, cudaStream_t stream) {
  if (M <= 0 || N <= 0) return B200_OK;
  // 16-bit operands in tensor-core layouts: the tcgen05 GEMM (fp32 accumulation, as below)
  if (gemm_dense_supported(a, adt, sam, sak, b, bdt, sbk, sbn, cdt, scn, M, N, K, accdt))
    return launch_gemm_dense(a, adt, sam, b, sbn, c, cdt, scm, M, N, K, stream);
  const dim3 grid((unsigned)((N + 15) / 16), (unsigned)((M + 15) / 16));
  if (grid.y > 65535u) return b200_set_error(B200_ERR_UNSUPPORTED, "generic matmul: M=%lld too large", (long long)M);
  switch (accdt) {
    case B200_DT_F16: case B200_DT_BF16: case B200_DT_F32:
      matmul_generic_kernel<float><<<grid, 256, 0, stream>>>(a, adt, sam, sak, b, bdt, sbk, sbn, c, cdt, scm, scn, M, N, K);
      break;
    case B200_DT_F64:
      matmul_generic_kernel<double><<<grid, 256, 0, stream>>>(a, adt, sam, sak, b, bdt, sbk, sbn, c, cdt, scm, scn, M, N, K);
      break;
    case B200_DT_I32: case B200_DT_I64: case B200_DT_I8: case B200_DT_I16: case B200_DT_BOOL:
      matmul_generic_kernel<int64_t><<<grid, 256, 0, stream>>>(a, adt, sam, sak, b, bdt, sbk, sbn, c, cdt, scm, scn, M, N, K);
      break;
    case B200_DT_U32: case B200_DT_U64: case B200_DT_U8: case B200_DT_U16:
      matmul_generic_kernel<uint64_t><<<grid, 256, 0, stream>>>(a, adt, sam, sak, b, bdt, sbk, sbn, c, cdt, scm, scn, M, N, K);
      break;
    default: return b200_set_error(B200_ERR_UNSUPPORTED, "generic matmul: accumulator dtype %d", accdt);
  }
  B200_LAUNCH_CHECK();
  return B200_OK;
}

__global__ void cast_kernel(const void *src, int sdt, void *dst, int ddt, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    if (!dt_is_float(sdt) && !dt_is_float(ddt)) store_i64(dst, i, ddt, load_as_i64(src, i, sdt));
    else if (sdt == B200_DT_F64 || ddt == B200_DT_F64 || !dt_is_float(sdt)) store_f64(dst, i, ddt, load_as_f64(src, i, sdt));
    else store_f32(dst, i, ddt, load_as_f32(src, i, sdt));
  }
}

// Same-dtype copy in 16-byte vectors (the staging copy of a decode step's activations from
// pinned host memory: one load per thread over the host link). It lets a dependent kernel
// launched with programmatic dependent launch start at once (that kernel streams its weights
// while this copy runs and waits for it before reading the copy).
__global__ void copy16_kernel(const uint4 *src, uint4 *dst, int64_t n16) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = src[i];
}

int32_t launch_cast(const void *src, int sdt, void *dst, int ddt, int64_t n, cudaStream_t stream) {
  if (n <= 0) return B200_OK;
  const int64_t bytes = n * dt_size(sdt);
  if (sdt == ddt && bytes % 16 == 0 && (uintptr_t)src % 16 == 0 && (uintptr_t)dst % 16 == 0) {
    const int64_t n16 = bytes / 16;
    int64_t blocks = (n16 + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    copy16_kernel<<<(unsigned)blocks, 256, 0, stream>>>(static_cast<const uint4 *>(src), static_cast<uint4 *>(dst), n16);
    B200_LAUNCH_CHECK();
    return B200_OK;
  }
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  cast_kernel<<<(unsigned)blocks, 256, 0, stream>>>(src, sdt, dst, ddt, n);
  B200_LAUNCH_CHECK();
  return B200_OK;
}

// Bounded spin on a flag: never traps, always terminates after max_spins polls.
__global__ void wait_flag_kernel(const int32_t *flag, int32_t expect, int64_t max_spins, int32_t *status) {
  const volatile int32_t *f = flag;
  for (int64_t i = 0; i < max_spins; ++i) {
    if (*f == expect) {
      *status = B200_OK;
      return;
    }
    __nanosleep(256);
  }
  *status = B200_ERR_TIMEOUT;
}

int32_t launch_wait_flag(const int32_t *flag, int32_t expect, int64_t max_spins, int32_t *status, cudaStream_t stream) {
  wait_flag_kernel<<<1, 1, 0, stream>>>(flag, expect, max_spins, status);
  B200_LAUNCH_CHECK();
  return B200_OK;
}

}  // namespace b200
