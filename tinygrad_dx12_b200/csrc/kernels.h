// kernels.h -- host-side launchers shared between the C-ABI (capi.cu) and kernel files.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/b200_packed.h"

namespace b200 {

// Arguments of a fused packed linear y[m, n] = sum_k x[m, k] * W[n, k].
struct LinearArgs {
  const uint8_t *w;  // packed bytes
  const void *scales;
  int fmt, sdt;
  int64_t rows, cols, block, nblk;
  const void *x;
  int xdt;
  int64_t m, ldx;  // x row stride in elements (k stride is 1)
  void *y;
  int ydt;
  int64_t ldy_m, ldy_n;
  int flags;  // B200_FLAG_* bits
  void *ycopy[7];  // further destinations that receive the same y (decode GEMV epilogues)
  int ncopy;
};

int32_t launch_dequant(const b200_packed_desc *w, int64_t begin, int64_t count, void *out, int32_t out_dtype,
                       bool fp8_exact, cudaStream_t stream);

// fp32 CUDA-core fused kernel (any M; x f16/bf16/f32).
bool simt_supported(const LinearArgs &a);
int32_t launch_gemv_simt(const LinearArgs &a, cudaStream_t stream);

// tensor-core decode GEMV (M <= 32; x f16/bf16).
bool gemv_tc_supported(const LinearArgs &a);
int32_t launch_gemv_tc(const LinearArgs &a, cudaStream_t stream);

// tcgen05 GEMM (M > 32; x f16/bf16).
bool gemm_supported(const LinearArgs &a);
int32_t launch_gemm(const LinearArgs &a, cudaStream_t stream);
int32_t gemm_device_error(unsigned int *v, bool clear);

// 2-D tiled TMA descriptor (defined in gemm_sm100.cu); base 16-byte aligned, row_bytes % 16 == 0.
int32_t make_tma_2d(CUtensorMap *map, CUtensorMapDataType dt, const void *base, uint64_t inner, uint64_t outer,
                    uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz);

// streamed (TMA) decode GEMV for M <= 2 (gemv.cu)
bool gemv_stream_supported(const LinearArgs &a);
int32_t launch_gemv_stream(const LinearArgs &a, cudaStream_t stream);
int32_t gemv_device_error(unsigned int *v, bool clear);

// split-K mma.sync decode GEMM for 3 <= M <= 32, 4-bit formats (skinny.cu); also 33 <= M <= 64
// with per-32 fp16 / bf16 / fp32 or wider group scales
bool skinny_supported(const LinearArgs &a);
int32_t launch_skinny(const LinearArgs &a, cudaStream_t stream);
int32_t skinny_device_error(unsigned int *v, bool clear);
// same kernel, split-K scratch from a fixed device array instead of a library workspace
int32_t launch_skinny_noalloc(const LinearArgs &a, cudaStream_t stream);

// block-scaled tcgen05 decode kernel (kind::mxf8f6f4) for FP4 / FP6 weights and 1..64 tokens
// (gemv_mx.cu): the packed codes are the MMA's A operand, x is split into exact E4M3 pieces
bool mx_supported(const LinearArgs &a);
bool mx_ready(cudaStream_t stream);  // its workspace exists or can be allocated now
int32_t launch_mx(const LinearArgs &a, cudaStream_t stream);
int32_t mx_device_error(unsigned int *v, bool clear);
int32_t mx_reset_tickets();  // after a device error: zero the split-tile tickets on this device
// the resident-pieces FP4 kernel (gemv_mxs.cu) for 1..4 tokens is faster than the decode GEMV here
bool mx_preferred(const LinearArgs &a);

// dense fp16 / bf16 tcgen05 GEMM for ordinary matmuls (gemm_dense.cu): c = a @ b with a
// row-major (k contiguous) and b K-major (k contiguous per column), fp32 accumulation
bool gemm_dense_supported(const void *a, int adt, int64_t sam, int64_t sak, const void *b, int bdt, int64_t sbk,
                          int64_t sbn, int cdt, int64_t scn, int64_t M, int64_t N, int64_t K, int accdt);
int32_t launch_gemm_dense(const void *a, int adt, int64_t sam, const void *b, int64_t sbn, void *c, int cdt,
                          int64_t scm, int64_t M, int64_t N, int64_t K, cudaStream_t stream);
int32_t gemm_dense_device_error(unsigned int *v, bool clear);

int32_t launch_matmul_generic(const void *a, int adt, int64_t sam, int64_t sak, const void *b, int bdt, int64_t sbk,
                              int64_t sbn, void *c, int cdt, int64_t scm, int64_t scn, int64_t M, int64_t N, int64_t K,
                              int accdt, cudaStream_t stream);
int32_t launch_cast(const void *src, int sdt, void *dst, int ddt, int64_t n, cudaStream_t stream);
int32_t launch_add_rmsnorm(void *h, int hdt, const float *partial, void *x, int xdt, int64_t M, int64_t H, float eps,
                           cudaStream_t stream);
int32_t launch_peer_reduce_rmsnorm(const void *const *partials, uint32_t *const *flags, uint32_t *epoch, int rank,
                                   int world, int64_t rows_max, int64_t timeout_ns, void *h, int hdt, void *x, int xdt,
                                   int64_t M, int64_t H, float eps, cudaStream_t stream);
int32_t stackops_device_error(unsigned int *v, bool clear);
int32_t launch_gate_mul(const void *gu, int gdt, void *out, int odt, int64_t M, int64_t I, cudaStream_t stream);
int32_t launch_wait_flag(const int32_t *flag, int32_t expect, int64_t max_spins, int32_t *status, cudaStream_t stream);

}  // namespace b200
