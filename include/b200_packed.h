/*
 * b200_packed.h -- C-ABI of the B200 (sm_100a) packed low-bit matmul library.
 *
 * This is the native boundary that replaces tinygrad-dx12's DX12 path for packed
 * low-bit (INT4 / UINT4 / FP4 E2M1 / FP6 E2M3 / FP6 E3M2) weights:
 *
 *   - decode + dequant  : src/tinygrad_dx12/codegen/decomp/dx12.py:49-106 (PackedTensor.unpack)
 *   - packed matmul     : src/tinygrad_dx12/codegen/linalg.py:136-223 (matmul), :226-298 (matvec),
 *                         lowered there to renderer/linalg.py:38-167 (HLSL LinAlg kernels)
 *   - runtime           : src/tinygrad_dx12/runtime/ops_dx12.py (DX12Device / DX12Allocator /
 *                         DX12Program / fences), reached there through COM vtables via ctypes
 *                         (runtime/support/dx12.py:21-59)
 *
 * Conventions (mirroring runtime/support/dx12.py:11-15, which raises on a failed HRESULT):
 *   - every function returns int32 status: 0 = ok, < 0 = error (B200_ERR_*);
 *   - b200_last_error() copies the calling thread's last error message;
 *   - all pointers to tensors are device pointers owned by the caller. The compute entry
 *     points allocate nothing, with one exception: b200_packed_linear on a few tokens
 *     (3 <= m <= 64) splits K across CTAs and, on its first such call on a (device, stream),
 *     allocates a 16 MiB split-K workspace kept for the life of the process
 *     (b200_packed_linear_noalloc is the allocation-free form). Other allocations are the
 *     explicit b200_malloc / b200_stream_create / b200_event_create calls;
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream);
 *     all compute entry points are asynchronous on that stream.
 *   - thread-safe: no global mutable state on the compute paths except the per-thread
 *     error message and the test-only failure injector.
 */
#ifndef B200_PACKED_H
#define B200_PACKED_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------------- */
#define B200_OK 0
#define B200_ERR_INVALID (-1)     /* malformed arguments (Python: ValueError)             */
#define B200_ERR_UNSUPPORTED (-2) /* valid, but this path does not handle it             */
#define B200_ERR_CUDA (-3)        /* a CUDA runtime call failed; message has the name    */
#define B200_ERR_TIMEOUT (-4)     /* a bounded wait ran out (host or device side)        */
#define B200_ERR_INJECTED (-5)    /* failure injected by b200_inject_failure (tests)     */

/* ---- packed formats: same table as FORMATS, codegen/decomp/dx12.py:10 ------------- */
#define B200_FMT_INT4 0     /* (4 bits, signed two's complement nibble)  */
#define B200_FMT_UINT4 1    /* (4 bits, unsigned)                        */
#define B200_FMT_FP4_E2M1 2 /* (4, e2, m1, bias 1)                        */
#define B200_FMT_FP6_E2M3 3 /* (6, e2, m3, bias 1)                        */
#define B200_FMT_FP6_E3M2 4 /* (6, e3, m2, bias 3)                        */

/* ---- element types (tinygrad dtype names in comments) ----------------------------- */
#define B200_DT_NONE 0
#define B200_DT_BOOL 1
#define B200_DT_I8 2      /* int8    */
#define B200_DT_U8 3      /* uint8   */
#define B200_DT_I16 4     /* int16   */
#define B200_DT_U16 5     /* uint16  */
#define B200_DT_I32 6     /* int32   */
#define B200_DT_U32 7     /* uint32  */
#define B200_DT_I64 8     /* int64   */
#define B200_DT_U64 9     /* uint64  */
#define B200_DT_F8E4M3 10 /* fp8e4m3 (E4M3FN) */
#define B200_DT_F8E5M2 11 /* fp8e5m2 */
#define B200_DT_F16 12    /* float16 */
#define B200_DT_BF16 13   /* bfloat16 */
#define B200_DT_F32 14    /* float32 */
#define B200_DT_F64 15    /* float64 */
#define B200_DT_E8M0 16   /* decoded-by-definition power-of-two scale byte (2^(b-127)) */

/* ---- matmul path selection (b200_packed_linear `path`) ----------------------------- */
#define B200_PATH_AUTO 0    /* the best kernel that takes the operands (below)          */
#define B200_PATH_GEMV 1    /* force the mma.sync decode GEMV / few-token GEMM (m <= 64) */
#define B200_PATH_GEMM 2    /* force the tcgen05 GEMM                                   */
#define B200_PATH_SIMT 3    /* force the fp32 CUDA-core fused kernel                    */
#define B200_PATH_MX 4      /* force the block-scaled tcgen05 decode kernel: FP4 / FP6
                               weights (per-32 E8M0 with K % 512 == 0, per-row or no
                               scales), bf16 x up to 64 tokens or fp16 x up to 42,
                               K % 256 == 0. AUTO takes it for FP4 weights at 1..4 tokens
                               when each SM streams at least 32 (1..2 tokens) or 64
                               (3..4 tokens) 128-row x 256-deep K stages */
/* OR-able flag: launch with programmatic dependent launch (PDL). The kernel may start while
 * the previous kernel on the stream is still running; it streams its packed weights and
 * scales at once and waits for that kernel before it reads x or writes y. Only valid when
 * the weights and scales are not written by the immediately preceding kernels (true for
 * inference weights); the activation dependency is always honoured. Honoured by the decode
 * GEMV (M <= 2) and the decode GEMM for 3..64 tokens; the other kernels ignore it. */
#define B200_FLAG_PDL 0x100
/* OR-able flag: the caller guarantees that no E8M0 scale byte of the matrix is 0x00 (2^-127)
 * or 0xFF (NaN). The decode GEMV then converts every byte with a shift and skips its per-stage
 * test for those two bytes (about 5 % of a one-token call), and the decode GEMM for 3..64
 * tokens runs its shift-only instantiation (about 9 % at 8 tokens). Results with such a byte present
 * and the flag set are undefined; without the flag every byte is decoded exactly. The Python
 * layer sets it per weight after checking the scales once. Ignored for other scale types. */
#define B200_FLAG_SCALES_ORDINARY 0x200

/*
 * Packed operand descriptor: the fields of PackedTensor (codegen/decomp/dx12.py:26-30)
 * flattened to a 2-D view. `rows` = prod(shape[:-1]), `cols` = shape[-1] (K).
 * The byte stream is the reference layout: consecutive payloads, least-significant bit
 * first, four elements per 2 bytes (4-bit) or per 3 bytes (6-bit); row r starts at bit
 * r*cols*bits. `scales`, when present, is row-major [rows, ceil(cols/block_size)] of
 * `scale_dtype`.
 */
typedef struct b200_packed_desc {
  const void *data;    /* device pointer to packed bytes                          */
  int64_t data_bytes;  /* bytes available at `data` (>= ceil(rows*cols*bits/8))    */
  int32_t format;      /* B200_FMT_*                                              */
  int32_t scale_dtype; /* B200_DT_NONE when unscaled, else F16/BF16/F32/F64/E8M0   */
  int64_t rows;
  int64_t cols;
  int64_t block_size;  /* >= 1                                                    */
  const void *scales;  /* device pointer or NULL                                  */
} b200_packed_desc;

/* ---- library / errors ------------------------------------------------------------- */
int32_t b200_version(void);
/* Copy the calling thread's last error message (NUL-terminated, truncated to len). */
int32_t b200_last_error(char *buf, size_t len);
/* Test hook: the `after`-th following compute entry call returns `code` instead of
 * running (after=0 disables). Replaces the injected submit failure of
 * test/device/test_execution.py:128-165. */
int32_t b200_inject_failure(int32_t after, int32_t code);

/* Validation of PackedTensor.__post_init__ (codegen/decomp/dx12.py:32-47). */
int32_t b200_validate(const b200_packed_desc *w);

/* ---- decode / dequant: PackedTensor.unpack (codegen/decomp/dx12.py:49-106) ---------
 * Writes flat elements [elem_begin, elem_begin + elem_count) of the decoded tensor to
 * `out` (contiguous, `out_dtype`). Arithmetic is the reference's: FP payloads decode to
 * float32 exactly, scales multiply in least_upper(float32, scale_dtype, out_dtype) (float32
 * or float64), then a numeric cast to out_dtype. Unscaled FP4/FP6 with an FP8 out_dtype
 * use the exact bit encoding of dx12.py:78-92. Bit-exact with the CPU restatement. */
int32_t b200_dequant(const b200_packed_desc *w, int64_t elem_begin, int64_t elem_count, void *out,
                     int32_t out_dtype, void *stream);

/* ---- fused packed linear: y[m, n] = sum_k x[m, k] * W[n, k] --------------------------
 * The call form linalg.matmul(W, x.T) (codegen/linalg.py:136-223) and
 * linalg.matvec(W, v) (:226-298, m = 1), with the decode of dx12.py:49-106 fused in.
 * x: `x_dtype` in {F16, BF16, F32}, element (m, k) at x + m*x_stride_m + k*x_stride_k
 * (element strides). y: `y_dtype` in {F16, BF16, F32}, element (m, n) at
 * y + m*y_stride_m + n*y_stride_n. Accumulation is float32 in every path. */
int32_t b200_packed_linear(const b200_packed_desc *w, const void *x, int32_t x_dtype, int64_t m,
                           int64_t x_stride_m, int64_t x_stride_k, void *y, int32_t y_dtype,
                           int64_t y_stride_m, int64_t y_stride_n, int32_t path, void *stream);

/* Which kernel b200_packed_linear would run for these arguments (B200_PATH_*), or < 0
 * when unsupported. No launch. */
int32_t b200_packed_linear_plan(const b200_packed_desc *w, int32_t x_dtype, int64_t m, int32_t y_dtype,
                                int32_t path);

/* ---- ordinary matmul ("tiled" scope, codegen/linalg.py:188-189): c = a @ b ----------
 * a [M,K], b [K,N], c [M,N] with element strides; operands are converted to `acc_dtype`
 * (F32, F64, I32, U32, I64, U64) before multiply-accumulate; c written as c_dtype. */
int32_t b200_matmul_generic(const void *a, int32_t a_dtype, int64_t sa_m, int64_t sa_k, const void *b,
                            int32_t b_dtype, int64_t sb_k, int64_t sb_n, void *c, int32_t c_dtype,
                            int64_t sc_m, int64_t sc_n, int64_t M, int64_t N, int64_t K, int32_t acc_dtype,
                            void *stream);

/* Elementwise numeric cast between dtypes (contiguous), used for the `.cast(...)`
 * of unpacked operands and outputs. */
int32_t b200_cast(const void *src, int32_t src_dtype, void *dst, int32_t dst_dtype, int64_t count, void *stream);

/* ---- runtime: replaces runtime/ops_dx12.py (allocator, queue, fences) --------------- */
int32_t b200_device_count(int32_t *count);
int32_t b200_malloc(int32_t device, size_t bytes, void **ptr);   /* DX12Allocator._alloc  */
int32_t b200_free(int32_t device, void *ptr);                     /* DX12Allocator._free   */
/* kind: 0 host->device, 1 device->host, 2 device->device (DX12Allocator._copyin/_copyout) */
int32_t b200_memcpy(void *dst, const void *src, size_t bytes, int32_t kind, void *stream);
int32_t b200_stream_create(int32_t device, void **stream);        /* command queue          */
int32_t b200_stream_destroy(void *stream);
/* Bounded wait for all work on `stream` (DX12Device.wait, ops_dx12.py:206-228): polls with
 * a deadline and returns B200_ERR_TIMEOUT instead of hanging; timeout_ms < 0 waits forever. */
int32_t b200_stream_wait(void *stream, int64_t timeout_ms);
int32_t b200_event_create(void **event);
int32_t b200_event_record(void *event, void *stream);
int32_t b200_event_elapsed_ms(void *start, void *end, float *ms);
int32_t b200_event_destroy(void *event);

/* Sticky device-side error bits of the library's kernels on `device` (bit 0: a bounded
 * mbarrier / flag wait gave up and the kernel returned early). Synchronous; `clear` != 0
 * resets them. Replaces the sticky `failure` of runtime/ops_dx12.py:171,195-198. */
int32_t b200_device_status(int32_t device, uint32_t *flags, int32_t clear);

/* Device-side bounded wait (failure detection without a GPU fault): a one-thread kernel
 * spins until *flag == expect or `max_spins` polls have passed, then writes 0 (seen) or
 * B200_ERR_TIMEOUT to *status. Never traps. */
int32_t b200_device_wait_flag(const int32_t *flag, int32_t expect, int64_t max_spins, int32_t *status,
                              void *stream);

/* b200_packed_linear (unit k / n strides; `flags` = a B200_PATH_* in the low byte, AUTO = 0,
 * OR-ed with B200_FLAG_* bits) writing the same result to n_y <= 8
 * destinations of one layout -- e.g. this rank's slot in every rank's peer-mapped buffer, the
 * push half of the tensor-parallel reduction. The decode GEMV (m <= 2) stores every destination
 * from its epilogue; other kernels compute into y[0] and copy. No counterpart in the reference. */
int32_t b200_packed_linear_multi(const b200_packed_desc *w, const void *x, int32_t x_dtype, int64_t m,
                                 int64_t x_stride_m, void *const *y, int32_t n_y, int32_t y_dtype, int64_t y_stride_m,
                                 int32_t flags, void *stream);

/* Allocation-free form of b200_packed_linear for a few tokens (3 <= m <= 32, 4-bit formats,
 * the split-K decode GEMM). No counterpart in the reference. Same arguments and result as
 * b200_packed_linear with path B200_PATH_GEMV and unit k / n strides; bitwise the same result.
 * It never calls an allocator: its split-K scratch is a fixed 2 MiB device array of the
 * library (per device), resolved on the first call on a device -- make that first call before
 * any stream capture. With CUDA's default lazy module loading, that first call (or any first
 * call of this library's kernels) also loads the library's device code and commits the 2 MiB
 * array on the device: make one warm-up call before the caller hands all free HBM to its own
 * pool, or run the process with CUDA_MODULE_LOADING=EAGER. Shapes whose split-K partials
 * would not fit (splits x m x N x 4 bytes beyond the 2 MiB less 16 KiB of row-block tickets,
 * or more than 4096 row blocks of 128 rows; on a 148-SM B200 e.g. m = 32 with N >= 8192)
 * return B200_ERR_UNSUPPORTED; shapes the kernel does not take return the same error.
 * Calls that overlap in time on one device (several streams or threads) share the array and
 * race: serialise them. */
int32_t b200_packed_linear_noalloc(const b200_packed_desc *w, const void *x, int32_t x_dtype, int64_t m,
                                   int64_t x_stride_m, void *y, int32_t y_dtype, int64_t y_stride_m, void *stream);

/* ---- projection-stack glue (benchmark configs c4 / c5) --------------------------------
 * No counterpart in the reference, whose packed path ends at one matmul
 * (codegen/linalg.py:136-223); these are the elementwise steps between the packed
 * projections of the multi-layer tensor-parallel stacks. Rows (tokens) are independent. */

/* For each of the M rows of h (M x H, dtype h_dtype, row-major): if `partial` (fp32, M x H)
 * is given, h += partial (fp32 add, rounded back to h_dtype in place); then, if `x` is given,
 * x = h * rsqrt(mean(h^2) + eps) computed in fp32 and rounded to x_dtype. */
int32_t b200_add_rmsnorm(void *h, int32_t h_dtype, const float *partial, void *x, int32_t x_dtype, int64_t M,
                         int64_t H, float eps, void *stream);

/* out[m, i] = gu[m, i] * gu[m, I + i] for gu (M x 2I) -- the gated product of a fused
 * gate|up projection -- as an fp32 product rounded to out_dtype. */
int32_t b200_gate_mul(const void *gu, int32_t gu_dtype, void *out, int32_t out_dtype, int64_t M, int64_t I,
                      void *stream);

/* Tensor-parallel reduction of the row-parallel projections over peer memory, fused with the
 * residual add and RMS norm (the all-reduce step of the stacks). No counterpart in the
 * reference. `partials[q]` is rank q's fp32 partial (M x H rows, row-major) as mapped in this
 * process, `flags[q]` rank q's flag array (world x rows_max uint32, zeroed before first use),
 * `epoch` this rank's counters (rows_max uint32, zeroed before first use). Per row the kernel
 * publishes its epoch to every rank, waits for every rank's (giving up after timeout_ns with
 * the device error bit set), then h += sum over q = 0..world-1 of partials[q] (fixed order)
 * and x = h * rsqrt(mean(h^2) + eps). M <= rows_max, world <= 8. */
int32_t b200_peer_allreduce_add_rmsnorm(const void *const *partials, uint32_t *const *flags, uint32_t *epoch,
                                        int32_t rank, int32_t world, int64_t rows_max, int64_t timeout_ns, void *h,
                                        int32_t h_dtype, void *x, int32_t x_dtype, int64_t M, int64_t H, float eps,
                                        void *stream);

/* CUDA IPC plumbing for the peer buffers: export a handle (64 bytes) of a b200_malloc'd
 * allocation, open a peer's handle in this process, close it. */
int32_t b200_ipc_get_handle(void *dev_ptr, void *handle64);
int32_t b200_ipc_open(const void *handle64, void **dev_ptr);
int32_t b200_ipc_close(void *dev_ptr);

#ifdef __cplusplus
}
#endif

#endif /* B200_PACKED_H */
