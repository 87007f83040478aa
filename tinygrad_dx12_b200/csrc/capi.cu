// capi.cu -- the extern "C" boundary declared in include/b200_packed.h.
//
// Replaces, for the packed low-bit path, what tinygrad-dx12 reaches through COM vtables
// (src/tinygrad_dx12/runtime/support/dx12.py:21-59) and its DX12 runtime
// (src/tinygrad_dx12/runtime/ops_dx12.py): argument validation, kernel selection, launch on
// the caller's stream, a thread-local error message, bounded waits, and a failure injector
// for tests (test/device/test_execution.py:128-165 injects a failing submit the same way).
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <chrono>
#include <thread>

#include "common.cuh"
#include "kernels.h"

#define B200_VERSION 100

static thread_local char g_err[1024];
static std::atomic<int32_t> g_inject_after{0};
static std::atomic<int32_t> g_inject_code{0};

int32_t b200_set_error(int32_t code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

// Returns non-zero (the injected code) when this call should fail.
static int32_t injected() {
  int32_t after = g_inject_after.load();
  while (after > 0) {
    if (g_inject_after.compare_exchange_weak(after, after - 1)) {
      if (after == 1) {
        const int32_t code = g_inject_code.load();
        return b200_set_error(code, "injected failure (code %d)", code);
      }
      return 0;
    }
  }
  return 0;
}

using namespace b200;

static int32_t validate_desc(const b200_packed_desc *w) {
  // codegen/decomp/dx12.py:32-47
  if (w == nullptr) return b200_set_error(B200_ERR_INVALID, "null packed descriptor");
  if (w->format < B200_FMT_INT4 || w->format > B200_FMT_FP6_E3M2)
    return b200_set_error(B200_ERR_INVALID, "unknown packed format %d", w->format);
  if (w->rows < 0 || w->cols < 0) return b200_set_error(B200_ERR_INVALID, "packed shape must contain nonnegative dimensions");
  const int bits = fmt_bits(w->format);
  const int64_t need = (w->rows * w->cols * bits + 7) / 8;
  if (w->data_bytes < need) return b200_set_error(B200_ERR_INVALID, "packed storage is smaller than the declared shape");
  if (w->block_size < 1) return b200_set_error(B200_ERR_INVALID, "packed block size must be positive");
  if (w->scales != nullptr) {
    switch (w->scale_dtype) {
      case B200_DT_F16: case B200_DT_BF16: case B200_DT_F32: case B200_DT_F64: case B200_DT_E8M0:
      case B200_DT_I8: case B200_DT_U8: case B200_DT_I16: case B200_DT_U16: case B200_DT_I32: case B200_DT_U32:
      case B200_DT_I64: case B200_DT_U64: case B200_DT_F8E4M3: case B200_DT_F8E5M2: break;
      default: return b200_set_error(B200_ERR_INVALID, "unsupported scale dtype %d", w->scale_dtype);
    }
  }
  if (need > 0 && w->data == nullptr) return b200_set_error(B200_ERR_INVALID, "null packed data");
  return B200_OK;
}

extern "C" {

int32_t b200_version(void) { return B200_VERSION; }

int32_t b200_last_error(char *buf, size_t len) {
  if (buf == nullptr || len == 0) return (int32_t)strlen(g_err);
  strncpy(buf, g_err, len - 1);
  buf[len - 1] = 0;
  return (int32_t)strlen(buf);
}

int32_t b200_inject_failure(int32_t after, int32_t code) {
  g_inject_code.store(code);
  g_inject_after.store(after < 0 ? 0 : after);
  return B200_OK;
}

int32_t b200_validate(const b200_packed_desc *w) { return validate_desc(w); }

int32_t b200_dequant(const b200_packed_desc *w, int64_t elem_begin, int64_t elem_count, void *out, int32_t out_dtype,
                     void *stream) {
  if (int32_t rc = injected()) return rc;
  if (int32_t rc = validate_desc(w)) return rc;
  const int64_t total = w->rows * w->cols;
  if (elem_begin < 0 || elem_count < 0 || elem_begin + elem_count > total)
    return b200_set_error(B200_ERR_INVALID, "element window [%lld, %lld) outside %lld elements", (long long)elem_begin,
                          (long long)(elem_begin + elem_count), (long long)total);
  if (dt_size(out_dtype) == 0 || out_dtype == B200_DT_E8M0)
    return b200_set_error(B200_ERR_INVALID, "unsupported output dtype %d", out_dtype);
  if (elem_count > 0 && out == nullptr) return b200_set_error(B200_ERR_INVALID, "null output");
  const bool fp_fmt = w->format >= B200_FMT_FP4_E2M1;
  // dx12.py:11,78: exact FP8 candidates per format
  const bool cand = (out_dtype == B200_DT_F8E4M3 && fp_fmt) ||
                    (out_dtype == B200_DT_F8E5M2 && (w->format == B200_FMT_FP4_E2M1 || w->format == B200_FMT_FP6_E3M2));
  const bool exact = w->scales == nullptr && cand;
  return launch_dequant(w, elem_begin, elem_count, out, out_dtype, exact, (cudaStream_t)stream);
}

static bool fill_linear(const b200_packed_desc *w, const void *x, int32_t x_dtype, int64_t m, int64_t x_stride_m,
                        int64_t x_stride_k, void *y, int32_t y_dtype, int64_t y_stride_m, int64_t y_stride_n,
                        LinearArgs &a) {
  a.w = (const uint8_t *)w->data;
  a.scales = w->scales;
  a.fmt = w->format;
  a.sdt = w->scales ? w->scale_dtype : B200_DT_NONE;
  a.rows = w->rows;
  a.cols = w->cols;
  a.block = w->block_size;
  a.nblk = (w->cols + w->block_size - 1) / w->block_size;
  a.x = x;
  a.xdt = x_dtype;
  a.m = m;
  a.ldx = x_stride_m;
  a.y = y;
  a.ydt = y_dtype;
  a.ldy_m = y_stride_m;
  a.ldy_n = y_stride_n;
  a.flags = 0;
  a.ncopy = 0;
  for (int i = 0; i < 7; ++i) a.ycopy[i] = nullptr;
  return x_stride_k == 1;
}

// Kernel for these operands. `mx_ok` = false leaves the block-scaled decode kernel out (its
// workspace cannot be allocated during a stream capture).
static int32_t plan(const LinearArgs &a, bool kstride_ok, int32_t path, bool mx_ok = true) {
  if (!kstride_ok) return B200_ERR_UNSUPPORTED;
  path &= 0xFF;  // flag bits (B200_FLAG_*) do not select a kernel
  const bool tc = gemv_tc_supported(a) || skinny_supported(a), gm = gemm_supported(a), simt = simt_supported(a);
  const bool mx = mx_ok && mx_supported(a);
  switch (path) {
    case B200_PATH_MX: return mx ? B200_PATH_MX : B200_ERR_UNSUPPORTED;
    case B200_PATH_AUTO:
      if (mx && a.m <= 4 && mx_preferred(a)) return B200_PATH_MX;  // FP4 with many stages per SM
      if (a.m <= 32 && tc) return B200_PATH_GEMV;
      if (a.m > 32 && gm) return B200_PATH_GEMM;
      if (a.m <= 64 && skinny_supported(a)) return B200_PATH_GEMV;  // scales the GEMM declines
      if (simt) return B200_PATH_SIMT;
      return B200_ERR_UNSUPPORTED;
    case B200_PATH_GEMV: return tc ? B200_PATH_GEMV : B200_ERR_UNSUPPORTED;
    case B200_PATH_GEMM: return gm ? B200_PATH_GEMM : B200_ERR_UNSUPPORTED;
    case B200_PATH_SIMT: return simt ? B200_PATH_SIMT : B200_ERR_UNSUPPORTED;
  }
  return B200_ERR_INVALID;
}

int32_t b200_packed_linear_plan(const b200_packed_desc *w, int32_t x_dtype, int64_t m, int32_t y_dtype, int32_t path) {
  if (int32_t rc = validate_desc(w)) return rc;
  LinearArgs a;
  // alignment-neutral probe: pretend x is aligned and contiguous
  fill_linear(w, (const void *)(uintptr_t)256, x_dtype, m, w->cols, 1, (void *)(uintptr_t)256, y_dtype, w->rows, 1, a);
  return plan(a, true, path);
}

int32_t b200_packed_linear(const b200_packed_desc *w, const void *x, int32_t x_dtype, int64_t m, int64_t x_stride_m,
                           int64_t x_stride_k, void *y, int32_t y_dtype, int64_t y_stride_m, int64_t y_stride_n,
                           int32_t path, void *stream) {
  if (int32_t rc = injected()) return rc;
  if (int32_t rc = validate_desc(w)) return rc;
  if (m < 0) return b200_set_error(B200_ERR_INVALID, "negative m");
  if (m == 0 || w->rows == 0) return B200_OK;
  if (x == nullptr || y == nullptr) return b200_set_error(B200_ERR_INVALID, "null x or y");
  LinearArgs a;
  const bool ks = fill_linear(w, x, x_dtype, m, x_stride_m, x_stride_k, y, y_dtype, y_stride_m, y_stride_n, a);
  a.flags = path & ~0xFF;
  cudaStream_t s = (cudaStream_t)stream;
  const int32_t p = plan(a, ks, path, mx_ready(s));
  switch (p) {
    case B200_PATH_MX: return launch_mx(a, s);
    case B200_PATH_GEMV:
      if (a.m > 2) return launch_skinny(a, s);
      return gemv_stream_supported(a) ? launch_gemv_stream(a, s) : launch_gemv_tc(a, s);
    case B200_PATH_GEMM: return launch_gemm(a, s);
    case B200_PATH_SIMT: return launch_gemv_simt(a, s);
  }
  return b200_set_error(B200_ERR_UNSUPPORTED,
                        "no fused kernel for format=%d scale_dtype=%d block=%lld K=%lld x_dtype=%d y_dtype=%d m=%lld "
                        "path=%d (x k-stride %lld)",
                        a.fmt, a.sdt, (long long)a.block, (long long)a.cols, a.xdt, a.ydt, (long long)m, path,
                        (long long)x_stride_k);
}

int32_t b200_matmul_generic(const void *a, int32_t a_dtype, int64_t sa_m, int64_t sa_k, const void *b, int32_t b_dtype,
                            int64_t sb_k, int64_t sb_n, void *c, int32_t c_dtype, int64_t sc_m, int64_t sc_n, int64_t M,
                            int64_t N, int64_t K, int32_t acc_dtype, void *stream) {
  if (int32_t rc = injected()) return rc;
  if (M < 0 || N < 0 || K < 0) return b200_set_error(B200_ERR_INVALID, "negative matmul dims");
  if (dt_size(a_dtype) == 0 || dt_size(b_dtype) == 0 || dt_size(c_dtype) == 0)
    return b200_set_error(B200_ERR_INVALID, "bad matmul dtype");
  return launch_matmul_generic(a, a_dtype, sa_m, sa_k, b, b_dtype, sb_k, sb_n, c, c_dtype, sc_m, sc_n, M, N, K,
                               acc_dtype, (cudaStream_t)stream);
}

int32_t b200_cast(const void *src, int32_t src_dtype, void *dst, int32_t dst_dtype, int64_t count, void *stream) {
  if (int32_t rc = injected()) return rc;
  if (dt_size(src_dtype) == 0 || dt_size(dst_dtype) == 0) return b200_set_error(B200_ERR_INVALID, "bad cast dtype");
  return launch_cast(src, src_dtype, dst, dst_dtype, count, (cudaStream_t)stream);
}

// ---- runtime -------------------------------------------------------------------------
int32_t b200_device_count(int32_t *count) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  if (count) *count = n;
  return B200_OK;
}

int32_t b200_malloc(int32_t device, size_t bytes, void **ptr) {
  if (ptr == nullptr) return b200_set_error(B200_ERR_INVALID, "null out pointer");
  B200_CUDA_TRY(cudaSetDevice(device));
  B200_CUDA_TRY(cudaMalloc(ptr, bytes));
  return B200_OK;
}

int32_t b200_free(int32_t device, void *ptr) {
  B200_CUDA_TRY(cudaSetDevice(device));
  B200_CUDA_TRY(cudaFree(ptr));
  return B200_OK;
}

int32_t b200_memcpy(void *dst, const void *src, size_t bytes, int32_t kind, void *stream) {
  cudaMemcpyKind k = kind == 0 ? cudaMemcpyHostToDevice : kind == 1 ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
  if (kind < 0 || kind > 2) return b200_set_error(B200_ERR_INVALID, "bad copy kind %d", kind);
  B200_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, k, (cudaStream_t)stream));
  return B200_OK;
}

int32_t b200_stream_create(int32_t device, void **stream) {
  B200_CUDA_TRY(cudaSetDevice(device));
  cudaStream_t s;
  B200_CUDA_TRY(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  *stream = (void *)s;
  return B200_OK;
}

int32_t b200_stream_destroy(void *stream) {
  B200_CUDA_TRY(cudaStreamDestroy((cudaStream_t)stream));
  return B200_OK;
}

int32_t b200_stream_wait(void *stream, int64_t timeout_ms) {
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t e = cudaStreamQuery((cudaStream_t)stream);
    if (e == cudaSuccess) return B200_OK;
    if (e != cudaErrorNotReady)
      return b200_set_error(B200_ERR_CUDA, "stream wait: %s", cudaGetErrorString(e));
    if (timeout_ms >= 0) {
      const auto el = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0);
      if (el.count() >= timeout_ms)
        return b200_set_error(B200_ERR_TIMEOUT, "stream wait timed out after %lld ms", (long long)timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

int32_t b200_event_create(void **event) {
  cudaEvent_t e;
  B200_CUDA_TRY(cudaEventCreate(&e));
  *event = (void *)e;
  return B200_OK;
}

int32_t b200_event_record(void *event, void *stream) {
  B200_CUDA_TRY(cudaEventRecord((cudaEvent_t)event, (cudaStream_t)stream));
  return B200_OK;
}

int32_t b200_event_elapsed_ms(void *start, void *end, float *ms) {
  B200_CUDA_TRY(cudaEventElapsedTime(ms, (cudaEvent_t)start, (cudaEvent_t)end));
  return B200_OK;
}

int32_t b200_event_destroy(void *event) {
  B200_CUDA_TRY(cudaEventDestroy((cudaEvent_t)event));
  return B200_OK;
}

int32_t b200_device_status(int32_t device, uint32_t *flags, int32_t clear) {
  if (flags == nullptr) return b200_set_error(B200_ERR_INVALID, "null flags");
  B200_CUDA_TRY(cudaSetDevice(device));
  unsigned int v = 0, u = 0;
  if (int32_t rc = gemm_device_error(&v, clear != 0)) return rc;
  if (int32_t rc = gemv_device_error(&u, clear != 0)) return rc;
  unsigned int w = 0, z = 0, dd = 0, mxe = 0;
  if (int32_t rc = skinny_device_error(&w, clear != 0)) return rc;
  if (int32_t rc = stackops_device_error(&z, clear != 0)) return rc;
  if (int32_t rc = gemm_dense_device_error(&dd, clear != 0)) return rc;
  if (int32_t rc = mx_device_error(&mxe, clear != 0)) return rc;
  *flags = v | u | w | z | dd | mxe;
  if (clear != 0 && *flags != 0)  // a kernel gave up mid-way: its split-tile tickets may be half counted
    if (int32_t rc = mx_reset_tickets()) return rc;
  return B200_OK;
}

int32_t b200_packed_linear_multi(const b200_packed_desc *w, const void *x, int32_t x_dtype, int64_t m,
                                 int64_t x_stride_m, void *const *y, int32_t n_y, int32_t y_dtype, int64_t y_stride_m,
                                 int32_t flags, void *stream) {
  if (int32_t rc = injected()) return rc;
  if (int32_t rc = validate_desc(w)) return rc;
  if (m < 0 || n_y < 1 || n_y > 8 || y == nullptr) return b200_set_error(B200_ERR_INVALID, "bad m or destinations");
  for (int i = 0; i < n_y; ++i)
    if (y[i] == nullptr) return b200_set_error(B200_ERR_INVALID, "null destination %d", i);
  if (m == 0 || w->rows == 0) return B200_OK;
  if (x == nullptr) return b200_set_error(B200_ERR_INVALID, "null x");
  LinearArgs a;
  const bool ks = fill_linear(w, x, x_dtype, m, x_stride_m, 1, y[0], y_dtype, y_stride_m, 1, a);
  a.flags = flags & ~0xFF;
  cudaStream_t s = (cudaStream_t)stream;
  const int32_t p = plan(a, ks, flags, mx_ready(s));  // the low byte selects a path, as in b200_packed_linear
  if (p == B200_PATH_MX || (p == B200_PATH_GEMV && a.m <= 2)) {  // these epilogues write every destination
    a.ncopy = n_y - 1;
    for (int i = 1; i < n_y; ++i) a.ycopy[i - 1] = y[i];
    if (p == B200_PATH_MX) return launch_mx(a, s);
    return gemv_stream_supported(a) ? launch_gemv_stream(a, s) : launch_gemv_tc(a, s);
  }
  int32_t rc = B200_ERR_UNSUPPORTED;
  switch (p) {
    case B200_PATH_GEMV: rc = launch_skinny(a, s); break;
    case B200_PATH_GEMM: rc = launch_gemm(a, s); break;
    case B200_PATH_SIMT: rc = launch_gemv_simt(a, s); break;
    default: return b200_set_error(B200_ERR_UNSUPPORTED, "no fused kernel for these operands");
  }
  if (rc != B200_OK) return rc;
  const size_t row_bytes = (size_t)w->rows * dt_size(y_dtype), pitch = (size_t)y_stride_m * dt_size(y_dtype);
  for (int i = 1; i < n_y; ++i)
    B200_CUDA_TRY(cudaMemcpy2DAsync(y[i], pitch, y[0], pitch, row_bytes, (size_t)m, cudaMemcpyDeviceToDevice, s));
  return B200_OK;
}

int32_t b200_packed_linear_noalloc(const b200_packed_desc *w, const void *x, int32_t x_dtype, int64_t m,
                                   int64_t x_stride_m, void *y, int32_t y_dtype, int64_t y_stride_m, void *stream) {
  if (int32_t rc = injected()) return rc;
  if (int32_t rc = validate_desc(w)) return rc;
  if (m < 0) return b200_set_error(B200_ERR_INVALID, "negative m");
  if (m == 0 || w->rows == 0) return B200_OK;
  if (x == nullptr || y == nullptr) return b200_set_error(B200_ERR_INVALID, "null x or y");
  LinearArgs a;
  fill_linear(w, x, x_dtype, m, x_stride_m, 1, y, y_dtype, y_stride_m, 1, a);
  if (m < 3 || m > 32 || !skinny_supported(a))
    return b200_set_error(B200_ERR_UNSUPPORTED,
                          "packed_linear_noalloc: no split-K decode GEMM for format=%d scale_dtype=%d block=%lld "
                          "K=%lld x_dtype=%d y_dtype=%d m=%lld",
                          a.fmt, a.sdt, (long long)a.block, (long long)a.cols, a.xdt, a.ydt, (long long)m);
  return launch_skinny_noalloc(a, (cudaStream_t)stream);
}

int32_t b200_add_rmsnorm(void *h, int32_t h_dtype, const float *partial, void *x, int32_t x_dtype, int64_t M,
                         int64_t H, float eps, void *stream) {
  if (int32_t rc = injected()) return rc;
  if (h == nullptr || M < 0 || H < 0) return b200_set_error(B200_ERR_INVALID, "bad add_rmsnorm arguments");
  if (!dt_is_float(h_dtype) || (x != nullptr && !dt_is_float(x_dtype)))
    return b200_set_error(B200_ERR_INVALID, "add_rmsnorm needs floating-point h / x");
  return launch_add_rmsnorm(h, h_dtype, partial, x, x_dtype, M, H, eps, (cudaStream_t)stream);
}

int32_t b200_gate_mul(const void *gu, int32_t gu_dtype, void *out, int32_t out_dtype, int64_t M, int64_t I,
                      void *stream) {
  if (int32_t rc = injected()) return rc;
  if (gu == nullptr || out == nullptr || M < 0 || I < 0) return b200_set_error(B200_ERR_INVALID, "bad gate_mul arguments");
  if (!dt_is_float(gu_dtype) || !dt_is_float(out_dtype))
    return b200_set_error(B200_ERR_INVALID, "gate_mul needs floating-point tensors");
  return launch_gate_mul(gu, gu_dtype, out, out_dtype, M, I, (cudaStream_t)stream);
}

int32_t b200_peer_allreduce_add_rmsnorm(const void *const *partials, uint32_t *const *flags, uint32_t *epoch,
                                        int32_t rank, int32_t world, int64_t rows_max, int64_t timeout_ns, void *h,
                                        int32_t h_dtype, void *x, int32_t x_dtype, int64_t M, int64_t H, float eps,
                                        void *stream) {
  if (int32_t rc = injected()) return rc;
  if (partials == nullptr || flags == nullptr || epoch == nullptr || h == nullptr)
    return b200_set_error(B200_ERR_INVALID, "peer reduce: null pointer");
  if (world < 1 || world > 8 || rank < 0 || rank >= world || M < 0 || M > rows_max || H < 0 || timeout_ns <= 0)
    return b200_set_error(B200_ERR_INVALID, "peer reduce: bad rank/world/rows/timeout");
  for (int q = 0; q < world; ++q)
    if (partials[q] == nullptr || flags[q] == nullptr) return b200_set_error(B200_ERR_INVALID, "peer reduce: null peer");
  if (!dt_is_float(h_dtype) || (x != nullptr && !dt_is_float(x_dtype)))
    return b200_set_error(B200_ERR_INVALID, "peer reduce needs floating-point h / x");
  return launch_peer_reduce_rmsnorm(partials, flags, epoch, rank, world, rows_max, timeout_ns, h, h_dtype, x, x_dtype, M,
                                    H, eps, (cudaStream_t)stream);
}

int32_t b200_ipc_get_handle(void *dev_ptr, void *handle64) {
  if (dev_ptr == nullptr || handle64 == nullptr) return b200_set_error(B200_ERR_INVALID, "ipc: null pointer");
  cudaIpcMemHandle_t hd;
  B200_CUDA_TRY(cudaIpcGetMemHandle(&hd, dev_ptr));
  memcpy(handle64, &hd, sizeof(hd));
  return B200_OK;
}

int32_t b200_ipc_open(const void *handle64, void **dev_ptr) {
  if (dev_ptr == nullptr || handle64 == nullptr) return b200_set_error(B200_ERR_INVALID, "ipc: null pointer");
  cudaIpcMemHandle_t hd;
  memcpy(&hd, handle64, sizeof(hd));
  B200_CUDA_TRY(cudaIpcOpenMemHandle(dev_ptr, hd, cudaIpcMemLazyEnablePeerAccess));
  return B200_OK;
}

int32_t b200_ipc_close(void *dev_ptr) {
  if (dev_ptr == nullptr) return b200_set_error(B200_ERR_INVALID, "ipc: null pointer");
  B200_CUDA_TRY(cudaIpcCloseMemHandle(dev_ptr));
  return B200_OK;
}

int32_t b200_device_wait_flag(const int32_t *flag, int32_t expect, int64_t max_spins, int32_t *status, void *stream) {
  if (flag == nullptr || status == nullptr) return b200_set_error(B200_ERR_INVALID, "null flag/status");
  if (max_spins < 0) return b200_set_error(B200_ERR_INVALID, "max_spins must be bounded");
  return launch_wait_flag(flag, expect, max_spins, status, (cudaStream_t)stream);
}

}  // extern "C"
