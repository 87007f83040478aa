// stack_ops.cu -- the elementwise steps between the packed projections of a decoder layer
// stack (benchmark configs c4 / c5): residual add of an fp32 partial + RMS normalisation, and
// the gate * up product. One launch each per sub-layer; rows (tokens) are independent.
//
// The reference has no layer stack (its packed path ends at one matmul); these kernels exist
// so the multi-layer configurations run without a torch elementwise chain between kernels.
#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace b200 {
namespace stackops {

constexpr int THREADS = 512;

__device__ __forceinline__ float block_sum(float v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
  if (warp == 0) {
    s = lane < THREADS / 32 ? red[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[THREADS / 32] = s;
  }
  __syncthreads();
  return red[THREADS / 32];
}

// One CTA per row: h = h + partial (if given, fp32 add then rounding to h's dtype);
// x = h * rsqrt(mean(h^2) + eps) in fp32, stored in x's dtype.
__device__ __forceinline__ void pdl_enter() {
  // launched with programmatic stream serialization: let the next kernel start its prologue,
  // then wait until the previous kernel's results are visible before reading them
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Launch with the programmatic-dependent-launch attribute (every kernel here calls pdl_enter
// before touching memory, so the attribute is always safe).
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

__global__ void __launch_bounds__(THREADS) add_rmsnorm_kernel(void *h, int hdt, const float *partial, void *x,
                                                              int xdt, int64_t H, float eps) {
  __shared__ float red[THREADS / 32 + 1];
  pdl_enter();
  const int64_t row = blockIdx.x;
  const int64_t base = row * H;
  float ss = 0.f;
  for (int64_t i = threadIdx.x; i < H; i += THREADS) {
    float v = load_as_f32(h, base + i, hdt);
    if (partial != nullptr) {
      v += partial[base + i];
      store_f32(h, base + i, hdt, v);
      v = load_as_f32(h, base + i, hdt);  // the stored (rounded) value is what the next layer sees
    }
    ss += v * v;
  }
  const float total = block_sum(ss, red);
  const float inv = rsqrtf(total / (float)H + eps);
  if (x != nullptr)
    for (int64_t i = threadIdx.x; i < H; i += THREADS) store_f32(x, base + i, xdt, load_as_f32(h, base + i, hdt) * inv);
}

// ---- vectorised, typed row kernels (one CTA of RT threads per row, H <= RT * 4 * RV) ---------
constexpr int RT = 1024, RV = 4;

template <typename T>
__device__ __forceinline__ void load4(const T *p, float (&f)[4]);
template <>
__device__ __forceinline__ void load4<__half>(const __half *p, float (&f)[4]) {
  const uint2 u = *reinterpret_cast<const uint2 *>(p);
  const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u.x)),
               b = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
  f[0] = a.x, f[1] = a.y, f[2] = b.x, f[3] = b.y;
}
template <>
__device__ __forceinline__ void load4<__nv_bfloat16>(const __nv_bfloat16 *p, float (&f)[4]) {
  const uint2 u = *reinterpret_cast<const uint2 *>(p);
  f[0] = __uint_as_float(u.x << 16), f[1] = __uint_as_float(u.x & 0xFFFF0000u);
  f[2] = __uint_as_float(u.y << 16), f[3] = __uint_as_float(u.y & 0xFFFF0000u);
}
template <>
__device__ __forceinline__ void load4<float>(const float *p, float (&f)[4]) {
  const float4 u = *reinterpret_cast<const float4 *>(p);
  f[0] = u.x, f[1] = u.y, f[2] = u.z, f[3] = u.w;
}
template <typename T>
__device__ __forceinline__ void store4(T *p, const float (&f)[4]);
template <>
__device__ __forceinline__ void store4<__half>(__half *p, const float (&f)[4]) {
  const __half2 a = __floats2half2_rn(f[0], f[1]), b = __floats2half2_rn(f[2], f[3]);
  *reinterpret_cast<uint2 *>(p) = make_uint2(*reinterpret_cast<const uint32_t *>(&a), *reinterpret_cast<const uint32_t *>(&b));
}
template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16 *p, const float (&f)[4]) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(f[0], f[1]), b = __floats2bfloat162_rn(f[2], f[3]);
  *reinterpret_cast<uint2 *>(p) = make_uint2(*reinterpret_cast<const uint32_t *>(&a), *reinterpret_cast<const uint32_t *>(&b));
}
template <>
__device__ __forceinline__ void store4<float>(float *p, const float (&f)[4]) {
  *reinterpret_cast<float4 *>(p) = make_float4(f[0], f[1], f[2], f[3]);
}
template <typename T>
__device__ __forceinline__ float round_t(float v);
template <>
__device__ __forceinline__ float round_t<__half>(float v) { return __half2float(__float2half_rn(v)); }
template <>
__device__ __forceinline__ float round_t<__nv_bfloat16>(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
template <>
__device__ __forceinline__ float round_t<float>(float v) { return v; }

__device__ __forceinline__ float block_sum_rt(float v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float t = lane < RT / 32 ? red[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) red[RT / 32] = t;
  }
  __syncthreads();
  return red[RT / 32];
}

// h += partial (rounded to T), then x = rmsnorm(h); every value stays in registers.
template <typename T>
__global__ void __launch_bounds__(RT) add_rmsnorm_vec_kernel(T *h, const float *partial, T *x, int64_t H, float eps) {
  __shared__ float red[RT / 32 + 1];
  pdl_enter();
  const int64_t row = blockIdx.x;
  T *hr = h + row * H;
  const float *pr = partial != nullptr ? partial + row * H : nullptr;
  const int nv = (int)(H / 4);
  float val[RV][4];
  float ss = 0.f;
#pragma unroll
  for (int it = 0; it < RV; ++it) {
    const int v = threadIdx.x + it * RT;
    if (v < nv) {
      float f[4];
      load4<T>(hr + 4 * v, f);
      if (pr != nullptr) {
        const float4 q = reinterpret_cast<const float4 *>(pr)[v];
        f[0] = round_t<T>(f[0] + q.x), f[1] = round_t<T>(f[1] + q.y);
        f[2] = round_t<T>(f[2] + q.z), f[3] = round_t<T>(f[3] + q.w);
        store4<T>(hr + 4 * v, f);
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) ss += f[c] * f[c], val[it][c] = f[c];
    }
  }
  const float inv = rsqrtf(block_sum_rt(ss, red) / (float)H + eps);
  if (x != nullptr) {
    T *xr = x + row * H;
#pragma unroll
    for (int it = 0; it < RV; ++it) {
      const int v = threadIdx.x + it * RT;
      if (v < nv) {
        const float o[4] = {val[it][0] * inv, val[it][1] * inv, val[it][2] * inv, val[it][3] * inv};
        store4<T>(xr + 4 * v, o);
      }
    }
  }
}

// out[m, i] = gu[m, i] * gu[m, I + i] (fp32 product, rounded to out's dtype).
__global__ void gate_mul_kernel(const void *gu, int gdt, void *out, int odt, int64_t M, int64_t I) {
  pdl_enter();
  const int64_t n = M * I;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = t / I, i = t - m * I;
    const float g = load_as_f32(gu, m * 2 * I + i, gdt), u = load_as_f32(gu, m * 2 * I + I + i, gdt);
    store_f32(out, t, odt, g * u);
  }
}

}  // namespace stackops

int32_t launch_add_rmsnorm(void *h, int hdt, const float *partial, void *x, int xdt, int64_t M, int64_t H, float eps,
                           cudaStream_t stream) {
  if (M <= 0 || H <= 0) return B200_OK;
  using namespace stackops;
  const int esz = dt_size(hdt);
  const bool vec = (x == nullptr || xdt == hdt) && H % 4 == 0 && H <= (int64_t)RT * 4 * RV &&
                   (uintptr_t)h % (4 * esz) == 0 && (x == nullptr || (uintptr_t)x % (4 * esz) == 0) &&
                   (partial == nullptr || (uintptr_t)partial % 16 == 0);
  if (vec && hdt == B200_DT_F16) {
    B200_CUDA_TRY(launch_pdl(add_rmsnorm_vec_kernel<__half>, dim3((unsigned)M), dim3(RT), stream, (__half *)h, partial,
                             (__half *)x, H, eps));
  } else if (vec && hdt == B200_DT_BF16) {
    B200_CUDA_TRY(launch_pdl(add_rmsnorm_vec_kernel<__nv_bfloat16>, dim3((unsigned)M), dim3(RT), stream,
                             (__nv_bfloat16 *)h, partial, (__nv_bfloat16 *)x, H, eps));
  } else if (vec && hdt == B200_DT_F32) {
    B200_CUDA_TRY(launch_pdl(add_rmsnorm_vec_kernel<float>, dim3((unsigned)M), dim3(RT), stream, (float *)h, partial,
                             (float *)x, H, eps));
  } else {
    B200_CUDA_TRY(launch_pdl(add_rmsnorm_kernel, dim3((unsigned)M), dim3(THREADS), stream, h, hdt, partial, x, xdt, H,
                             eps));
  }
  return B200_OK;
}

int32_t launch_gate_mul(const void *gu, int gdt, void *out, int odt, int64_t M, int64_t I, cudaStream_t stream) {
  const int64_t n = M * I;
  if (n <= 0) return B200_OK;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  B200_CUDA_TRY(stackops::launch_pdl(stackops::gate_mul_kernel, dim3((unsigned)blocks), dim3(256), stream, gu, gdt, out,
                                     odt, M, I));
  return B200_OK;
}

}  // namespace b200

// ---- tensor-parallel reduction over peer memory (one-shot, fused with add + RMS norm) -------
// Each rank's row-parallel projection has written its fp32 partial (M x H) into its own buffer,
// which every peer has mapped (CUDA IPC). For row r, CTA r:
//   1. e = ++epoch[r] (this rank's count of reductions of row r; the same on every rank);
//   2. publishes e in flags[rank][r] of every rank and 3. waits until flags[q][r] >= e locally
//      for every rank q -- thread q talks to rank q, with a system-scope fence before its store
//      and after its last load (bounded; on give-up it flags the device error word and continues);
//   4. sums the partial rows of ranks 0..world-1 in that order (identical on every rank, so h
//      stays bitwise replicated), adds the sum to h and writes x = rmsnorm(h).
// A rank reuses a partial buffer only two reductions later, after every peer has signalled
// the reduction in between, i.e. after every peer has finished reading it.

namespace b200 {

int32_t stackops_device_error(unsigned int *v, bool clear) {
  B200_CUDA_TRY(tu_device_error(v, clear));
  return B200_OK;
}

namespace stackops {

constexpr int MAX_PEERS = 8;
struct PeerReduce {
  const float *partial[MAX_PEERS];  // rank q's partial buffer (M x H fp32), mapped here
  uint32_t *flags[MAX_PEERS];       // rank q's flag array [world][rows_max], mapped here
  uint32_t *epoch;                  // this rank's epoch counters [rows_max]
  int rank, world;
  int64_t rows_max;
  int64_t timeout_ns;
};

__device__ __forceinline__ void st_relaxed_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

constexpr int PR_THREADS = 1024;
constexpr int PR_VEC = 2;  // float4 per thread per rank held in registers at once (H <= 8192 per pass)

template <typename T>
__device__ __forceinline__ float round_to(float v);
template <>
__device__ __forceinline__ float round_to<__half>(float v) { return __half2float(__float2half_rn(v)); }
template <>
__device__ __forceinline__ float round_to<__nv_bfloat16>(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
template <>
__device__ __forceinline__ float round_to<float>(float v) { return v; }

template <typename T>
__global__ void __launch_bounds__(PR_THREADS) peer_reduce_rmsnorm_kernel(PeerReduce pr, T *__restrict__ h,
                                                                         void *x, int xdt, int64_t H, float eps) {
  __shared__ float red[PR_THREADS / 32 + 1];
  const int64_t row = blockIdx.x;
  pdl_enter();  // this rank's partial is complete from here on
  __shared__ uint32_t e_sh;
  if (threadIdx.x == 0) {
    e_sh = pr.epoch[row] + 1u;
    pr.epoch[row] = e_sh;
  }
  __syncthreads();
  const uint32_t e = e_sh;
  if (threadIdx.x < pr.world) {
    // thread q signals rank q and waits for rank q's signal: one NVLink round trip overall
    const int q = threadIdx.x;
    asm volatile("fence.acq_rel.sys;" ::: "memory");  // the partial is visible before the flag
    st_relaxed_sys(pr.flags[q] + (int64_t)pr.rank * pr.rows_max + row, e);
    const uint32_t *f = pr.flags[pr.rank] + (int64_t)q * pr.rows_max + row;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 0;; ++i) {
      if ((int32_t)(ld_relaxed_sys(f) - e) >= 0) break;
      if ((i & 255u) == 255u && globaltimer() - t0 > (uint64_t)pr.timeout_ns) {
        atomicOr(&g_device_error, B200_DEVERR_MBAR_TIMEOUT);
        break;
      }
    }
    asm volatile("fence.acq_rel.sys;" ::: "memory");  // rank q's partial is read after its flag
  }
  __syncthreads();
  T *hr = h + row * H;
  const int64_t base = row * H;
  float ss = 0.f;
  if (H % 4 == 0) {
    const int64_t nv = H / 4;
    for (int64_t v0 = 0; v0 < nv; v0 += (int64_t)PR_THREADS * PR_VEC) {
      float4 acc[PR_VEC];
      float4 got[MAX_PEERS][PR_VEC];
#pragma unroll
      for (int q = 0; q < MAX_PEERS; ++q)  // every peer load issued before any is used
#pragma unroll
        for (int u = 0; u < PR_VEC; ++u) {
          const int64_t v = v0 + threadIdx.x + (int64_t)u * PR_THREADS;
          got[q][u] = (q < pr.world && v < nv) ? __ldcv(reinterpret_cast<const float4 *>(pr.partial[q] + base) + v)
                                               : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
      for (int u = 0; u < PR_VEC; ++u) {
        acc[u] = got[0][u];
#pragma unroll
        for (int q = 1; q < MAX_PEERS; ++q)
          if (q < pr.world) acc[u].x += got[q][u].x, acc[u].y += got[q][u].y, acc[u].z += got[q][u].z, acc[u].w += got[q][u].w;
        const int64_t v = v0 + threadIdx.x + (int64_t)u * PR_THREADS;
        if (v < nv) {
          const float r[4] = {acc[u].x, acc[u].y, acc[u].z, acc[u].w};
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const float hv = round_to<T>((float)hr[4 * v + c] + r[c]);
            hr[4 * v + c] = (T)hv;
            ss += hv * hv;
          }
        }
      }
    }
  } else {
    for (int64_t i = threadIdx.x; i < H; i += PR_THREADS) {
      float sum = 0.f;
      for (int q = 0; q < pr.world; ++q) sum += __ldcv(pr.partial[q] + base + i);
      const float hv = round_to<T>((float)hr[i] + sum);
      hr[i] = (T)hv;
      ss += hv * hv;
    }
  }
  // block sum of squares
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    float t = lane < PR_THREADS / 32 ? red[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) red[PR_THREADS / 32] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[PR_THREADS / 32] / (float)H + eps);
  if (x != nullptr)
    for (int64_t i = threadIdx.x; i < H; i += PR_THREADS) store_f32(x, base + i, xdt, (float)hr[i] * inv);
}

}  // namespace stackops

namespace stackops {

// The register-resident form of peer_reduce_rmsnorm_kernel (x in h's dtype, H % 4 == 0).
template <typename T>
__global__ void __launch_bounds__(RT) peer_reduce_vec_kernel(PeerReduce pr, T *__restrict__ h, T *x, int64_t H,
                                                             float eps) {
  __shared__ float red[RT / 32 + 1];
  __shared__ uint32_t e_sh;
  const int64_t row = blockIdx.x;
  pdl_enter();  // this rank's partial is complete from here on
  if (threadIdx.x == 0) {
    e_sh = pr.epoch[row] + 1u;
    pr.epoch[row] = e_sh;
  }
  __syncthreads();
  const uint32_t e = e_sh;
  if (threadIdx.x < pr.world) {  // thread q signals rank q and waits for rank q's signal
    const int q = threadIdx.x;
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    st_relaxed_sys(pr.flags[q] + (int64_t)pr.rank * pr.rows_max + row, e);
    const uint32_t *f = pr.flags[pr.rank] + (int64_t)q * pr.rows_max + row;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 0;; ++i) {
      if ((int32_t)(ld_relaxed_sys(f) - e) >= 0) break;
      if ((i & 255u) == 255u && globaltimer() - t0 > (uint64_t)pr.timeout_ns) {
        atomicOr(&g_device_error, B200_DEVERR_MBAR_TIMEOUT);
        break;
      }
    }
    asm volatile("fence.acq_rel.sys;" ::: "memory");
  }
  __syncthreads();
  T *hr = h + row * H;
  const int64_t base = row * H;
  const int nv = (int)(H / 4);
  float val[RV][4];
  float ss = 0.f;
#pragma unroll
  for (int it = 0; it < RV; ++it) {
    const int v = threadIdx.x + it * RT;
    if (v < nv) {
      float4 got[MAX_PEERS];
#pragma unroll
      for (int q = 0; q < MAX_PEERS; ++q)  // every peer load in flight before any is used
        got[q] = q < pr.world ? __ldcv(reinterpret_cast<const float4 *>(pr.partial[q] + base) + v)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
      float4 sum = got[0];
#pragma unroll
      for (int q = 1; q < MAX_PEERS; ++q)
        if (q < pr.world) sum.x += got[q].x, sum.y += got[q].y, sum.z += got[q].z, sum.w += got[q].w;
      float f[4];
      load4<T>(hr + 4 * v, f);
      f[0] = round_t<T>(f[0] + sum.x), f[1] = round_t<T>(f[1] + sum.y);
      f[2] = round_t<T>(f[2] + sum.z), f[3] = round_t<T>(f[3] + sum.w);
      store4<T>(hr + 4 * v, f);
#pragma unroll
      for (int c = 0; c < 4; ++c) ss += f[c] * f[c], val[it][c] = f[c];
    }
  }
  const float inv = rsqrtf(block_sum_rt(ss, red) / (float)H + eps);
  if (x != nullptr) {
    T *xr = x + row * H;
#pragma unroll
    for (int it = 0; it < RV; ++it) {
      const int v = threadIdx.x + it * RT;
      if (v < nv) {
        const float o[4] = {val[it][0] * inv, val[it][1] * inv, val[it][2] * inv, val[it][3] * inv};
        store4<T>(xr + 4 * v, o);
      }
    }
  }
}

}  // namespace stackops

int32_t launch_peer_reduce_rmsnorm(const void *const *partials, uint32_t *const *flags, uint32_t *epoch, int rank,
                                   int world, int64_t rows_max, int64_t timeout_ns, void *h, int hdt, void *x, int xdt,
                                   int64_t M, int64_t H, float eps, cudaStream_t stream) {
  if (M <= 0 || H <= 0) return B200_OK;
  stackops::PeerReduce pr = {};
  for (int q = 0; q < world; ++q) {
    pr.partial[q] = static_cast<const float *>(partials[q]);
    pr.flags[q] = flags[q];
  }
  pr.epoch = epoch;
  pr.rank = rank;
  pr.world = world;
  pr.rows_max = rows_max;
  pr.timeout_ns = timeout_ns;
  using namespace stackops;
  const int esz = dt_size(hdt);
  bool vec = (x == nullptr || xdt == hdt) && H % 4 == 0 && H <= (int64_t)RT * 4 * RV &&
             (uintptr_t)h % (4 * esz) == 0 && (x == nullptr || (uintptr_t)x % (4 * esz) == 0);
  for (int q = 0; q < world; ++q) vec = vec && (uintptr_t)partials[q] % 16 == 0;
  if (vec && hdt == B200_DT_F16) {
    B200_CUDA_TRY(launch_pdl(peer_reduce_vec_kernel<__half>, dim3((unsigned)M), dim3(RT), stream, pr, (__half *)h,
                             (__half *)x, H, eps));
    return B200_OK;
  }
  if (vec && hdt == B200_DT_BF16) {
    B200_CUDA_TRY(launch_pdl(peer_reduce_vec_kernel<__nv_bfloat16>, dim3((unsigned)M), dim3(RT), stream, pr,
                             (__nv_bfloat16 *)h, (__nv_bfloat16 *)x, H, eps));
    return B200_OK;
  }
  if (vec && hdt == B200_DT_F32) {
    B200_CUDA_TRY(launch_pdl(peer_reduce_vec_kernel<float>, dim3((unsigned)M), dim3(RT), stream, pr, (float *)h,
                             (float *)x, H, eps));
    return B200_OK;
  }
  switch (hdt) {
    case B200_DT_F16:
      B200_CUDA_TRY(launch_pdl(peer_reduce_rmsnorm_kernel<__half>, dim3((unsigned)M), dim3(PR_THREADS), stream, pr,
                               (__half *)h, x, xdt, H, eps));
      break;
    case B200_DT_BF16:
      B200_CUDA_TRY(launch_pdl(peer_reduce_rmsnorm_kernel<__nv_bfloat16>, dim3((unsigned)M), dim3(PR_THREADS), stream,
                               pr, (__nv_bfloat16 *)h, x, xdt, H, eps));
      break;
    case B200_DT_F32:
      B200_CUDA_TRY(launch_pdl(peer_reduce_rmsnorm_kernel<float>, dim3((unsigned)M), dim3(PR_THREADS), stream, pr,
                               (float *)h, x, xdt, H, eps));
      break;
    default:
      return b200_set_error(B200_ERR_UNSUPPORTED, "peer reduce: h dtype %d (f16, bf16, f32)", hdt);
  }
  return B200_OK;
}

}  // namespace b200
