// gemm_dense.cu -- ordinary fp16 / bf16 matmul on the 5th-generation tensor cores.
//
//   c[m, n] = sum_k a[m, k] * b[k, n]     (a: M x K, k contiguous; b given K-major, i.e. b^T
//                                           is N x K with k contiguous; fp32 accumulation)
//
// The "tiled" / ordinary matmul of the reference's matrix API (tinygrad-dx12
// src/tinygrad_dx12/codegen/linalg.py:188-189, lowered to the LinAlg kernel of
// renderer/linalg.py:38-124) for plain 16-bit operands: the packed GEMM (gemm_sm100.cu)
// without its dequant stage. Persistent, one CTA per SM, tiles of 128 (n) x bt (m <= 256):
//   warp 0 lane 0  TMA producer: b^T tile (128 x 64) and a tile (bt x 64), both 128-byte
//                  swizzled K-major, into a 4-stage ring (full[s]);
//   warp 1 lane 0  MMA issuer: 4 x tcgen05.mma.kind::f16 (M=128, N=bt, K=16) per stage, both
//                  operands from shared memory, into one of two fp32 TMEM accumulators
//                  (2 x 256 columns), so each tile's epilogue overlaps the next main loop;
//   warps 2..5     epilogue: tcgen05.ld of 32-column chunks, cast, staged in shared memory and
//                  written with a TMA store (direct stores when c's layout does not allow TMA).
// K tails are zero-filled by TMA. Every wait is bounded (sm100.cuh).
#include <cudaTypedefs.h>
#include <string.h>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace b200 {

int32_t gemm_dense_device_error(unsigned int *v, bool clear) {
  B200_CUDA_TRY(tu_device_error(v, clear));
  return B200_OK;
}

namespace dense {

constexpr int BW = 128, BT_MAX = 256, BK = 64, STAGES = 4, ACC = 2;
constexpr int EPI_WARPS = 4, THREADS = (2 + EPI_WARPS) * 32;
constexpr int X_BYTES = BT_MAX * BK * 2;  // 32 KB
constexpr int W_BYTES = BW * BK * 2;      // 16 KB
constexpr int EPI_CHUNK = 32;
constexpr int STG_BYTES = EPI_CHUNK * BW * 4;
constexpr int TMEM_COLS = ACC * BT_MAX;  // 512
constexpr int SMEM_BYTES = 1024 + STAGES * (X_BYTES + W_BYTES) + 2 * STG_BYTES + 256;

struct Params {
  int64_t M, N, K;
  void *c;
  int cdt;
  int64_t ldc;
  int wblocks, tblocks, bt, nk;
  int tma_store;
};

template <typename T>
__device__ __forceinline__ T cvt_out(float v);
template <>
__device__ __forceinline__ __half cvt_out<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 cvt_out<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ float cvt_out<float>(float v) { return v; }

template <typename T>
__device__ __forceinline__ void stage32(uint8_t *stg, int r, const uint32_t (&v)[32]) {
  T *dst = (T *)stg + r;
#pragma unroll
  for (int j = 0; j < 32; ++j) dst[j * BW] = cvt_out<T>(__uint_as_float(v[j]));
}
template <typename T>
__device__ __forceinline__ void store32(const Params &p, int64_t m, int64_t n, const uint32_t (&v)[32]) {
  T *dst = (T *)p.c + m * p.ldc + n;
  const int64_t lim = p.M - m;
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (j < lim) dst[(int64_t)j * p.ldc] = cvt_out<T>(__uint_as_float(v[j]));
}

__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, %0;" ::"n"(EPI_WARPS * 32) : "memory"); }

template <bool BF16>
__global__ void __launch_bounds__(THREADS, 1)
    dense_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmb,
                 const __grid_constant__ CUtensorMap tmc, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *xs = base;                          // a tiles (B operand)
  uint8_t *ws = xs + STAGES * X_BYTES;         // b^T tiles (A operand)
  uint8_t *stg = ws + STAGES * W_BYTES;        // [2][STG_BYTES]
  uint64_t *full = (uint64_t *)(stg + 2 * STG_BYTES);
  uint64_t *empty = full + STAGES;
  uint64_t *accfull = empty + STAGES;  // [ACC]
  uint64_t *accempty = accfull + ACC;  // [ACC]
  uint64_t *done = accempty + ACC;
  uint32_t *tmem_slot = (uint32_t *)(done + 1);
  volatile uint32_t *abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = p.wblocks * p.tblocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < ACC; ++a) {
      mbar_init(&accfull[a], 1);
      mbar_init(&accempty[a], EPI_WARPS);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tma);
    prefetch_tmap(&tmb);
    if (p.tma_store) prefetch_tmap(&tmc);
  }
  __syncwarp();
  if (warp == 0) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t tx = (uint32_t)(p.bt * BK * 2 + W_BYTES);
      int idx = 0, issued = 0;
      uint32_t ph = 0;
      for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const int tb = tile % p.tblocks, wb = tile / p.tblocks;
        for (int kb = 0; kb < p.nk; ++kb) {
          if (issued >= STAGES && !mbar_wait(&empty[idx], ph ^ 1u, abort_flag)) break;
          if (*abort_flag) break;
          mbar_arrive_expect_tx(&full[idx], tx);
          tma_load_2d(xs + idx * X_BYTES, &tma, kb * BK, tb * p.bt, &full[idx]);
          tma_load_2d(ws + idx * W_BYTES, &tmb, kb * BK, wb * BW, &full[idx]);
          ++issued;
          if (++idx == STAGES) idx = 0, ph ^= 1u;
        }
        if (*abort_flag) break;
      }
      if (*abort_flag) {
        for (int i = 0; i < STAGES && i < issued; ++i) {
          int s = idx - 1 - i;
          uint32_t q = ph;
          if (s < 0) s += STAGES, q ^= 1u;
          mbar_wait(&full[s], q, abort_flag, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(BF16 ? 1u : 0u, BW, (uint32_t)p.bt);
      int idx = 0, i = 0;
      uint32_t ph = 0;
      for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++i) {
        const int ab = i % ACC;
        if (i >= ACC) mbar_wait_sleep(&accempty[ab], (uint32_t)((i / ACC - 1) & 1), abort_flag);
        tc_fence_after();
        const uint32_t tacc = tmem + (uint32_t)(ab * BT_MAX);
        for (int kb = 0; kb < p.nk; ++kb) {
          if (mbar_wait_sleep(&full[idx], ph, abort_flag)) {
            tc_fence_after();
            const uint64_t a0 = sw128_kmajor_desc(ws + idx * W_BYTES), b0 = sw128_kmajor_desc(xs + idx * X_BYTES);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              mma_f16_ss(tacc, a0 + (uint64_t)(2 * k), b0 + (uint64_t)(2 * k), idesc, (kb | k) != 0);
            mma_commit(&empty[idx]);
          }
          if (++idx == STAGES) idx = 0, ph ^= 1u;
        }
        mma_commit(&accfull[ab]);
      }
      mma_commit(done);
      mbar_wait(done, 0, abort_flag, 500000000ull);
    }
  } else {
    const int qd = warp & 3;
    const int r = qd * 32 + lane;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const bool issuer = warp == 2 && lane == 0;
    int i = 0, chunk = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++i) {
      const int ab = i % ACC;
      const int64_t n0 = (int64_t)(tile / p.tblocks) * BW, n = n0 + r;
      const int64_t m0 = (int64_t)(tile % p.tblocks) * p.bt;
      bool ok = mbar_wait(&accfull[ab], (uint32_t)((i / ACC) & 1), abort_flag) && !*abort_flag;
      ok = __all_sync(0xffffffffu, ok);
      tc_fence_after();
      const uint32_t tacc = tmem + lane_base + (uint32_t)(ab * BT_MAX);
      for (int c = 0; c < p.bt; c += EPI_CHUNK, ++chunk) {
        uint32_t v[32];
        if (ok) {
          tmem_ld_32x32b_x32(tacc + (uint32_t)c, v);
          tmem_ld_wait();
        }
        if (c + EPI_CHUNK >= p.bt) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&accempty[ab]);
        }
        const bool live = ok && m0 + c < p.M;
        if (p.tma_store) {
          uint8_t *sb = stg + (chunk & 1) * STG_BYTES;
          if (issuer) bulk_wait_read<1>();
          epi_sync();
          if (live) {
            if (p.cdt == B200_DT_F16) stage32<__half>(sb, r, v);
            else if (p.cdt == B200_DT_BF16) stage32<__nv_bfloat16>(sb, r, v);
            else stage32<float>(sb, r, v);
          }
          fence_proxy_async_smem();
          epi_sync();
          if (issuer && live) {
            tma_store_2d(&tmc, sb, (int32_t)n0, (int32_t)(m0 + c));
            bulk_commit();
          }
        } else if (live && n < p.N) {
          if (p.cdt == B200_DT_F16) store32<__half>(p, m0 + c, n, v);
          else if (p.cdt == B200_DT_BF16) store32<__nv_bfloat16>(p, m0 + c, n, v);
          else store32<float>(p, m0 + c, n, v);
        }
      }
    }
    if (issuer) bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, TMEM_COLS);
}

}  // namespace dense

bool gemm_dense_supported(const void *a, int adt, int64_t sam, int64_t sak, const void *b, int bdt, int64_t sbk,
                          int64_t sbn, int cdt, int64_t scn, int64_t M, int64_t N, int64_t K, int accdt) {
  if (adt != bdt || (adt != B200_DT_F16 && adt != B200_DT_BF16)) return false;
  if (accdt != B200_DT_F16 && accdt != B200_DT_BF16 && accdt != B200_DT_F32) return false;
  if (cdt != B200_DT_F16 && cdt != B200_DT_BF16 && cdt != B200_DT_F32) return false;
  if (sak != 1 || sbk != 1 || scn != 1 || M < 1 || N < 1 || K < 16) return false;
  if ((uintptr_t)a % 16 != 0 || (uintptr_t)b % 16 != 0) return false;
  if ((sam * 2) % 16 != 0 || (sbn * 2) % 16 != 0 || sam < K || sbn < K) return false;
  if ((M + 255) / 256 * ((N + 127) / 128) > (int64_t)INT32_MAX) return false;
  return true;
}

int32_t launch_gemm_dense(const void *a, int adt, int64_t sam, const void *b, int64_t sbn, void *c, int cdt,
                          int64_t scm, int64_t M, int64_t N, int64_t K, cudaStream_t stream) {
  using namespace dense;
  const bool bf = adt == B200_DT_BF16;
  int sms = 0;
  B200_CUDA_TRY(device_sms(&sms));
  if (bf)
    B200_CUDA_TRY((ensure_dynamic_smem<dense_kernel<true>>(SMEM_BYTES)));
  else
    B200_CUDA_TRY((ensure_dynamic_smem<dense_kernel<false>>(SMEM_BYTES)));
  int bt = (int)((M + 31) / 32 * 32);
  if (bt > BT_MAX) bt = BT_MAX;
  const CUtensorMapDataType dt = bf ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tma, tmb, tmc;
  if (int32_t rc = make_tma_2d(&tma, dt, a, (uint64_t)K, (uint64_t)M, (uint64_t)sam * 2, BK, (uint32_t)bt,
                               CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  if (int32_t rc = make_tma_2d(&tmb, dt, b, (uint64_t)K, (uint64_t)N, (uint64_t)sbn * 2, BK, BW,
                               CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  const int csz = cdt == B200_DT_F32 ? 4 : 2;
  memset(&tmc, 0, sizeof(tmc));
  const bool tma_store = (uintptr_t)c % 16 == 0 && (scm * csz) % 16 == 0 && scm >= N;
  if (tma_store) {
    const CUtensorMapDataType cdtt = cdt == B200_DT_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                     : cdt == B200_DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                           : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    if (int32_t rc = make_tma_2d(&tmc, cdtt, c, (uint64_t)N, (uint64_t)M, (uint64_t)scm * csz, BW, EPI_CHUNK,
                                 CU_TENSOR_MAP_SWIZZLE_NONE))
      return rc;
  }
  Params p;
  p.M = M, p.N = N, p.K = K;
  p.c = c, p.cdt = cdt, p.ldc = scm;
  p.bt = bt;
  p.wblocks = (int)((N + BW - 1) / BW);
  p.tblocks = (int)((M + bt - 1) / bt);
  p.nk = (int)((K + BK - 1) / BK);
  p.tma_store = tma_store ? 1 : 0;
  const int64_t tiles = (int64_t)p.wblocks * p.tblocks;
  const unsigned grid = (unsigned)(tiles < sms ? tiles : sms);
  if (bf)
    dense_kernel<true><<<grid, THREADS, SMEM_BYTES, stream>>>(tma, tmb, tmc, p);
  else
    dense_kernel<false><<<grid, THREADS, SMEM_BYTES, stream>>>(tma, tmb, tmc, p);
  B200_LAUNCH_CHECK();
  return B200_OK;
}

}  // namespace b200
