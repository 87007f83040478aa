// gemm_sm100.cu -- packed low-bit prefill GEMM on the 5th-generation tensor cores.
//
//   y[m, n] = sum_k x[m, k] * dequant(W)[n, k]        (x fp16/bf16 row-major, W packed (N, K))
//
// The B200 replacement of the reference's LinAlg matrix kernel (tinygrad-dx12
// src/tinygrad_dx12/renderer/linalg.py:38-124) for packed operands, with the decode of
// src/tinygrad_dx12/codegen/decomp/dx12.py:69-106 fused on chip instead of materialised.
//
// Persistent kernel: one CTA per SM walks 128 (weight rows n) x bt (tokens m, <= 256) output
// tiles; K advances 64 elements per stage. The weights are the MMA's A operand and live in
// tensor memory (decoded there by CUDA cores), so shared memory carries only the TMA traffic
// (x tiles and packed codes) and the tensor core's x reads.
//   warp 0 lane 0  TMA producer: x tile (bt x 64, 128-byte swizzle) and the tile's packed weight
//                  bytes (128 rows x 32/48 bytes) into a 5-stage ring, signalled on full[s];
//   warp 1 lane 0  MMA issuer: 4 x tcgen05.mma.kind::f16 (M=128, N=bt, K=16, A from tensor
//                  memory) per stage into one fp32 accumulator (128 lanes x bt columns);
//                  tcgen05.commit frees the shared stage (empty[s]) and the A stage (afree[a])
//                  and, after a tile's last stage, publishes the accumulator (accfull);
//   warps 2..9     dequant warps: thread (lane quarter q, K half h) decodes weight row
//                  32q + lane, 32 payloads per stage, to exact fp16/bf16 (decode.cuh) and
//                  writes them with tcgen05.st into a 4-stage A ring in tensor memory (aready);
//   warps 10..13   epilogue warpgroup: tcgen05.ld of the finished accumulator (lane = weight row,
//                  column = token), per-row scale, cast, store y[m, n]; it releases the
//                  accumulator (accempty) as soon as the last columns are read.
// Every mbarrier wait is bounded (sm100.cuh): on give-up the CTA drains its copies and MMAs,
// frees TMEM and returns, and the library's device error flag is set.
//
// Exactness: every payload value is exactly representable in fp16 and bf16 (<= 4 significant
// bits, small exponent range). Per-row scales (block_size >= K) multiply the fp32 accumulator
// in the epilogue; per-group E8M0 scales are powers of two and multiply the operand exactly
// (barring fp16 overflow). Products are exact in the fp32 accumulator, so results equal the
// reference's fp32 arithmetic up to summation order.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"
#include "decode.cuh"

namespace b200 {

int32_t gemm_device_error(unsigned int *v, bool clear) {
  B200_CUDA_TRY(tu_device_error(v, clear));
  return B200_OK;
}

namespace gemm {

constexpr int BW = 128;           // weight rows per tile = MMA M = TMEM lanes
constexpr int BT_MAX = 256;       // tokens per tile = MMA N (runtime bt <= 256, multiple of 32)
constexpr int BK = 64;            // K per pipeline stage
constexpr int STAGES = 5;         // shared-memory ring: x tile + packed weight tile per stage
constexpr int NA = 4;             // decoded-weight (A operand) stages in tensor memory
constexpr int ACC_COLS = BT_MAX;  // fp32 accumulator: 128 lanes x bt columns
constexpr int A_COLS = BK / 2;    // one A stage: 64 fp16/bf16 per row = 32 columns
constexpr int TMEM_COLS = 512;    // ACC_COLS + NA * A_COLS = 384, allocated as a power of two
constexpr int DQ_WARPS = 8;       // dequant warps: (TMEM lane quarter, K half) pairs
constexpr int THREADS = (2 + DQ_WARPS + 4) * 32;  // producer, MMA, dequant, 4 epilogue warps
constexpr int X_BYTES = BT_MAX * BK * 2;          // 32 KB
constexpr int P_STAGE = 6144;                     // packed bytes slot (128 rows x 48 B max)
constexpr int SMEM_BYTES = 1024 /*align slack*/ + STAGES * (X_BYTES + P_STAGE) + 256 /*barriers*/;
static_assert(ACC_COLS + NA * A_COLS <= TMEM_COLS, "tensor memory budget");
enum ScaleMode { SCALE_NONE = 0, SCALE_ROW = 1, SCALE_E8M0 = 2 };

struct Params {
  int64_t M, N, K;
  const void *scales;
  int sdt;
  int64_t nblk, block;
  int scale_mode;
  void *y;
  int ydt;
  int64_t ldy;
  int wblocks, tblocks;  // tile grid: weight-row blocks x token blocks
  int bt;                // tokens per tile (MMA N)
};

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }

// One thread's accumulator row (weight row n) for 32 consecutive tokens -> y[m, n] (stride ldy).
template <typename T>
__device__ __forceinline__ void store_col32(const Params &p, int64_t m, int64_t n, const uint32_t (&v)[32],
                                            float sc) {
  T *dst = (T *)p.y + m * p.ldy + n;
  const int64_t lim = p.M - m;
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (j < lim) dst[(int64_t)j * p.ldy] = from_f32<T>(__uint_as_float(v[j]) * sc);
}

template <int FMT, bool BF16>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw, Params p) {
  constexpr int BITS = Fmt<FMT>::bits;
  constexpr int PB = BK * BITS / 8;  // packed bytes per row per stage: 32 or 48
  extern __shared__ uint8_t smem_raw[];
  uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *xs = base;
  uint8_t *ps = xs + STAGES * X_BYTES;
  uint64_t *full = (uint64_t *)(ps + STAGES * P_STAGE);  // [STAGES] x + packed tile landed
  uint64_t *empty = full + STAGES;                        // [STAGES] stage's MMAs retired
  uint64_t *aready = empty + STAGES;                      // [NA] decoded A stage written to TMEM
  uint64_t *afree = aready + NA;                          // [NA] A stage's MMAs retired
  uint64_t *accfull = afree + NA;                         // tile's accumulator complete
  uint64_t *accempty = accfull + 1;                       // accumulator drained by the epilogue
  uint64_t *done = accempty + 1;                          // all MMAs of this CTA retired (exit path)
  uint32_t *tmem_slot = (uint32_t *)(done + 1);
  volatile uint32_t *abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = (int)(p.K / BK);
  const int ntiles = p.wblocks * p.tblocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < NA; ++a) {
      mbar_init(&aready[a], DQ_WARPS * 32);
      mbar_init(&afree[a], 1);
    }
    mbar_init(accfull, 1);
    mbar_init(accempty, 128);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmx);
    prefetch_tmap(&tmw);
  }
  __syncwarp();
  if (warp == 0) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tacc = tmem, ta = tmem + ACC_COLS;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const uint32_t tx_bytes = (uint32_t)(p.bt * BK * 2 + BW * PB);  // full boxes (OOB rows zero-filled)
      int64_t q = 0, issued = 0;
      for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const int tb = tile % p.tblocks, wb = tile / p.tblocks;
        for (int kb = 0; kb < nk; ++kb, ++q) {
          const int s = (int)(q % STAGES);
          if (q >= STAGES && !mbar_wait(&empty[s], (uint32_t)((q / STAGES - 1) & 1), abort_flag)) continue;
          if (*abort_flag) continue;
          mbar_arrive_expect_tx(&full[s], tx_bytes);
          tma_load_2d(xs + s * X_BYTES, &tmx, kb * BK, tb * p.bt, &full[s]);
          tma_load_2d(ps + s * P_STAGE, &tmw, kb * PB, wb * BW, &full[s]);
          issued = q + 1;
        }
      }
      if (*abort_flag) {  // drain this CTA's copies still in flight before it exits
        for (int64_t r = (issued > STAGES ? issued - STAGES : 0); r < issued; ++r)
          mbar_wait(&full[r % STAGES], (uint32_t)((r / STAGES) & 1), abort_flag, 200000000ull);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: D[128 x bt] += A[tmem 128 x 16] * x[bt x 16]^T ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(BF16 ? 1u : 0u, BW, (uint32_t)p.bt);
      int64_t q = 0;
      int i = 0;
      for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++i) {
        if (i > 0) mbar_wait(accempty, (uint32_t)((i - 1) & 1), abort_flag);
        tc_fence_after();
        for (int kb = 0; kb < nk; ++kb, ++q) {
          const int s = (int)(q % STAGES), a = (int)(q % NA);
          if (!mbar_wait(&full[s], (uint32_t)((q / STAGES) & 1), abort_flag) ||
              !mbar_wait(&aready[a], (uint32_t)((q / NA) & 1), abort_flag))
            continue;
          tc_fence_after();
          const uint64_t b0 = sw128_kmajor_desc(xs + s * X_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)  // A: 8 columns per K=16; B: +32 bytes inside the swizzle atom
            mma_f16_ts(tacc, ta + (uint32_t)(a * A_COLS + 8 * k), b0 + (uint64_t)(2 * k), idesc, (kb | k) != 0);
          mma_commit(&empty[s]);
          mma_commit(&afree[a]);
        }
        mma_commit(accfull);  // arrives once this tile's MMAs have completed
      }
      mma_commit(done);
      mbar_wait(done, 0, abort_flag, 500000000ull);
    }
  } else if (warp < 2 + DQ_WARPS) {
    // ---------------- dequant: thread = (weight row r = TMEM lane, K half h) ----------------
    const int qd = warp & 3, h = (warp - 2) >> 2;
    const int r = qd * 32 + lane;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const bool scaled = p.scale_mode == SCALE_E8M0;
    int64_t q = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
      const int64_t n = (int64_t)(tile / p.tblocks) * BW + r;
      for (int kb = 0; kb < nk; ++kb, ++q) {
        const int s = (int)(q % STAGES), a = (int)(q % NA);
        bool ok = mbar_wait(&full[s], (uint32_t)((q / STAGES) & 1), abort_flag);
        if (ok && q >= NA) ok = mbar_wait(&afree[a], (uint32_t)((q / NA - 1) & 1), abort_flag);
        if (!__all_sync(0xffffffffu, ok)) continue;  // tcgen05.st is warp-collective
        const uint8_t *src = ps + s * P_STAGE + r * PB + h * (PB / 2);
        uint32_t w[PB / 8];
        if constexpr (BITS == 4) {
          const uint4 u = *reinterpret_cast<const uint4 *>(src);
          w[0] = u.x, w[1] = u.y, w[2] = u.z, w[3] = u.w;
        } else {
#pragma unroll
          for (int j = 0; j < 3; ++j) {
            const uint2 u = *reinterpret_cast<const uint2 *>(src + 8 * j);
            w[2 * j] = u.x, w[2 * j + 1] = u.y;
          }
        }
        float gf = 1.f;
        if (scaled && n < p.N)
          gf = e8m0_to_f32(((const uint8_t *)p.scales)[n * p.nblk + (kb * BK + 32 * h) / p.block]);
        uint32_t out[16];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {  // 8 payloads per unit, pairs (2i, 2i+1) in natural K order
          uint32_t o[4];
          gemv::decode8_natural<FMT, BF16>(w, cc, o);
          if (scaled) {  // power-of-two block scale: exact while the product stays in range
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              if constexpr (BF16) {
                const __nv_bfloat162 v =
                    __hmul2(*reinterpret_cast<const __nv_bfloat162 *>(&o[j]), __float2bfloat162_rn(gf));
                o[j] = *reinterpret_cast<const uint32_t *>(&v);
              } else {
                const __half2 v = __hmul2(*reinterpret_cast<const __half2 *>(&o[j]), __float2half2_rn(gf));
                o[j] = *reinterpret_cast<const uint32_t *>(&v);
              }
            }
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) out[4 * cc + j] = o[j];
        }
        // K elements kb*64 + 32h + 2c, +1 -> column a*32 + 16h + c of lane r
        tmem_st_32x32b_x16(ta + lane_base + (uint32_t)(a * A_COLS + 16 * h), out);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&aready[a]);
      }
    }
  } else {
    // ---------------- epilogue: lane = weight row n, columns = tokens ----------------
    const int qd = warp & 3;
    const int r = qd * 32 + lane;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    int i = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++i) {
      const int64_t n = (int64_t)(tile / p.tblocks) * BW + r;
      const int64_t m0 = (int64_t)(tile % p.tblocks) * p.bt;
      float sc = 1.f;
      if (p.scale_mode == SCALE_ROW && n < p.N) sc = load_as_f32(p.scales, n * p.nblk, p.sdt);
      bool ok = mbar_wait(accfull, (uint32_t)(i & 1), abort_flag) && !*abort_flag;
      ok = __all_sync(0xffffffffu, ok);
      tc_fence_after();
      for (int c = 0; c < p.bt; c += 32) {
        uint32_t v[32];
        if (ok) {
          tmem_ld_32x32b_x32(tacc + lane_base + (uint32_t)c, v);
          tmem_ld_wait();
        }
        if (c + 32 >= p.bt) {  // last columns read: the next tile may overwrite the accumulator
          tc_fence_before();
          mbar_arrive(accempty);
        }
        if (ok && n < p.N && m0 + c < p.M) {
          if (p.ydt == B200_DT_F16)
            store_col32<__half>(p, m0 + c, n, v, sc);
          else if (p.ydt == B200_DT_BF16)
            store_col32<__nv_bfloat16>(p, m0 + c, n, v, sc);
          else
            store_col32<float>(p, m0 + c, n, v, sc);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, TMEM_COLS);
}

// ---- host side ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)ptr;
  }
  return fn;
}

}  // namespace gemm

// 2-D tiled tensor map (no interleave, L2 256-byte promotion, zero fill out of bounds).
int32_t make_tma_2d(CUtensorMap *map, CUtensorMapDataType dt, const void *base, uint64_t inner, uint64_t outer,
                    uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
  auto fn = gemm::encode_fn();
  if (!fn) return b200_set_error(B200_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return b200_set_error(B200_ERR_CUDA, "cuTensorMapEncodeTiled failed: %d", (int)r);
  return B200_OK;
}

namespace gemm {

template <int FMT, bool BF16>
static int32_t launch_t(const LinearArgs &a, cudaStream_t stream) {
  constexpr int BITS = Fmt<FMT>::bits;
  static bool attr_set = false;
  static int sms = 0;
  if (!attr_set) {
    int dev = 0;
    B200_CUDA_TRY(cudaGetDevice(&dev));
    B200_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    B200_CUDA_TRY(cudaFuncSetAttribute(gemm_kernel<FMT, BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    attr_set = true;
  }
  int bt = (int)((a.m + 31) / 32 * 32);
  if (bt > BT_MAX) bt = BT_MAX;
  CUtensorMap tmx, tmw;
  if (int32_t rc = make_tma_2d(&tmx, BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.x,
                               (uint64_t)a.cols, (uint64_t)a.m, (uint64_t)a.ldx * 2, BK, (uint32_t)bt,
                               CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  const uint64_t row_bytes = (uint64_t)a.cols * BITS / 8;
  if (int32_t rc = make_tma_2d(&tmw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w, row_bytes, (uint64_t)a.rows, row_bytes,
                               BK * BITS / 8, BW, CU_TENSOR_MAP_SWIZZLE_NONE))
    return rc;
  Params p;
  p.M = a.m, p.N = a.rows, p.K = a.cols;
  p.scales = a.scales;
  p.sdt = a.sdt;
  p.nblk = a.nblk;
  p.block = a.block;
  p.scale_mode = a.scales == nullptr ? SCALE_NONE : (a.block >= a.cols ? SCALE_ROW : SCALE_E8M0);
  p.y = a.y;
  p.ydt = a.ydt;
  p.ldy = a.ldy_m;
  p.bt = bt;
  p.wblocks = (int)((a.rows + BW - 1) / BW);
  p.tblocks = (int)((a.m + bt - 1) / bt);
  const int64_t tiles = (int64_t)p.wblocks * p.tblocks;
  const unsigned grid = (unsigned)(tiles < sms ? tiles : sms);
  gemm_kernel<FMT, BF16><<<grid, THREADS, SMEM_BYTES, stream>>>(tmx, tmw, p);
  B200_LAUNCH_CHECK();
  return B200_OK;
}

}  // namespace gemm

bool gemm_supported(const LinearArgs &a) {
  using namespace gemm;
  if (a.xdt != B200_DT_F16 && a.xdt != B200_DT_BF16) return false;
  if (a.ydt != B200_DT_F16 && a.ydt != B200_DT_BF16 && a.ydt != B200_DT_F32) return false;
  if (a.cols < BK || a.cols % BK != 0 || a.rows <= 0 || a.m <= 0) return false;
  if ((a.m + 31) / 32 * ((a.rows + BW - 1) / BW) > (int64_t)INT32_MAX) return false;
  if (a.ldy_n != 1) return false;
  if ((uintptr_t)a.w % 16 != 0 || (uintptr_t)a.x % 16 != 0 || (a.ldx * 2) % 16 != 0) return false;
  if (a.scales != nullptr) {
    const bool row = a.block >= a.cols &&
                     (a.sdt == B200_DT_F16 || a.sdt == B200_DT_BF16 || a.sdt == B200_DT_F32 || a.sdt == B200_DT_E8M0);
    const bool grp = a.sdt == B200_DT_E8M0 && (a.block == 32 || a.block % BK == 0);
    if (!row && !grp) return false;
  }
  return true;
}

int32_t launch_gemm(const LinearArgs &a, cudaStream_t stream) {
  using namespace gemm;
  const bool bf = a.xdt == B200_DT_BF16;
#define B200_GEMM_CASE(F)                                                              \
  case F:                                                                              \
    return bf ? launch_t<F, true>(a, stream) : launch_t<F, false>(a, stream);
  switch (a.fmt) {
    B200_GEMM_CASE(B200_FMT_INT4)
    B200_GEMM_CASE(B200_FMT_UINT4)
    B200_GEMM_CASE(B200_FMT_FP4_E2M1)
    B200_GEMM_CASE(B200_FMT_FP6_E2M3)
    B200_GEMM_CASE(B200_FMT_FP6_E3M2)
  }
#undef B200_GEMM_CASE
  return b200_set_error(B200_ERR_INVALID, "unknown packed format %d", a.fmt);
}

}  // namespace b200
