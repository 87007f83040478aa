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
// (x tiles and packed codes), the tensor core's x reads and the epilogue's staging. The MMA is
// as wide as tensor memory allows (N = 256): narrower MMAs (N = 128, 192) measured slower on
// B200 even with a second accumulator to overlap the epilogue.
//   warp 0 lane 0  TMA producer: x tile (bt x 64, 128-byte swizzle) and the tile's packed weight
//                  bytes (128 rows x 32/48 bytes) into a 5-stage ring, signalled on full[s];
//   warp 1 lane 0  MMA issuer: 4 x tcgen05.mma.kind::f16 (M=128, N=bt, K=16, A from tensor
//                  memory) per stage into the fp32 accumulator (128 lanes x bt columns);
//                  tcgen05.commit frees the shared stage (empty[s]) and the A stage (afree[a])
//                  and, after a tile's last stage, publishes the accumulator (accfull);
//   warps 2..17    dequant warps: thread (lane quarter q, K quarter) decodes weight row
//                  32q + lane, 16 payloads per stage, to exact fp16/bf16 (decode.cuh) and
//                  writes them with tcgen05.st into a 4-stage A ring in tensor memory (aready,
//                  one arrival per warp);
//   warps 18..21   epilogue warpgroup: tcgen05.ld of the finished accumulator (lane = weight row,
//                  column = token), per-row scale, cast, staged as a 32-token x 128-row tile in
//                  shared memory and written to y with a TMA store; the accumulator is released
//                  (accempty) as soon as its last columns are read.
// Every mbarrier wait is bounded (sm100.cuh): on give-up the CTA drains its copies and MMAs,
// frees TMEM and returns, and the library's device error flag is set.
//
// Exactness: every payload value is exactly representable in fp16 and bf16 (<= 4 significant
// bits, small exponent range). Per-row scales (block_size >= K) multiply the fp32 accumulator
// in the epilogue; per-group E8M0 scales are powers of two and multiply the operand exactly
// (barring fp16 overflow). Products are exact in the fp32 accumulator, so results equal the
// reference's fp32 arithmetic up to summation order.
#include <cudaTypedefs.h>
#include <string.h>

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
constexpr int ACC = 1;            // fp32 accumulators (128 lanes x bt columns each)
constexpr int A_COLS = BK / 2;    // one A stage: 64 fp16/bf16 per row = 32 columns
constexpr int TMEM_COLS = 512;    // ACC * BT_MAX + NA * A_COLS <= 512
constexpr int DQ_WARPS = 16;      // dequant warps: (TMEM lane quarter, K quarter) pairs
constexpr int EPI_WARPS = 4;
constexpr int THREADS = (2 + DQ_WARPS + EPI_WARPS) * 32;  // producer, MMA, dequant, epilogue
constexpr int X_BYTES = BT_MAX * BK * 2;                    // 32 KB
constexpr int P_STAGE = 6144;                               // packed bytes slot (128 rows x 48 B max)
constexpr int EPI_CHUNK = 32;                               // tokens per epilogue store
constexpr int STG_BYTES = EPI_CHUNK * BW * 4;               // one staging buffer (fp32 worst case)
constexpr int SMEM_BYTES = 1024 /*align slack*/ + STAGES * (X_BYTES + P_STAGE) + 2 * STG_BYTES + 512 /*barriers*/;
static_assert(ACC * BT_MAX + NA * A_COLS <= TMEM_COLS, "tensor memory budget");
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
  int blk_stages;        // E8M0 group scales: K stages per scale block (0: block_size 32)
  int tma_store;         // y written through shared memory + TMA (else direct stores)
};

// Slot index and phase bit of a circular buffer of N stages, advanced once per use.
template <int N>
struct Ring {
  int idx = 0;
  uint32_t phase = 0;
  bool wrapped = false;  // every slot has been used at least once
  __device__ __forceinline__ void next() {
    if (++idx == N) {
      idx = 0;
      phase ^= 1u;
      wrapped = true;
    }
  }
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
// Same values into the staging tile stg[token j][row r] (row pitch BW elements).
template <typename T>
__device__ __forceinline__ void stage_col32(uint8_t *stg, int r, const uint32_t (&v)[32], float sc) {
  T *dst = (T *)stg + r;
#pragma unroll
  for (int j = 0; j < 32; ++j) dst[j * BW] = from_f32<T>(__uint_as_float(v[j]) * sc);
}

__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, %0;" ::"n"(EPI_WARPS * 32) : "memory"); }

template <int FMT, bool BF16>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw,
                const __grid_constant__ CUtensorMap tmy, Params p) {
  constexpr int BITS = Fmt<FMT>::bits;
  constexpr int PB = BK * BITS / 8;  // packed bytes per row per stage: 32 or 48
  constexpr int QB = PB / 4;         // packed bytes per row per K quarter: 8 or 12
  extern __shared__ uint8_t smem_raw[];
  uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *xs = base;
  uint8_t *ps = xs + STAGES * X_BYTES;
  uint8_t *stg = ps + STAGES * P_STAGE;                    // [2][STG_BYTES] epilogue staging
  uint64_t *full = (uint64_t *)(stg + 2 * STG_BYTES);     // [STAGES] x + packed tile landed
  uint64_t *empty = full + STAGES;                        // [STAGES] stage's MMAs retired
  uint64_t *aready = empty + STAGES;                      // [NA] decoded A stage written to TMEM
  uint64_t *afree = aready + NA;                          // [NA] A stage's MMAs retired
  uint64_t *accfull = afree + NA;                         // [ACC] tile's accumulator complete
  uint64_t *accempty = accfull + ACC;                     // [ACC] accumulator drained by the epilogue
  uint64_t *done = accempty + ACC;                        // all MMAs of this CTA retired (exit path)
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
      mbar_init(&aready[a], DQ_WARPS);
      mbar_init(&afree[a], 1);
    }
    for (int a = 0; a < ACC; ++a) {
      mbar_init(&accfull[a], 1);
      mbar_init(&accempty[a], EPI_WARPS);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmx);
    prefetch_tmap(&tmw);
    if (p.tma_store) prefetch_tmap(&tmy);
  }
  __syncwarp();
  if (warp == 0) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t ta = tmem + ACC * BT_MAX;  // A ring after the accumulators

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const uint32_t tx_bytes = (uint32_t)(p.bt * BK * 2 + BW * PB);  // full boxes (OOB rows zero-filled)
      Ring<STAGES> st;
      int issued = 0;
      for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const int tb = tile % p.tblocks, wb = tile / p.tblocks;
        for (int kb = 0; kb < nk; ++kb, st.next()) {
          if (st.wrapped && !mbar_wait(&empty[st.idx], st.phase ^ 1u, abort_flag)) continue;
          if (*abort_flag) continue;
          mbar_arrive_expect_tx(&full[st.idx], tx_bytes);
          tma_load_2d(xs + st.idx * X_BYTES, &tmx, kb * BK, tb * p.bt, &full[st.idx]);
          tma_load_2d(ps + st.idx * P_STAGE, &tmw, kb * PB, wb * BW, &full[st.idx]);
          ++issued;
        }
      }
      if (*abort_flag) {  // drain the copies still in flight (at most the last STAGES uses) before exit
        for (int i = 0; i < STAGES && i < issued; ++i) {
          int idx = st.idx - 1 - i;
          uint32_t ph = st.phase;
          if (idx < 0) idx += STAGES, ph ^= 1u;
          mbar_wait(&full[idx], ph, abort_flag, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: D[128 x bt] += A[tmem 128 x 16] * x[bt x 16]^T ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(BF16 ? 1u : 0u, BW, (uint32_t)p.bt);
      Ring<STAGES> st;
      Ring<NA> ar;
      int i = 0;
      for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++i) {
        const int ab = i % ACC;
        if (i >= ACC) mbar_wait(&accempty[ab], (uint32_t)((i / ACC - 1) & 1), abort_flag);
        tc_fence_after();
        const uint32_t tacc = tmem + (uint32_t)(ab * BT_MAX);
        for (int kb = 0; kb < nk; ++kb, st.next(), ar.next()) {
          if (!mbar_wait_sleep(&full[st.idx], st.phase, abort_flag) || !mbar_wait_sleep(&aready[ar.idx], ar.phase, abort_flag))
            continue;
          tc_fence_after();
          const uint64_t b0 = sw128_kmajor_desc(xs + st.idx * X_BYTES);
          const uint32_t a0 = ta + (uint32_t)(ar.idx * A_COLS);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)  // A: 8 columns per K=16; B: +32 bytes inside the swizzle atom
            mma_f16_ts(tacc, a0 + (uint32_t)(8 * k), b0 + (uint64_t)(2 * k), idesc, (kb | k) != 0);
          mma_commit(&empty[st.idx]);
          mma_commit(&afree[ar.idx]);
        }
        mma_commit(&accfull[ab]);  // arrives once this tile's MMAs have completed
      }
      mma_commit(done);
      mbar_wait(done, 0, abort_flag, 500000000ull);
    }
  } else if (warp < 2 + DQ_WARPS) {
    // ---------------- dequant: thread = (weight row r = TMEM lane, K quarter kq) ----------------
    const int qd = warp & 3, kq = (warp - 2) >> 2;
    const int r = qd * 32 + lane;
    const uint32_t tdst = ta + ((uint32_t)(qd * 32) << 16) + (uint32_t)(8 * kq);
    const bool scaled = p.scale_mode == SCALE_E8M0;
    const uint8_t *srow = ps + r * PB + kq * QB;
    Ring<STAGES> st;
    Ring<NA> ar;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
      const int64_t n = (int64_t)(tile / p.tblocks) * BW + r;
      const uint8_t *scl = scaled && n < p.N ? (const uint8_t *)p.scales + n * p.nblk : nullptr;
      for (int kb = 0; kb < nk; ++kb, st.next(), ar.next()) {
        bool ok = mbar_wait(&full[st.idx], st.phase, abort_flag);
        if (ok && ar.wrapped) ok = mbar_wait(&afree[ar.idx], ar.phase ^ 1u, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) continue;  // tcgen05.st is warp-collective
        const uint8_t *src = srow + st.idx * P_STAGE;
        uint32_t w[QB / 4];
        if constexpr (BITS == 4) {
          const uint2 u = *reinterpret_cast<const uint2 *>(src);
          w[0] = u.x, w[1] = u.y;
        } else {
#pragma unroll
          for (int j = 0; j < 3; ++j) w[j] = reinterpret_cast<const uint32_t *>(src)[j];
        }
        float gf = 1.f;
        if (scl != nullptr)
          gf = e8m0_to_f32(scl[p.blk_stages == 0 ? 2 * kb + (kq >> 1) : (unsigned)kb / (unsigned)p.blk_stages]);
        uint32_t out[8];
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {  // 8 payloads per unit, pairs (2i, 2i+1) in natural K order
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
        // K elements kb*64 + 16kq + 2c, +1 -> column a*32 + 8kq + c of lane r
        tmem_st_32x32b_x8(tdst + (uint32_t)(ar.idx * A_COLS), out);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&aready[ar.idx]);
      }
    }
  } else {
    // ---------------- epilogue: lane = weight row n, columns = tokens ----------------
    const int qd = warp & 3;
    const int r = qd * 32 + lane;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const bool issuer = warp == 2 + DQ_WARPS && lane == 0;
    int i = 0, chunk = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++i) {
      const int ab = i % ACC;
      const int64_t n0 = (int64_t)(tile / p.tblocks) * BW, n = n0 + r;
      const int64_t m0 = (int64_t)(tile % p.tblocks) * p.bt;
      float sc = 1.f;
      if (p.scale_mode == SCALE_ROW && n < p.N) sc = load_as_f32(p.scales, n * p.nblk, p.sdt);
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
        if (c + EPI_CHUNK >= p.bt) {  // last columns read: tile i + ACC may overwrite this accumulator
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&accempty[ab]);
        }
        const bool live = ok && m0 + c < p.M;
        if (p.tma_store) {
          uint8_t *sb = stg + (chunk & 1) * STG_BYTES;
          if (issuer) bulk_wait_read<1>();  // the store issued from this buffer two chunks ago has read it
          epi_sync();
          if (live) {
            if (p.ydt == B200_DT_F16)
              stage_col32<__half>(sb, r, v, sc);
            else if (p.ydt == B200_DT_BF16)
              stage_col32<__nv_bfloat16>(sb, r, v, sc);
            else
              stage_col32<float>(sb, r, v, sc);
          }
          fence_proxy_async_smem();
          epi_sync();
          if (issuer && live) {
            tma_store_2d(&tmy, sb, (int32_t)n0, (int32_t)(m0 + c));  // rows >= M, columns >= N clipped
            bulk_commit();
          }
        } else if (live && n < p.N) {
          if (p.ydt == B200_DT_F16)
            store_col32<__half>(p, m0 + c, n, v, sc);
          else if (p.ydt == B200_DT_BF16)
            store_col32<__nv_bfloat16>(p, m0 + c, n, v, sc);
          else
            store_col32<float>(p, m0 + c, n, v, sc);
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
  int sms = 0;
  B200_CUDA_TRY(device_sms(&sms));
  B200_CUDA_TRY((ensure_dynamic_smem<gemm_kernel<FMT, BF16>>(SMEM_BYTES)));
  int bt = (int)((a.m + 31) / 32 * 32);
  if (bt > BT_MAX) bt = BT_MAX;
  const int ysz = a.ydt == B200_DT_F32 ? 4 : 2;
  CUtensorMap tmy;
  memset(&tmy, 0, sizeof(tmy));
  const bool tma_store = (uintptr_t)a.y % 16 == 0 && (a.ldy_m * ysz) % 16 == 0 && a.ldy_m >= a.rows;
  if (tma_store) {
    const CUtensorMapDataType ydt = a.ydt == B200_DT_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                    : a.ydt == B200_DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                            : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    if (int32_t rc = make_tma_2d(&tmy, ydt, a.y, (uint64_t)a.rows, (uint64_t)a.m, (uint64_t)a.ldy_m * ysz, BW,
                                 EPI_CHUNK, CU_TENSOR_MAP_SWIZZLE_NONE))
      return rc;
  }
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
  p.tma_store = tma_store ? 1 : 0;
  p.blk_stages = (a.scales != nullptr && a.block < a.cols && a.block != 32) ? (int)(a.block / BK) : 0;
  p.wblocks = (int)((a.rows + BW - 1) / BW);
  p.tblocks = (int)((a.m + bt - 1) / bt);
  const int64_t tiles = (int64_t)p.wblocks * p.tblocks;
  const unsigned grid = (unsigned)(tiles < sms ? tiles : sms);
  gemm_kernel<FMT, BF16><<<grid, THREADS, SMEM_BYTES, stream>>>(tmx, tmw, tmy, p);
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
