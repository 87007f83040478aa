// gemm_sm100.cu -- packed low-bit prefill GEMM on the 5th-generation tensor cores.
//
//   y[m, n] = sum_k x[m, k] * dequant(W)[n, k]        (x fp16/bf16 row-major, W packed (N, K))
//
// The B200 replacement of the reference's LinAlg matrix kernel (tinygrad-dx12
// src/tinygrad_dx12/renderer/linalg.py:38-124) for packed operands, with the decode of
// src/tinygrad_dx12/codegen/decomp/dx12.py:69-106 fused on chip instead of materialised.
//
// Persistent kernel: one CTA per SM walks 128 (m) x 128 (n) output tiles; K advances 64
// elements per stage through a 4-stage shared-memory ring that runs continuously across tiles.
//   warp 0 lane 0  TMA producer: x tile (128 x 64, 128-byte swizzle) and the tile's packed weight
//                  bytes (128 rows x 32/48 bytes), both signalled on full[s];
//   warp 1 lane 0  MMA issuer: 4 x tcgen05.mma.kind::f16 (M=128, N=128, K=16) per stage into one
//                  of two 128-column fp32 TMEM accumulators; tcgen05.commit frees the stage
//                  (empty[s]) and, after the last stage of a tile, publishes the accumulator;
//   warps 2..9     dequant warps (256 threads): each pair of threads decodes one weight row of
//                  the stage (32 payloads each) to exact fp16/bf16 (decode.cuh) and writes it in
//                  the 128-byte swizzled K-major layout the MMA reads (bready[s]);
//   warps 10..13   epilogue warpgroup: tcgen05.ld of the finished accumulator, per-column scale,
//                  cast, store; it frees the accumulator so the next-but-one tile can reuse it,
//                  which overlaps each epilogue with the next tile's main loop.
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

constexpr int BM = 128, BN = 128, BK = 64, STAGES = 4, ACC = 2;
constexpr int DQ_WARPS = 8;           // dequant warps: two threads per weight row
constexpr int THREADS = (2 + DQ_WARPS + 4) * 32;  // producer, MMA, dequant, 4 epilogue warps
constexpr int X_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_BYTES = BN * BK * 2;  // 16 KB
constexpr int P_STAGE = 6144;         // packed bytes slot (128 rows x 48 B max), 1024-aligned
constexpr int SMEM_BYTES = 1024 /*align slack*/ + STAGES * (X_BYTES + B_BYTES + P_STAGE) + 1024 /*bars etc*/ +
                           ACC * BN * 4;
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
  int mblocks, nblocks;  // tile grid
};

template <int FMT, bool BF16>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw, Params p) {
  constexpr int BITS = Fmt<FMT>::bits;
  constexpr int PB = BK * BITS / 8;  // packed bytes per row per stage: 32 or 48
  constexpr uint32_t TX_BYTES = X_BYTES + BN * PB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *xs = base;
  uint8_t *bsm = xs + STAGES * X_BYTES;
  uint8_t *ps = bsm + STAGES * B_BYTES;
  uint64_t *full = (uint64_t *)(ps + STAGES * P_STAGE);
  uint64_t *bready = full + STAGES;
  uint64_t *empty = bready + STAGES;
  uint64_t *accf = empty + STAGES;  // [ACC] accumulator ready for the epilogue
  uint64_t *acce = accf + ACC;      // [ACC] accumulator drained by the epilogue
  uint64_t *done = acce + ACC;      // all MMAs of this CTA retired (exit path)
  uint32_t *tmem_slot = (uint32_t *)(done + 1);
  volatile uint32_t *abort_flag = tmem_slot + 1;
  float *colscale = (float *)(tmem_slot + 4);  // [ACC][BN]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = (int)(p.K / BK);
  const int ntiles = p.mblocks * p.nblocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&bready[s], DQ_WARPS * 32);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < ACC; ++a) {
      mbar_init(&accf[a], 1);
      mbar_init(&acce[a], 128);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmx);
    prefetch_tmap(&tmw);
  }
  __syncwarp();
  if (warp == 0) tmem_alloc(tmem_slot, ACC * BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int64_t q = 0, issued = 0;
      for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const int mb = tile % p.mblocks, nb = tile / p.mblocks;
        for (int kb = 0; kb < nk; ++kb, ++q) {
          const int s = (int)(q % STAGES);
          if (q >= STAGES && !mbar_wait(&empty[s], (uint32_t)((q / STAGES - 1) & 1), abort_flag)) continue;
          if (*abort_flag) continue;
          mbar_arrive_expect_tx(&full[s], TX_BYTES);
          tma_load_2d(xs + s * X_BYTES, &tmx, kb * BK, mb * BM, &full[s]);
          tma_load_2d(ps + s * P_STAGE, &tmw, kb * PB, nb * BN, &full[s]);
          issued = q + 1;
        }
      }
      if (*abort_flag) {  // drain this CTA's copies still in flight before it exits
        for (int64_t r = (issued > STAGES ? issued - STAGES : 0); r < issued; ++r)
          mbar_wait(&full[r % STAGES], (uint32_t)((r / STAGES) & 1), abort_flag, 200000000ull);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(BF16 ? 1u : 0u, BM, BN);
      int64_t q = 0;
      int i = 0;
      for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++i) {
        const int a = i & 1;
        if (i >= ACC) mbar_wait(&acce[a], (uint32_t)((i / ACC - 1) & 1), abort_flag);
        tc_fence_after();
        const uint32_t dacc = tmem + (uint32_t)(a * BN);
        for (int kb = 0; kb < nk; ++kb, ++q) {
          const int s = (int)(q % STAGES);
          const uint32_t ph = (uint32_t)((q / STAGES) & 1);
          if (!mbar_wait(&full[s], ph, abort_flag) || !mbar_wait(&bready[s], ph, abort_flag)) continue;
          tc_fence_after();
          const uint64_t a0 = sw128_kmajor_desc(xs + s * X_BYTES);
          const uint64_t b0 = sw128_kmajor_desc(bsm + s * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)  // +32 bytes per K=16 step inside the swizzle atom
            mma_f16_ss(dacc, a0 + (uint64_t)(2 * k), b0 + (uint64_t)(2 * k), idesc, (kb | k) != 0);
          mma_commit(&empty[s]);
        }
        mma_commit(&accf[a]);  // arrives once this tile's MMAs have completed
      }
      mma_commit(done);
      mbar_wait(done, 0, abort_flag, 500000000ull);
    }
  } else if (warp < 2 + DQ_WARPS) {
    // ---------------- dequant warps: thread = (row t, half h) of the stage ----------------
    const int dt = threadIdx.x - 64;
    const int t = dt & (BN - 1), h = dt / BN;  // weight row within the tile, 32-payload half
    const bool scaled = p.scale_mode == SCALE_E8M0;
    int64_t q = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
      const int64_t n = (int64_t)(tile / p.mblocks) * BN + t;
      for (int kb = 0; kb < nk; ++kb, ++q) {
        const int s = (int)(q % STAGES);
        if (!mbar_wait(&full[s], (uint32_t)((q / STAGES) & 1), abort_flag)) continue;
        const uint8_t *src = ps + s * P_STAGE + t * PB + h * (PB / 2);
        uint32_t w[PB / 8];
        if constexpr (BITS == 4) {
          const uint4 u = *reinterpret_cast<const uint4 *>(src);
          w[0] = u.x, w[1] = u.y, w[2] = u.z, w[3] = u.w;
        } else {
#pragma unroll
          for (int i = 0; i < 3; ++i) {
            const uint2 u = *reinterpret_cast<const uint2 *>(src + 8 * i);
            w[2 * i] = u.x, w[2 * i + 1] = u.y;
          }
        }
        float gf = 1.f;
        if (scaled && n < p.N)
          gf = e8m0_to_f32(((const uint8_t *)p.scales)[n * p.nblk + (kb * BK + 32 * h) / p.block]);
        uint8_t *dst = bsm + s * B_BYTES + (t >> 3) * 1024 + (t & 7) * 128;
#pragma unroll
        for (int cc = 0; cc < BK / 16; ++cc) {  // 16-byte chunk = 8 payloads, natural K order
          const int c = h * (BK / 16) + cc;
          uint32_t out[4];
          gemv::decode8_natural<FMT, BF16>(w, cc, out);
          if (scaled) {  // power-of-two block scale: exact while the product stays in range
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              if constexpr (BF16) {
                const __nv_bfloat162 r =
                    __hmul2(*reinterpret_cast<const __nv_bfloat162 *>(&out[j]), __float2bfloat162_rn(gf));
                out[j] = *reinterpret_cast<const uint32_t *>(&r);
              } else {
                const __half2 r = __hmul2(*reinterpret_cast<const __half2 *>(&out[j]), __float2half2_rn(gf));
                out[j] = *reinterpret_cast<const uint32_t *>(&r);
              }
            }
          }
          *reinterpret_cast<uint4 *>(dst + ((c ^ (t & 7)) << 4)) = make_uint4(out[0], out[1], out[2], out[3]);
        }
        fence_proxy_async_smem();
        mbar_arrive(&bready[s]);
      }
    }
  } else {
    // ---------------- epilogue warpgroup ----------------
    const int et = threadIdx.x - (2 + DQ_WARPS) * 32;  // 0..127
    const int qd = warp & 3;           // TMEM lane quarter this warp may access
    const int row = qd * 32 + lane;
    const int esz = p.ydt == B200_DT_F32 ? 4 : 2;
    const bool vec_ok = ((uintptr_t)p.y % 16 == 0) && ((p.ldy * esz) % 16 == 0);
    int i = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++i) {
      const int a = i & 1;
      const int64_t m0 = (int64_t)(tile % p.mblocks) * BM, n0 = (int64_t)(tile / p.mblocks) * BN;
      {
        const int64_t n = n0 + et;
        float s = 1.f;
        if (p.scale_mode == SCALE_ROW && n < p.N) s = load_as_f32(p.scales, n * p.nblk, p.sdt);
        colscale[a * BN + et] = s;
      }
      asm volatile("bar.sync 2, 128;" ::: "memory");
      const bool ok = mbar_wait(&accf[a], (uint32_t)((i / ACC) & 1), abort_flag) && !*abort_flag;
      tc_fence_after();
      const int64_t m = m0 + row;
      const float *cs = colscale + a * BN;
      for (int c = 0; c < BN; c += 16) {
        uint32_t r[16];
        if (ok) {
          tmem_ld_32x32b_x16(tmem + ((uint32_t)(qd * 32) << 16) + (uint32_t)(a * BN + c), r);
          tmem_ld_wait();
        }
        if (ok && m < p.M) {
          float v[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]) * cs[c + j];
          const int64_t off = m * p.ldy + n0 + c;
          if (vec_ok && n0 + c + 16 <= p.N) {
            if (p.ydt == B200_DT_F32) {
              float4 *d = reinterpret_cast<float4 *>((float *)p.y + off);
#pragma unroll
              for (int j = 0; j < 4; ++j) d[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            } else {
              uint32_t h[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                if (p.ydt == B200_DT_BF16) {
                  __nv_bfloat162 b = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
                  h[j] = *reinterpret_cast<uint32_t *>(&b);
                } else {
                  __half2 b = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
                  h[j] = *reinterpret_cast<uint32_t *>(&b);
                }
              }
              uint4 *d = reinterpret_cast<uint4 *>((uint16_t *)p.y + off);
              d[0] = make_uint4(h[0], h[1], h[2], h[3]);
              d[1] = make_uint4(h[4], h[5], h[6], h[7]);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (n0 + c + j < p.N) store_f32(p.y, off + j, p.ydt, v[j]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acce[a]);  // the accumulator may be overwritten by tile i + ACC
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, ACC * BN);
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
  CUtensorMap tmx, tmw;
  if (int32_t rc = make_tma_2d(&tmx, BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.x,
                               (uint64_t)a.cols, (uint64_t)a.m, (uint64_t)a.ldx * 2, BK, BM,
                               CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  const uint64_t row_bytes = (uint64_t)a.cols * BITS / 8;
  if (int32_t rc = make_tma_2d(&tmw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w, row_bytes, (uint64_t)a.rows, row_bytes,
                               BK * BITS / 8, BN, CU_TENSOR_MAP_SWIZZLE_NONE))
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
  p.mblocks = (int)((a.m + BM - 1) / BM);
  p.nblocks = (int)((a.rows + BN - 1) / BN);
  const int64_t tiles = (int64_t)p.mblocks * p.nblocks;
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
  if ((a.m + BM - 1) / BM * ((a.rows + BN - 1) / BN) > (int64_t)INT32_MAX) return false;
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
