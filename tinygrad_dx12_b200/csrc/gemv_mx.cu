// gemv_mx.cu -- block-scaled tcgen05 decode kernel for FP4 / FP6 weights and 1..64 tokens.
//
//   y[m, n] = sum_k x[m, k] * dequant(W)[n, k]
//
// The decode half of the reference's packed matmul (tinygrad-dx12
// src/tinygrad_dx12/codegen/linalg.py:136-245 over the decode of codegen/decomp/dx12.py:69-106)
// with no decode instructions at all: the tensor cores read the packed FP4 E2M1 / FP6 E2M3 /
// FP6 E3M2 codes as the A operand of tcgen05.mma kind::mxf8f6f4 and apply the per-32 E8M0 weight
// scales themselves (scale-factor A in tensor memory). Every FP4/FP6 code is an exact value of
// its OCP format, and 2^(e-127) is exactly the reference's decoded scale (dx12.py:102-106), so
// the MMA multiplies exactly the reference's dequantised weight.
//
// Activations keep their precision: x (bf16 or fp16) is split per 32-element block into E4M3
// pieces with one E8M0 block scale 2^E (E chosen so the block maximum lands in [128, 256)):
//   x / 2^E = p1 + p2 (+ p3),  p1 = rn_e4m3(x / 2^E),  p2 = rn_e4m3(x / 2^E - p1), ...
// A bf16 value has 8 significant bits and two 4-bit pieces hold it exactly (three for fp16's
// 11) unless it is 2^17 below its block maximum, where the last piece leaves the E4M3 range:
// the representation error is below 2^-17 of the block maximum. The pieces are extra B rows
// (token m, piece p -> MMA column m * P + p) and the epilogue adds them in fp32, so one MMA
// with N = 8 * ceil(m * P / 8) columns carries all pieces of all tokens.
//
// Work split (stream-K): units = (128-row weight tile, 256-deep K stage); CTA c of the
// persistent grid (one per SM) takes units [c * U / G, (c + 1) * U / G), so every SM streams
// the same number of bytes whatever the matrix shape. A tile split across CTAs is finished by
// the last contributor (acquire-release ticket), which adds the fp32 partials of its tile in
// CTA order (deterministic) and stores y.
//
// Roles (672 threads): warps 0-3 issue the TMA loads of a shared-memory ring (per stage the
// weight codes -- one 128-byte box of packed FP4 for kind::mxf4, else two boxes through the
// 16U4/16U6 "align 16B" tensor-map types, which lay each 16-code group into the 16-byte slot the
// MMA reads -- and the stage's E8M0 weight scales); a thread's TMA issues are serialised at
// several hundred cycles per box, so up to four threads issue alternate stages. Warps 17-20
// split the stage's x into pieces straight into the ring's B tiles and their scale bytes. Warps
// 8-15 (two sets of four, one tensor-memory lane quarter per warp; a set owns the ring slots of
// one parity) write both scale-factor operands into tensor memory with tcgen05.st (row r ->
// lane r % 32 in every quarter, column r / 32, byte = K block). Warp 16 lane 0 issues the MMAs
// into one of two fp32 accumulators; warps 4-7 read the accumulators (tcgen05.ld) and finish
// the rows.
// Every wait is bounded (sm100.cuh); on give-up the kernel flags the device error word.
#include <map>
#include <mutex>

#include "mx.cuh"

namespace b200 {

int32_t mx_device_error(unsigned int *v, bool clear) {
  B200_CUDA_TRY(tu_device_error(v, clear));
  return B200_OK;
}

namespace mx {

// warps: 0-3 TMA producers, 4-7 epilogue, 8-15 scale-factor writers (two sets of four that take
// alternate stages; in each, warp w writes tensor-memory lane quarter w % 4), 16 MMA issuer,
// 17-20 x converters
constexpr int PROD_WARPS = 4, EPI_WARP0 = 4, SF_WARP0 = 8, MMA_WARP = 16, CONV_WARP0 = 17, CONV_WARPS = 4;
constexpr int THREADS = 21 * 32;
constexpr int MAX_STAGES = 8;
constexpr int MAX_COLS = 128;     // m * pieces per call
// tensor memory: two accumulators (columns [0, d1) and [d1, 2 d1)), then one scale-factor set of
// 16 columns per ring slot (A box 0, A box 1, B box 0, B box 1: 4 columns each); the allocation
// is the power of two that holds them, so small calls leave room for the next call's CTA on the SM

struct Params {
  int64_t rows, cols;
  int nst, ntiles;       // K stages per tile, 128-row tiles
  int64_t units;         // ntiles * nst
  int grid;              // CTAs
  int m, P, N;           // tokens, pieces per token, MMA N
  int stages;            // ring depth
  int nact;              // producers and converters in use: min(4, stages). An actor that owns
                         // the stages i = a (mod nact) never gets more than one ring round ahead
                         // of the consumers, so a slot's barrier phase parity is never ambiguous
  // per stage: codes [2][128 rows][128 B] at 0, x pieces [2][N rows][128 B] at b_off, raw
  // weight scales [128 rows][16 B] at sraw_off, x-piece scales [128 rows][8 K blocks] at xsf_off
  uint32_t stage_bytes, b_off, sraw_off, xsf_off;
  uint32_t tx;           // TMA transaction bytes per stage
  uint32_t d1_col, sf_col, tmem_cols;  // tensor-memory layout
  uint32_t idesc;        // instruction descriptor without scale-factor ids
  const uint16_t *x;     // activations (bf16 or fp16), row stride ldx
  int64_t ldx;
  const void *rscale;    // per-row weight scales (SM_ROW)
  int sdt;
  void *y;
  int ydt;
  int64_t ldy_m;
  void *ycopy[7];
  int ncopy;
  float *part;           // [grid][2][m][128] fp32 partials of split tiles
  unsigned int *tickets; // [ntiles]
};

// P = 8: kind::mxf4 (FP4 weights, x in eight FP4 pieces, 256 packed codes per 128-byte row);
// P = 2 or 3: kind::mxf8f6f4 (FP4 / FP6 weights, x in E4M3 pieces, two 128-code boxes per stage).
template <int FMT, int SMODE, int P, bool XBF16>
__global__ void __launch_bounds__(THREADS, 1)
    mx_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tms, const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *ring = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int S = p.stages;
  uint64_t *full = reinterpret_cast<uint64_t *>(ring + (size_t)S * p.stage_bytes);
  uint64_t *sfready = full + S;
  uint64_t *bready = sfready + S;
  uint64_t *empty = bready + S;
  uint64_t *accfull = empty + S;
  uint64_t *accempty = accfull + 2;
  uint64_t *drain = accempty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile uint32_t *abort_flag = tmem_slot + 1;
  volatile uint32_t *last_flag = tmem_slot + 2;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t u0 = unit_start(p, blockIdx.x), u1 = unit_start(p, blockIdx.x + 1);
  const int64_t n = u1 - u0;
  constexpr bool MXF4 = P == 8;
  constexpr int NBOX = MXF4 ? 1 : 2;          // boxes of codes (and of x pieces) per stage
  const uint32_t bbox = (uint32_t)p.N * 128;  // bytes of one box of x pieces

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&sfready[s], 4);
      mbar_init(&bready[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accfull[b], 1);
      mbar_init(&accempty[b], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  // x-piece rows past m * P stay zero, their scale bytes 2^0: written once here for every slot
  for (int s = 0; s < S; ++s) {
    uint8_t *st = ring + (size_t)s * p.stage_bytes;
    for (uint32_t o = threadIdx.x * 16; o < NBOX * bbox; o += THREADS * 16)
      *reinterpret_cast<uint4 *>(st + p.b_off + o) = make_uint4(0u, 0u, 0u, 0u);
    for (uint32_t o = threadIdx.x * 16; o < TM * 8; o += THREADS * 16)
      *reinterpret_cast<uint4 *>(st + p.xsf_off + o) = make_uint4(0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu);
  }
  fence_proxy_async_smem();
  if (warp == MMA_WARP) tmem_alloc(tmem_slot, p.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp < PROD_WARPS) {
    // ---------------- TMA producers: weight codes and scales (no dependency on x) ----------------
    // A thread's TMA issues are serialised (about one box per several hundred cycles), so four
    // warps issue the stages i = warp (mod 4), each stage's boxes from one thread.
    if (lane == 0) {
      prefetch_tmap(&tmw);
      if constexpr (SMODE == SM_E8M0) prefetch_tmap(&tms);
      int64_t i = warp;
      for (; i < n && warp < p.nact; i += p.nact) {
        const int slot = (int)(i % S);
        const uint32_t round = (uint32_t)(i / S);
        if (i >= S && !mbar_wait(&empty[slot], (round - 1u) & 1u, abort_flag)) break;
        const int64_t u = u0 + i;
        const int t = (int)(u / p.nst), s = (int)(u % p.nst);
        uint8_t *st = ring + (size_t)slot * p.stage_bytes;
        mbar_arrive_expect_tx(&full[slot], p.tx);
        if constexpr (MXF4) {  // 256 packed codes = 128 bytes per row
          tma_load_2d(st, &tmw, s * (KS / 2), t * TM, &full[slot]);
        } else {
          tma_load_2d(st, &tmw, s * KS, t * TM, &full[slot]);
          tma_load_2d(st + TM * KB, &tmw, s * KS + KB, t * TM, &full[slot]);
        }
        if constexpr (SMODE == SM_E8M0) tma_load_2d(st + p.sraw_off, &tms, (s * 8) & ~15, t * TM, &full[slot]);
      }
      if (*abort_flag) {  // let this thread's copies in flight land before the CTA exits
        for (int64_t q = warp; q < (i < n ? i : n); q += p.nact)
          if (q + S >= i) mbar_wait(&full[q % S], (uint32_t)((q / S) & 1), abort_flag, 200000000ull);
      }
    }
  } else if (warp >= CONV_WARP0 && warp < CONV_WARP0 + CONV_WARPS) {
    // ---------------- x -> pieces, straight into the stage's B tiles ----------------
    // converter warp cw takes the stages i = cw (mod 4) for every token
    const int cw = warp - CONV_WARP0;
    asm volatile("griddepcontrol.wait;" ::: "memory");  // x is the previous kernel's output
    for (int64_t i = cw; i < n && cw < p.nact; i += p.nact) {
      const int slot = (int)(i % S);
      const uint32_t round = (uint32_t)(i / S);
      if (i >= S && !mbar_wait(&empty[slot], (round - 1u) & 1u, abort_flag)) break;
      const int s = (int)((u0 + i) % p.nst);
      const uint16_t *xs = p.x + (int64_t)s * KS + 8 * lane;
      uint8_t *stg = ring + (size_t)slot * p.stage_bytes;
      if constexpr (MXF4) {
        // lane l: elements 8l..8l+7 = bytes 4l..4l+3 of each piece row, K block l / 4
        uint8_t *xsf = stg + p.xsf_off + (lane >> 2);
        const uint32_t chunk = (uint32_t)lane >> 2, off = (uint32_t)(lane & 3) * 4;
        for (int mm = 0; mm < p.m; ++mm) {
          float v[8];
          load8<XBF16>(xs + (int64_t)mm * p.ldx, v);
          uint32_t pc[P];
          const uint32_t byte0 = split_fp4<P>(v, pc);
#pragma unroll
          for (int c = 0; c < P; ++c) {
            const uint32_t j = (uint32_t)(mm * P + c);
            *reinterpret_cast<uint32_t *>(stg + p.b_off + j * 128 + ((chunk ^ (j & 7)) << 4) + off) = pc[c];
            if ((lane & 3) == 0) xsf[j * 8] = (uint8_t)(byte0 == 255u ? (c == 0 ? 255u : 127u) : byte0 - 2u * c);
          }
        }
      } else {
        // lane l: elements 8l..8l+7 of the stage's 256 (box l / 16, K block l / 4), four tokens'
        // loads in flight at once
        const int box = lane >> 4, kb = (lane >> 2) & 3;
        const uint32_t chunk = (uint32_t)(lane & 15) >> 1, half = (uint32_t)(lane & 1) * 8;
        uint8_t *bt = stg + p.b_off + box * bbox;
        uint8_t *xsf = stg + p.xsf_off + box * 4 + kb;
        for (int m0 = 0; m0 < p.m; m0 += 4) {
          float v[4][8];
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (m0 + q < p.m) load8<XBF16>(xs + (int64_t)(m0 + q) * p.ldx, v[q]);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if (m0 + q >= p.m) break;
            uint2 pc[P];
            const uint32_t byte = split_pieces<P>(v[q], pc);
#pragma unroll
            for (int c = 0; c < P; ++c) {
              const uint32_t j = (uint32_t)((m0 + q) * P + c);  // B row (MMA column) of this token's piece c
              *reinterpret_cast<uint2 *>(bt + j * 128 + ((chunk ^ (j & 7)) << 4) + half) = pc[c];
              if ((lane & 3) == 0) xsf[j * 8] = (uint8_t)byte;
            }
          }
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bready[slot]);
    }
  } else if (warp == MMA_WARP) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t d_col[2] = {0u, p.d1_col};
      int slot = 0;
      uint32_t round = 0;
      int seg = -1;
      bool ok = true;
      for (int64_t i = 0; i < n && ok; ++i) {
        const int64_t u = u0 + i;
        const int s = (int)(u % p.nst);
        const bool seg_start = i == 0 || s == 0;
        const bool seg_end = i == n - 1 || s == p.nst - 1;
        if (seg_start) {
          ++seg;
          if (seg >= 2 && !mbar_wait(&accempty[seg & 1], (uint32_t)((seg / 2 - 1) & 1), abort_flag)) break;
        }
        ok = mbar_wait(&sfready[slot], round & 1u, abort_flag);  // implies the codes, pieces and scales
        if (!ok) break;
        tc_fence_after();
        const uint8_t *st = ring + (size_t)slot * p.stage_bytes;
        const uint32_t dcol = tmem + d_col[seg & 1];
        const uint32_t sf = tmem + p.sf_col + 16u * (uint32_t)slot;
        if constexpr (MXF4) {
          const uint64_t ad = sw128_kmajor_desc(st), bd = sw128_kmajor_desc(st + p.b_off);
#pragma unroll
          for (int j = 0; j < 4; ++j) {  // K = 64 per MMA (32 bytes along the rows); K blocks 2j, 2j+1
            const uint32_t h = (uint32_t)(j & 1) * 2, col = 4u * (uint32_t)(j >> 1);
            mma_mxf4(dcol, ad + (uint64_t)(2 * j), bd + (uint64_t)(2 * j), p.idesc | (h << 4) | (h << 29),
                     (seg_start && j == 0) ? 0u : 1u, (sf + col) | (h << 30), (sf + 8u + col) | (h << 30));
          }
        } else {
#pragma unroll
          for (int b = 0; b < 2; ++b) {
            const uint64_t ad = sw128_kmajor_desc(st + TM * KB * b), bd = sw128_kmajor_desc(st + p.b_off + bbox * b);
#pragma unroll
            for (int j = 0; j < 4; ++j) {  // K = 32 per MMA: 32 bytes further along the 128-byte rows
              const uint32_t id = p.idesc | ((uint32_t)j << 4) | ((uint32_t)j << 29);
              mma_mx(dcol, ad + (uint64_t)(2 * j), bd + (uint64_t)(2 * j), id, (seg_start && b == 0 && j == 0) ? 0u : 1u,
                     (sf + 4u * b) | ((uint32_t)j << 30), (sf + 8u + 4u * b) | ((uint32_t)j << 30));
            }
          }
        }
        mma_commit(&empty[slot]);
        if (seg_end) mma_commit(&accfull[seg & 1]);
        if (++slot == S) slot = 0, ++round;
      }
      // every MMA issued has completed before the CTA frees its tensor memory
      mma_commit(drain);
      mbar_wait(drain, 0, abort_flag, 200000000ull);
    }
  } else if (warp >= SF_WARP0 && warp < SF_WARP0 + 8) {
    // ---------------- scale factors -> tensor memory (one lane quarter per warp) ----------------
    // Row r of a 128-row operand has its E8M0 scale of K block b at lane r % 32 (in every lane
    // quarter), column 4 * box + r / 32 of the slot's set, byte b: thread i0 of each of these
    // warps writes the words of rows i0, i0 + 32, i0 + 64, i0 + 96 into its own quarter.
    // The set of a stage is its ring slot's parity: a set that owns a slot has waited on the
    // slot's previous phase itself, so its next wait on that slot is never a phase ahead of it
    // (stages split by index parity would not be, with an odd ring depth).
    const uint32_t quarter = (uint32_t)(warp & 3);
    const int set = (warp - SF_WARP0) >> 2;
    int slot = 0;
    uint32_t round = 0;
    for (int64_t i = 0; i < n; ++i, (++slot == S ? (slot = 0, ++round) : 0u)) {
      if ((slot & 1) != set) continue;
      bool ok = mbar_wait(&bready[slot], round & 1u, abort_flag);
      if (SMODE == SM_E8M0) ok = ok && mbar_wait(&full[slot], round & 1u, abort_flag);
      if (!ok) break;
      const int s = (int)((u0 + i) % p.nst);
      const uint8_t *st = ring + (size_t)slot * p.stage_bytes;
      uint32_t w[16];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int r = lane + 32 * q;
        uint2 a = make_uint2(0x7F7F7F7Fu, 0x7F7F7F7Fu);
        if constexpr (SMODE == SM_E8M0) a = *reinterpret_cast<const uint2 *>(st + p.sraw_off + r * 16 + ((s * 8) & 15));
        const uint2 bx = *reinterpret_cast<const uint2 *>(st + p.xsf_off + r * 8);
        w[q] = a.x, w[4 + q] = a.y, w[8 + q] = bx.x, w[12 + q] = bx.y;
      }
      tmem_st_32x32b_x16(tmem + ((32u * quarter) << 16) + p.sf_col + 16u * (uint32_t)slot, w);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sfready[slot]);
    }
  } else if (warp >= EPI_WARP0 && warp < EPI_WARP0 + 4) {
    // ---------------- epilogue: rows of the tile, one per thread ----------------
    const int r = (warp - EPI_WARP0) * 32 + lane;  // row within the tile = tensor-memory lane
    const uint32_t lane_base = (uint32_t)((warp - EPI_WARP0) * 32) << 16;
    const uint32_t d_col[2] = {0u, p.d1_col};
    constexpr int TOK = P == 8 ? 1 : 8;  // tokens per accumulator read: TOK * P / 8 loads of 8 columns
    bool waited = false;
    int seg = 0;
    for (int64_t i = 0; i < n;) {
      const int64_t u = u0 + i;
      const int t = (int)(u / p.nst), s0 = (int)(u % p.nst);
      const int64_t len = (p.nst - s0) < (n - i) ? (p.nst - s0) : (n - i);
      const bool whole = s0 == 0 && len == p.nst;
      i += len;
      const int buf = seg & 1;
      if (!mbar_wait(&accfull[buf], (uint32_t)((seg / 2) & 1), abort_flag)) break;  // no sleep: the tail is latency
      tc_fence_after();
      if (!waited) {  // y, the partials and the tickets belong to the stream order
        asm volatile("griddepcontrol.wait;" ::: "memory");
        waited = true;
      }
      const int64_t row = (int64_t)t * TM + r;
      float rs = 1.f;
      if constexpr (SMODE == SM_ROW)
        if (row < p.rows) rs = load_as_f32(p.rscale, row, p.sdt);
      const int e = (u0 / p.nst == t) ? 0 : 1;  // this CTA's first or last tile
      float *mypart = p.part + ((size_t)blockIdx.x * 2 + e) * p.m * TM;
      // TOK tokens at a time: P * TOK accumulator columns
      for (int m0 = 0; m0 < p.m; m0 += TOK) {
        float acc[TOK];
#pragma unroll
        for (int q = 0; q < TOK; ++q) acc[q] = 0.f;
#pragma unroll
        for (int c = 0; c < P * TOK / 8; ++c) {
          float v[8];
          tmem_ld_x8(tmem + lane_base + d_col[buf] + (uint32_t)(m0 * P + 8 * c), v);
#pragma unroll
          for (int q = 0; q < 8; ++q) acc[(8 * c + q) / P] += v[q];  // column m0*P + 8c + q: token (8c+q)/P
        }
#pragma unroll
        for (int q = 0; q < TOK; ++q) {
          const int mm = m0 + q;
          if (mm >= p.m) break;
          if (whole) {
            if (row < p.rows) {
              const float yv = acc[q] * rs;
              store_f32(p.y, mm * p.ldy_m + row, p.ydt, yv);
              for (int cp = 0; cp < p.ncopy; ++cp) store_f32(p.ycopy[cp], mm * p.ldy_m + row, p.ydt, yv);
            }
          } else {
            mypart[(size_t)mm * TM + r] = acc[q];
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty[buf]);
      ++seg;
      if (!whole) {
        // the last contributor of the tile adds every contributor's partial in CTA order
        // (the barrier orders every epilogue thread's partial stores before thread 0's fence, which
        // is cumulative: one gpu-scope fence and an acq_rel ticket publish them all, and the
        // barrier after the ticket orders the winner's loads after its acquire)
        const int cf = owner(p, (int64_t)t * p.nst), cl = owner(p, (int64_t)t * p.nst + p.nst - 1);
        epi_sync();
        if (threadIdx.x == EPI_WARP0 * 32) {
          __threadfence();
          unsigned int old;
          asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], 1;" : "=r"(old) : "l"(&p.tickets[t]) : "memory");
          *last_flag = old == (unsigned int)(cl - cf) ? 1u : 0u;
        }
        epi_sync();
        if (*last_flag) {
          if (row < p.rows) {
            for (int m0 = 0; m0 < p.m; m0 += 8) {  // 8 tokens at a time: all their loads in flight together
              float sum[8];
#pragma unroll
              for (int q = 0; q < 8; ++q) sum[q] = 0.f;
              for (int cc = cf; cc <= cl; ++cc) {
                const int ee = (unit_start(p, cc) / p.nst == t) ? 0 : 1;
                const float *src = p.part + ((size_t)cc * 2 + ee) * p.m * TM + r;
                float v[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) v[q] = m0 + q < p.m ? __ldcg(src + (size_t)(m0 + q) * TM) : 0.f;
#pragma unroll
                for (int q = 0; q < 8; ++q) sum[q] += v[q];
              }
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                const int mm = m0 + q;
                if (mm >= p.m) break;
                const float yv = sum[q] * rs;
                store_f32(p.y, mm * p.ldy_m + row, p.ydt, yv);
                for (int cp = 0; cp < p.ncopy; ++cp) store_f32(p.ycopy[cp], mm * p.ldy_m + row, p.ydt, yv);
              }
            }
          }
          if (threadIdx.x == EPI_WARP0 * 32) p.tickets[t] = 0u;  // ready for the next call
        }
        epi_sync();
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == MMA_WARP) tmem_dealloc(tmem, p.tmem_cols);
}

// ---- per-(device, stream) workspace: fp32 partials of shared tiles and their tickets ----------

static std::mutex g_ws_mutex;
static std::map<std::pair<int, cudaStream_t>, Workspace> g_ws;

int32_t workspace_for(cudaStream_t stream, bool may_allocate, Workspace *&out) {
  int dev = 0;
  B200_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(g_ws_mutex);
  auto it = g_ws.find({dev, stream});
  if (it != g_ws.end()) {
    out = &it->second;
    return B200_OK;
  }
  out = nullptr;
  if (!may_allocate) return B200_OK;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  B200_CUDA_TRY(cudaStreamIsCapturing(stream, &cs));
  if (cs != cudaStreamCaptureStatusNone) return B200_OK;  // no allocation while capturing
  int sms = 0;
  B200_CUDA_TRY(device_sms(&sms));
  Workspace w;
  w.part_bytes = (size_t)sms * 2 * 64 * TM * sizeof(float);
  w.tickets_n = TICKETS;
  B200_CUDA_TRY(cudaMalloc((void **)&w.part, w.part_bytes));
  B200_CUDA_TRY(cudaMalloc((void **)&w.tickets, w.tickets_n * sizeof(unsigned int)));
  B200_CUDA_TRY(cudaMemset(w.tickets, 0, w.tickets_n * sizeof(unsigned int)));
  B200_CUDA_TRY(cudaDeviceSynchronize());
  out = &(g_ws[{dev, stream}] = w);
  return B200_OK;
}

static int pieces_of(int xdt) { return xdt == B200_DT_BF16 ? 2 : 3; }


static size_t smem_for(const Params &p) { return 1024 + (size_t)p.stages * p.stage_bytes + 8 * (4 * p.stages + 5) + 16; }

template <int FMT, int SMODE, int P, bool XBF16>
static int32_t launch_t(const LinearArgs &a, const Workspace &w, cudaStream_t stream) {
  constexpr int BITS = Fmt<FMT>::bits;
  constexpr bool MXF4 = P == 8;
  int sms = 0;
  B200_CUDA_TRY(device_sms(&sms));
  Params p;
  memset(&p, 0, sizeof(p));
  p.rows = a.rows;
  p.cols = a.cols;
  p.nst = (int)(a.cols / KS);
  p.ntiles = (int)((a.rows + TM - 1) / TM);
  p.units = (int64_t)p.ntiles * p.nst;
  p.grid = (int)(p.units < sms ? p.units : sms);
  p.m = (int)a.m;
  p.P = P;
  p.N = (p.m * P + 7) / 8 * 8;
  const uint32_t bbox = (uint32_t)p.N * 128;
  const uint32_t nbox = MXF4 ? 1 : 2;
  p.b_off = nbox * TM * KB;  // 16 KB of packed FP4 codes, or 32 KB of codes in 16-byte slots
  p.sraw_off = p.b_off + (nbox * bbox + 1023) / 1024 * 1024;
  p.xsf_off = p.sraw_off + TM * 16;
  p.stage_bytes = (p.xsf_off + TM * 8 + 1023) / 1024 * 1024;
  // Up to ~100 KB of shared memory when five stages fit there, so that the next call's CTA can
  // take the other half of the SM and stream its weights while this one finishes (programmatic
  // dependent launch); otherwise one CTA per SM with a deeper ring.
  int stages = (int)((100 * 1024 - 2048) / p.stage_bytes);
  if (stages < 5) stages = (int)((200 * 1024 - 2048) / p.stage_bytes);
  if (stages > MAX_STAGES) stages = MAX_STAGES;
  if (stages < 2) return b200_set_error(B200_ERR_UNSUPPORTED, "mx decode: %d tokens do not fit the ring", p.m);
  p.stages = stages;
  p.nact = stages < PROD_WARPS ? stages : PROD_WARPS;
  {
    const int tok = P == 8 ? 1 : 8;
    const uint32_t read_cols = (uint32_t)((p.m + tok - 1) / tok * tok * P);  // columns the epilogue reads
    const uint32_t width = ((read_cols > (uint32_t)p.N ? read_cols : (uint32_t)p.N) + 15) / 16 * 16;
    p.d1_col = width;
    p.sf_col = 2 * width;
    const uint32_t need = p.sf_col + 16u * (uint32_t)stages;
    p.tmem_cols = 32;
    while (p.tmem_cols < need) p.tmem_cols *= 2;
    if (p.tmem_cols > 512) return b200_set_error(B200_ERR_UNSUPPORTED, "mx decode: %d tokens exceed tensor memory", p.m);
  }
  // transaction bytes: the stage's packed codes as stored in global memory (128 rows x 256 codes,
  // one box or two) and the scale box
  p.tx = (uint32_t)(TM * KS * BITS / 8) + (SMODE == SM_E8M0 ? TM * 16 : 0);
  if constexpr (MXF4)  // kind::mxf4: A and B E2M1 (format 1), E8M0 scales, K = 64
    p.idesc = (1u << 7) | (1u << 10) | ((uint32_t)(p.N >> 3) << 17) | (1u << 23) | ((uint32_t)(TM >> 4) << 24);
  else  // kind::mxf8f6f4: A the weight format, B E4M3 (format 0), E8M0 scales, K = 32
    p.idesc = (a_format<FMT>() << 7) | (0u << 10) | ((uint32_t)(p.N >> 3) << 17) | (1u << 23) |
              ((uint32_t)(TM >> 4) << 24);
  p.x = static_cast<const uint16_t *>(a.x);
  p.ldx = a.ldx;
  p.rscale = a.scales;
  p.sdt = a.sdt;
  p.y = a.y;
  p.ydt = a.ydt;
  p.ldy_m = a.ldy_m;
  p.ncopy = a.ncopy;
  for (int i = 0; i < 7; ++i) p.ycopy[i] = i < a.ncopy ? a.ycopy[i] : nullptr;
  p.part = w.part;
  p.tickets = w.tickets;

  CUtensorMap tmw, tms;
  const uint64_t row_bytes = (uint64_t)a.cols * BITS / 8;
  if constexpr (MXF4) {
    if (int32_t rc = make_tma_2d(&tmw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w, row_bytes, (uint64_t)a.rows, row_bytes, 128,
                                 TM, CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  } else {
    if (int32_t rc = make_tma_2d(&tmw,
                                 BITS == 4 ? CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B : CU_TENSOR_MAP_DATA_TYPE_16U6_ALIGN16B,
                                 a.w, (uint64_t)a.cols, (uint64_t)a.rows, row_bytes, KB, TM, CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  }
  if constexpr (SMODE == SM_E8M0) {
    if (int32_t rc = make_tma_2d(&tms, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.scales, (uint64_t)a.nblk, (uint64_t)a.rows,
                                 (uint64_t)a.nblk, 16, TM, CU_TENSOR_MAP_SWIZZLE_NONE))
      return rc;
  } else {
    tms = tmw;
  }
  const size_t smem = smem_for(p);
  B200_CUDA_TRY((ensure_dynamic_smem<mx_kernel<FMT, SMODE, P, XBF16>>(210 * 1024)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.grid);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[1];
  attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = (a.flags & B200_FLAG_PDL) ? 1 : 0;
  B200_CUDA_TRY(cudaLaunchKernelEx(&cfg, mx_kernel<FMT, SMODE, P, XBF16>, tmw, tms, p));
  return B200_OK;
}

// FP4 weights at 1..MXF4_MAX_M tokens: kind::mxf4 with eight FP4 pieces per token; otherwise
// kind::mxf8f6f4 with two E4M3 pieces per bf16 token, three per fp16 token
constexpr int MXF4_MAX_M = 2;
template <int FMT, int SMODE>
static int32_t dispatch_x(const LinearArgs &a, const Workspace &w, cudaStream_t stream) {
  const bool bf = a.xdt == B200_DT_BF16;
  if constexpr (FMT == B200_FMT_FP4_E2M1)
    if (a.m <= MXF4_MAX_M) return bf ? launch_t<FMT, SMODE, 8, true>(a, w, stream) : launch_t<FMT, SMODE, 8, false>(a, w, stream);
  return bf ? launch_t<FMT, SMODE, 2, true>(a, w, stream) : launch_t<FMT, SMODE, 3, false>(a, w, stream);
}

template <int FMT>
static int32_t dispatch(const LinearArgs &a, const Workspace &w, cudaStream_t stream) {
  switch (scale_mode(a)) {
    case SM_E8M0: return dispatch_x<FMT, SM_E8M0>(a, w, stream);
    case SM_ROW: return dispatch_x<FMT, SM_ROW>(a, w, stream);
    default: return dispatch_x<FMT, SM_NONE>(a, w, stream);
  }
}

}  // namespace mx

// Shapes the block-scaled kernel takes (independent of whether its workspace exists yet).
bool mx_supported(const LinearArgs &a) {
  using namespace mx;
  if (!(a.fmt == B200_FMT_FP4_E2M1 || a.fmt == B200_FMT_FP6_E2M3 || a.fmt == B200_FMT_FP6_E3M2)) return false;
  if (a.xdt != B200_DT_BF16 && a.xdt != B200_DT_F16) return false;
  if (a.ydt != B200_DT_F16 && a.ydt != B200_DT_BF16 && a.ydt != B200_DT_F32) return false;
  if (a.m < 1 || a.m * pieces_of(a.xdt) > MAX_COLS) return false;
  if (a.ldy_n != 1 || a.rows < 1 || a.rows > (int64_t)TICKETS * TM) return false;
  if (a.cols < KS || a.cols % KS != 0 || a.cols > (1 << 24)) return false;
  const int bits = fmt_bits(a.fmt);
  if ((uintptr_t)a.w % 32 != 0 || ((uint64_t)a.cols * bits / 8) % 32 != 0) return false;
  if ((uintptr_t)a.x % 16 != 0 || (a.m > 1 && (a.ldx * 2) % 16 != 0)) return false;
  switch (scale_mode(a)) {
    case SM_E8M0:
      if (a.sdt != B200_DT_E8M0 || a.block != 32) return false;
      if (a.nblk % 16 != 0 || (uintptr_t)a.scales % 16 != 0) return false;
      break;
    case SM_ROW:
      if (!(a.sdt == B200_DT_F16 || a.sdt == B200_DT_BF16 || a.sdt == B200_DT_F32)) return false;
      break;
    default: break;
  }
  return true;
}

// Runs the kernel if its workspace exists or can be allocated now; B200_ERR_UNSUPPORTED otherwise
// (a first call inside a stream capture), so the caller can take another kernel.
int32_t launch_mx(const LinearArgs &a, cudaStream_t stream) {
  using namespace mx;
  Workspace *w = nullptr;
  if (int32_t rc = workspace_for(stream, true, w)) return rc;
  if (w == nullptr) return b200_set_error(B200_ERR_UNSUPPORTED, "mx decode: no workspace while capturing");
  int sms = 0;
  B200_CUDA_TRY(device_sms(&sms));
  if ((size_t)sms * 2 * a.m * TM * sizeof(float) > w->part_bytes)
    return b200_set_error(B200_ERR_UNSUPPORTED, "mx decode: shape beyond the workspace");
  if (mxs_supported(a)) return launch_mxs(a, *w, stream);
  switch (a.fmt) {
    case B200_FMT_FP4_E2M1: return dispatch<B200_FMT_FP4_E2M1>(a, *w, stream);
    case B200_FMT_FP6_E2M3: return dispatch<B200_FMT_FP6_E2M3>(a, *w, stream);
    case B200_FMT_FP6_E3M2: return dispatch<B200_FMT_FP6_E3M2>(a, *w, stream);
  }
  return b200_set_error(B200_ERR_UNSUPPORTED, "mx decode: format %d", a.fmt);
}

// Zero the tile tickets of every workspace on the current device: after a kernel gave up on a
// bounded wait (device status bit set), a split tile may have been left half counted.
int32_t mx_reset_tickets() {
  using namespace mx;
  int dev = 0;
  B200_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(g_ws_mutex);
  for (auto &kv : g_ws)
    if (kv.first.first == dev) B200_CUDA_TRY(cudaMemset(kv.second.tickets, 0, kv.second.tickets_n * sizeof(unsigned int)));
  B200_CUDA_TRY(cudaDeviceSynchronize());
  return B200_OK;
}

// Whether a call on `stream` could run now: the workspace exists, or may be allocated (not capturing).
bool mx_ready(cudaStream_t stream) {
  using namespace mx;
  Workspace *w = nullptr;
  if (workspace_for(stream, false, w) != B200_OK) return false;
  if (w != nullptr) return true;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) return false;
  return cs == cudaStreamCaptureStatusNone;
}

}  // namespace b200
