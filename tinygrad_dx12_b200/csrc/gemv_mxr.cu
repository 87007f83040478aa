// gemv_mxr.cu -- row-split block-scaled tcgen05 decode GEMV for FP4 E2M1 weights at one token.
//
//   y[n] = sum_k x[k] * dequant(W)[n, k]
//
// The one-column matrix path of the reference's packed matmul (tinygrad-dx12
// src/tinygrad_dx12/codegen/linalg.py:226-245 over the decode of codegen/decomp/dx12.py:69-106)
// for FP4 weights, with no decode instructions: the packed E2M1 codes are read by the tensor
// cores as operand B of tcgen05.mma kind::mxf4 (K = 64), and the per-32 E8M0 weight scales are
// scale-factor B (every E2M1 code is an exact value, and 2^(e-127) is exactly the reference's
// decoded scale, dx12.py:102-106).
//
// Work split: every CTA (one per SM) owns a contiguous range of weight rows over the WHOLE of K
// (8-row blocks, ~56 rows per SM at 8192 rows), so no CTA shares an output with another and a
// call has no split-K fixup; rows go through the MMA in tiles of at most 64 (the MMA's N).
//
// x is the A operand: it is split once per call into eight FP4 pieces under ONE scale for the
// whole vector (piece q at 2^(E-2q), E from max|x|: error at most 2^-17 of max|x|), piece q being
// A row q. The MMA's M is 128, so rows 8..127 of A read whatever shared memory follows the
// pieces (FP4 codes are all finite; those accumulator rows are never read). Because the x scale
// is one number per piece, scale-factor A is a constant written once per call, and the weight
// scales of a row tile (all K stages) are copied into tensor memory once per tile: a K stage is
// then a TMA load of 8 KB of codes and four MMAs.
//
// Roles (512 threads):
//   warps 14-15 lane 0: TMA producers of the weight codes (one box of the tile's rows x 256 codes
//     per stage, 128-byte swizzle; a tensor map per tile height), stages of their parity;
//   warps 12-13 lane 0: MMA issuers, stages of their parity into their own accumulator pair
//     (one thread issues one MMA per ~36 ns, so two share the stages); each copies its own scale
//     factors with tcgen05.cp (copies and MMAs of one thread execute in issue order);
//   warps 4-7: weight-scale atoms of each tile (32 rows x 16 bytes per stage: rows r and r + 32,
//     both K-block groups), straight from global memory;
//   warps 0-3 and 8-11: converters (max|x|, then the pieces of their stages); warp 0 is also the
//     epilogue: it adds the issuers' accumulators and the eight piece rows and stores y.
// Every wait is bounded (sm100.cuh); on give-up the kernel flags the device error word and
// returns.
#include "mx.cuh"

namespace b200 {
namespace mxr {
using namespace mx;

constexpr int SF_WARP0 = 4, MMA_WARP0 = 12, PROD_WARP0 = 14;
constexpr int THREADS = 16 * 32;
constexpr int TMEM_THREADS = PROD_WARP0 * 32;  // every warp but the producers
constexpr int MAX_H = 64;                      // weight rows per tile (the MMA's N)
constexpr int MAX_NST = 32;                    // K <= 8192
constexpr int G = 2;                           // K stages per ring slot (one TMA box)
constexpr int STAGE_BYTES = MAX_H * 128;       // one stage: up to 64 rows x 256 codes
constexpr int SLOT_BYTES = G * STAGE_BYTES;
constexpr int MAX_STAGES = 8;                  // ring depth (even)

struct Maps {
  CUtensorMap m[8];  // weight codes as {128-byte K chunk, row, chunk}: box {128, 8 (i + 1) rows, G
                     // chunks}, 128-byte swizzle; a box lands as G [rows][128 B] stage tiles
};

struct Params {
  int64_t rows, cols;
  int nst;           // K stages of 256
  int nb8;           // 8-row blocks
  int grid;
  int stages;        // ring slots (even), G K stages each; issuer k's producer fills k, k + nmma, ...
  int ngroups;       // slots per tile: ceil(nst / G)
  int nmma;          // MMA issuers: 2, or 1 when K is a single group
  uint32_t xp_off, ring_off, sfb_off, sfa_off, bar_off;
  uint32_t idesc;    // kind::mxf4, M = 128, without N
  const uint16_t *x;
  const uint8_t *scales;  // E8M0 bytes [rows][nblk] (SM_E8M0)
  int64_t nblk;
  const void *rscale;     // per-row scales (SM_ROW)
  int sdt;
  void *y;
  int ydt;
  void *ycopy[7];
  int ncopy;
};

// CTA c's 8-row blocks [b0, b0 + nblocks), split into ntiles tiles of at most 8 blocks.
struct Tiles {
  int b0, nblocks, ntiles;
};
__host__ __device__ inline Tiles tiles_of(int nb8, int grid, int c) {
  Tiles t;
  t.b0 = (int)((int64_t)nb8 * c / grid);
  t.nblocks = (int)((int64_t)nb8 * (c + 1) / grid) - t.b0;
  t.ntiles = (t.nblocks + 7) / 8;
  return t;
}
__host__ __device__ inline void tile_rows(const Tiles &t, int j, int &first_block, int &blocks) {
  const int lo = t.nblocks * j / t.ntiles, hi = t.nblocks * (j + 1) / t.ntiles;
  first_block = t.b0 + lo;
  blocks = hi - lo;  // 1..8
}

__device__ __forceinline__ void conv_sync() { asm volatile("bar.sync 3, 256;" ::: "memory"); }
__device__ __forceinline__ void tmem_sync() { asm volatile("bar.sync 2, %0;" ::"n"(TMEM_THREADS) : "memory"); }

// Shared-memory descriptor of a 32-row x 16-byte scale-factor atom (rows 16 bytes apart).
__device__ __forceinline__ uint64_t sf_atom_desc(const void *atom) {
  const uint64_t addr = smem_u32(atom);
  return ((addr & 0x3FFFFull) >> 4) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(128 >> 4) << 32) | (1ull << 46);
}
__device__ __forceinline__ void sf_copy(uint32_t taddr, uint64_t desc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(desc) : "memory");
}

template <int SMODE, bool XBF16>
__global__ void __launch_bounds__(THREADS, 1)
    mxr_kernel(const __grid_constant__ Maps maps, const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *xp = base + p.xp_off;        // [nst][8 rows][128 B] x pieces (128-byte swizzle)
  uint8_t *ring = base + p.ring_off;    // [slots][G][64 rows][128 B] weight codes
  uint8_t *sfb_atoms = base + p.sfb_off;  // [2 tiles][nst][512 B]
  uint8_t *sfa_atom = base + p.sfa_off;   // [512 B]
  const int S = p.stages, nst = p.nst, nm = p.nmma;
  uint64_t *full = reinterpret_cast<uint64_t *>(base + p.bar_off);
  uint64_t *empty = full + S;
  uint64_t *bready = empty + S;       // [nst] x pieces of stage s, one phase
  uint64_t *sfbready = bready + nst;  // [2] a tile's weight-scale atoms
  uint64_t *sfbfree = sfbready + 2;   // [2] their shared memory is free again
  uint64_t *sfaready = sfbfree + 2;   // x-piece scale atom
  uint64_t *accfull = sfaready + 1;   // [issuer][buffer]
  uint64_t *accempty = accfull + 4;   // [buffer]
  uint64_t *drain = accempty + 2;     // [issuer]
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 2);
  volatile uint32_t *abort_flag = tmem_slot + 1;
  float *red = reinterpret_cast<float *>(tmem_slot + 2);  // [8] max|x| per converter warp
  uint32_t *bad = tmem_slot + 10;                          // [8] non-finite x seen

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Tiles tl = tiles_of(p.nb8, p.grid, blockIdx.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < nst; ++s) mbar_init(&bready[s], 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sfbready[b], 4);
      mbar_init(&sfbfree[b], nm);
      mbar_init(&accempty[b], 1);
      mbar_init(&drain[b], 1);
    }
    mbar_init(sfaready, 1);
    for (int b = 0; b < 4; ++b) mbar_init(&accfull[b], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp >= PROD_WARP0) {
    // ---------------- TMA producers: weight codes, groups g = k (mod nmma) of every tile ---------
    const int k = warp - PROD_WARP0;
    const int ng = p.ngroups;
    if (lane == 0 && k < nm) {
      {
        int fb, nbk;
        tile_rows(tl, 0, fb, nbk);
        prefetch_tmap(&maps.m[nbk - 1]);  // the first tile's map (only the heights used are encoded)
      }
      const int spi = S / nm;  // ring slots of this producer: k, k + nm, ...
      int j = 0;
      for (int ti = 0; ti < tl.ntiles && !*abort_flag; ++ti) {
        int fb, nbk;
        tile_rows(tl, ti, fb, nbk);
        const CUtensorMap *map = &maps.m[nbk - 1];
        for (int g = k; g < ng; g += nm, ++j) {
          const int slot = k + nm * (j % spi);
          const uint32_t round = (uint32_t)(j / spi);
          if (j >= spi && !mbar_wait(&empty[slot], (round - 1u) & 1u, abort_flag)) break;
          mbar_arrive_expect_tx(&full[slot], (uint32_t)(G * nbk * 8 * 128));
          tma_load_3d(ring + (size_t)slot * SLOT_BYTES, map, 0, fb * 8, g * G, &full[slot]);
        }
      }
      if (*abort_flag) {  // let this thread's copies in flight land before the CTA exits
        for (int q = j - spi < 0 ? 0 : j - spi; q < j; ++q)
          mbar_wait(&full[k + nm * (q % spi)], (uint32_t)((q / spi) & 1), abort_flag, 200000000ull);
      }
    }
    return;  // the producers take no part in the tensor-memory barriers below
  }

  if (warp == MMA_WARP0) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  tmem_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // tensor memory: accumulators [issuer][buffer] of 64 columns at 0..255, the issuers' copies of
  // scale-factor A at 256 + 4 k, the weight-scale factors of the tile at 264 + 4 s
  constexpr uint32_t SFA_COL = 256, SFB_COL = 264;

  if (warp < 4 || (warp >= 8 && warp < 12)) {
    // ---------------- converters: x -> eight FP4 pieces under one scale ----------------
    const int cw = warp < 4 ? warp : warp - 4;  // 0..7: stages s = cw (mod 8)
    asm volatile("griddepcontrol.wait;" ::: "memory");  // x is the previous kernel's output
    uint4 raw[MAX_NST / 8];
    float amax = 0.f;
    uint32_t nonfinite = 0;
#pragma unroll
    for (int i = 0; i < MAX_NST / 8; ++i) {
      const int s = cw + 8 * i;
      if (s < nst) {
        raw[i] = *reinterpret_cast<const uint4 *>(p.x + (int64_t)s * KS + 8 * lane);
        float v[8];
        raw_to_f32<XBF16>(raw[i], v);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float a = fabsf(v[e]);
          nonfinite |= a <= 3.4e38f ? 0u : 1u;
          amax = fmaxf(amax, a);
        }
      }
    }
    for (int o = 16; o > 0; o >>= 1) {
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      nonfinite |= __shfl_xor_sync(0xffffffffu, nonfinite, o);
    }
    if (lane == 0) red[cw] = amax, bad[cw] = nonfinite;
    conv_sync();
    amax = 0.f;
    nonfinite = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) amax = fmaxf(amax, red[w]), nonfinite |= bad[w];
    // piece 0's scale puts max|x| in [2, 4); a non-finite x makes every output NaN (scale byte
    // 255 on piece 0), an all-zero x gives zeros
    uint32_t byte0;
    if (nonfinite) byte0 = 255u;
    else if (amax == 0.f) byte0 = 141u;
    else {
      const int b = ilogbf(amax) + 126;
      byte0 = (uint32_t)(b < 15 ? 15 : b > 253 ? 253 : b);
    }
    if (cw == 0) {  // scale-factor A: row q (q < 8) = piece q, the other rows 2^0
      uint32_t w = 0x7F7F7F7Fu;
      if (lane < 8) {
        const uint32_t bq = byte0 == 255u ? (lane == 0 ? 255u : 127u) : byte0 - 2u * (uint32_t)lane;
        w = bq * 0x01010101u;
      }
      reinterpret_cast<uint4 *>(sfa_atom)[lane] = make_uint4(w, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(sfaready);
    }
    const uint32_t chunk = (uint32_t)lane >> 2, off = (uint32_t)(lane & 3) * 4;
#pragma unroll
    for (int i = 0; i < MAX_NST / 8; ++i) {
      const int s = cw + 8 * i;
      if (s >= nst) break;
      float v[8];
      raw_to_f32<XBF16>(raw[i], v);
      uint32_t pc[8];
      if (byte0 == 255u) {
#pragma unroll
        for (int q = 0; q < 8; ++q) pc[q] = 0u;
      } else {
        fp4_pieces<8>(v, byte0, pc);
      }
      uint8_t *st = xp + (size_t)s * 1024;
#pragma unroll
      for (int q = 0; q < 8; ++q)  // A row q of the stage's 8-row, 128-byte-swizzled atom
        *reinterpret_cast<uint32_t *>(st + q * 128 + ((chunk ^ (uint32_t)q) << 4) + off) = pc[q];
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bready[s]);
    }
  } else if (warp >= SF_WARP0 && warp < SF_WARP0 + 4) {
    // ---------------- weight-scale atoms of each tile: stages s = w (mod 4) ----------------
    // atom of stage s, row l: [K blocks 0-3 of tile row l, of row l + 32, K blocks 4-7 of row l,
    // of row l + 32] -> tensor-memory columns c, c + 1 (blocks 0-3) and c + 2, c + 3 (blocks 4-7)
    const int hw = warp - SF_WARP0;
    for (int ti = 0; ti < tl.ntiles; ++ti) {
      const int b = ti & 1;
      if (ti >= 2 && !mbar_wait(&sfbfree[b], (uint32_t)((ti / 2 - 1) & 1), abort_flag)) break;
      int fb, nbk;
      tile_rows(tl, ti, fb, nbk);
      const int64_t r0 = (int64_t)fb * 8 + lane, r1 = r0 + 32;
      const bool ok0 = lane < nbk * 8 && r0 < p.rows, ok1 = lane + 32 < nbk * 8 && r1 < p.rows;
      for (int s = hw; s < nst; s += 4) {
        uint2 a0 = make_uint2(0x7F7F7F7Fu, 0x7F7F7F7Fu), a1 = a0;
        if constexpr (SMODE == SM_E8M0) {
          if (ok0) a0 = __ldg(reinterpret_cast<const uint2 *>(p.scales + r0 * p.nblk + 8 * s));
          if (ok1) a1 = __ldg(reinterpret_cast<const uint2 *>(p.scales + r1 * p.nblk + 8 * s));
        }
        reinterpret_cast<uint4 *>(sfb_atoms + ((size_t)b * nst + s) * 512)[lane] = make_uint4(a0.x, a1.x, a0.y, a1.y);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sfbready[b]);
    }
  } else if (warp >= MMA_WARP0 && warp < MMA_WARP0 + 2) {
    // ---------------- MMA issuers: groups g = k (mod nmma) of every tile ----------------
    const int k = warp - MMA_WARP0;
    const int ng = p.ngroups;
    if (lane == 0 && k < nm) {
      const uint32_t hi = 2u << 30;
      const int spi = S / nm;
      bool ok = mbar_wait(sfaready, 0u, abort_flag);
      tc_fence_after();
      const uint32_t sfa = tmem + SFA_COL + 4u * (uint32_t)k;  // this issuer's copy
      if (ok) sf_copy(sfa, sf_atom_desc(sfa_atom));
      int j = 0;
      for (int ti = 0; ti < tl.ntiles && ok; ++ti) {
        int fb, nbk;
        tile_rows(tl, ti, fb, nbk);
        const uint32_t id0 = p.idesc | ((uint32_t)nbk << 17);  // N = 8 * nbk (field N >> 3)
        const uint32_t id2 = id0 | (2u << 4) | (2u << 29);
        const uint32_t tile_bytes = (uint32_t)nbk * 8u * 128u;  // one stage of the slot
        const int buf = ti & 1;
        if (ti >= 2 && !(ok = mbar_wait(&accempty[buf], (uint32_t)((ti / 2 - 1) & 1), abort_flag))) break;
        if (!(ok = mbar_wait(&sfbready[buf], (uint32_t)((ti / 2) & 1), abort_flag))) break;
        tc_fence_after();
        for (int g = k; g < ng; g += nm)
          for (int s = g * G; s < g * G + G && s < nst; ++s)
            sf_copy(tmem + SFB_COL + 4u * (uint32_t)s, sf_atom_desc(sfb_atoms + ((size_t)buf * nst + s) * 512));
        mma_commit(&sfbfree[buf]);  // the atoms' shared memory is free once these copies are done
        const uint32_t dcol = tmem + (uint32_t)(2 * k + buf) * 64u;
        bool first = true;
        for (int g = k; g < ng; g += nm, ++j) {
          if (ti == 0)
            for (int s = g * G; s < g * G + G && s < nst && ok; ++s) ok = mbar_wait(&bready[s], 0u, abort_flag);
          const int slot = k + nm * (j % spi);
          if (!ok || !(ok = mbar_wait(&full[slot], (uint32_t)((j / spi) & 1), abort_flag))) break;
          tc_fence_after();
          for (int st = 0; st < G && g * G + st < nst; ++st) {
            const int s = g * G + st;
            const uint64_t ad = sw128_kmajor_desc(xp + (size_t)s * 1024);
            const uint64_t bd = sw128_kmajor_desc(ring + (size_t)slot * SLOT_BYTES + (size_t)st * tile_bytes);
            const uint32_t sfb = tmem + SFB_COL + 4u * (uint32_t)s;
            mma_mxf4(dcol, ad, bd, id0, first ? 0u : 1u, sfa, sfb);
            mma_mxf4(dcol, ad + 2, bd + 2, id2, 1u, sfa | hi, sfb | hi);
            mma_mxf4(dcol, ad + 4, bd + 4, id0, 1u, sfa, sfb + 2u);
            mma_mxf4(dcol, ad + 6, bd + 6, id2, 1u, sfa | hi, (sfb + 2u) | hi);
            first = false;
          }
          mma_commit(&empty[slot]);
        }
        if (!ok) break;
        mma_commit(&accfull[2 * k + buf]);
      }
      // every MMA and copy issued has completed before the CTA frees its tensor memory
      mma_commit(&drain[k]);
      mbar_wait(&drain[k], 0, abort_flag, 200000000ull);
    }
  }
  if (warp == 0) {
    // ---------------- epilogue: y of each tile from the issuers' accumulators ----------------
    // Lane q < 8 holds accumulator row q (x piece q) in every column (tile row); the eight rows
    // are added across lanes, then lane q stores columns q, q + 8, ...
    uint32_t ph = 0;
    for (int ti = 0; ti < tl.ntiles; ++ti) {
      int fb, nbk;
      tile_rows(tl, ti, fb, nbk);
      const int buf = ti & 1;
      bool ok = true;
      for (int k = 0; k < nm; ++k) {
        const int a = 2 * k + buf;
        ok = ok && mbar_wait(&accfull[a], (ph >> a) & 1u, abort_flag);
        ph ^= 1u << a;
      }
      if (!ok) break;
      tc_fence_after();
      for (int h = 0; h < 2 && 32 * h < nbk * 8; ++h) {
        float acc[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) acc[c] = 0.f;
        for (int k = 0; k < nm; ++k) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tmem + (uint32_t)(2 * k + buf) * 64u + 32u * (uint32_t)h, v);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 32; ++c) acc[c] += __uint_as_float(v[c]);
        }
#pragma unroll
        for (int c = 0; c < 32; ++c) {  // add the eight piece rows (lanes q, q ^ 1, ...)
          acc[c] += __shfl_xor_sync(0xffffffffu, acc[c], 1);
          acc[c] += __shfl_xor_sync(0xffffffffu, acc[c], 2);
          acc[c] += __shfl_xor_sync(0xffffffffu, acc[c], 4);
        }
        float mine[4];  // columns lane, lane + 8, lane + 16, lane + 24 (static register selection)
#pragma unroll
        for (int c = 0; c < 32; ++c)
          if ((c & 7) == (lane & 7)) mine[c >> 3] = acc[c];
        if (lane < 8) {
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const int n = 32 * h + lane + 8 * jj;
            const int64_t row = (int64_t)fb * 8 + n;
            if (n < nbk * 8 && row < p.rows) {
              float yv = mine[jj];
              if constexpr (SMODE == SM_ROW) yv *= load_as_f32(p.rscale, row, p.sdt);
              store_f32(p.y, row, p.ydt, yv);
              for (int cp = 0; cp < p.ncopy; ++cp) store_f32(p.ycopy[cp], row, p.ydt, yv);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty[buf]);
    }
  }
  tc_fence_before();
  tmem_sync();
  tc_fence_after();
  if (warp == MMA_WARP0) tmem_dealloc(tmem, 512);
}

struct Layout {
  int stages;
  uint32_t xp_off, ring_off, sfb_off, sfa_off, bar_off;
  size_t smem;
};

static Layout layout_for(int nst) {
  Layout l = {};
  l.xp_off = 0;
  l.ring_off = (uint32_t)nst * 1024;  // the ring follows the pieces: A rows 8..127 of the last
                                      // stage read up to 15 KB past them, inside the ring
  l.stages = MAX_STAGES;
  l.sfb_off = l.ring_off + (uint32_t)l.stages * SLOT_BYTES;
  l.sfa_off = l.sfb_off + 2u * (uint32_t)nst * 512u;
  l.bar_off = l.sfa_off + 512;
  l.smem = 1024 + l.bar_off + 8 * (2 * (size_t)l.stages + nst + 2 + 2 + 1 + 4 + 2 + 2) + 4 * 18 + 16;
  return l;
}

template <int SMODE, bool XBF16>
static int32_t launch_t(const LinearArgs &a, cudaStream_t stream) {
  int sms = 0;
  B200_CUDA_TRY(device_sms(&sms));
  Params p;
  memset(&p, 0, sizeof(p));
  p.rows = a.rows;
  p.cols = a.cols;
  p.nst = (int)(a.cols / KS);
  p.nb8 = (int)((a.rows + 7) / 8);
  p.grid = p.nb8 < sms ? p.nb8 : sms;
  p.ngroups = (p.nst + G - 1) / G;
  p.nmma = p.ngroups >= 2 ? 2 : 1;
  const Layout l = layout_for(p.nst);
  p.stages = l.stages;
  p.xp_off = l.xp_off;
  p.ring_off = l.ring_off;
  p.sfb_off = l.sfb_off;
  p.sfa_off = l.sfa_off;
  p.bar_off = l.bar_off;
  // kind::mxf4: A and B E2M1 (format 1), E8M0 scales, M = 128 (N per tile in the kernel)
  p.idesc = (1u << 7) | (1u << 10) | (1u << 23) | ((uint32_t)(TM >> 4) << 24);
  p.x = static_cast<const uint16_t *>(a.x);
  p.scales = static_cast<const uint8_t *>(a.scales);
  p.nblk = a.nblk;
  p.rscale = a.scales;
  p.sdt = a.sdt;
  p.y = a.y;
  p.ydt = a.ydt;
  p.ncopy = a.ncopy;
  for (int i = 0; i < 7; ++i) p.ycopy[i] = i < a.ncopy ? a.ycopy[i] : nullptr;

  // one tensor map per tile height the grid uses (8..64 rows)
  Maps maps;
  memset(&maps, 0, sizeof(maps));
  bool need[8] = {false, false, false, false, false, false, false, false};
  for (int c = 0; c < p.grid; ++c) {
    const Tiles t = tiles_of(p.nb8, p.grid, c);
    for (int j = 0; j < t.ntiles; ++j) {
      int fb, nbk;
      tile_rows(t, j, fb, nbk);
      need[nbk - 1] = true;
    }
  }
  const uint64_t row_bytes = (uint64_t)a.cols / 2;
  for (int h = 0; h < 8; ++h)
    if (need[h])
      if (int32_t rc = make_tma_3d(&maps.m[h], CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w, 128, (uint64_t)a.rows,
                                   (uint64_t)p.nst, row_bytes, 128, 128, (uint32_t)(8 * (h + 1)), (uint32_t)G,
                                   CU_TENSOR_MAP_SWIZZLE_128B))
        return rc;
  B200_CUDA_TRY((ensure_dynamic_smem<mxr_kernel<SMODE, XBF16>>(210 * 1024)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.grid);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = l.smem < 116 * 1024 ? 116 * 1024 : l.smem;  // one CTA per SM
  cfg.stream = stream;
  cudaLaunchAttribute attrs[1];
  attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = (a.flags & B200_FLAG_PDL) ? 1 : 0;
  B200_CUDA_TRY(cudaLaunchKernelEx(&cfg, mxr_kernel<SMODE, XBF16>, maps, p));
  return B200_OK;
}

}  // namespace mxr

// FP4 weights, one token, K a multiple of 256 up to 8192; the caller has checked mx_supported.
bool mxr_supported(const LinearArgs &a) {
  using namespace mxr;
  if (a.fmt != B200_FMT_FP4_E2M1 || a.m != 1) return false;
  if (a.cols % KS != 0 || a.cols / KS > MAX_NST) return false;
  if ((uintptr_t)a.w % 16 != 0 || (uintptr_t)a.x % 16 != 0) return false;
  if (mx::scale_mode(a) == SM_E8M0 && (uintptr_t)a.scales % 8 != 0) return false;
  return true;
}

int32_t launch_mxr(const LinearArgs &a, cudaStream_t stream) {
  using namespace mxr;
  const bool bf = a.xdt == B200_DT_BF16;
  switch (mx::scale_mode(a)) {
    case SM_E8M0: return bf ? launch_t<SM_E8M0, true>(a, stream) : launch_t<SM_E8M0, false>(a, stream);
    case SM_ROW: return bf ? launch_t<SM_ROW, true>(a, stream) : launch_t<SM_ROW, false>(a, stream);
    default: return bf ? launch_t<SM_NONE, true>(a, stream) : launch_t<SM_NONE, false>(a, stream);
  }
}

}  // namespace b200
