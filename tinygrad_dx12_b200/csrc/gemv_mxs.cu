// gemv_mxs.cu -- block-scaled tcgen05 decode GEMV for FP4 E2M1 weights and 1..4 tokens, with
// the activation pieces resident in shared memory.
//
//   y[m, n] = sum_k x[m, k] * dequant(W)[n, k]
//
// The decode GEMV of the reference's packed matmul (tinygrad-dx12
// src/tinygrad_dx12/codegen/linalg.py:226-245, the one-column matrix path, over the decode of
// codegen/decomp/dx12.py:69-106) for FP4 weights, with no decode instructions: the tensor cores
// read the packed E2M1 codes as the A operand of tcgen05.mma kind::mxf4 (K = 64) and apply the
// per-32 E8M0 weight scales themselves (scale-factor A in tensor memory); every E2M1 code is an
// exact value and 2^(e-127) is exactly the reference's decoded scale (dx12.py:102-106).
//
// x is split once per call into eight FP4 pieces per element (mx.cuh split_fp4: piece q carries
// E8M0 scale 2^(e-2q), error at most 2^-17 of the 32-block maximum), piece q of token m being B
// row 8m + q, so one MMA with N = 8m columns carries every piece of every token and the epilogue
// adds each token's eight columns in fp32.
//
// What differs from gemv_mx.cu (the general kernel, x pieces per ring stage): a decode call
// streams ~10-100 stages per CTA, and per-stage side work there (converting x, writing the
// scale operands with tcgen05.st and waiting for them) took longer than a stage's 16 KB of
// weight codes take to arrive. Here
//   * the CTA's x pieces for all the K stages it touches (at most one per K stage of the matrix)
//     are converted once, at the start, into a resident shared-memory array with their
//     scale-factor atoms;
//   * the weight scales of a stage are laid out as two 32-row scale-factor atoms by a helper
//     warp, from global memory, and the MMA thread copies them into tensor memory with
//     tcgen05.cp right before the stage's four MMAs (copies and MMAs execute in issue order, so
//     nothing waits for them); the copies rotate over eight column sets, so a copy never
//     overwrites scales an MMA in flight still reads;
//   * every loop advances its tile / stage / slot counters incrementally (measured: a thread
//     issues one MMA per ~36 ns in a loop without divisions, ~126 ns with a 64-bit modulo per
//     unit), and two threads issue the MMAs of alternate units (the tensor pipe takes one
//     K = 64 MMA per ~21 ns at these N; HBM supplies a 16 KB unit per ~370 ns per SM).
//
// Work split (stream-K, as gemv_mx.cu): units = (128-row weight tile, 256-deep K stage), CTA c
// of the persistent grid takes units [c U / G, (c + 1) U / G); a tile split across CTAs is
// finished by its last contributor (acquire-release ticket) adding the fp32 partials in CTA
// order (deterministic). Unit i of a CTA reads K stage (u0 + i) % nst, whose x pieces sit in
// resident slot i % nst: the first min(units, nst) units of a CTA touch distinct stages.
// Pair split (matrices of at most SMs / 2 tiles, an even stage count): the grid is two CTAs per
// tile, launched as 2-CTA clusters, CTA 2t + h taking K half h of tile t (the same unit ranges
// as stream-K over that grid). The second CTA pushes its fp32 partials into the first one's
// shared memory (st.shared::cluster, one release-arrive per thread on the first CTA's mbarrier)
// and the first adds them after its own, in the stream-K order: no global partials, fence or
// ticket, whose dependent L2 round trips made up most of a one-token call's tail.
//
// Roles (512 threads): two pipelines, for the even and the odd units of the CTA. Warps 14-15
// lane 0 issue the TMA loads of the weight codes (one 128-row x 128-byte box = 256 codes per row
// per stage, 128-byte swizzle) into the ring slots of their parity; they start before the
// tensor-memory allocation, so a call launched with programmatic dependent launch streams its
// first stages while the previous call's CTA on the SM finishes. Warps 12-13 lane 0 each issue
// the copies and MMAs of their units into their own pair of fp32 accumulators (one thread issues
// an MMA with two scale copies about every 70 ns; two threads do so concurrently). Warps 8-11
// convert x into the resident pieces; warps 4-7 build the weight-scale atoms of alternate
// units; warps 0-3 read the accumulators (tcgen05.ld), add the two issuers' sums and finish the
// rows. Every wait is bounded (sm100.cuh); on give-up the kernel flags the device error word and
// returns.
#include "mx.cuh"

namespace b200 {
namespace mxs {
using namespace mx;

constexpr int EPI_WARP0 = 0, SF_WARP0 = 4, CONV_WARP0 = 8, MMA_WARP0 = 12, PROD_WARP0 = 14, PROD_WARPS = 2;
constexpr int THREADS = 16 * 32;
constexpr int TMEM_THREADS = PROD_WARP0 * 32;  // every warp but the producers
constexpr int STAGE_BYTES = TM * 128;          // 128 rows x 256 FP4 codes
constexpr int SFR = 8;                         // scale-factor atom ring (units in flight)
constexpr int MAX_M = 4;
constexpr int MAX_STAGES = 8;
constexpr int SMEM_MAX = 227 * 1024;            // dynamic shared memory a CTA may take

struct Params {
  int64_t rows, cols;
  int nst, ntiles;          // K stages per tile, 128-row tiles
  int64_t units;            // ntiles * nst
  int grid;                 // CTAs
  int m, N;                 // tokens, MMA N = 8 m
  int stages;               // weight-code ring depth
  int nb;                   // resident x-piece slots: min(max units per CTA, nst)
  int nmma;                 // MMA issuers (1 or 2): issuer k takes the units i = k (mod nmma)
  uint32_t b_off, sfb_off, sfa_off, bar_off;  // smem: pieces [nb][N][128 B], SFB atoms every N x 16 B,
                                              // SFA atom ring [SFR][2][512 B], barriers
  uint32_t width, sfa_col, sfb_col, tmem_cols;  // accumulator [issuer k][buffer] at (2 k + buffer) * width
  uint32_t idesc;
  const uint16_t *x;        // activations (bf16 or fp16), row stride ldx
  int64_t ldx;
  const uint8_t *scales;    // E8M0 bytes [rows][nblk] (SM_E8M0)
  int64_t nblk;
  const void *rscale;       // per-row weight scales (SM_ROW)
  int sdt;
  void *y;
  int ydt;
  int64_t ldy_m;
  void *ycopy[7];
  int ncopy;
  float *part;              // [grid][2][m][128] fp32 partials of split tiles
  unsigned int *tickets;    // [ntiles]
  int pair;                 // pair split (2-CTA clusters), see above
  uint32_t pair_off;        // smem: [MAX_M][128] fp32 partials pushed by the cluster partner
};

__device__ __forceinline__ void tmem_sync() { asm volatile("bar.sync 2, %0;" ::"n"(TMEM_THREADS) : "memory"); }

// Shared-memory descriptor of a 32-row x 16-byte scale-factor atom (rows 16 bytes apart, no
// swizzle), the source of tcgen05.cp .32x128b.
__device__ __forceinline__ uint64_t sf_atom_desc(const void *atom) {
  const uint64_t addr = smem_u32(atom);
  return ((addr & 0x3FFFFull) >> 4) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(128 >> 4) << 32) | (1ull << 46);
}
// Copy one atom into 4 tensor-memory columns of every lane quarter (row l -> lane l of each).
__device__ __forceinline__ void sf_copy(uint32_t taddr, uint64_t desc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(desc) : "memory");
}

// ---- 2-CTA cluster helpers of the pair split ----
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Every thread of both CTAs arrives once per phase and waits once per phase (non-aligned forms:
// the threads of a warp reach them at different points).
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire;" ::: "memory"); }
// This CTA's shared-memory address `a` as seen in the shared window of cluster CTA `rank`.
__device__ __forceinline__ uint32_t map_rank(uint32_t a, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t a, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t a) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(a) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait with cluster-scope acquire (the arrivals come from the partner CTA).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, volatile uint32_t *abort_flag) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((i & 63) == 0) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > 2000000000ull) {
        *abort_flag = 1;
        atomicOr(&g_device_error, B200_DEVERR_MBAR_TIMEOUT);
        return false;
      }
    }
  }
}

template <int SMODE, bool XBF16>
__global__ void __launch_bounds__(THREADS, 1) mxs_kernel(const __grid_constant__ CUtensorMap tmw, const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *ring = base;
  uint8_t *bres = base + p.b_off;
  uint8_t *sfb_atoms = base + p.sfb_off;
  uint8_t *sfa_atoms = base + p.sfa_off;
  const int S = p.stages;
  uint64_t *full = reinterpret_cast<uint64_t *>(base + p.bar_off);
  uint64_t *empty = full + S;
  uint64_t *sfready = empty + S;
  uint64_t *sffree = sfready + SFR;
  uint64_t *accfull = sffree + SFR;  // [issuer][buffer]
  uint64_t *accempty = accfull + 4;
  uint64_t *drain = accempty + 2;  // [issuer]
  uint64_t *bready = drain + 2;  // [nb], one phase each
  uint64_t *pairbar = bready + p.nb;  // pair split: the partner's 128 pushes
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(pairbar + 1);
  volatile uint32_t *abort_flag = tmem_slot + 1;
  volatile uint32_t *last_flag = tmem_slot + 2;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t u0 = unit_start(p, blockIdx.x), u1 = unit_start(p, blockIdx.x + 1);
  const int n = (int)(u1 - u0);
  const int nb = p.nb, nst = p.nst;
  const int t0 = (int)(u0 / nst), s0 = (int)(u0 % nst);  // first unit's tile and K stage

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int r = 0; r < SFR; ++r) {
      mbar_init(&sfready[r], 1);
      mbar_init(&sffree[r], 1);
    }
    for (int b = 0; b < 4; ++b) mbar_init(&accfull[b], 1);
    for (int b = 0; b < 2; ++b) mbar_init(&accempty[b], 4);
    mbar_init(&drain[0], 1);
    mbar_init(&drain[1], 1);
    for (int b = 0; b < nb; ++b) mbar_init(&bready[b], 1);
    mbar_init(pairbar, TM);
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  // pair split: phase 0 of the cluster barrier publishes the initialised mbarriers to the
  // partner (waited for before the first remote access); phase 1 at the end keeps this CTA's
  // shared memory alive until the partner is done with it
  if (p.pair) cluster_arrive();
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp >= PROD_WARP0) {
    // ---------------- TMA producers: weight codes (no dependency on the previous kernel) -------
    // producer pw fills the ring slots of parity pw (the ring depth is even), i.e. the units
    // i = pw (mod 2): with two MMA issuers, producer k and issuer k form one pipeline
    const int pw = warp - PROD_WARP0;
    const int nact = PROD_WARPS;
    if (lane == 0) {
      prefetch_tmap(&tmw);
      int t = t0, s = s0 + pw;
      while (s >= nst) s -= nst, ++t;
      int i = pw;
      for (; i < n; i += nact) {
        const int slot = i % S;
        const uint32_t round = (uint32_t)(i / S);
        if (i >= S && !mbar_wait(&empty[slot], (round - 1u) & 1u, abort_flag)) break;
        mbar_arrive_expect_tx(&full[slot], STAGE_BYTES);
        tma_load_2d(ring + (size_t)slot * STAGE_BYTES, &tmw, s * 128, t * TM, &full[slot]);
        s += nact;
        while (s >= nst) s -= nst, ++t;
      }
      if (*abort_flag) {  // let this thread's copies in flight land before the CTA exits
        for (int q = pw; q < (i < n ? i : n); q += nact)
          if (q + S >= i) mbar_wait(&full[q % S], (uint32_t)((q / S) & 1), abort_flag, 200000000ull);
      }
    }
    if (p.pair) {
      cluster_wait();
      cluster_arrive();
      cluster_wait();
    }
    return;  // the producers take no part in the tensor-memory barriers below
  }
  bool cluster_phase0 = false;  // pair split: this thread has waited for phase 0

  if (warp == MMA_WARP0) tmem_alloc(tmem_slot, p.tmem_cols);
  tc_fence_before();
  tmem_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4 || (warp >= CONV_WARP0 && warp < CONV_WARP0 + 4)) {
    // ---------------- x -> eight FP4 pieces per token, resident slots b = cw (mod 8) -----------
    // Converters: warps 8-11 and the epilogue warps 0-3, which take their epilogue role after.
    // Slot b holds K stage (s0 + b) % nst: B rows 8 mm + c (token mm, piece c) of 128 bytes
    // (128-byte swizzle), and its scale-factor atom (row j: bytes 0-3 = K blocks 0-3 of B row j,
    // bytes 8-11 = K blocks 4-7, so tensor-memory columns c and c + 2 hold the two groups).
    const int cw = warp < 4 ? warp : warp - CONV_WARP0 + 4;  // converter 0..7
    const uint32_t chunk = (uint32_t)lane >> 2, off = (uint32_t)(lane & 3) * 4;
    const int kb = lane >> 2;  // this lane's K block of the stage (elements 8 lane .. 8 lane + 7)
    // An atom's rows 0..N-1 are B rows; the copy also reads its rows N..31, which land in
    // tensor-memory lanes no MMA of N columns reads, so atom b + 1 starts N rows after atom b.
    const uint32_t sfbs = (uint32_t)p.N * 16;
    for (int b = cw; b < nb; b += 8)  // pad bytes of the atoms' B rows: scale 2^0
      if (lane < p.N)
        reinterpret_cast<uint4 *>(sfb_atoms + (size_t)b * sfbs)[lane] = make_uint4(0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu, 0x7F7F7F7Fu);
    __syncwarp();
    asm volatile("griddepcontrol.wait;" ::: "memory");  // x is the previous kernel's output
    // (slot, token) pairs of this warp in slot-major order, four pairs' loads in flight at once
    const int myslots = nb > cw ? (nb - cw + 7) / 8 : 0;
    const int pairs = myslots * p.m;
    for (int q0 = 0; q0 < pairs; q0 += 4) {
      uint4 raw[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (q0 + q >= pairs) break;
        const int b = cw + 8 * ((q0 + q) / p.m), mm = (q0 + q) % p.m;
        int s = s0 + b;
        if (s >= nst) s -= nst;  // b < nst
        raw[q] = *reinterpret_cast<const uint4 *>(p.x + (int64_t)mm * p.ldx + (int64_t)s * KS + 8 * lane);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (q0 + q >= pairs) break;
        const int b = cw + 8 * ((q0 + q) / p.m), mm = (q0 + q) % p.m;
        float v[8];
        raw_to_f32<XBF16>(raw[q], v);
        uint32_t pc[8];
        const uint32_t byte0 = split_fp4<8>(v, pc);
        uint8_t *bt = bres + (size_t)b * p.N * 128;
        uint8_t *atom = sfb_atoms + (size_t)b * sfbs + (kb < 4 ? kb : 4 + kb);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint32_t j = (uint32_t)(mm * 8 + c);  // B row of token mm's piece c
          *reinterpret_cast<uint32_t *>(bt + j * 128 + ((chunk ^ (j & 7)) << 4) + off) = pc[c];
          if ((lane & 3) == 0) atom[j * 16] = (uint8_t)(byte0 == 255u ? (c == 0 ? 255u : 127u) : byte0 - 2u * c);
        }
        if (mm == p.m - 1) {  // the slot's last token: its pieces and scales are ready (publishing
          fence_proxy_async_smem();  // each slot at once measured faster than converting four
          __syncwarp();              // slots' pieces together and publishing them after)
          if (lane == 0) mbar_arrive(&bready[b]);
        }
      }
    }
  } else if (warp >= SF_WARP0 && warp < SF_WARP0 + 4) {
    // ---------------- weight scales -> scale-factor atoms, units i = w (mod 4) -----------------
    // Unit i's two atoms (K blocks 0-3 and 4-7 of its stage): row l = the words of tile rows
    // l, l + 32, l + 64, l + 96, i.e. tensor-memory columns q = row / 32 of lane row % 32.
    // The next unit's scale loads are issued before this unit's atoms are written (keeping more
    // in flight measured slower: they delay the x loads that the first MMA waits for).
    const int sw = warp - SF_WARP0;
    int t = t0, s = s0 + sw;
    while (s >= nst) s -= nst, ++t;
    auto load_unit = [&](int tt, int ss, uint2 (&a)[4]) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        a[q] = make_uint2(0x7F7F7F7Fu, 0x7F7F7F7Fu);
        if constexpr (SMODE == SM_E8M0) {
          const int64_t row = (int64_t)tt * TM + lane + 32 * q;
          if (row < p.rows) a[q] = __ldg(reinterpret_cast<const uint2 *>(p.scales + row * p.nblk + 8 * ss));
        }
      }
    };
    uint2 cur[4];
    if (sw < n) load_unit(t, s, cur);
    for (int i = sw; i < n; i += 4) {
      s += 4;
      while (s >= nst) s -= nst, ++t;
      uint2 nxt[4];
      if (i + 4 < n) load_unit(t, s, nxt);
      const int r = i % SFR;
      if (i >= SFR && !mbar_wait(&sffree[r], (uint32_t)((i / SFR - 1) & 1), abort_flag)) break;
      uint8_t *atom = sfa_atoms + (size_t)r * 1024 + 16 * lane;
      *reinterpret_cast<uint4 *>(atom) = make_uint4(cur[0].x, cur[1].x, cur[2].x, cur[3].x);
      *reinterpret_cast<uint4 *>(atom + 512) = make_uint4(cur[0].y, cur[1].y, cur[2].y, cur[3].y);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sfready[r]);
#pragma unroll
      for (int q = 0; q < 4; ++q) cur[q] = nxt[q];
    }
  } else if (warp >= MMA_WARP0 && warp < MMA_WARP0 + 2) {
    // ---------------- MMA issuers: per unit two scale copies and four K = 64 MMAs ----------------
    // Issuer k takes the units i = k (mod nmma) into its own accumulator pair; a tile segment's
    // result is the sum of the issuers' accumulators. Unit i's segment is (s0 + i) / nst.
    const int k = warp - MMA_WARP0;
    if (lane == 0 && k < p.nmma) {
      const int nm = p.nmma;
      const uint32_t id0 = p.idesc, id2 = p.idesc | (2u << 4) | (2u << 29);  // scale bytes 0-1 | 2-3
      const uint32_t hi = 2u << 30;
      int slot = k, r = k, set = k, b = k % nst, s = s0 + k, seg = 0;
      while (s >= nst) s -= nst, ++seg;
      uint32_t round = 0, rround = 0;
      for (int i = k; i < n; i += nm) {
        const bool first = i < nm || s < nm;              // this issuer's first unit of the segment
        const bool last = i + nm >= n || s + nm >= nst;   // ... and its last
        const int buf = seg & 1;
        if (first && seg >= 2 && !mbar_wait(&accempty[buf], (uint32_t)((seg / 2 - 1) & 1), abort_flag)) break;
        const uint32_t sfb = tmem + p.sfb_col + 4u * (uint32_t)b;
        if (i < nb) {  // first use of resident slot b (== i): its x pieces and their scales
          if (!mbar_wait(&bready[b], 0u, abort_flag)) break;
          tc_fence_after();
          sf_copy(sfb, sf_atom_desc(sfb_atoms + (size_t)b * p.N * 16));
        }
        if (!mbar_wait(&sfready[r], rround & 1u, abort_flag)) break;
        if (!mbar_wait(&full[slot], round & 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t sfa = tmem + p.sfa_col + 8u * (uint32_t)set;
        sf_copy(sfa, sf_atom_desc(sfa_atoms + (size_t)r * 1024));
        sf_copy(sfa + 4u, sf_atom_desc(sfa_atoms + (size_t)r * 1024 + 512));
        const uint64_t ad = sw128_kmajor_desc(ring + (size_t)slot * STAGE_BYTES);
        const uint64_t bd = sw128_kmajor_desc(bres + (size_t)b * p.N * 128);
        const uint32_t dcol = tmem + (uint32_t)(2 * k + buf) * p.width;
        mma_mxf4(dcol, ad, bd, id0, first ? 0u : 1u, sfa, sfb);
        mma_mxf4(dcol, ad + 2, bd + 2, id2, 1u, sfa | hi, sfb | hi);
        mma_mxf4(dcol, ad + 4, bd + 4, id0, 1u, sfa + 4u, sfb + 2u);
        mma_mxf4(dcol, ad + 6, bd + 6, id2, 1u, (sfa + 4u) | hi, (sfb + 2u) | hi);
        mma_commit(&empty[slot]);
        mma_commit(&sffree[r]);
        if (last) mma_commit(&accfull[2 * k + buf]);
        if ((slot += nm) >= S) slot -= S, ++round;
        if ((r += nm) >= SFR) r -= SFR, ++rround;
        set = (set + nm) & 7;
        b += nm;
        while (b >= nst) b -= nst;
        s += nm;
        while (s >= nst) s -= nst, ++seg;
      }
      // every MMA issued has completed before the CTA frees its tensor memory
      mma_commit(&drain[k]);
      mbar_wait(&drain[k], 0, abort_flag, 200000000ull);
    }
  }
  if (warp < 4) {
    // ---------------- epilogue (warps 0-3): rows of the tile, one per thread ----------------
    // Whole tiles are stored at once; a tile shared with other CTAs (at most this CTA's first and
    // last) is published right after its partial sums are stored, and its last contributor adds
    // every contributor's partial in CTA order. (Publishing both at the end instead measured
    // slower: the two tickets and reductions then pile up on the same late CTAs.)
    const int r = warp * 32 + lane;  // row within the tile = tensor-memory lane
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    bool waited = false, ok = true;
    const uint32_t prank = p.pair ? cluster_rank() : 0u;
    float *pairbuf = reinterpret_cast<float *>(base + p.pair_off);
    if (p.pair) {
      cluster_wait();
      cluster_phase0 = true;
    }
    uint32_t ph = 0;  // phase bit of accfull[issuer][buffer]
    int seg = 0;
    for (int i = 0; i < n && ok;) {
      const int64_t u = u0 + i;
      const int t = (int)(u / p.nst), s0 = (int)(u % p.nst);
      const int len = (p.nst - s0) < (n - i) ? (p.nst - s0) : (n - i);
      const bool whole = s0 == 0 && len == p.nst;
      const int buf = seg & 1;
      // issuers with a unit in this segment (units i .. i + len - 1, issuer k has i = k mod nmma)
      const uint32_t contrib = p.nmma == 1 ? 1u : len >= 2 ? 3u : (1u << (i & 1));
      i += len;
      for (int k = 0; k < 2; ++k)
        if (contrib >> k & 1u) {
          const int a = 2 * k + buf;
          ok = ok && mbar_wait(&accfull[a], (ph >> a) & 1u, abort_flag);  // no sleep: the tail is latency
          ph ^= 1u << a;
        }
      if (!ok) break;
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
      float mine[MAX_M];
#pragma unroll
      for (int q = 0; q < MAX_M; ++q) mine[q] = 0.f;
      for (int mm = 0; mm < p.m; ++mm) {
        float acc = 0.f;
        for (int k = 0; k < 2; ++k)
          if (contrib >> k & 1u) {
            float v[8];  // token mm's eight pieces in issuer k's accumulator
            tmem_ld_x8(tmem + lane_base + (uint32_t)(2 * k + buf) * p.width + 8u * (uint32_t)mm, v);
            acc += ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
          }
        if (whole) {
          if (row < p.rows) {
            const float yv = acc * rs;
            store_f32(p.y, mm * p.ldy_m + row, p.ydt, yv);
            for (int cp = 0; cp < p.ncopy; ++cp) store_f32(p.ycopy[cp], mm * p.ldy_m + row, p.ydt, yv);
          }
        } else if (p.pair) {
          if (prank == 1u) st_cluster_f32(map_rank(smem_u32(pairbuf + mm * TM + r), 0u), acc);
#pragma unroll
          for (int q = 0; q < MAX_M; ++q)
            if (q == mm) mine[q] = acc;
        } else {
          mypart[(size_t)mm * TM + r] = acc;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty[buf]);
      ++seg;
      if (whole) continue;
      if (p.pair) {
        // second half: publish this thread's pushes; first half: add them after its own sums
        if (prank == 1u) {
          mbar_arrive_cluster(map_rank(smem_u32(pairbar), 0u));
        } else {
          ok = mbar_wait_cluster(pairbar, 0u, abort_flag);
          if (ok && row < p.rows) {
            for (int mm = 0; mm < p.m; ++mm) {
              float mv = 0.f;
#pragma unroll
              for (int q = 0; q < MAX_M; ++q)
                if (q == mm) mv = mine[q];
              const float yv = (mv + pairbuf[mm * TM + r]) * rs;
              store_f32(p.y, mm * p.ldy_m + row, p.ydt, yv);
              for (int cp = 0; cp < p.ncopy; ++cp) store_f32(p.ycopy[cp], mm * p.ldy_m + row, p.ydt, yv);
            }
          }
        }
        continue;
      }
      // (the barrier orders every epilogue thread's partial stores before thread 0's fence, which
      // is cumulative: one gpu-scope fence and the acq_rel ticket publish them all, and the
      // barrier after the ticket orders the winner's loads after thread 0's acquire)
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
          float sum[MAX_M];
#pragma unroll
          for (int q = 0; q < MAX_M; ++q) sum[q] = 0.f;
          for (int c0 = cf; c0 <= cl; c0 += 4) {  // four contributors' loads in flight, summed in CTA order
            float v[4][MAX_M];
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              const int cc = c0 + jj;
              const int ee = cc <= cl && (unit_start(p, cc) / p.nst == t) ? 0 : 1;
              const float *src = p.part + ((size_t)cc * 2 + ee) * p.m * TM + r;
#pragma unroll
              for (int q = 0; q < MAX_M; ++q) v[jj][q] = (cc <= cl && q < p.m) ? __ldcg(src + (size_t)q * TM) : 0.f;
            }
#pragma unroll
            for (int jj = 0; jj < 4; ++jj)
#pragma unroll
              for (int q = 0; q < MAX_M; ++q) sum[q] += v[jj][q];
          }
#pragma unroll
          for (int q = 0; q < MAX_M; ++q) {
            if (q >= p.m) break;
            const float yv = sum[q] * rs;
            store_f32(p.y, q * p.ldy_m + row, p.ydt, yv);
            for (int cp = 0; cp < p.ncopy; ++cp) store_f32(p.ycopy[cp], q * p.ldy_m + row, p.ydt, yv);
          }
        }
        if (threadIdx.x == EPI_WARP0 * 32) p.tickets[t] = 0u;  // ready for the next call
      }
      epi_sync();
    }
  }
  tc_fence_before();
  tmem_sync();
  tc_fence_after();
  if (warp == MMA_WARP0) tmem_dealloc(tmem, p.tmem_cols);
  if (p.pair) {
    if (!cluster_phase0) cluster_wait();
    cluster_arrive();
    cluster_wait();
  }
}

// Shared-memory layout and even ring depth (stages == 0: the resident slots do not fit), and
// the tensor-memory columns: four accumulators of `width` ([issuer][buffer]), SFR sets of 8 SFA
// columns, 4 SFB columns per resident slot (256 or 512 columns; one CTA per SM).
struct Layout {
  int stages, nb;
  uint32_t b_off, sfb_off, sfa_off, pair_off, bar_off;
  uint32_t width, sfa_col, sfb_col, tmem_cols;
  size_t smem;
};

static Layout layout_for(int64_t units, int grid, int nst, int N) {
  Layout l = {};
  const int64_t nmax = (units + grid - 1) / grid;
  l.nb = (int)(nmax < nst ? nmax : nst);
  l.width = N <= 16 ? 16u : 32u;
  l.sfa_col = 4 * l.width;
  l.sfb_col = l.sfa_col + 8 * SFR;
  const uint32_t need = l.sfb_col + 4u * (uint32_t)l.nb;
  if (need > 512) return Layout{};
  l.tmem_cols = need <= 256 ? 256u : 512u;
  const size_t bbytes = (size_t)l.nb * N * 128, sfbbytes = (size_t)(l.nb - 1) * N * 16 + 512;
  const size_t sfabytes = (size_t)SFR * 1024;
  const size_t pairbytes = (size_t)MAX_M * TM * 4;
  auto total = [&](int s) {
    const size_t bars = 8 * (2 * (size_t)s + 2 * SFR + 4 + 2 + 2 + l.nb + 1) + 16;
    return 1024 + (size_t)s * STAGE_BYTES + bbytes + sfbbytes + sfabytes + pairbytes + bars;
  };
  // one CTA per SM (shared memory above half the SM's): two CTAs of one grid on an SM would
  // split its bandwidth while another SM idles (measured: a ~5 us tail at c2 with ~113 KB CTAs)
  int s = 0;
  while (s + 2 <= MAX_STAGES && total(s + 2) <= (size_t)SMEM_MAX) s += 2;
  if (s < 2) return Layout{};
  l.stages = s;
  l.b_off = (uint32_t)s * STAGE_BYTES;
  l.sfb_off = l.b_off + (uint32_t)bbytes;
  l.sfa_off = l.sfb_off + (uint32_t)sfbbytes;
  l.pair_off = l.sfa_off + (uint32_t)sfabytes;
  l.bar_off = l.pair_off + (uint32_t)pairbytes;
  l.smem = total(s);
  if (l.smem < 116 * 1024) l.smem = 116 * 1024;
  return l;
}

// Pair split: an even stage count and two CTAs per tile fitting one wave.
static bool pair_split(int64_t ntiles, int nst, int sms) { return nst % 2 == 0 && 2 * ntiles <= sms; }

// The grid a call gets: two CTAs per tile (pair split) or one persistent CTA per SM.
static int grid_for(int64_t ntiles, int nst, int sms) {
  const int64_t units = ntiles * nst;
  return pair_split(ntiles, nst, sms) ? (int)(2 * ntiles) : (int)(units < sms ? units : sms);
}

template <int SMODE, bool XBF16>
static int32_t launch_t(const LinearArgs &a, const Workspace &w, cudaStream_t stream) {
  int sms = 0;
  B200_CUDA_TRY(device_sms(&sms));
  Params p;
  memset(&p, 0, sizeof(p));
  p.rows = a.rows;
  p.cols = a.cols;
  p.nst = (int)(a.cols / KS);
  p.ntiles = (int)((a.rows + TM - 1) / TM);
  p.units = (int64_t)p.ntiles * p.nst;
  p.pair = pair_split(p.ntiles, p.nst, sms) ? 1 : 0;
  p.grid = grid_for(p.ntiles, p.nst, sms);
  p.m = (int)a.m;
  p.N = 8 * p.m;
  const Layout l = layout_for(p.units, p.grid, p.nst, p.N);
  if (l.stages == 0) return b200_set_error(B200_ERR_UNSUPPORTED, "mx decode: x pieces do not fit shared memory");
  p.stages = l.stages;
  p.nb = l.nb;
  p.b_off = l.b_off;
  p.sfb_off = l.sfb_off;
  p.sfa_off = l.sfa_off;
  p.pair_off = l.pair_off;
  p.bar_off = l.bar_off;
  p.width = l.width;
  p.sfa_col = l.sfa_col;
  p.sfb_col = l.sfb_col;
  p.tmem_cols = l.tmem_cols;
  // two issuers unless a CTA wraps around K with an odd stage count (a resident slot would then
  // be used by both issuers, and its scale copy is ordered only within one issuer's stream)
  const int64_t nmax = (p.units + p.grid - 1) / p.grid;
  p.nmma = (nmax <= p.nst || p.nst % 2 == 0) ? 2 : 1;
  // kind::mxf4: A and B E2M1 (format 1), E8M0 scales, M = 128, N = 8 m
  p.idesc = (1u << 7) | (1u << 10) | ((uint32_t)(p.N >> 3) << 17) | (1u << 23) | ((uint32_t)(TM >> 4) << 24);
  p.x = static_cast<const uint16_t *>(a.x);
  p.ldx = a.ldx;
  p.scales = static_cast<const uint8_t *>(a.scales);
  p.nblk = a.nblk;
  p.rscale = a.scales;
  p.sdt = a.sdt;
  p.y = a.y;
  p.ydt = a.ydt;
  p.ldy_m = a.ldy_m;
  p.ncopy = a.ncopy;
  for (int i = 0; i < 7; ++i) p.ycopy[i] = i < a.ncopy ? a.ycopy[i] : nullptr;
  p.part = w.part;
  p.tickets = w.tickets;

  CUtensorMap tmw;
  const uint64_t row_bytes = (uint64_t)a.cols / 2;
  if (int32_t rc = make_tma_2d(&tmw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w, row_bytes, (uint64_t)a.rows, row_bytes, 128, TM,
                               CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  B200_CUDA_TRY((ensure_dynamic_smem<mxs_kernel<SMODE, XBF16>>(SMEM_MAX)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.grid);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = l.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  unsigned nattr = 0;
  if (a.flags & B200_FLAG_PDL) {
    attrs[nattr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[nattr++].val.programmaticStreamSerializationAllowed = 1;
  }
  if (p.pair) {
    attrs[nattr].id = cudaLaunchAttributeClusterDimension;
    attrs[nattr].val.clusterDim.x = 2;
    attrs[nattr].val.clusterDim.y = 1;
    attrs[nattr++].val.clusterDim.z = 1;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = nattr;
  B200_CUDA_TRY(cudaLaunchKernelEx(&cfg, mxs_kernel<SMODE, XBF16>, tmw, p));
  return B200_OK;
}

}  // namespace mxs

// FP4 weights, 1..4 tokens, and the resident x pieces fit (checked against the grid the call
// would get); the rest of mx_supported's conditions hold for the caller.
bool mxs_supported(const LinearArgs &a) {
  using namespace mxs;
  if (a.fmt != B200_FMT_FP4_E2M1 || a.m < 1 || a.m > MAX_M) return false;
  if (mx::scale_mode(a) == SM_E8M0 && (uintptr_t)a.scales % 8 != 0) return false;
  int sms = 0;
  if (device_sms(&sms) != cudaSuccess) return false;
  const int nst = (int)(a.cols / KS);
  const int64_t ntiles = (a.rows + TM - 1) / TM;
  const int64_t units = ntiles * (int64_t)nst;
  return layout_for(units, grid_for(ntiles, nst, sms), nst, 8 * (int)a.m).stages != 0;
}

// Whether the automatic path should take this kernel over the mma.sync decode GEMV: only when
// every CTA streams enough stages to amortise the fixed costs of a call (after the previous
// kernel completes: the x load, queued behind the weight stream, and its conversion, ~2.5 us;
// after the last unit: the epilogue and the pair or ticket reduction, ~2.5 us). Measured, FP4
// E8M0 bf16, CUDA-graph replay with PDL, stream-K units per CTA in brackets, this kernel vs
// the mma.sync kernels: 57344 x 8192 [97] M=1 45.6 vs 49.0 us, M=2 48.8 vs 61.1, M=4 56.3 vs
// 92.6; 8192 x 28672 [48, pair split] M=1 30.2 vs 36.2, M=2 33.8 vs 114.4, M=4 48.2 vs 44.1;
// 10240 x 8192 [18] M=1 16.7 vs 15.8; 8192 x 8192 [14, pair split] M=1 12.4 vs 10.6, M=2 14.3
// vs 13.1; 7168 x 8192 [pair split] M=1 12.1 vs 10.1.
bool mx_preferred(const LinearArgs &a) {
  using namespace mxs;
  if (!mxs_supported(a)) return false;
  int sms = 0;
  if (device_sms(&sms) != cudaSuccess) return false;
  const int64_t units = ((a.rows + TM - 1) / TM) * (a.cols / KS);
  const int64_t grid = units < sms ? units : sms;
  const int64_t per_cta = (units + grid - 1) / grid;
  return a.m <= 2 ? per_cta >= 32 : per_cta >= 64;
}

int32_t launch_mxs(const LinearArgs &a, const mx::Workspace &w, cudaStream_t stream) {
  using namespace mxs;
  const bool bf = a.xdt == B200_DT_BF16;
  switch (mx::scale_mode(a)) {
    case SM_E8M0: return bf ? launch_t<SM_E8M0, true>(a, w, stream) : launch_t<SM_E8M0, false>(a, w, stream);
    case SM_ROW: return bf ? launch_t<SM_ROW, true>(a, w, stream) : launch_t<SM_ROW, false>(a, w, stream);
    default: return bf ? launch_t<SM_NONE, true>(a, w, stream) : launch_t<SM_NONE, false>(a, w, stream);
  }
}

}  // namespace b200
