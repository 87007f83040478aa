// gemv.cu -- streamed decode GEMV for M <= 2 (the M=1 / M=2 path of linalg.matvec / matmul).
//
//   y[m, n] = sum_k x[m, k] * dequant(W)[n, k]
//
// Replaces the reference's one-column matrix path over a packed operand (tinygrad-dx12
// src/tinygrad_dx12/codegen/linalg.py:226-245 -> renderer/linalg.py) with the decode of
// src/tinygrad_dx12/codegen/decomp/dx12.py:69-106 fused in registers.
//
// Structure (Blackwell-native streaming):
//   * persistent CTAs (as many per SM as fit); CTA c owns a contiguous range of 32-row blocks;
//   * the last warp's lane 0 is a TMA producer: for each row block it streams 32 rows x 512
//     payloads per stage (256 B/row for 4-bit, 384 B/row for 6-bit) plus the stage's per-32
//     block scales (or a 16-byte box of its 64..512-payload group scales) into a shared-memory
//     ring (~80 KB in flight per CTA, no registers),
//     signalled by mbarrier transaction counts; it starts before the programmatic-dependency
//     wait because weights and scales are parameters, not outputs of the previous kernel;
//   * warps 0-7 (0-15 when no CTA takes more than one row block) consume: four warps per
//     stage, one 128-payload chunk each. A lane reads its 32-payload blocks of rows g, g+8,
//     g+16, g+24 from shared memory, decodes them to exact
//     fp16 (gemv_tc.cuh) and feeds two independent mma.sync m16n8k16 chains with the
//     block-diagonal activation operand, so every accumulator column is one block's partial
//     sum, scaled in fp32 (exact for every scale dtype);
//   * x is staged once per CTA as fp16 (power-of-two prescale when bf16 would overflow);
//   * per row block the consumer warps reduce through shared memory and store y.
// All mbarrier waits are bounded; on give-up the kernel flags the device error word and
// returns without hanging.
#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"
#include "gemv_tc.cuh"

namespace b200 {

int32_t gemv_device_error(unsigned int *v, bool clear) {
  B200_CUDA_TRY(tu_device_error(v, clear));
  return B200_OK;
}

namespace gemvs {
using namespace gemv;

// NC consumer warps (8 or 16) plus one TMA producer warp; the consumers form NC / CPS groups and
// group q takes the stages st with st % (NC / CPS) == q.
template <int NC>
__host__ __device__ constexpr int threads() {
  return (NC + 1) * 32;
}
constexpr int CPS = 4;               // 128-payload chunks per stage (one per consumer warp of a group)
constexpr int KSTAGE = CPS * CHUNK;  // payloads per row per stage (512)
constexpr int RB = 32;               // rows per block: two m16 row groups per lane

template <int BITS>
__host__ __device__ constexpr int wrow() {  // packed bytes per row per stage
  return KSTAGE * BITS / 8;
}
__host__ __device__ constexpr int slot_bytes(int bits, int sesz) {
  return ((RB * KSTAGE * bits / 8 + RB * (KSTAGE / 32) * sesz) + 127) / 128 * 128;
}
template <int BITS>
__host__ __device__ constexpr int ring_stages() {  // ~80 KB of packed bytes in flight per CTA
  return BITS == 4 ? 10 : 6;
}
template <int SK>
__host__ __device__ constexpr int scale_esz() {
  return SK == SK_E8M0 ? 1 : SK == SK_F16 || SK == SK_BF16 ? 2 : SK == SK_F32 ? 4 : 0;
}

// E8M0 byte -> 2^(b-127) as float32, branch-free: b=0 is the subnormal 2^-127, b=255 is NaN.
__device__ __forceinline__ float e8m0_fast(uint32_t b) {
  const uint32_t bits = b == 0xFFu ? 0x7FC00000u : max(b << 23, 0x00400000u);
  return __uint_as_float(bits);
}

template <int SK>
__device__ __forceinline__ float smem_scale(const uint8_t *s) {
  if constexpr (SK == SK_F16) return __half2float(*reinterpret_cast<const __half *>(s));
  else if constexpr (SK == SK_BF16) return __uint_as_float((uint32_t)*reinterpret_cast<const uint16_t *>(s) << 16);
  else if constexpr (SK == SK_F32) return *reinterpret_cast<const float *>(s);
  else return 1.f;
}

template <int SK>
__device__ __forceinline__ void smem_scale_pair(const uint8_t *s, float &s0, float &s1) {
  if constexpr (SK == SK_E8M0) {
    const uint32_t v = *reinterpret_cast<const uint16_t *>(s);
    s0 = e8m0_fast(v & 0xFFu);
    s1 = e8m0_fast(v >> 8);
  } else if constexpr (SK == SK_F16) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(s));
    s0 = f.x, s1 = f.y;
  } else if constexpr (SK == SK_BF16) {
    const uint32_t v = *reinterpret_cast<const uint32_t *>(s);
    s0 = __uint_as_float(v << 16), s1 = __uint_as_float(v & 0xFFFF0000u);
  } else if constexpr (SK == SK_F32) {
    const float2 f = *reinterpret_cast<const float2 *>(s);
    s0 = f.x, s1 = f.y;
  } else {
    s0 = s1 = 1.f;
  }
}

// One lane's chunk for four rows (two m16 row groups) and its accumulator-column scales.
template <int BITS>
struct Chunk4 {
  Chunk<BITS> lo, hi;  // rows g, g+8 | rows g+16, g+24
};

// E8M0 bytes -> float32 scales, four per word (byte i -> out[i]). Bytes 1..254 are 2^(b-127) =
// float bits b << 23; bytes 0 (2^-127, subnormal) and 255 (NaN) take the exact conversion, a
// warp-uniform branch that ordinary scales never take. The zero-byte test of v and of ~v
// ((v - 0x01..) & ~v & 0x80..) finds both without per-byte compares.
// With `ordinary` (the caller's B200_FLAG_SCALES_ORDINARY: no byte 0 or 255 in the matrix) the
// test is skipped.
__device__ __forceinline__ void e8m0_scales8(uint32_t v01, uint32_t v23, float (&lo)[4], float (&hi)[4],
                                             bool ordinary) {
  constexpr uint32_t K1 = 0x01010101u, H = 0x80808080u;
  bool exact = false;
  if (!ordinary) {  // kernel parameter: uniform
    const uint32_t sp = (((v01 - K1) & ~v01) | ((~v01 - K1) & v01) | ((v23 - K1) & ~v23) | ((~v23 - K1) & v23)) & H;
    exact = __any_sync(0xffffffffu, sp != 0u);
  }
  if (exact) {
#pragma unroll
    for (int i = 0; i < 4; ++i) lo[i] = e8m0_fast((v01 >> (8 * i)) & 0xFFu), hi[i] = e8m0_fast((v23 >> (8 * i)) & 0xFFu);
  } else {
    lo[0] = __uint_as_float((v01 & 0xFFu) << 23), lo[1] = __uint_as_float((v01 & 0xFF00u) << 15);
    lo[2] = __uint_as_float((v01 & 0xFF0000u) << 7), lo[3] = __uint_as_float((v01 & 0xFF000000u) >> 1);
    hi[0] = __uint_as_float((v23 & 0xFFu) << 23), hi[1] = __uint_as_float((v23 & 0xFF00u) << 15);
    hi[2] = __uint_as_float((v23 & 0xFF0000u) << 7), hi[3] = __uint_as_float((v23 & 0xFF000000u) >> 1);
  }
}

// The MMAs of one chunk, then its per-block scales: for E8M0, `e01` / `e23` hold the raw scale
// bytes (rows g, g+8 | g+16, g+24; blocks blk, blk+1 of each) and are converted after the MMAs
// are issued, so the conversion fills the MMA latency instead of preceding it.
template <int FMT, int SK>
__device__ __forceinline__ void compute_chunk4(const Chunk4<Fmt<FMT>::bits> &r, const __half *xblk, float (&acc)[4],
                                               uint32_t e01 = 0u, uint32_t e23 = 0u, bool ordinary = false) {
  constexpr int BITS = Fmt<FMT>::bits;
  float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int u = 0; u < 4; ++u) {  // 8-payload unit u of this lane's block
    uint32_t pa[4], pb[4], pc[4], pd[4];
    if constexpr (BITS == 4) {
      decode8_4bit<FMT>(r.lo.a[u], pa);
      decode8_4bit<FMT>(r.lo.b[u], pb);
      decode8_4bit<FMT>(r.hi.a[u], pc);
      decode8_4bit<FMT>(r.hi.b[u], pd);
    } else {
      const int bit = 48 * u, wi = bit >> 5, sh = bit & 31;  // the unit lies in words wi, wi+1
      decode8_6bit<FMT>((((uint64_t)r.lo.a[wi + 1] << 32) | r.lo.a[wi]) >> sh, pa);
      decode8_6bit<FMT>((((uint64_t)r.lo.b[wi + 1] << 32) | r.lo.b[wi]) >> sh, pb);
      decode8_6bit<FMT>((((uint64_t)r.hi.a[wi + 1] << 32) | r.hi.a[wi]) >> sh, pc);
      decode8_6bit<FMT>((((uint64_t)r.hi.b[wi + 1] << 32) | r.hi.b[wi]) >> sh, pd);
    }
    const uint4 xv = *reinterpret_cast<const uint4 *>(xblk + 8 * u);  // shared by both groups
    const uint32_t a0[4] = {pa[0], pb[0], pa[1], pb[1]}, a1[4] = {pa[2], pb[2], pa[3], pb[3]};
    const uint32_t c0[4] = {pc[0], pd[0], pc[1], pd[1]}, c1[4] = {pc[2], pd[2], pc[3], pd[3]};
    mma16816(d0, a0, xv.x, xv.y);
    mma16816(d1, c0, xv.x, xv.y);
    mma16816(d0, a1, xv.z, xv.w);
    mma16816(d1, c1, xv.z, xv.w);
  }
  // d = {D[g][2t], D[g][2t+1], D[g+8][2t], D[g+8][2t+1]}: per-block partial sums
  if constexpr (SK == SK_NONE || SK == SK_ROW) {
    acc[0] += d0[0] + d0[1];
    acc[1] += d0[2] + d0[3];
    acc[2] += d1[0] + d1[1];
    acc[3] += d1[2] + d1[3];
  } else if constexpr (SK == SK_E8M0) {
    float lo[4], hi[4];
    e8m0_scales8(e01, e23, lo, hi, ordinary);
    acc[0] = fmaf(d0[0], lo[0], fmaf(d0[1], lo[1], acc[0]));
    acc[1] = fmaf(d0[2], lo[2], fmaf(d0[3], lo[3], acc[1]));
    acc[2] = fmaf(d1[0], hi[0], fmaf(d1[1], hi[1], acc[2]));
    acc[3] = fmaf(d1[2], hi[2], fmaf(d1[3], hi[3], acc[3]));
  } else {
    acc[0] = fmaf(d0[0], r.lo.sa0, fmaf(d0[1], r.lo.sa1, acc[0]));
    acc[1] = fmaf(d0[2], r.lo.sb0, fmaf(d0[3], r.lo.sb1, acc[1]));
    acc[2] = fmaf(d1[0], r.hi.sa0, fmaf(d1[1], r.hi.sa1, acc[2]));
    acc[3] = fmaf(d1[2], r.hi.sb0, fmaf(d1[3], r.hi.sb1, acc[3]));
  }
}

template <int BITS>
__device__ __forceinline__ void read_rows(Chunk<BITS> &c, const uint8_t *base, int ra, int rb, int sub, int t) {
  constexpr int WR = wrow<BITS>();
  if constexpr (BITS == 4) {
    const uint4 ua = *reinterpret_cast<const uint4 *>(base + ra * WR + sub * 64 + 16 * t);
    const uint4 ub = *reinterpret_cast<const uint4 *>(base + rb * WR + sub * 64 + 16 * t);
    c.a[0] = ua.x, c.a[1] = ua.y, c.a[2] = ua.z, c.a[3] = ua.w;
    c.b[0] = ub.x, c.b[1] = ub.y, c.b[2] = ub.z, c.b[3] = ub.w;
  } else {  // two 192-byte boxes per stage: chunks 0,1 in the first, 2,3 in the second
    const uint8_t *hb = base + (sub >> 1) * RB * (WR / 2) + (sub & 1) * 96 + 24 * t;
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      const uint2 ua = *reinterpret_cast<const uint2 *>(hb + ra * (WR / 2) + 8 * q);
      const uint2 ub = *reinterpret_cast<const uint2 *>(hb + rb * (WR / 2) + 8 * q);
      c.a[2 * q] = ua.x, c.a[2 * q + 1] = ua.y, c.b[2 * q] = ub.x, c.b[2 * q + 1] = ub.y;
    }
  }
}

struct StreamParams {
  Params p;
  int64_t nrb;  // row blocks
  int nst;      // stages per row block
  int xbf16;
  int ordinary;  // B200_FLAG_SCALES_ORDINARY: E8M0 scale bytes known to lie in 1..254
  // Staged scales: gshift = log2(block / 32) (0: one scale per 32-payload block; 1..4: group
  // scales of 64..512 payloads). Each stage loads a box of sbe scales per row that starts at a
  // multiple of sbe, since a TMA box is at least 16 bytes wide (four fp16 group-128 scales
  // are 8): the stage's first scale sits at offset (st * (16 >> gshift)) % sbe of the box.
  int gshift, sbe;
  uint32_t tx;  // bytes per stage (codes + scale box)
};

// stage x[m][K] as fp16 in decode pair order (consumer threads only). Each thread issues up to
// XB 16-byte loads before converting any, so the staging costs about one memory round trip.
template <int FMT, int NC>
__device__ __forceinline__ bool stage_x_consumers(const Params &p, __half *xs, int K, int tid, bool xbf16,
                                                  float prescale) {
  constexpr int XB = 4;
  bool ok = true;
  const int n8 = K >> 3;
  for (int mm = 0; mm < (int)p.m; ++mm) {
    const uint4 *src = reinterpret_cast<const uint4 *>((const uint16_t *)p.x + (int64_t)mm * p.ldx);
    for (int k0 = tid; k0 < n8; k0 += XB * NC * 32) {
      uint4 u[XB];
#pragma unroll
      for (int j = 0; j < XB; ++j) {
        const int k8 = k0 + j * NC * 32;
        u[j] = k8 < n8 ? __ldg(src + k8) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int j = 0; j < XB; ++j) {
        const int k8 = k0 + j * NC * 32;
        if (k8 >= n8) break;
        const uint32_t wv[4] = {u[j].x, u[j].y, u[j].z, u[j].w};
        uint32_t hh[4];  // fp16 pairs (elements 2i, 2i+1)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (xbf16 && prescale == 1.f) {
            // one f32x2 -> f16x2 convert per pair; |x| >= 65536 (bf16 magnitude bits >= 0x4780:
            // the largest bf16 below, 65280, is finite in fp16) or Inf / NaN sets bit 15 of a
            // 16-bit lane of (bits & 0x7FFF) + 0x3880, with no carry into the other lane
            const __half2 h2 = __floats2half2_rn(__uint_as_float(wv[i] << 16), __uint_as_float(wv[i] & 0xFFFF0000u));
            hh[i] = *reinterpret_cast<const uint32_t *>(&h2);
            ok = ok && (((wv[i] & 0x7FFF7FFFu) + 0x38803880u) & 0x80008000u) == 0u;
          } else if (xbf16) {
            const __half lo = __float2half_rn(__uint_as_float(wv[i] << 16) * prescale);
            const __half hi = __float2half_rn(__uint_as_float(wv[i] & 0xFFFF0000u) * prescale);
            ok = ok && !(__hisinf(lo) | __hisinf(hi));
            hh[i] = (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
          } else {
            hh[i] = wv[i];
          }
        }
        uint4 o;
        if constexpr (pairs_04<FMT>())  // (e0, e4), (e1, e5), (e2, e6), (e3, e7)
          o = make_uint4(__byte_perm(hh[0], hh[2], 0x5410), __byte_perm(hh[0], hh[2], 0x7632),
                         __byte_perm(hh[1], hh[3], 0x5410), __byte_perm(hh[1], hh[3], 0x7632));
        else
          o = make_uint4(hh[0], hh[1], hh[2], hh[3]);
        *reinterpret_cast<uint4 *>(xs + (int64_t)mm * K + 8 * k8) = o;
      }
    }
  }
  return ok;
}

template <int NC>
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"r"(NC * 32) : "memory");
}

template <int FMT, int SK, int NC, bool GS>
__global__ void __launch_bounds__(threads<NC>(), 1)
    gemv_stream_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tms,
                       StreamParams sp) {
  constexpr int BITS = Fmt<FMT>::bits;
  constexpr int WR = wrow<BITS>();
  constexpr int SESZ = scale_esz<SK>();
  constexpr bool GROUP = SESZ > 0;
  constexpr int SLOT = slot_bytes(BITS, SESZ);
  constexpr int STAGES = ring_stages<BITS>();
  constexpr uint32_t TX = RB * WR + (GROUP ? RB * (KSTAGE / 32) * SESZ : 0);
  const Params &p = sp.p;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t *ring = (uint8_t *)(((uintptr_t)smem_raw + 127) & ~(uintptr_t)127);
  uint64_t *full = reinterpret_cast<uint64_t *>(ring + STAGES * SLOT);
  uint64_t *empty = full + STAGES;
  volatile uint32_t *abort_flag = reinterpret_cast<uint32_t *>(empty + STAGES);
  volatile uint32_t *ovf_flag = abort_flag + 1;
  // 16-byte aligned: zslot and xs below take 128-bit stores
  float *red = reinterpret_cast<float *>(((uintptr_t)(empty + STAGES + 1) + 15) & ~(uintptr_t)15);  // [2][NC][2][RB]
  __half *zslot = reinterpret_cast<__half *>(red + 2 * NC * 2 * RB);  // CHUNK zeros
  __half *xs = zslot + CHUNK;                                              // [m][K]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = (int)p.cols;
  const int64_t rb_begin = (sp.nrb * blockIdx.x) / gridDim.x, rb_end = (sp.nrb * (blockIdx.x + 1)) / gridDim.x;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], CPS);
    }
    *abort_flag = 0;
    *ovf_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == NC) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tmap(&tmw);
      if constexpr (GROUP) prefetch_tmap(&tms);
      int64_t gs = 0;
      int slot = 0;        // gs % STAGES, kept incrementally (no 64-bit division in the loop)
      uint32_t round = 0;  // (gs / STAGES) & 1
      for (int64_t rbk = rb_begin; rbk < rb_end; ++rbk) {
        for (int st = 0; st < sp.nst; ++st, ++gs, (++slot == STAGES ? (slot = 0, round ^= 1u) : 0u)) {
          if (gs >= STAGES && !mbar_wait(&empty[slot], round ^ 1u, abort_flag)) continue;
          if (*abort_flag) continue;
          uint8_t *dst = ring + slot * SLOT;
          mbar_arrive_expect_tx(&full[slot], GS ? sp.tx : TX);
          if constexpr (BITS == 4) {
            tma_load_2d(dst, &tmw, st * WR, (int32_t)(rbk * RB), &full[slot]);
          } else {  // 384 B per row: two 192-byte boxes
            tma_load_2d(dst, &tmw, st * WR, (int32_t)(rbk * RB), &full[slot]);
            tma_load_2d(dst + RB * (WR / 2), &tmw, st * WR + WR / 2, (int32_t)(rbk * RB), &full[slot]);
          }
          if constexpr (GROUP)
            tma_load_2d(dst + RB * WR, &tms, GS ? (st * (16 >> sp.gshift)) & ~(sp.sbe - 1) : st * (KSTAGE / 32),
                        (int32_t)(rbk * RB), &full[slot]);
        }
      }
      if (*abort_flag) {  // drain copies still in flight before exiting
        const int64_t first = gs > STAGES ? gs - STAGES : 0;
        for (int64_t q = first; q < gs; ++q)
          mbar_wait(&full[q % STAGES], (uint32_t)((q / STAGES) & 1), abort_flag, 200000000ull);
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  const int g = lane >> 2, t = lane & 3;
  const int cm = t >> 1, cblk = 2 * (t & 1);
  const int sub = warp % CPS;     // chunk within a stage
  const int group = warp / CPS;  // this warp consumes stages st with st % (NC / CPS) == group
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (tid < CHUNK / 8) reinterpret_cast<uint4 *>(zslot)[tid] = make_uint4(0u, 0u, 0u, 0u);
  float prescale = 1.f;
  if (!stage_x_consumers<FMT, NC>(p, xs, K, tid, sp.xbf16 != 0, 1.f)) *ovf_flag = 1;
  consumer_sync<NC>();
  if (*ovf_flag) {  // rare: bf16 beyond fp16 range -> power-of-two prescale so max|x| < 2^15
    float amax = 0.f;
    for (int mm = 0; mm < (int)p.m; ++mm)
      for (int k = tid; k < K; k += NC * 32)
        amax = fmaxf(amax, fabsf(__bfloat162float(((const __nv_bfloat16 *)p.x)[(int64_t)mm * p.ldx + k])));
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) red[warp] = amax;
    consumer_sync<NC>();
    for (int wv = 0; wv < NC; ++wv) amax = fmaxf(amax, red[wv]);
    const int ex = ((__float_as_int(amax) >> 23) & 0xFF) - 127;
    prescale = __int_as_float((127 - (ex - 14)) << 23);
    stage_x_consumers<FMT, NC>(p, xs, K, tid, true, prescale);
    consumer_sync<NC>();
  }

  const int bm = g >> 2;
  const bool owner = (t == (g & 3)) && bm < p.m;
  const __half *xrow = xs + (int64_t)bm * K + 32 * t;
  int slot = 0;        // ring slot of the current stage, kept incrementally
  uint32_t round = 0;  // its phase parity
  int buf = 0;
  for (int64_t rbk = rb_begin; rbk < rb_end; ++rbk) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};  // rows g, g+8, g+16, g+24 for m = cm
    for (int st = 0; st < sp.nst; ++st, (++slot == STAGES ? (slot = 0, round ^= 1u) : 0u)) {
      if ((unsigned)st % (NC / CPS) != (unsigned)group) continue;
      const bool got = mbar_wait(&full[slot], round, abort_flag);
      const uint8_t *base = ring + slot * SLOT;
      Chunk4<BITS> r;
      uint32_t e01 = 0u, e23 = 0u;  // E8M0: raw scale bytes, converted after the chunk's MMAs
      if (got) {
        read_rows<BITS>(r.lo, base, g, g + 8, sub, t);
        read_rows<BITS>(r.hi, base, g + 16, g + 24, sub, t);
        if constexpr (SK == SK_E8M0) {
          const uint8_t *sb = base + RB * WR;
          const int blk = sub * 4 + cblk;
          const uint32_t u0 = *reinterpret_cast<const uint16_t *>(sb + (g * (KSTAGE / 32) + blk));
          const uint32_t u1 = *reinterpret_cast<const uint16_t *>(sb + ((g + 8) * (KSTAGE / 32) + blk));
          const uint32_t u2 = *reinterpret_cast<const uint16_t *>(sb + ((g + 16) * (KSTAGE / 32) + blk));
          const uint32_t u3 = *reinterpret_cast<const uint16_t *>(sb + ((g + 24) * (KSTAGE / 32) + blk));
          e01 = u0 | (u1 << 16), e23 = u2 | (u3 << 16);
        } else if constexpr (GROUP) {
          const uint8_t *sb = base + RB * WR;
          const int blk = sub * 4 + cblk;  // block index within the stage's 16 blocks per row (even)
          if constexpr (!GS) {
            smem_scale_pair<SK>(sb + (g * (KSTAGE / 32) + blk) * SESZ, r.lo.sa0, r.lo.sa1);
            smem_scale_pair<SK>(sb + ((g + 8) * (KSTAGE / 32) + blk) * SESZ, r.lo.sb0, r.lo.sb1);
            smem_scale_pair<SK>(sb + ((g + 16) * (KSTAGE / 32) + blk) * SESZ, r.hi.sa0, r.hi.sa1);
            smem_scale_pair<SK>(sb + ((g + 24) * (KSTAGE / 32) + blk) * SESZ, r.hi.sb0, r.hi.sb1);
          } else {  // blocks blk, blk + 1 share one group scale
            const int gi = ((st * (16 >> sp.gshift)) & (sp.sbe - 1)) + (blk >> sp.gshift);
            r.lo.sa0 = r.lo.sa1 = smem_scale<SK>(sb + (g * sp.sbe + gi) * SESZ);
            r.lo.sb0 = r.lo.sb1 = smem_scale<SK>(sb + ((g + 8) * sp.sbe + gi) * SESZ);
            r.hi.sa0 = r.hi.sa1 = smem_scale<SK>(sb + ((g + 16) * sp.sbe + gi) * SESZ);
            r.hi.sb0 = r.hi.sb1 = smem_scale<SK>(sb + ((g + 24) * sp.sbe + gi) * SESZ);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);  // the slot's data now lives in registers
      if (got) {
        const int chunk = st * CPS + sub;
        compute_chunk4<FMT, SK>(r, owner ? xrow + (int64_t)chunk * CHUNK : zslot, acc, e01, e23, sp.ordinary != 0);
      }
    }
    // ---- reduce this row block over the NC consumer warps and store ----
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 1);
    float *rb = red + buf * (NC * 2 * RB);
    if ((t & 1) == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i) rb[(warp * 2 + cm) * RB + g + 8 * i] = acc[i];
    }
    consumer_sync<NC>();
    if (tid < 2 * RB) {
      const int mm = tid / RB, rr = tid % RB;
      const int64_t n = rbk * RB + rr;
      if (mm < p.m && n < p.rows && !*abort_flag) {
        float s = 0.f;
#pragma unroll
        for (int wv = 0; wv < NC; ++wv) s += rb[(wv * 2 + mm) * RB + rr];
        s *= place_factor<FMT>() / prescale;
        if constexpr (SK == SK_ROW) s *= load_as_f32(p.scales, n * p.nblk, p.sdt);
        store_f32(p.y, mm * p.ldy_m + n * p.ldy_n, p.ydt, s);
        for (int i = 0; i < p.ncopy; ++i) store_f32(p.ycopy[i], mm * p.ldy_m + n * p.ldy_n, p.ydt, s);
      }
    }
    buf ^= 1;
  }
}

template <int BITS, int SESZ, int NC>
static size_t smem_bytes(int64_t m, int64_t cols) {
  return 128 + (size_t)ring_stages<BITS>() * slot_bytes(BITS, SESZ) + 2 * ring_stages<BITS>() * 8 + 8 + 16 +
         2 * NC * 2 * RB * 4 + CHUNK * 2 + (size_t)m * cols * 2;
}

template <int FMT, int SK, int NC, bool GS>
static int32_t launch_t(const LinearArgs &a, cudaStream_t stream) {
  constexpr int BITS = Fmt<FMT>::bits;
  constexpr int SESZ = scale_esz<SK>();
  const size_t smem = smem_bytes<BITS, SESZ, NC>(a.m, a.cols);
  int sms = 0;
  B200_CUDA_TRY(device_sms(&sms));
  B200_CUDA_TRY((ensure_dynamic_smem<gemv_stream_kernel<FMT, SK, NC, GS>>(200 * 1024)));
  int per_sm = 0;
  B200_CUDA_TRY((occupancy_cached<gemv_stream_kernel<FMT, SK, NC, GS>>(&per_sm, threads<NC>(), smem)));
  if (per_sm < 1) return b200_set_error(B200_ERR_UNSUPPORTED, "streamed GEMV: no CTA fits (%zu B smem)", smem);
  CUtensorMap tmw, tms;
  const uint64_t row_bytes = (uint64_t)a.cols * BITS / 8;
  int gshift = 0;  // group scales: block = 32 << gshift payloads
  while (GS && (32 << gshift) < a.block) ++gshift;
  const int gps = (KSTAGE / 32) >> gshift;  // scales per row and stage
  const int sbe = gshift == 0 ? KSTAGE / 32 : (gps * SESZ >= 16 ? gps : 16 / (SESZ > 0 ? SESZ : 1));
  if (int32_t rc = make_tma_2d(&tmw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w, row_bytes, (uint64_t)a.rows, row_bytes,
                               BITS == 4 ? wrow<BITS>() : wrow<BITS>() / 2, RB, CU_TENSOR_MAP_SWIZZLE_NONE))
    return rc;
  if constexpr (SESZ > 0) {
    const CUtensorMapDataType dt = SESZ == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                   : SESZ == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : SK == SK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    if (int32_t rc = make_tma_2d(&tms, dt, a.scales, (uint64_t)a.nblk, (uint64_t)a.rows, (uint64_t)a.nblk * SESZ,
                                 (uint32_t)sbe, RB, CU_TENSOR_MAP_SWIZZLE_NONE))
      return rc;
  } else {
    tms = tmw;
  }
  StreamParams sp;
  Params &p = sp.p;
  p.w = a.w, p.scales = a.scales, p.sdt = a.sdt, p.rows = a.rows, p.cols = a.cols, p.nblk = a.nblk, p.block = a.block;
  p.x = a.x, p.m = a.m, p.ldx = a.m > 1 ? a.ldx : a.cols, p.y = a.y, p.ydt = a.ydt, p.ldy_m = a.ldy_m,
  p.ldy_n = a.ldy_n, p.pdl = 0;
  p.ncopy = a.ncopy;
  for (int i = 0; i < 7; ++i) p.ycopy[i] = i < a.ncopy ? a.ycopy[i] : nullptr;
  sp.nrb = (a.rows + RB - 1) / RB;
  sp.nst = (int)(a.cols / KSTAGE);
  sp.xbf16 = a.xdt == B200_DT_BF16;
  sp.ordinary = (a.flags & B200_FLAG_SCALES_ORDINARY) != 0;
  sp.gshift = gshift;
  sp.sbe = sbe;
  sp.tx = (uint32_t)(RB * wrow<BITS>() + RB * sbe * SESZ);
  const int64_t slots = (int64_t)sms * per_sm;
  const int64_t grid = sp.nrb < slots ? sp.nrb : slots;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(threads<NC>());
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[1];
  attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = (a.flags & B200_FLAG_PDL) ? 1 : 0;
  B200_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_stream_kernel<FMT, SK, NC, GS>, tmw, tms, sp));
  return B200_OK;
}

// 16 consumer warps when no CTA takes more than one row block: a lone row block is latency
// bound and twice the warps halve its stage rounds (FP4, M=1: 1280 x 8192 8.7 -> 6.4 us,
// 4096 x 4096 5.8 -> 4.3 us). CTAs that stream several row blocks keep 8 (16 measured slower:
// 8192 x 8192 10.5 -> 11.4 us, 28672 x 8192 28.9 -> 34 us).
// GS: group scales (block 64..512) in the per-dtype kernels; a separate instantiation keeps the
// per-32 kernels' registers (and two CTAs per SM) as they are
template <int FMT, int SK, bool GS = false>
static int32_t launch_nc(const LinearArgs &a, cudaStream_t stream) {
  int sms = 0;
  B200_CUDA_TRY(device_sms(&sms));
  const int64_t nrb = (a.rows + RB - 1) / RB;
  if (nrb <= sms && smem_bytes<Fmt<FMT>::bits, scale_esz<SK>(), 16>(a.m, a.cols) <= 200 * 1024)
    return launch_t<FMT, SK, 16, GS>(a, stream);
  return launch_t<FMT, SK, 8, GS>(a, stream);
}

template <int FMT>
static int32_t dispatch_sk(const LinearArgs &a, int sk, cudaStream_t stream) {
  switch (sk) {
    case SK_NONE: return launch_nc<FMT, SK_NONE>(a, stream);
    case SK_ROW: return launch_nc<FMT, SK_ROW>(a, stream);
    case SK_E8M0: return launch_nc<FMT, SK_E8M0>(a, stream);
    case SK_F16: return launch_nc<FMT, SK_F16>(a, stream);
    case SK_BF16: return launch_nc<FMT, SK_BF16>(a, stream);
    case SK_F32: return launch_nc<FMT, SK_F32>(a, stream);
    case SK_GROUP:  // the per-dtype kernels with gshift > 0
      return a.sdt == B200_DT_F16    ? launch_nc<FMT, SK_F16, true>(a, stream)
             : a.sdt == B200_DT_BF16 ? launch_nc<FMT, SK_BF16, true>(a, stream)
                                     : launch_nc<FMT, SK_F32, true>(a, stream);
  }
  return b200_set_error(B200_ERR_UNSUPPORTED, "streamed GEMV: scale layout");
}

}  // namespace gemvs

bool gemv_stream_supported(const LinearArgs &a) {
  using namespace gemvs;
  if (!gemv_tc_supported(a)) return false;
  if (a.cols % KSTAGE != 0 || a.cols > (1 << 24)) return false;
  const int sk = gemv::scale_kind(a);
  // group scales wider than 32 (block 64..512): staged per stage like per-32 scales (a TMA box
  // of at least 16 bytes per row); E8M0 group scales stay on the register-ring GEMV
  if (sk == gemv::SK_GROUP) {
    if (!(a.sdt == B200_DT_F16 || a.sdt == B200_DT_BF16 || a.sdt == B200_DT_F32)) return false;
    if (!(a.block == 64 || a.block == 128 || a.block == 256 || a.block == 512)) return false;
  }
  if (sk >= gemv::SK_E8M0) {
    const int esz = dt_size(a.sdt);
    if ((a.nblk * esz) % 16 != 0 || (uintptr_t)a.scales % 16 != 0) return false;
  }
  const int bits = fmt_bits(a.fmt);
  if ((uintptr_t)a.w % 16 != 0 || ((uint64_t)a.cols * bits / 8) % 16 != 0) return false;
  const size_t smem = bits == 4 ? smem_bytes<4, 4, 8>(a.m, a.cols) : smem_bytes<6, 4, 8>(a.m, a.cols);
  return smem <= 200 * 1024;
}

int32_t launch_gemv_stream(const LinearArgs &a, cudaStream_t stream) {
  using namespace gemvs;
  const int sk = gemv::scale_kind(a);
  switch (a.fmt) {
    case B200_FMT_INT4: return dispatch_sk<B200_FMT_INT4>(a, sk, stream);
    case B200_FMT_UINT4: return dispatch_sk<B200_FMT_UINT4>(a, sk, stream);
    case B200_FMT_FP4_E2M1: return dispatch_sk<B200_FMT_FP4_E2M1>(a, sk, stream);
    case B200_FMT_FP6_E2M3: return dispatch_sk<B200_FMT_FP6_E2M3>(a, sk, stream);
    case B200_FMT_FP6_E3M2: return dispatch_sk<B200_FMT_FP6_E3M2>(a, sk, stream);
  }
  return b200_set_error(B200_ERR_INVALID, "unknown packed format %d", a.fmt);
}

}  // namespace b200
