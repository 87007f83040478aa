// skinny.cu -- packed decode GEMM for a few tokens (3 <= M <= 32; up to 64 for the scale layouts
// the tcgen05 GEMM declines), 4-bit formats.
//
//   y[m, n] = sum_k x[m, k] * dequant(W)[n, k]
//
// The small-batch case of the reference's packed matmul (tinygrad-dx12
// src/tinygrad_dx12/codegen/linalg.py:136-223 over dx12.py:69-106 decodes): too many tokens
// for the M <= 2 streamed GEMV, too few for the tcgen05 GEMM, whose CUDA-core dequant costs
// more instructions per weight than an HBM-bound pass can afford.
//
// One CTA owns 128 weight rows and one K slice (split-K keeps every SM busy when N is small):
//   * warp 8, lane 0 streams per stage (512 K) the rows' packed codes (two 128-byte-swizzled
//     TMA boxes), x[0:8*NT, stage] (eight 128-byte-swizzled boxes, rows past M zero-filled)
//     and, for per-32 scales, the stage's scale tile into a shared-memory ring;
//   * warps 0-7 consume: warp w owns rows 16w..16w+15 (the 32-token tile runs warps 0-15, warp
//     w and w+8 sharing rows 16(w%8).. and taking the first / second half of each stage's
//     blocks, then adding their sums through shared memory). ldmatrix hands lane (g, t) payloads
//     8t..8t+7 of one 32-payload block for rows g and g+8; the sm_100a conversions decode them
//     to exact fp16; two mma.sync m16n8k16 per block and token tile give the block's partial
//     sum for 8 tokens, scaled in fp32 by the block's scale (exact for every scale dtype).
//     bf16 x is converted to fp16 in shared memory per stage with a per-token power-of-two
//     prescale (max |x| of the chunk brought to [2^14, 2^15)), undone on the fp32 partials;
//   * with one K slice the CTA stores y; otherwise it writes fp32 partials to a workspace,
//     and the last CTA of the row block (atomic ticket) sums the slices in fixed order and
//     stores y, then resets the ticket.
// Every wait is bounded (sm100.cuh); on give-up the kernel flags the device error word.
#include <map>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"
#define B200_GEMV_TC_NO_ENTRY
#include "gemv_tc.cuh"

namespace b200 {

int32_t skinny_device_error(unsigned int *v, bool clear) {
  B200_CUDA_TRY(tu_device_error(v, clear));
  return B200_OK;
}

namespace skinny {
using namespace gemv;

constexpr int RB = 128;                 // weight rows per CTA (16 per consumer row group)
// Consumer warps: eight row groups of 16 rows. The 32-token tile (one CTA per SM) runs two warps
// per row group, each taking half of every stage's 32-payload blocks, so that the SM keeps 16
// consumer warps (M=32, FP4 E8M0: 52 -> 47 us); the smaller tiles run one warp per row group and
// two CTAs per SM. Wide group scales and per-32 fp32 scales keep one warp per row group: their
// scale registers would not fit the 96 registers that 17 warps leave per thread.
template <int NT, int SK>
__host__ __device__ constexpr int consumers() {
  return NT == 4 && SK != gemv::SK_GROUP && SK != gemv::SK_F32 ? 16 : 8;
}
template <int NT, int SK>
__host__ __device__ constexpr int threads() {
  return (consumers<NT, SK>() + 1) * 32;
}
constexpr int KST = 512;                // payloads per row per stage
constexpr int W_BYTES = RB * KST / 2;   // 4-bit codes: 32 KB per stage
template <int NT>
__host__ __device__ constexpr int ctas_per_sm() {  // two resident CTAs while their rings fit
  return NT <= 2 ? 2 : 1;
}
template <int NT>
__host__ __device__ constexpr int smem_cap() {
  return NT <= 2 ? 108 * 1024 : 210 * 1024;
}

template <int NT>
__host__ __device__ constexpr int x_bytes() {  // 8 boxes of (8*NT tokens x 64 halves)
  return 8 * (8 * NT) * 128;
}
__host__ __device__ constexpr int s_bytes(int esz) { return RB * (KST / 32) * esz; }
template <int NT>
__host__ __device__ constexpr int slot_bytes(int esz) {
  return (W_BYTES + x_bytes<NT>() + s_bytes(esz) + 1023) / 1024 * 1024;
}
template <int NT>
__host__ __device__ constexpr int stages(int esz) {
  return smem_cap<NT>() / slot_bytes<NT>(esz) > 4   ? 4
         : smem_cap<NT>() / slot_bytes<NT>(esz) < 2 ? 2
                                                     : smem_cap<NT>() / slot_bytes<NT>(esz);
}

// Group scales (64..512 payloads, fp16 / bf16 / fp32) staged like the per-32 kinds: per stage
// one 16-byte box of scales per row (TMA boxes are at least 16 bytes wide; four fp16 group-128
// scales are 8), starting at a multiple of the box; the stage's groups begin at offset
// (stage * groups per stage) mod box. SK_GROUP reads group scales from global memory instead
// (other shapes: E8M0 groups, scale rows that are not 16-byte multiples, fp32 group-64).
constexpr int SK_GSTAGED = 16;
// Per-32 E8M0 scales under B200_FLAG_SCALES_ORDINARY (no byte 0 or 255 in the matrix): the same
// kernel with 2^(b-127) taken as float bits b << 23, one shift instead of the exact conversion.
constexpr int SK_E8M0_ORD = 17;
template <int SK>
__host__ __device__ constexpr bool is_e8m0() {
  return SK == gemv::SK_E8M0 || SK == SK_E8M0_ORD;
}

template <int SK>
__host__ __device__ constexpr int tile_esz() {  // staged scale bytes per 32-payload block and row
  return is_e8m0<SK>() || SK == SK_GSTAGED ? 1 : SK == SK_F16 || SK == SK_BF16 ? 2 : SK == SK_F32 ? 4 : 0;
}

struct SkParams {
  const void *scales;
  int sdt;
  int64_t nblk, block;
  int block_log2;
  const void *x;
  int64_t m;
  void *y;
  int ydt;
  int64_t ldy_m, ldy_n;
  int64_t rows;
  int nst;       // stages along K
  int gps, gbox;  // SK_GSTAGED: group scales per stage and row, scales per 16-byte box
  int splits;    // K slices
  int xbf16;
  float *ws;     // [splits][m][rows] fp32 partials (splits > 1)
  unsigned int *tickets;  // [row blocks]
};

// E8M0 byte -> 2^(b-127), branch-free (b = 0: 2^-127 subnormal; b = 255: NaN).
__device__ __forceinline__ float e8m0_val(uint32_t b) {
  const uint32_t bits = b == 0xFFu ? 0x7FC00000u : max(b << 23, 0x00400000u);
  return __uint_as_float(bits);
}

template <int SK>
__device__ __forceinline__ float tile_scale(const uint8_t *srow, int b) {
  if constexpr (SK == SK_E8M0_ORD) return __uint_as_float((uint32_t)srow[b] << 23);
  else if constexpr (SK == SK_E8M0) return e8m0_val(srow[b]);
  else if constexpr (SK == SK_F16) return __half2float(reinterpret_cast<const __half *>(srow)[b]);
  else if constexpr (SK == SK_BF16) return __uint_as_float((uint32_t)reinterpret_cast<const uint16_t *>(srow)[b] << 16);
  else if constexpr (SK == SK_F32) return reinterpret_cast<const float *>(srow)[b];
  else return 1.f;
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t &d0, uint32_t &d1, uint32_t &d2, uint32_t &d3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
               : "r"(addr));
}

template <int NC>
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(NC * 32) : "memory");
}

// compile-time choice between two same-typed arrays (no runtime indexing of registers)
template <bool FIRST, typename T>
__device__ __forceinline__ T &pick(T &a, T &b) {
  if constexpr (FIRST) return a;
  else return b;
}

// bf16 x chunk of the slot -> fp16 in place with a per-token power-of-two prescale; writes
// the inverse factors to inv[8*NT]. Tokens are the box rows (8*NT per box, 8 boxes).
template <int NT, int NC>
__device__ __forceinline__ void convert_x(uint8_t *xs, float *inv, int tid) {
  constexpr int TOK = 8 * NT, TPT = NC * 32 / TOK;  // threads per token
  const int tok = tid / TPT, part = tid % TPT;
  // each token row holds 8 boxes x 8 chunks of 16 bytes = 64 chunks (positions are swizzled,
  // which does not matter for an elementwise conversion)
  float amax = 0.f;
  for (int c = part; c < 64; c += TPT) {
    const uint4 u = *reinterpret_cast<const uint4 *>(xs + (c >> 3) * (TOK * 128) + tok * 128 + (c & 7) * 16);
    const uint32_t v[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
      amax = fmaxf(amax, fmaxf(fabsf(__uint_as_float(v[i] << 16)), fabsf(__uint_as_float(v[i] & 0xFFFF0000u))));
  }
#pragma unroll
  for (int o = TPT / 2; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  // prescale 2^(14 - e) with e the exponent of amax (amax = 0: factor 1)
  int e = amax > 0.f ? ((__float_as_int(amax) >> 23) & 0xFF) - 127 : 14;
  e = e > 126 ? 126 : (e < -112 ? -112 : e);  // both factors stay normal floats
  const float ps = __int_as_float((127 + 14 - e) << 23);
  if (part == 0) inv[tok] = __int_as_float((127 - 14 + e) << 23);
  for (int c = part; c < 64; c += TPT) {
    uint4 *p = reinterpret_cast<uint4 *>(xs + (c >> 3) * (TOK * 128) + tok * 128 + (c & 7) * 16);
    const uint4 u = *p;
    const uint32_t v[4] = {u.x, u.y, u.z, u.w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half2 h = __floats2half2_rn(__uint_as_float(v[i] << 16) * ps, __uint_as_float(v[i] & 0xFFFF0000u) * ps);
      o[i] = *reinterpret_cast<const uint32_t *>(&h);
    }
    *p = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

template <int FMT, int NT, int SK, bool XBF16>
__global__ void __launch_bounds__(threads<NT, SK>(), ctas_per_sm<NT>())
    skinny_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx,
                  const __grid_constant__ CUtensorMap tms, SkParams p) {
  constexpr int ESZ = tile_esz<SK>();
  constexpr bool STAGE_SCALES = ESZ > 0;                        // TMA stages a scale tile
  constexpr bool TILE_SCALES = STAGE_SCALES && SK != SK_GSTAGED;  // per-32 scales
  constexpr bool GROUPED = SK == SK_GROUP || SK == SK_GSTAGED;
  constexpr int SLOT = slot_bytes<NT>(ESZ);
  constexpr int STAGES = stages<NT>(ESZ);
  constexpr int TOK = 8 * NT;
  constexpr int NC = consumers<NT, SK>();
  constexpr int KH = NC / 8;         // warps per row group; each takes 1/KH of a stage's blocks
  constexpr int NB = KST / 32 / KH;  // 32-payload blocks per warp and stage
  constexpr uint32_t TX = W_BYTES + x_bytes<NT>() + (STAGE_SCALES ? s_bytes(ESZ) : 0);
  extern __shared__ uint8_t smem_raw[];
  uint8_t *ring = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t *full = reinterpret_cast<uint64_t *>(ring + STAGES * SLOT);
  uint64_t *empty = full + STAGES;
  volatile uint32_t *abort_flag = reinterpret_cast<uint32_t *>(empty + STAGES);
  volatile uint32_t *last_flag = abort_flag + 1;
  float *inv = const_cast<float *>(reinterpret_cast<volatile float *>(abort_flag + 2));  // [STAGES][TOK]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rblk = blockIdx.x / p.splits, split = blockIdx.x % p.splits;
  const int st0 = (int)((int64_t)p.nst * split / p.splits), st1 = (int)((int64_t)p.nst * (split + 1) / p.splits);

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NC);
    }
    *abort_flag = 0;
    *last_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == NC) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tmap(&tmw);
      prefetch_tmap(&tmx);
      if constexpr (STAGE_SCALES) prefetch_tmap(&tms);
      // codes and scales are parameters: the first ring's worth is requested before the
      // programmatic-dependency wait (x may be the previous kernel's output)
      auto load_wscales = [&](int st, int slot) {
        uint8_t *dst = ring + slot * SLOT;
        mbar_arrive_expect_tx(&full[slot], TX);
        tma_load_2d(dst, &tmw, st * (KST / 2), rblk * RB, &full[slot]);
        tma_load_2d(dst + RB * 128, &tmw, st * (KST / 2) + 128, rblk * RB, &full[slot]);
        if constexpr (STAGE_SCALES)
          tma_load_2d(dst + W_BYTES + x_bytes<NT>(), &tms,
                      SK == SK_GSTAGED ? (st * p.gps) & ~(p.gbox - 1) : st * (KST / 32), rblk * RB, &full[slot]);
      };
      const int pre = st1 - st0 < STAGES ? st1 - st0 : STAGES;
      for (int i = 0; i < pre; ++i) load_wscales(st0 + i, i);
      asm volatile("griddepcontrol.wait;" ::: "memory");
      int slot = 0, issued = 0;
      uint32_t ph = 0;
      for (int st = st0; st < st1; ++st) {
        if (issued >= pre) {
          if (issued >= STAGES && !mbar_wait(&empty[slot], ph ^ 1u, abort_flag)) break;
          if (*abort_flag) break;
          load_wscales(st, slot);
        }
        uint8_t *dst = ring + slot * SLOT;
#pragma unroll
        for (int j = 0; j < 8; ++j) tma_load_2d(dst + W_BYTES + j * (TOK * 128), &tmx, st * KST + 64 * j, 0, &full[slot]);
        ++issued;
        if (++slot == STAGES) slot = 0, ph ^= 1u;
      }
      if (*abort_flag) {  // drain copies still in flight before exiting
        for (int i = 0; i < STAGES && i < issued; ++i) {
          int s = slot - 1 - i;
          uint32_t q = ph;
          if (s < 0) s += STAGES, q ^= 1u;
          mbar_wait(&full[s], q, abort_flag, 200000000ull);
        }
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  // x, y and the split-K workspace belong to the stream order: wait for the previous kernel
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int g = lane >> 2, t = lane & 3;
  const int kh = KH == 1 ? 0 : warp / 8;  // which part of each stage's blocks this warp takes
  const int r0 = (KH == 1 ? warp : warp % 8) * 16;  // rows r0 + g, r0 + g + 8 (within the CTA's 128)
  const int64_t nlo = (int64_t)rblk * RB + r0 + g, nhi = nlo + 8;
  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  // ldmatrix row address for this lane: matrix q = lane / 8 (rows +0/+8, chunk +0/+1), row i
  const int lq = lane >> 3, li = lane & 7;
  const int lrow = r0 + (lq & 1) * 8 + li;
  const int lchunk = lq >> 1;
  // x fragment offsets within a box: token row g, 16-byte chunk t (even block) / 4 + t (odd)
  const int xoff[2] = {g * 128 + ((t ^ g) << 4), g * 128 + (((4 + t) ^ g) << 4)};

  int slot = 0;
  uint32_t ph = 0;
  for (int st = st0; st < st1; ++st) {
    // SK_GROUP: the scales of the groups that end in this stage, indexed by their last block
    // (prefetched before the stage wait; compile-time indices keep them in registers)
    float sgl[NB], sgh[NB];  // indexed by the warp's local block j (stage block kh * NB + j)
    if constexpr (SK == SK_GROUP) {
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        const int bb = kh * NB + j;
        sgl[j] = sgh[j] = 0.f;
        if (((32 * (bb + 1)) & (p.block - 1)) == 0) {
          const int64_t gi = ((int64_t)st * KST + 32 * bb) >> p.block_log2;
          if (nlo < p.rows) sgl[j] = load_as_f32(p.scales, nlo * p.nblk + gi, p.sdt);
          if (nhi < p.rows) sgh[j] = load_as_f32(p.scales, nhi * p.nblk + gi, p.sdt);
        }
      }
    }
    const bool got = mbar_wait(&full[slot], ph, abort_flag);
    uint8_t *base = ring + slot * SLOT;
    uint8_t *xs = base + W_BYTES;
    float *sinv = inv + slot * TOK;
    if constexpr (XBF16) {
      if (got) convert_x<NT, NC>(xs, sinv, tid);
      consumer_sync<NC>();
    }
    // the stage's partial sums: a separate array with bf16 x (its per-token prescale is undone
    // per stage), the running sums themselves with fp16 x (saves 4 * NT registers)
    float sacc_bf[NT][4];  // unused (and eliminated) with fp16 x
    float(&sacc)[NT][4] = pick<XBF16>(sacc_bf, acc);
    if constexpr (XBF16) {
#pragma unroll
      for (int j = 0; j < NT; ++j) sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.f;
    }
    if (got) {
      const uint8_t *srow_lo = base + W_BYTES + x_bytes<NT>() + (r0 + g) * (KST / 32) * ESZ;
      const uint8_t *srow_hi = srow_lo + 8 * (KST / 32) * ESZ;
      const uint32_t wbase = smem_u32(base);
      // the E8M0 scales of this warp's NB blocks, rows g / g+8 (word i holds local blocks 4i..4i+3)
      // (applied to each block's fp32 MMA result: folding them into the fp16 operand with HMUL2
      // measured slower on every tile, FP4 8192^2 M=8 20.98 vs 20.03 us, M=32 fp16 x 32.7 vs 29.5)
      uint32_t e8l[is_e8m0<SK>() ? NB / 4 : 1] = {}, e8h[is_e8m0<SK>() ? NB / 4 : 1] = {};
      if constexpr (is_e8m0<SK>()) {
        if constexpr (NB == 16) {
          const uint4 ul = *reinterpret_cast<const uint4 *>(srow_lo), uh = *reinterpret_cast<const uint4 *>(srow_hi);
          e8l[0] = ul.x, e8l[1] = ul.y, e8l[2] = ul.z, e8l[3] = ul.w;
          e8h[0] = uh.x, e8h[1] = uh.y, e8h[2] = uh.z, e8h[3] = uh.w;
        } else {
          const uint2 ul = *reinterpret_cast<const uint2 *>(srow_lo + kh * NB);
          const uint2 uh = *reinterpret_cast<const uint2 *>(srow_hi + kh * NB);
          e8l[0] = ul.x, e8l[1] = ul.y, e8h[0] = uh.x, e8h[1] = uh.y;
        }
      }
      float gd[NT][4];  // running partial of the current scale group (group kinds)
#pragma unroll
      for (int j = 0; j < NT; ++j) gd[j][0] = gd[j][1] = gd[j][2] = gd[j][3] = 0.f;
#pragma unroll
      for (int jp = 0; jp < NB / 2; ++jp) {  // pairs of this warp's 32-payload blocks
        const int b = kh * NB + 2 * jp;
        const int box = b >> 3, chunk = (b & 7) + lchunk;
        uint32_t wl0, wh0, wl1, wh1;  // rows g / g+8 of blocks b / b+1
        ldmatrix_x4(wbase + box * (RB * 128) + lrow * 128 + (((chunk) ^ (lrow & 7)) << 4), wl0, wh0, wl1, wh1);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int bb = b + h;
          uint32_t ol[4], oh[4];
          const uint32_t wl = h ? wl1 : wl0, wh = h ? wh1 : wh0;
          decode8_natural<FMT, false>(&wl, 0, ol);
          decode8_natural<FMT, false>(&wh, 0, oh);
          const int xbox = bb >> 1;
          float sl = 1.f, sh = 1.f;
          if constexpr (is_e8m0<SK>()) {
            const int jb = 2 * jp + h;  // local block: compile-time word and byte
            const uint32_t bl = (e8l[jb >> 2] >> (8 * (jb & 3))) & 0xFFu, bh = (e8h[jb >> 2] >> (8 * (jb & 3))) & 0xFFu;
            if constexpr (SK == SK_E8M0_ORD) {
              sl = __uint_as_float(bl << 23);
              sh = __uint_as_float(bh << 23);
            } else {
              sl = e8m0_val(bl);
              sh = e8m0_val(bh);
            }
          } else if constexpr (TILE_SCALES) {
            sl = tile_scale<SK>(srow_lo, bb);
            sh = tile_scale<SK>(srow_hi, bb);
          }
          const uint32_t a0[4] = {ol[0], oh[0], ol[1], oh[1]}, a1[4] = {ol[2], oh[2], ol[3], oh[3]};
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            const uint4 xv = *reinterpret_cast<const uint4 *>(xs + xbox * (TOK * 128) + (8 * j) * 128 + xoff[bb & 1]);
            if constexpr (TILE_SCALES) {
              float d[4] = {0.f, 0.f, 0.f, 0.f};
              mma16816(d, a0, xv.x, xv.y);
              mma16816(d, a1, xv.z, xv.w);
              sacc[j][0] = fmaf(d[0], sl, sacc[j][0]);
              sacc[j][1] = fmaf(d[1], sl, sacc[j][1]);
              sacc[j][2] = fmaf(d[2], sh, sacc[j][2]);
              sacc[j][3] = fmaf(d[3], sh, sacc[j][3]);
            } else if constexpr (GROUPED) {
              mma16816(gd[j], a0, xv.x, xv.y);
              mma16816(gd[j], a1, xv.z, xv.w);
            } else {
              mma16816(sacc[j], a0, xv.x, xv.y);
              mma16816(sacc[j], a1, xv.z, xv.w);
            }
          }
          if constexpr (GROUPED) {
            if (((32 * (bb + 1)) & (p.block - 1)) == 0) {  // the group ends with this block
              float gl, gh;
              if constexpr (SK == SK_GSTAGED) {
                const int e = ((st * p.gps) & (p.gbox - 1)) + ((bb + 1) >> (p.block_log2 - 5)) - 1;
                gl = load_as_f32(srow_lo, e, p.sdt);
                gh = load_as_f32(srow_hi, e, p.sdt);
              } else {
                gl = sgl[2 * jp + h], gh = sgh[2 * jp + h];
              }
#pragma unroll
              for (int j = 0; j < NT; ++j) {
                sacc[j][0] = fmaf(gd[j][0], gl, sacc[j][0]);
                sacc[j][1] = fmaf(gd[j][1], gl, sacc[j][1]);
                sacc[j][2] = fmaf(gd[j][2], gh, sacc[j][2]);
                sacc[j][3] = fmaf(gd[j][3], gh, sacc[j][3]);
                gd[j][0] = gd[j][1] = gd[j][2] = gd[j][3] = 0.f;
              }
            }
          }
        }
      }
    }
    // the slot's bytes are no longer needed (generic-proxy writes ordered before the next TMA fill)
    if constexpr (XBF16) fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    if constexpr (XBF16) {
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const float f0 = sinv[8 * j + 2 * t], f1 = sinv[8 * j + 2 * t + 1];
        acc[j][0] = fmaf(sacc[j][0], f0, acc[j][0]);
        acc[j][1] = fmaf(sacc[j][1], f1, acc[j][1]);
        acc[j][2] = fmaf(sacc[j][2], f0, acc[j][2]);
        acc[j][3] = fmaf(sacc[j][3], f1, acc[j][3]);
      }
    }
    if (++slot == STAGES) slot = 0, ph ^= 1u;
  }

  if constexpr (KH == 2) {
    // the second warp of each row group hands its sums to the first through the ring, which is
    // idle now: every stage has been consumed, so no copy is in flight
    float *pair = reinterpret_cast<float *>(ring);  // [8 row groups][NT * 4][32 lanes]
    consumer_sync<NC>();
    if (kh == 1) {
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) pair[((warp - 8) * NT * 4 + 4 * j + i) * 32 + lane] = acc[j][i];
    }
    consumer_sync<NC>();
    if (kh == 0) {
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[j][i] += pair[(warp * NT * 4 + 4 * j + i) * 32 + lane];
    }
  }

  // ---------------- epilogue (first warp of each row group) ----------------
  const bool ok = !*abort_flag;
  float rs_lo = 1.f, rs_hi = 1.f;
  if constexpr (SK == SK_ROW) {
    if (nlo < p.rows) rs_lo = load_as_f32(p.scales, nlo * p.nblk, p.sdt);
    if (nhi < p.rows) rs_hi = load_as_f32(p.scales, nhi * p.nblk, p.sdt);
  }
  if (p.splits == 1) {
    if (!ok || kh != 0) return;
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int64_t m = 8 * j + 2 * t + (i & 1), n = i < 2 ? nlo : nhi;
        if (m < p.m && n < p.rows) store_f32(p.y, m * p.ldy_m + n * p.ldy_n, p.ydt, acc[j][i] * (i < 2 ? rs_lo : rs_hi));
      }
    return;
  }
  // split-K: partials to the workspace, then the last CTA of the row block reduces
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t m = 8 * j + 2 * t + (i & 1), n = i < 2 ? nlo : nhi;
      if (kh == 0 && m < p.m && n < p.rows) p.ws[((int64_t)split * p.m + m) * p.rows + n] = acc[j][i];
    }
  // one thread publishes the CTA's partials (the barrier orders every thread's stores before its
  // release) and, if it is the last slice, acquires the others' (the barrier after it orders the
  // reads below): cheaper than a full fence in every thread
  consumer_sync<NC>();
  if (tid == 0) {
    unsigned int ticket;
    asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], 1;" : "=r"(ticket) : "l"(&p.tickets[rblk]) : "memory");
    *last_flag = ticket == (unsigned int)(p.splits - 1);
  }
  consumer_sync<NC>();
  if (!*last_flag) return;
  const int64_t n0 = (int64_t)rblk * RB;
  for (int e = tid; e < RB * (int)p.m; e += NC * 32) {
    const int64_t m = e / RB, n = n0 + e % RB;
    if (n >= p.rows) continue;
    float s = 0.f;
    for (int sp = 0; sp < p.splits; ++sp) s += __ldcg(&p.ws[((int64_t)sp * p.m + m) * p.rows + n]);
    if constexpr (SK == SK_ROW) s *= load_as_f32(p.scales, n * p.nblk, p.sdt);
    if (ok) store_f32(p.y, m * p.ldy_m + n * p.ldy_n, p.ydt, s);
  }
  if (tid == 0) p.tickets[rblk] = 0u;  // ready for the next call on this workspace
}

template <int NT>
static size_t smem_bytes(int esz) {
  return 1024 + (size_t)stages<NT>(esz) * slot_bytes<NT>(esz) + 2 * 4 * 8 + 16 + 4 * 8 * NT * 4;
}

// ---- per-(device, stream) split-K workspace --------------------------------------------------
struct Workspace {
  float *ws = nullptr;
  unsigned int *tickets = nullptr;
  size_t ws_bytes = 0, tickets_n = 0;
};
constexpr size_t WS_BYTES = 16u << 20;  // fp32 partials (max splits x M x N)
constexpr size_t TICKETS = 16384;       // row blocks (N up to 2M rows)

static std::mutex g_ws_mutex;
static std::map<std::pair<int, cudaStream_t>, Workspace> g_ws;

static int32_t workspace_for(cudaStream_t stream, Workspace *&out) {
  int dev = 0;
  B200_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(g_ws_mutex);
  auto it = g_ws.find({dev, stream});
  if (it != g_ws.end()) {
    out = &it->second;
    return B200_OK;
  }
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  B200_CUDA_TRY(cudaStreamIsCapturing(stream, &cs));
  if (cs != cudaStreamCaptureStatusNone) {  // no allocation while capturing: run unsplit
    out = nullptr;
    return B200_OK;
  }
  Workspace w;
  B200_CUDA_TRY(cudaMalloc((void **)&w.ws, WS_BYTES));
  B200_CUDA_TRY(cudaMalloc((void **)&w.tickets, TICKETS * sizeof(unsigned int)));
  // on the caller's stream, the only one that uses this workspace: ordered before its kernels
  // even when that stream does not synchronise with the legacy default stream
  B200_CUDA_TRY(cudaMemsetAsync(w.tickets, 0, TICKETS * sizeof(unsigned int), stream));
  w.ws_bytes = WS_BYTES;
  w.tickets_n = TICKETS;
  out = &(g_ws[{dev, stream}] = w);
  return B200_OK;
}

template <int FMT, int NT, int SK, bool XBF16>
static int32_t launch_t(const LinearArgs &a, int splits, float *ws, unsigned int *tickets, cudaStream_t stream) {
  constexpr int ESZ = tile_esz<SK>();
  const size_t smem = smem_bytes<NT>(ESZ);
  B200_CUDA_TRY((ensure_dynamic_smem<skinny_kernel<FMT, NT, SK, XBF16>>((int)smem)));
  CUtensorMap tmw, tmx, tms;
  const uint64_t row_bytes = (uint64_t)a.cols / 2;
  if (int32_t rc = make_tma_2d(&tmw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w, row_bytes, (uint64_t)a.rows, row_bytes, 128,
                               RB, CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  if (int32_t rc = make_tma_2d(&tmx, XBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.x,
                               (uint64_t)a.cols, (uint64_t)a.m, (uint64_t)a.ldx * 2, 64, 8 * NT,
                               CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  if constexpr (SK == SK_GSTAGED) {
    const int esz = dt_size(a.sdt);
    const CUtensorMapDataType dt = a.sdt == B200_DT_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : a.sdt == B200_DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                           : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    if (int32_t rc = make_tma_2d(&tms, dt, a.scales, (uint64_t)a.nblk, (uint64_t)a.rows, (uint64_t)a.nblk * esz,
                                 (uint32_t)(16 / esz), RB, CU_TENSOR_MAP_SWIZZLE_NONE))
      return rc;
  } else if constexpr (ESZ > 0) {
    const CUtensorMapDataType dt = ESZ == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                   : ESZ == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : SK == SK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    if (int32_t rc = make_tma_2d(&tms, dt, a.scales, (uint64_t)a.nblk, (uint64_t)a.rows, (uint64_t)a.nblk * ESZ,
                                 KST / 32, RB, CU_TENSOR_MAP_SWIZZLE_NONE))
      return rc;
  } else {
    tms = tmw;
  }
  SkParams p;
  p.scales = a.scales, p.sdt = a.sdt, p.nblk = a.nblk, p.block = a.block;
  p.block_log2 = 0;
  while (((int64_t)1 << p.block_log2) < a.block) ++p.block_log2;
  p.gps = (int)(KST / (a.block > 0 ? a.block : KST));
  p.gbox = SK == SK_GSTAGED ? 16 / dt_size(a.sdt) : 1;
  p.x = a.x, p.m = a.m, p.y = a.y, p.ydt = a.ydt, p.ldy_m = a.ldy_m, p.ldy_n = a.ldy_n, p.rows = a.rows;
  p.nst = (int)(a.cols / KST);
  p.splits = splits;
  p.xbf16 = XBF16;
  p.ws = ws;
  p.tickets = tickets;
  const int64_t nrb = (a.rows + RB - 1) / RB;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(nrb * splits));
  cfg.blockDim = dim3(threads<NT, SK>());
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[1];
  attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = (a.flags & B200_FLAG_PDL) ? 1 : 0;
  B200_CUDA_TRY(cudaLaunchKernelEx(&cfg, skinny_kernel<FMT, NT, SK, XBF16>, tmw, tmx, tms, p));
  return B200_OK;
}

template <int FMT, int NT, int SK>
static int32_t launch_x(const LinearArgs &a, int splits, float *ws, unsigned int *tk, cudaStream_t s) {
  return a.xdt == B200_DT_BF16 ? launch_t<FMT, NT, SK, true>(a, splits, ws, tk, s)
                               : launch_t<FMT, NT, SK, false>(a, splits, ws, tk, s);
}

// Group scales that fit the staged layout: fp16 / bf16 / fp32, a stage's groups within one
// 16-byte box, 16-byte scale rows and base.
static bool group_staged(const LinearArgs &a) {
  if (!(a.sdt == B200_DT_F16 || a.sdt == B200_DT_BF16 || a.sdt == B200_DT_F32)) return false;
  const int esz = dt_size(a.sdt);
  return (KST / a.block) * esz <= 16 && (a.nblk * esz) % 16 == 0 && (uintptr_t)a.scales % 16 == 0;
}

template <int FMT, int NT>
static int32_t launch_sk(const LinearArgs &a, int sk, int splits, float *ws, unsigned int *tk, cudaStream_t s) {
  switch (sk) {
    case SK_NONE: return launch_x<FMT, NT, SK_NONE>(a, splits, ws, tk, s);
    case SK_ROW: return launch_x<FMT, NT, SK_ROW>(a, splits, ws, tk, s);
    case SK_E8M0:
      return (a.flags & B200_FLAG_SCALES_ORDINARY) ? launch_x<FMT, NT, SK_E8M0_ORD>(a, splits, ws, tk, s)
                                                   : launch_x<FMT, NT, SK_E8M0>(a, splits, ws, tk, s);
    case SK_F16: return launch_x<FMT, NT, SK_F16>(a, splits, ws, tk, s);
    case SK_BF16: return launch_x<FMT, NT, SK_BF16>(a, splits, ws, tk, s);
    case SK_F32: return launch_x<FMT, NT, SK_F32>(a, splits, ws, tk, s);
    case SK_GROUP:
      return group_staged(a) ? launch_x<FMT, NT, SK_GSTAGED>(a, splits, ws, tk, s)
                             : launch_x<FMT, NT, SK_GROUP>(a, splits, ws, tk, s);
  }
  return b200_set_error(B200_ERR_UNSUPPORTED, "skinny GEMM: scale layout");
}

// The 64-token tile serves 33..64 tokens for the scale layouts the tcgen05 GEMM declines (per-32
// fp16 / bf16 / fp32 scales and wider group scales, which it cannot fold into its operand exactly).
static bool wide_tile_scales(int sk) {
  return sk == SK_F16 || sk == SK_BF16 || sk == SK_F32 || sk == SK_GROUP;
}

template <int FMT>
static int32_t launch_sk64(const LinearArgs &a, int sk, int splits, float *ws, unsigned int *tk, cudaStream_t s) {
  switch (sk) {
    case SK_F16: return launch_x<FMT, 8, SK_F16>(a, splits, ws, tk, s);
    case SK_BF16: return launch_x<FMT, 8, SK_BF16>(a, splits, ws, tk, s);
    case SK_F32: return launch_x<FMT, 8, SK_F32>(a, splits, ws, tk, s);
    case SK_GROUP:
      return group_staged(a) ? launch_x<FMT, 8, SK_GSTAGED>(a, splits, ws, tk, s)
                             : launch_x<FMT, 8, SK_GROUP>(a, splits, ws, tk, s);
  }
  return b200_set_error(B200_ERR_UNSUPPORTED, "skinny GEMM: no 64-token tile for this scale layout");
}

template <int FMT>
static int32_t launch_nt(const LinearArgs &a, int sk, int splits, float *ws, unsigned int *tk, cudaStream_t s) {
  if (a.m <= 8) return launch_sk<FMT, 1>(a, sk, splits, ws, tk, s);
  if (a.m <= 16) return launch_sk<FMT, 2>(a, sk, splits, ws, tk, s);
  if (a.m <= 32) return launch_sk<FMT, 4>(a, sk, splits, ws, tk, s);
  return launch_sk64<FMT>(a, sk, splits, ws, tk, s);
}

static int choose_splits(const LinearArgs &a, int sms) {
  const int64_t nrb = (a.rows + RB - 1) / RB, nst = a.cols / KST;
  int64_t s = sms / nrb;
  if (s < 1) s = 1;
  if (s > nst) s = nst;
  if (s > 16) s = 16;
  return (int)s;
}

}  // namespace skinny

bool skinny_supported(const LinearArgs &a) {
  using namespace skinny;
  if (a.m < 3 || a.m > 64) return false;
  if (a.m > 32 && !wide_tile_scales(gemv::scale_kind(a))) return false;
  if (!(a.fmt == B200_FMT_INT4 || a.fmt == B200_FMT_UINT4 || a.fmt == B200_FMT_FP4_E2M1)) return false;
  if (a.xdt != B200_DT_F16 && a.xdt != B200_DT_BF16) return false;
  if (a.ydt != B200_DT_F16 && a.ydt != B200_DT_BF16 && a.ydt != B200_DT_F32) return false;
  if (a.cols < KST || a.cols % KST != 0 || a.cols > ((int64_t)1 << 26) || a.rows <= 0) return false;
  if ((a.rows + RB - 1) / RB * 16 > (int64_t)INT32_MAX) return false;
  if ((uintptr_t)a.w % 16 != 0 || (uintptr_t)a.x % 16 != 0 || (a.ldx * 2) % 16 != 0) return false;
  if (a.scales != nullptr) {
    const int sk = gemv::scale_kind(a);
    if (sk == gemv::SK_GROUP) {
      if (!(a.block == 64 || a.block == 128 || a.block == 256 || a.block == 512)) return false;
      if (!(a.sdt == B200_DT_F16 || a.sdt == B200_DT_BF16 || a.sdt == B200_DT_F32 || a.sdt == B200_DT_E8M0)) return false;
    } else if (sk >= gemv::SK_E8M0) {
      if ((a.nblk * dt_size(a.sdt)) % 16 != 0 || (uintptr_t)a.scales % 16 != 0) return false;
    } else if (sk == gemv::SK_ROW) {
      if (!(a.sdt == B200_DT_F16 || a.sdt == B200_DT_BF16 || a.sdt == B200_DT_F32 || a.sdt == B200_DT_E8M0)) return false;
    }
  }
  return true;
}

int32_t launch_skinny(const LinearArgs &a, cudaStream_t stream) {
  using namespace skinny;
  int sms = 0;
  B200_CUDA_TRY(device_sms(&sms));
  int splits = choose_splits(a, sms * (a.m <= 16 ? 2 : 1));
  float *ws = nullptr;
  unsigned int *tickets = nullptr;
  if (splits > 1) {
    Workspace *w = nullptr;
    if (int32_t rc = workspace_for(stream, w)) return rc;
    const int64_t nrb = (a.rows + RB - 1) / RB;
    const size_t per_split = (size_t)a.m * a.rows * sizeof(float);
    if (w == nullptr || (size_t)nrb > w->tickets_n) {
      splits = 1;
    } else {
      while (splits > 1 && (size_t)splits * per_split > w->ws_bytes) --splits;
      ws = w->ws;
      tickets = w->tickets;
    }
  }
  const int sk = gemv::scale_kind(a);
  switch (a.fmt) {
    case B200_FMT_INT4: return launch_nt<B200_FMT_INT4>(a, sk, splits, ws, tickets, stream);
    case B200_FMT_UINT4: return launch_nt<B200_FMT_UINT4>(a, sk, splits, ws, tickets, stream);
    case B200_FMT_FP4_E2M1: return launch_nt<B200_FMT_FP4_E2M1>(a, sk, splits, ws, tickets, stream);
  }
  return b200_set_error(B200_ERR_UNSUPPORTED, "skinny GEMM: format %d", a.fmt);
}

}  // namespace b200

// ---- allocation-free variant (b200_packed_linear_noalloc) ---------------------------------
// The split-K scratch (row-block tickets, then fp32 partials) lives in one fixed device array
// of this translation unit; nothing is allocated. The tickets must start at zero: the array is
// zero-initialised when the module loads and every reducing CTA resets its ticket, so set-up
// writes nothing (a memset there would be unordered against a caller's non-blocking stream).
// Calls that overlap in time on one device share the array and race.
namespace b200 {
namespace skinny {

constexpr size_t NOALLOC_SCRATCH_BYTES = 2u << 20;  // 2 MiB per device
constexpr size_t NOALLOC_TICKETS = 4096;            // row blocks of 128 rows (N <= 524288)
static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

static std::mutex g_noalloc_mutex;
static std::map<int, unsigned char *> g_noalloc_base;  // device -> address of the array

// Resolve the array's device address once per device (with that device current).
static int32_t noalloc_scratch(unsigned char *&base) {
  int dev = 0;
  B200_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  auto it = g_noalloc_base.find(dev);
  if (it != g_noalloc_base.end()) {
    base = it->second;
    return B200_OK;
  }
  void *p = nullptr;
  B200_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
  base = static_cast<unsigned char *>(p);
  g_noalloc_base[dev] = base;
  return B200_OK;
}

}  // namespace skinny

int32_t launch_skinny_noalloc(const LinearArgs &a, cudaStream_t stream) {
  using namespace skinny;
  int sms = 0;
  B200_CUDA_TRY(device_sms(&sms));
  const int splits = choose_splits(a, sms * (a.m <= 16 ? 2 : 1));  // as b200_packed_linear
  float *ws = nullptr;
  unsigned int *tickets = nullptr;
  if (splits > 1) {
    const int64_t nrb = (a.rows + RB - 1) / RB;
    const size_t tbytes = NOALLOC_TICKETS * sizeof(unsigned int);
    const size_t need = (size_t)splits * a.m * a.rows * sizeof(float);
    if ((size_t)nrb > NOALLOC_TICKETS || need > NOALLOC_SCRATCH_BYTES - tbytes)
      return b200_set_error(B200_ERR_UNSUPPORTED,
                            "packed_linear_noalloc: needs %zu bytes of split-K scratch for %lld row blocks; the "
                            "fixed scratch holds %zu bytes and %zu row blocks",
                            need, (long long)nrb, NOALLOC_SCRATCH_BYTES - tbytes, NOALLOC_TICKETS);
    unsigned char *base = nullptr;
    if (int32_t rc = noalloc_scratch(base)) return rc;
    tickets = reinterpret_cast<unsigned int *>(base);
    ws = reinterpret_cast<float *>(base + tbytes);
  }
  const int sk = gemv::scale_kind(a);
  switch (a.fmt) {
    case B200_FMT_INT4: return launch_nt<B200_FMT_INT4>(a, sk, splits, ws, tickets, stream);
    case B200_FMT_UINT4: return launch_nt<B200_FMT_UINT4>(a, sk, splits, ws, tickets, stream);
    case B200_FMT_FP4_E2M1: return launch_nt<B200_FMT_FP4_E2M1>(a, sk, splits, ws, tickets, stream);
  }
  return b200_set_error(B200_ERR_UNSUPPORTED, "packed_linear_noalloc: format %d", a.fmt);
}

}  // namespace b200
