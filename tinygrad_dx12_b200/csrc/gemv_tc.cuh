// gemv_tc.cu -- decode GEMV for M <= 2: y[m, n] = sum_k x[m, k] * dequant(W)[n, k].
//
// The B200 replacement of the reference's matvec / one-column LinAlg matmul over a packed
// operand (tinygrad-dx12 src/tinygrad_dx12/codegen/linalg.py:226-245 -> renderer/linalg.py),
// with the decode of src/tinygrad_dx12/codegen/decomp/dx12.py:69-106 done in registers.
//
// Memory path. A CTA owns 16 weight rows; its 8 warps split K. Lane (g, t) = (lane/4, lane%4)
// streams, per 128-payload chunk, one 32-payload block of rows g and g+8 with a 128-bit load
// (4-bit formats) or three 64-bit loads (6-bit formats): every warp load instruction covers
// 8 rows x 64 (96) contiguous bytes. Activations are staged once per CTA in shared memory as
// fp16, ordered inside each 8-element group to match the register pairing of the decode.
//
// Math path. Payloads decode to exact fp16 values (INT4/UINT4 through the 0x6400 magic number,
// pairing payloads (i, i+4); FP4/FP6 through the sm_100a cvt.rn.f16x2.{e2m1,e2m3,e3m2}x2
// conversions, pairing (2i, 2i+1)) and feed mma.sync m16n8k16 (fp16 in, fp32 accumulate) as
// the A operand (16 rows x 16 k). Thread t
// supplies only payloads of its own 32-block, so column c of the B operand is made
// block-diagonal: B[k][c] holds x[m][k] when k belongs to block (c % 4) and c / 4 == m, else 0.
// Accumulator column c is then the exact per-block partial sum of block (c % 4) for row m, and
// is multiplied by that block's scale in fp32 -- the reference's per-block scaling, exact for
// every scale dtype (fp16 / bf16 / fp32 / E8M0), without cross-lane exchanges.
//
// bf16 activations are converted to fp16 with a per-CTA power-of-two prescale chosen from
// max|x| so nothing overflows; every bf16 value whose magnitude is >= 2^-17 of that range is
// exactly representable in fp16, smaller ones round with an absolute error below 2^-25 of the
// largest |x| (far inside the stated output tolerances).
#include "common.cuh"
#include "kernels.h"
#include "decode.cuh"

namespace b200 {
namespace gemv {

constexpr int WARPS = 8, ROWS = 16, CHUNK = 128;

struct Params {
  const uint8_t *w;
  const void *scales;
  int sdt;
  int64_t rows, cols, nblk, block;
  const void *x;
  int64_t m, ldx;
  void *y;
  int ydt;
  int64_t ldy_m, ldy_n;
  int pdl;  // launched with programmatic stream serialization
  void *ycopy[7];  // further destinations of y (same layout), e.g. peers' buffers
  int ncopy;
};


// Scale handling, a template parameter so the hot loop carries no dtype dispatch.
enum ScaleKind {
  SK_NONE = 0,   // unscaled
  SK_ROW = 1,    // one scale per row (block_size >= K): applied once to the fp32 result
  SK_E8M0 = 2,   // per-32 E8M0 bytes (block_size == 32)
  SK_F16 = 3,    // per-32 fp16
  SK_BF16 = 4,   // per-32 bf16
  SK_F32 = 5,    // per-32 fp32
  SK_GROUP = 6,  // any other block_size that is a multiple of 32, any scale dtype
};

// One lane's share of a 128-payload chunk: its 32-payload block of rows ra / rb and the
// scales of its two accumulator columns (blocks cblk, cblk+1 of the chunk).
template <int BITS>
struct Chunk {
  uint32_t a[BITS], b[BITS];  // 4 words (4-bit) or 6 words (6-bit) per row
  float sa0, sa1, sb0, sb1;
};

template <int SK>
__device__ __forceinline__ void load_scale_pair(const Params &p, int64_t row, int64_t k0, float &s0, float &s1) {
  if constexpr (SK == SK_E8M0) {  // two adjacent bytes -> 2^(b-127)
    const uint32_t v = __ldg(reinterpret_cast<const uint16_t *>((const uint8_t *)p.scales + row * p.nblk + (k0 >> 5)));
    s0 = e8m0_to_f32((uint8_t)(v & 0xFF));
    s1 = e8m0_to_f32((uint8_t)(v >> 8));
  } else if constexpr (SK == SK_F16) {
    const __half2 h = __ldg(reinterpret_cast<const __half2 *>((const __half *)p.scales + row * p.nblk + (k0 >> 5)));
    const float2 f = __half22float2(h);
    s0 = f.x, s1 = f.y;
  } else if constexpr (SK == SK_BF16) {
    const uint32_t v = __ldg(reinterpret_cast<const uint32_t *>((const uint16_t *)p.scales + row * p.nblk + (k0 >> 5)));
    s0 = __uint_as_float(v << 16), s1 = __uint_as_float(v & 0xFFFF0000u);
  } else if constexpr (SK == SK_F32) {
    const float2 f = __ldg(reinterpret_cast<const float2 *>((const float *)p.scales + row * p.nblk + (k0 >> 5)));
    s0 = f.x, s1 = f.y;
  } else if constexpr (SK == SK_GROUP) {
    s0 = load_as_f32(p.scales, row * p.nblk + (uint32_t)k0 / (uint32_t)p.block, p.sdt);
    s1 = load_as_f32(p.scales, row * p.nblk + (uint32_t)(k0 + 32) / (uint32_t)p.block, p.sdt);
  } else {
    s0 = s1 = 1.f;
  }
}

template <int BITS, int SK>
__device__ __forceinline__ void load_chunk(Chunk<BITS> &r, const Params &p, const uint8_t *wa, const uint8_t *wb,
                                           int c, int t, int cblk, int64_t ra, int64_t rb) {
  if constexpr (BITS == 4) {
    const uint4 ua = __ldg(reinterpret_cast<const uint4 *>(wa + (int64_t)c * 64 + 16 * t));
    const uint4 ub = __ldg(reinterpret_cast<const uint4 *>(wb + (int64_t)c * 64 + 16 * t));
    r.a[0] = ua.x, r.a[1] = ua.y, r.a[2] = ua.z, r.a[3] = ua.w;
    r.b[0] = ub.x, r.b[1] = ub.y, r.b[2] = ub.z, r.b[3] = ub.w;
  } else {
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      const uint2 ua = __ldg(reinterpret_cast<const uint2 *>(wa + (int64_t)c * 96 + 24 * t) + q);
      const uint2 ub = __ldg(reinterpret_cast<const uint2 *>(wb + (int64_t)c * 96 + 24 * t) + q);
      r.a[2 * q] = ua.x, r.a[2 * q + 1] = ua.y, r.b[2 * q] = ub.x, r.b[2 * q + 1] = ub.y;
    }
  }
  const int64_t k0 = (int64_t)c * CHUNK + 32 * cblk;
  load_scale_pair<SK>(p, ra, k0, r.sa0, r.sa1);
  load_scale_pair<SK>(p, rb, k0, r.sb0, r.sb1);
}

template <int FMT, int SK>
__device__ __forceinline__ void compute_chunk(const Chunk<Fmt<FMT>::bits> &r, const __half *xblk, float &acc_a,
                                              float &acc_b) {
  constexpr int BITS = Fmt<FMT>::bits;
  // two independent accumulator chains halve the serial mma latency of a chunk
  float d[4] = {0.f, 0.f, 0.f, 0.f}, e[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int u = 0; u < 4; ++u) {  // 8-payload unit u of this lane's block
    uint32_t pa[4], pb[4];
    if constexpr (BITS == 4) {
      decode8_4bit<FMT>(r.a[u], pa);
      decode8_4bit<FMT>(r.b[u], pb);
    } else {
      const int bit = 48 * u, wi = bit >> 5, sh = bit & 31;  // the unit lies in words wi, wi+1
      decode8_6bit<FMT>((((uint64_t)r.a[wi + 1] << 32) | r.a[wi]) >> sh, pa);
      decode8_6bit<FMT>((((uint64_t)r.b[wi + 1] << 32) | r.b[wi]) >> sh, pb);
    }
    // x of this unit in decode pair order; a zero slot for non-owner lanes
    const uint4 xv = *reinterpret_cast<const uint4 *>(xblk + 8 * u);
    const uint32_t a0[4] = {pa[0], pb[0], pa[1], pb[1]};
    mma16816(d, a0, xv.x, xv.y);
    const uint32_t a1[4] = {pa[2], pb[2], pa[3], pb[3]};
    mma16816(e, a1, xv.z, xv.w);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) d[i] += e[i];
  // d = {D[g][2t], D[g][2t+1], D[g+8][2t], D[g+8][2t+1]}: per-block partial sums
  if constexpr (SK == SK_NONE || SK == SK_ROW) {
    acc_a += d[0] + d[1];
    acc_b += d[2] + d[3];
  } else {
    acc_a = fmaf(d[0], r.sa0, fmaf(d[1], r.sa1, acc_a));
    acc_b = fmaf(d[2], r.sb0, fmaf(d[3], r.sb1, acc_b));
  }
}

// Stage x[m][K] into shared memory as fp16, permuted (0,4,1,5,2,6,3,7) within each 8-group.
// Returns false when a bf16 value overflowed fp16 after the prescale.
template <bool PERM04>
__device__ __forceinline__ bool stage_x(const Params &p, __half *xs, int K, bool xbf16, float prescale) {
  bool overflow = false;
  const int K8 = K >> 3;
  for (int mm = 0; mm < (int)p.m; ++mm) {
    const uint16_t *src = (const uint16_t *)p.x + (int64_t)mm * p.ldx;
    for (int k8 = threadIdx.x; k8 < K8; k8 += blockDim.x) {
      const uint4 u = __ldg(reinterpret_cast<const uint4 *>(src) + k8);
      const uint32_t wv[4] = {u.x, u.y, u.z, u.w};
      uint32_t h[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (xbf16) {
          const __half lo = __float2half_rn(__uint_as_float(wv[i] << 16) * prescale);
          const __half hi = __float2half_rn(__uint_as_float(wv[i] & 0xFFFF0000u) * prescale);
          overflow |= __hisinf(lo) | __hisinf(hi);
          h[2 * i] = __half_as_ushort(lo), h[2 * i + 1] = __half_as_ushort(hi);
        } else {
          h[2 * i] = wv[i] & 0xFFFFu, h[2 * i + 1] = wv[i] >> 16;
        }
      }
      if constexpr (PERM04)  // pairs (0,4),(1,5),(2,6),(3,7)
        *reinterpret_cast<uint4 *>(xs + (int64_t)mm * K + 8 * k8) =
            make_uint4(h[0] | (h[4] << 16), h[1] | (h[5] << 16), h[2] | (h[6] << 16), h[3] | (h[7] << 16));
      else  // natural pairs (0,1),(2,3),(4,5),(6,7)
        *reinterpret_cast<uint4 *>(xs + (int64_t)mm * K + 8 * k8) =
            make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16), h[6] | (h[7] << 16));
    }
  }
  return !overflow;
}

constexpr int PF = 2;  // chunks in flight per lane

template <int FMT, int SK>
__global__ void __launch_bounds__(WARPS * 32) gemv_bd_kernel(Params p, int xbf16) {
  constexpr int BITS = Fmt<FMT>::bits;
  extern __shared__ __align__(16) uint8_t smem[];
  const int K = (int)p.cols;
  __half *xs = reinterpret_cast<__half *>(smem);                         // [m][K] permuted fp16
  __half *zslot = xs + (size_t)p.m * K;                                  // CHUNK zeros
  float *red = reinterpret_cast<float *>(zslot + CHUNK);                 // [WARPS][2][ROWS]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int64_t n0 = (int64_t)blockIdx.x * ROWS;
  const int nchunks = K / CHUNK;
  const int c_begin = (nchunks * warp) / WARPS, c_end = (nchunks * (warp + 1)) / WARPS;
  const int64_t row_bytes = (int64_t)K * BITS / 8;
  // rows past the end read row 0 (results discarded) so no load is ever out of bounds
  const int64_t ra = n0 + g < p.rows ? n0 + g : 0, rb = n0 + g + 8 < p.rows ? n0 + g + 8 : 0;
  const uint8_t *wa = p.w + ra * row_bytes, *wb = p.w + rb * row_bytes;
  const int cm = t >> 1, cblk = 2 * (t & 1);  // accumulator columns 2t, 2t+1 -> (m, blocks)

  // Programmatic dependent launch: let the next kernel in the stream start its own weight
  // prefetch now (no-op unless it was launched with programmatic stream serialization).
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // weights and scales are parameters, not outputs of earlier kernels: start streaming them
  // before waiting on the previous kernel and before staging x
  Chunk<BITS> ring[PF];
#pragma unroll
  for (int j = 0; j < PF; ++j)
    if (c_begin + j < c_end) load_chunk<BITS, SK>(ring[j], p, wa, wb, c_begin + j, t, cblk, ra, rb);

  // x may be the previous kernel's output and y may still be read by it: wait for it to
  // finish (returns at once when this launch has no programmatic dependency)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (tid < CHUNK / 8) reinterpret_cast<uint4 *>(zslot)[tid] = make_uint4(0u, 0u, 0u, 0u);
  float prescale = 1.f;
  const bool ok = stage_x<pairs_04<FMT>()>(p, xs, K, xbf16 != 0, prescale);
  if (!__syncthreads_and(ok)) {  // rare: bf16 beyond fp16 range -> power-of-two prescale
    float amax = 0.f;
    for (int mm = 0; mm < (int)p.m; ++mm)
      for (int k = tid; k < K; k += blockDim.x)
        amax = fmaxf(amax, fabsf(__bfloat162float(((const __nv_bfloat16 *)p.x)[(int64_t)mm * p.ldx + k])));
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) red[warp] = amax;
    __syncthreads();
    for (int wv = 0; wv < WARPS; ++wv) amax = fmaxf(amax, red[wv]);
    const int ex = ((__float_as_int(amax) >> 23) & 0xFF) - 127;
    prescale = __int_as_float((127 - (ex - 14)) << 23);
    __syncthreads();
    stage_x<pairs_04<FMT>()>(p, xs, K, true, prescale);
  }
  __syncthreads();

  // B operand owner: lane (g, t) carries x of row m = g/4 for block t iff t == g % 4.
  const int bm = g >> 2;
  const bool owner = (t == (g & 3)) && bm < p.m;
  const __half *xrow = xs + (int64_t)bm * K + 32 * t;
  float acc_a = 0.f, acc_b = 0.f;  // rows g, g+8 for m = cm
  for (int c = c_begin; c < c_end; c += PF) {
#pragma unroll
    for (int j = 0; j < PF; ++j) {
      if (c + j < c_end) {
        compute_chunk<FMT, SK>(ring[j], owner ? xrow + (int64_t)(c + j) * CHUNK : zslot, acc_a, acc_b);
        if (c + j + PF < c_end) load_chunk<BITS, SK>(ring[j], p, wa, wb, c + j + PF, t, cblk, ra, rb);
      }
    }
  }
  // lanes t and t^1 hold the other two blocks of the same (m, rows)
  acc_a += __shfl_xor_sync(0xffffffffu, acc_a, 1);
  acc_b += __shfl_xor_sync(0xffffffffu, acc_b, 1);
  __syncthreads();
  if ((t & 1) == 0 && cm < p.m) {
    red[(warp * 2 + cm) * ROWS + g] = acc_a;
    red[(warp * 2 + cm) * ROWS + g + 8] = acc_b;
  }
  __syncthreads();
  if (tid < 2 * ROWS) {
    const int mm = tid / ROWS, r = tid % ROWS;
    const int64_t n = n0 + r;
    if (mm < p.m && n < p.rows) {
      float s = 0.f;
#pragma unroll
      for (int wv = 0; wv < WARPS; ++wv) s += red[(wv * 2 + mm) * ROWS + r];
      s *= place_factor<FMT>() / prescale;
      if constexpr (SK == SK_ROW) s *= load_as_f32(p.scales, n * p.nblk, p.sdt);
      store_f32(p.y, mm * p.ldy_m + n * p.ldy_n, p.ydt, s);
      for (int i = 0; i < p.ncopy; ++i) store_f32(p.ycopy[i], mm * p.ldy_m + n * p.ldy_n, p.ydt, s);
    }
  }
}

template <int FMT, int SK>
static int32_t launch_t(const Params &p, bool xbf16, cudaStream_t stream) {
  const size_t smem = (size_t)p.m * p.cols * 2 + CHUNK * 2 + WARPS * 2 * ROWS * sizeof(float);
  B200_CUDA_TRY((ensure_dynamic_smem<gemv_bd_kernel<FMT, SK>>(200 * 1024)));
  const unsigned grid = (unsigned)((p.rows + ROWS - 1) / ROWS);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(WARPS * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[1];
  attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = p.pdl ? 1 : 0;
  B200_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_bd_kernel<FMT, SK>, p, xbf16 ? 1 : 0));
  return B200_OK;
}

template <int FMT>
static int32_t dispatch_sk(const Params &p, int sk, bool xbf16, cudaStream_t stream) {
  switch (sk) {
    case SK_NONE: return launch_t<FMT, SK_NONE>(p, xbf16, stream);
    case SK_ROW: return launch_t<FMT, SK_ROW>(p, xbf16, stream);
    case SK_E8M0: return launch_t<FMT, SK_E8M0>(p, xbf16, stream);
    case SK_F16: return launch_t<FMT, SK_F16>(p, xbf16, stream);
    case SK_BF16: return launch_t<FMT, SK_BF16>(p, xbf16, stream);
    case SK_F32: return launch_t<FMT, SK_F32>(p, xbf16, stream);
    default: return launch_t<FMT, SK_GROUP>(p, xbf16, stream);
  }
}

static int scale_kind(const LinearArgs &a) {
  if (a.scales == nullptr) return SK_NONE;
  if (a.block >= a.cols) return SK_ROW;
  if (a.block == 32 && a.nblk % 2 == 0) {
    switch (a.sdt) {
      case B200_DT_E8M0: return SK_E8M0;
      case B200_DT_F16: return SK_F16;
      case B200_DT_BF16: return SK_BF16;
      case B200_DT_F32: return SK_F32;
    }
  }
  return SK_GROUP;
}

}  // namespace gemv

#ifndef B200_GEMV_TC_NO_ENTRY  // the entry points are defined once (gemv.cu); other users take the helpers
bool gemv_tc_supported(const LinearArgs &a) {
  using namespace gemv;
  if (a.m < 1 || a.m > 2) return false;
  if (a.xdt != B200_DT_F16 && a.xdt != B200_DT_BF16) return false;
  if (a.ydt != B200_DT_F16 && a.ydt != B200_DT_BF16 && a.ydt != B200_DT_F32) return false;
  if (a.cols < CHUNK || a.cols % CHUNK != 0 || a.rows <= 0 || a.cols > (int64_t)1 << 30) return false;
  if ((size_t)a.m * a.cols * 2 > 180 * 1024) return false;
  const int bits = fmt_bits(a.fmt);
  if ((uintptr_t)a.w % 16 != 0) return false;
  if (bits == 6 && (a.cols * 6 / 8) % 8 != 0) return false;
  if ((uintptr_t)a.x % 16 != 0 || (a.m > 1 && (a.ldx * 2) % 16 != 0)) return false;
  if (a.scales != nullptr) {
    if (!(a.sdt == B200_DT_F16 || a.sdt == B200_DT_BF16 || a.sdt == B200_DT_F32 || a.sdt == B200_DT_E8M0)) return false;
    if (!(a.block % 32 == 0 || a.block >= a.cols)) return false;
    const int esz = dt_size(a.sdt);
    if ((uintptr_t)a.scales % (2 * esz) != 0) return false;
  }
  return true;
}

int32_t launch_gemv_tc(const LinearArgs &a, cudaStream_t stream) {
  using namespace gemv;
  Params p;
  p.w = a.w;
  p.scales = a.scales;
  p.sdt = a.sdt;
  p.rows = a.rows;
  p.cols = a.cols;
  p.nblk = a.nblk;
  p.block = a.block;
  p.x = a.x;
  p.m = a.m;
  p.ldx = a.m > 1 ? a.ldx : a.cols;
  p.y = a.y;
  p.ydt = a.ydt;
  p.ldy_m = a.ldy_m;
  p.ldy_n = a.ldy_n;
  p.pdl = (a.flags & B200_FLAG_PDL) ? 1 : 0;
  p.ncopy = a.ncopy;
  for (int i = 0; i < 7; ++i) p.ycopy[i] = i < a.ncopy ? a.ycopy[i] : nullptr;
  const bool bf = a.xdt == B200_DT_BF16;
  const int sk = scale_kind(a);
  switch (a.fmt) {
    case B200_FMT_INT4: return dispatch_sk<B200_FMT_INT4>(p, sk, bf, stream);
    case B200_FMT_UINT4: return dispatch_sk<B200_FMT_UINT4>(p, sk, bf, stream);
    case B200_FMT_FP4_E2M1: return dispatch_sk<B200_FMT_FP4_E2M1>(p, sk, bf, stream);
    case B200_FMT_FP6_E2M3: return dispatch_sk<B200_FMT_FP6_E2M3>(p, sk, bf, stream);
    case B200_FMT_FP6_E3M2: return dispatch_sk<B200_FMT_FP6_E3M2>(p, sk, bf, stream);
  }
  return b200_set_error(B200_ERR_INVALID, "unknown packed format %d", a.fmt);
}

#endif  // B200_GEMV_TC_NO_ENTRY

}  // namespace b200
