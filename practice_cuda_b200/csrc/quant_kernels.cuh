// FP8 quantization kernels (HBM-bound): per-block / per-channel-row groups,
// per-channel columns (cluster + DSMEM reduction), per-tensor (two launches),
// and a generic strided fallback.  All produce bytes identical to the torch
// CPU restatement (see common.cuh for the scale arithmetic).
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"

namespace pcb {
namespace quant {

namespace cg = cooperative_groups;

constexpr int kThreads = 256;

enum ScaleMode : int {
  kDeqReciprocal = 0,  // dequant = 1 / quant_scale     (per-block, per-tensor)
  kDeqDivide = 1,      // dequant = amax / fp8_max       (per-channel)
  kDeqPow2 = 2,        // quant scale a power of two (E8M0), dequant = its reciprocal
  kQuantDivide = 3,    // dynamic float8 cast: quant scale = fp8_max / amax (one IEEE divide),
                       // and the stored scale is that quant scale
};

template <int MODE>
__device__ __forceinline__ float mode_quant_scale(float safe, float fp8_max) {
  if constexpr (MODE == kDeqPow2) return pow2_quant_scale(safe, fp8_max);
  else if constexpr (MODE == kQuantDivide) return __fdiv_rn(fp8_max, safe);
  else return quant_scale_from_amax(safe, fp8_max);
}

// The scale a kernel stores: the dequant scale, or (kQuantDivide) the quant scale.
template <int MODE>
__device__ __forceinline__ float mode_dequant_scale(float safe, float fp8_max, float qs) {
  if constexpr (MODE == kDeqDivide) return __fdiv_rn(safe, fp8_max);
  else if constexpr (MODE == kQuantDivide) return qs;
  else return __frcp_rn(qs);
}

struct GroupArgs {
  const void* x;
  int64_t sxb, sxm;  // x strides (elements); x is contiguous along n
  void* y;
  int64_t syb, sym;  // y strides (elements); y is contiguous along n
  float* scale;
  int64_t ssb, ssm, ssn;
  int64_t batch, m, n;
  int64_t gm, gn;        // group extent (rows, cols)
  int64_t groups_m, groups_n;
  int64_t num_groups;
  float eps;
};

// 16-byte chunk of input kept as raw bits (4 registers); converted to fp32
// element by element when needed.
template <int XT>
struct Chunk {
  using T = typename InType<XT>::T;
  static constexpr int VEC = 16 / (int)sizeof(T);
  uint4 raw;
  __device__ __forceinline__ void load(const T* p) { raw = __ldg(reinterpret_cast<const uint4*>(p)); }
  __device__ __forceinline__ uint32_t word(int i) const {
    return i == 0 ? raw.x : i == 1 ? raw.y : i == 2 ? raw.z : raw.w;
  }
  __device__ __forceinline__ float v(int i) const {
    if constexpr (XT == PCB_DTYPE_F32) {
      return __uint_as_float(word(i));
    } else if constexpr (XT == PCB_DTYPE_BF16) {
      const uint32_t w = word(i >> 1);
      return __uint_as_float((i & 1) ? (w & 0xffff0000u) : (w << 16));
    } else {
      const uint32_t w = word(i >> 1);
      return __half2float(__ushort_as_half((unsigned short)((i & 1) ? (w >> 16) : (w & 0xffffu))));
    }
  }
  // 16-bit inputs: max |x| over the chunk as raw 16-bit magnitude bits
  // (monotonic in |x| for bf16 and fp16, NaN above inf).
  __device__ __forceinline__ uint32_t amax16() const {
    const uint32_t m2 = __vmaxu2(__vmaxu2(raw.x & 0x7fff7fffu, raw.y & 0x7fff7fffu),
                                 __vmaxu2(raw.z & 0x7fff7fffu, raw.w & 0x7fff7fffu));
    return max(m2 & 0xffffu, m2 >> 16);
  }
  static __device__ __forceinline__ uint32_t bits16_to_f32_bits(uint32_t m) {
    if constexpr (XT == PCB_DTYPE_BF16) return m << 16;
    else return __float_as_uint(__half2float(__ushort_as_half((unsigned short)m)));
  }
  // max |x| over the chunk as fp32 bits (NaN compares above +inf).
  __device__ __forceinline__ uint32_t amax_bits() const {
    if constexpr (XT == PCB_DTYPE_F32) {
      return max(max(raw.x & 0x7fffffffu, raw.y & 0x7fffffffu), max(raw.z & 0x7fffffffu, raw.w & 0x7fffffffu));
    } else {
      const uint32_t m2 = __vmaxu2(__vmaxu2(raw.x & 0x7fff7fffu, raw.y & 0x7fff7fffu),
                                   __vmaxu2(raw.z & 0x7fff7fffu, raw.w & 0x7fff7fffu));
      const uint32_t m = max(m2 & 0xffffu, m2 >> 16);
      if constexpr (XT == PCB_DTYPE_BF16) {
        return m << 16;
      } else {
        return __float_as_uint(__half2float(__ushort_as_half((unsigned short)m)));
      }
    }
  }
  // Elements 2j, 2j+1 as fp32 (16-bit inputs).
  __device__ __forceinline__ float2 pair(int j) const {
    const uint32_t w = word(j);
    if constexpr (XT == PCB_DTYPE_BF16) {
      return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
    } else {
      return __half22float2(*reinterpret_cast<const __half2*>(&w));
    }
  }
  template <int YT>
  __device__ __forceinline__ void store(uint8_t* q, float qs) const {
    if constexpr (VEC == 8) {
      // Two IEEE fp32 products per FMUL2 (bit-identical to two __fmul_rn).
      const float2 q2 = make_float2(qs, qs);
      const float2 p0 = __fmul2_rn(pair(0), q2), p1 = __fmul2_rn(pair(1), q2);
      const float2 p2 = __fmul2_rn(pair(2), q2), p3 = __fmul2_rn(pair(3), q2);
      uint2 out;
      out.x = (uint32_t)cvt2_fp8<YT>(p0.x, p0.y) | ((uint32_t)cvt2_fp8<YT>(p1.x, p1.y) << 16);
      out.y = (uint32_t)cvt2_fp8<YT>(p2.x, p2.y) | ((uint32_t)cvt2_fp8<YT>(p3.x, p3.y) << 16);
      *reinterpret_cast<uint2*>(q) = out;
    } else {
      uint32_t out = (uint32_t)cvt2_fp8<YT>(__fmul_rn(v(0), qs), __fmul_rn(v(1), qs)) |
                     ((uint32_t)cvt2_fp8<YT>(__fmul_rn(v(2), qs), __fmul_rn(v(3), qs)) << 16);
      *reinterpret_cast<uint32_t*>(q) = out;
    }
  }
};

// Max-reduce `v` over a team of TEAM consecutive threads (TEAM a power of two
// <= 256).  Teams of <= 32 stay inside a warp; larger teams use `red` (one
// slot per warp of the CTA).
template <int TEAM>
__device__ __forceinline__ uint32_t team_max(uint32_t v, uint32_t* red) {
  if constexpr (TEAM <= 32) {
#pragma unroll
    for (int off = TEAM / 2; off > 0; off >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
  } else {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, off));
    constexpr int WARPS = TEAM / 32;
    const int warp = threadIdx.x >> 5;
    const int team_warp0 = (warp / WARPS) * WARPS;
    __syncwarp();
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    uint32_t r = 0;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) r = max(r, red[team_warp0 + w]);
    __syncthreads();
    return r;
  }
}

// One team of TEAM threads per quant group; each thread keeps up to CH
// 16-byte chunks in registers (larger groups re-read the remainder from L2).
// Grid-strided over groups.  Requires: x, y contiguous along n, 16-byte
// aligned rows of x, VEC-byte aligned rows of y, n % VEC == 0.
template <int XT, int YT, int TEAM, int CH, int MODE>
__global__ void __launch_bounds__(kThreads) quant_groups_kernel(const GroupArgs args) {
  using C = Chunk<XT>;
  using T = typename C::T;
  constexpr int VEC = C::VEC;
  constexpr int TEAMS_PER_CTA = kThreads / TEAM;
  __shared__ uint32_t red[kThreads / 32];

  const int t = threadIdx.x % TEAM;
  const int team_in_cta = threadIdx.x / TEAM;
  const int64_t team_stride = (int64_t)gridDim.x * TEAMS_PER_CTA;
  const float fp8_max = Fp8Max<YT>::value;
  const T* __restrict__ xbase = static_cast<const T*>(args.x);
  uint8_t* __restrict__ ybase = static_cast<uint8_t*>(args.y);

  // All teams of a CTA run the same number of iterations so the CTA-wide
  // reduction (TEAM > 32) never diverges around __syncthreads.
  const int64_t iters = (args.num_groups + team_stride - 1) / team_stride;
  for (int64_t it = 0; it < iters; ++it) {
    const int64_t g = it * team_stride + (int64_t)blockIdx.x * TEAMS_PER_CTA + team_in_cta;
    const bool active = g < args.num_groups;
    int64_t b = 0, gi = 0, gj = 0, row0 = 0, col0 = 0;
    int rows = 0, cpr = 1, nch = 0;
    if (active) {
      b = g / (args.groups_m * args.groups_n);
      const int64_t rem = g - b * args.groups_m * args.groups_n;
      gi = rem / args.groups_n;
      gj = rem - gi * args.groups_n;
      row0 = gi * args.gm;
      col0 = gj * args.gn;
      rows = (int)min(args.gm, args.m - row0);
      cpr = (int)(min(args.gn, args.n - col0) / VEC);
      nch = rows * cpr;
    }
    const T* xg = xbase + b * args.sxb + row0 * args.sxm + col0;
    uint8_t* yg = ybase + b * args.syb + row0 * args.sym + col0;

    C reg[CH];
    uint32_t amax = 0;
    if (nch == CH * TEAM && cpr == nch) {
      // A full single-row group: all CH loads issue before any of them is
      // used (per-chunk bounds checks would keep them in program order).
#pragma unroll
      for (int i = 0; i < CH; ++i) reg[i].load(xg + (i * TEAM + t) * VEC);
#pragma unroll
      for (int i = 0; i < CH; ++i) amax = max(amax, reg[i].amax_bits());
    } else {
#pragma unroll
      for (int i = 0; i < CH; ++i) {
        const int c = i * TEAM + t;
        if (c < nch) {
          const int r = c / cpr;
          const int cc = c - r * cpr;
          reg[i].load(xg + r * args.sxm + cc * VEC);
          amax = max(amax, reg[i].amax_bits());
        }
      }
    }
    for (int c = CH * TEAM + t; c < nch; c += TEAM) {  // groups larger than the register tile
      const int r = c / cpr;
      const int cc = c - r * cpr;
      C tmp;
      tmp.load(xg + r * args.sxm + cc * VEC);
      amax = max(amax, tmp.amax_bits());
    }
    amax = team_max<TEAM>(amax, red);

    const float safe = clamp_min_eps(__uint_as_float(amax), args.eps);
    const float qs = mode_quant_scale<MODE>(safe, fp8_max);
    if (active && t == 0) {
      const float deq = mode_dequant_scale<MODE>(safe, fp8_max, qs);
      args.scale[b * args.ssb + gi * args.ssm + gj * args.ssn] = deq;
    }
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      const int c = i * TEAM + t;
      if (c < nch) {
        const int r = c / cpr;
        const int cc = c - r * cpr;
        reg[i].template store<YT>(yg + r * args.sym + cc * VEC, qs);
      }
    }
    for (int c = CH * TEAM + t; c < nch; c += TEAM) {
      const int r = c / cpr;
      const int cc = c - r * cpr;
      C tmp;
      tmp.load(xg + r * args.sxm + cc * VEC);
      tmp.template store<YT>(yg + r * args.sym + cc * VEC, qs);
    }
  }
}

// Row groups (block_m == 1) of CPG <= 32 chunks, e.g. 1x128 tiles: each warp
// streams a contiguous span of 32*CH chunks of one row, so every load
// instruction covers 512 contiguous bytes and each thread keeps CH 16-byte
// loads in flight.  Register i of lane l holds chunk i*32+l of the span,
// which belongs to group (i*32+l)/CPG: the amax of register i reduces over
// aligned runs of CPG lanes.
struct RowSpanArgs {
  const void* x;
  int64_t sxb, sxm;
  void* y;
  int64_t syb, sym;
  float* scale;
  int64_t ssb, ssm, ssn;
  int64_t m, n;
  int64_t rows;           // batch * m
  int64_t spans_per_row;
  int64_t units;          // rows * spans_per_row
  float eps;
};

template <int XT, int YT, int CPG, int CH, int MODE>
__global__ void __launch_bounds__(kThreads, 3) quant_rowspan_kernel(const RowSpanArgs args) {
  using C = Chunk<XT>;
  using T = typename C::T;
  constexpr int VEC = C::VEC;
  constexpr int SPAN_CHUNKS = 32 * CH;
  constexpr int GN = CPG * VEC;  // group width in elements
  static_assert(CPG <= 32 && (32 % CPG) == 0, "groups must tile a warp");
  const int lane = threadIdx.x & 31;
  const int64_t warp_global = ((int64_t)blockIdx.x * kThreads + threadIdx.x) >> 5;
  const int64_t warp_stride = ((int64_t)gridDim.x * kThreads) >> 5;
  const float fp8_max = Fp8Max<YT>::value;
  const int64_t nchunks_row = args.n / VEC;
  for (int64_t u = warp_global; u < args.units; u += warp_stride) {
    const int64_t row = u / args.spans_per_row;
    const int64_t span = u - row * args.spans_per_row;
    const int64_t bi = row / args.m, r = row - bi * args.m;
    const T* xr = static_cast<const T*>(args.x) + bi * args.sxb + r * args.sxm;
    uint8_t* yr = static_cast<uint8_t*>(args.y) + bi * args.syb + r * args.sym;
    const int64_t c0 = span * SPAN_CHUNKS;
    // Chunks of this lane: c0 + i*32 + lane for i < CH, valid while < nchunks_row.
    const int64_t left = nchunks_row - c0 - lane;
    const int valid = (int)(left <= 0 ? 0 : (left + 31) / 32);
    const T* xs = xr + (c0 + lane) * VEC;
    uint8_t* ys = yr + (c0 + lane) * VEC;
    C reg[CH];
    uint32_t am[CH];
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      am[i] = 0;
      if (i < valid) {
        reg[i].load(xs + i * 32 * VEC);
        am[i] = reg[i].amax_bits();
      }
    }
#pragma unroll
    for (int i = 0; i < CH; ++i) {
#pragma unroll
      for (int off = CPG / 2; off > 0; off >>= 1) am[i] = max(am[i], __shfl_xor_sync(0xffffffffu, am[i], off));
    }
    float* srow = args.scale + bi * args.ssb + r * args.ssm;
    const int64_t g0 = ((c0 + lane) * VEC) / GN;  // group of register 0
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      if (i < valid) {
        const float safe = clamp_min_eps(__uint_as_float(am[i]), args.eps);
        const float qs = quant_scale_from_amax(safe, fp8_max);
        reg[i].template store<YT>(ys + i * 32 * VEC, qs);
        if ((lane % CPG) == 0) {
          const float deq = (MODE == kDeqReciprocal) ? __frcp_rn(qs) : __fdiv_rn(safe, fp8_max);
          srow[(g0 + i * (32 * VEC / GN)) * args.ssn] = deq;
        }
      }
    }
  }
}

// Generic fallback: one CTA per group, scalar strided loads, two passes.
struct GenericArgs {
  const void* x;
  int64_t sxb, sxm, sxn;
  void* y;
  int64_t syb, sym, syn;
  float* scale;
  int64_t ssb, ssm, ssn;
  int64_t batch, m, n;
  int64_t gm, gn, groups_m, groups_n, num_groups;
  float eps;
};

template <int XT, int YT, int MODE>
__global__ void __launch_bounds__(kThreads) quant_groups_generic_kernel(const GenericArgs args) {
  using T = typename InType<XT>::T;
  __shared__ uint32_t red[kThreads / 32];
  const float fp8_max = Fp8Max<YT>::value;
  const T* xbase = static_cast<const T*>(args.x);
  uint8_t* ybase = static_cast<uint8_t*>(args.y);
  for (int64_t g = blockIdx.x; g < args.num_groups; g += gridDim.x) {
    const int64_t b = g / (args.groups_m * args.groups_n);
    const int64_t rem = g - b * args.groups_m * args.groups_n;
    const int64_t gi = rem / args.groups_n;
    const int64_t gj = rem - gi * args.groups_n;
    const int64_t row0 = gi * args.gm, col0 = gj * args.gn;
    const int64_t rows = min(args.gm, args.m - row0);
    const int64_t cols = min(args.gn, args.n - col0);
    const int64_t count = rows * cols;
    uint32_t amax = 0;
    for (int64_t e = threadIdx.x; e < count; e += kThreads) {
      const int64_t r = e / cols, c = e - (e / cols) * cols;
      const T v = xbase[b * args.sxb + (row0 + r) * args.sxm + (col0 + c) * args.sxn];
      amax = max(amax, abs_bits(InType<XT>::to_f32(v)));
    }
    amax = team_max<kThreads>(amax, red);
    const float safe = clamp_min_eps(__uint_as_float(amax), args.eps);
    const float qs = mode_quant_scale<MODE>(safe, fp8_max);
    if (threadIdx.x == 0) args.scale[b * args.ssb + gi * args.ssm + gj * args.ssn] = mode_dequant_scale<MODE>(safe, fp8_max, qs);
    for (int64_t e = threadIdx.x; e < count; e += kThreads) {
      const int64_t r = e / cols, c = e - (e / cols) * cols;
      const float v =
          InType<XT>::to_f32(xbase[b * args.sxb + (row0 + r) * args.sxm + (col0 + c) * args.sxn]);
      ybase[b * args.syb + (row0 + r) * args.sym + (col0 + c) * args.syn] =
          cvt1_fp8<YT>(__fmul_rn(v, qs));
    }
  }
}

// Per-channel column quantization (one scale per column; reduce over rows) for
// row-major x.  A cluster of CL CTAs shares one strip of 8*VEC columns, each
// CTA taking a slice of the rows; the column amax is combined through
// distributed shared memory, then every CTA quantizes its slice (second read
// hits L2).
struct ColArgs {
  const void* x;
  int64_t sxb, sxm;
  void* y;
  int64_t syb, sym;
  float* scale;
  int64_t ssb, ssc;
  int64_t m, n;
  int rows_per_cta;
  float eps;
  int64_t ss_slab;  // SLAB mode: scale stride between row slabs
};

// SLAB = false: per-channel columns (one scale per column over all rows, the
//               rows split over a cluster, dequant = amax / fp8_max).
// SLAB = true:  per-block (rows_per_cta x 1) blocks, e.g. 128 x 1: CTA
//               blockIdx.y owns one row slab, dequant = 1 / quant_scale.
// Both passes over the slab (amax, then the cast, whose re-read hits L2) take
// the thread's rows kUnroll at a time with the loads issued first, so a CTA
// keeps kUnroll 16-byte loads per thread in flight.
constexpr int kColUnroll = 6;
template <int XT, int YT, bool SLAB = false, int MODE = kDeqReciprocal>
__global__ void __launch_bounds__(kThreads, 4) quant_cols_cluster_kernel(const ColArgs args) {
  using C = Chunk<XT>;
  using T = typename C::T;
  constexpr int VEC = C::VEC;
  constexpr int CHUNK_COLS = 8;               // chunks across the strip
  constexpr int SW = CHUNK_COLS * VEC;        // strip width in columns
  constexpr int ROW_LANES = kThreads / CHUNK_COLS;  // 32
  __shared__ uint32_t red[ROW_LANES][SW + 1];
  __shared__ uint32_t partial[SW];
  __shared__ float qs_s[SW];

  const float fp8_max = Fp8Max<YT>::value;
  int rank = 0, nranks = 1;
  if constexpr (!SLAB) {
    rank = (int)cg::this_cluster().block_rank();
    nranks = (int)cg::this_cluster().num_blocks();
  }

  const int64_t b = blockIdx.z;
  const int64_t col0 = (int64_t)blockIdx.x * SW;
  const int cc = threadIdx.x % CHUNK_COLS;
  const int rl = threadIdx.x / CHUNK_COLS;
  const int64_t col = col0 + (int64_t)cc * VEC;
  const bool col_ok = col < args.n;  // n % VEC == 0, so a chunk is all-in or all-out
  const int64_t slab = SLAB ? (int64_t)blockIdx.y : (int64_t)rank;
  const int64_t r_begin = slab * args.rows_per_cta;
  const int64_t r_end = min(args.m, r_begin + args.rows_per_cta);
  const T* xb = static_cast<const T*>(args.x) + b * args.sxb;
  uint8_t* yb = static_cast<uint8_t*>(args.y) + b * args.syb;

  // Column amax as ordered magnitude bits.  16-bit inputs keep two columns
  // per word and reduce them with packed unsigned 16-bit max (NaN compares
  // above inf), widened to fp32 bits once at the end.
  uint32_t am[VEC];
  uint32_t am2[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int i = 0; i < VEC; ++i) am[i] = 0;
  if (col_ok) {
    for (int64_t r0 = r_begin + rl; r0 < r_end; r0 += (int64_t)kColUnroll * ROW_LANES) {
      C ch[kColUnroll];
#pragma unroll
      for (int j = 0; j < kColUnroll; ++j) {
        const int64_t r = r0 + (int64_t)j * ROW_LANES;
        if (r < r_end) ch[j].load(xb + r * args.sxm + col);
        else ch[j].raw = make_uint4(0u, 0u, 0u, 0u);  // |0| leaves the amax unchanged
      }
#pragma unroll
      for (int j = 0; j < kColUnroll; ++j) {
        if constexpr (XT == PCB_DTYPE_F32) {
#pragma unroll
          for (int i = 0; i < VEC; ++i) am[i] = max(am[i], abs_bits(ch[j].v(i)));
        } else {
#pragma unroll
          for (int w = 0; w < 4; ++w) am2[w] = __vmaxu2(am2[w], ch[j].word(w) & 0x7fff7fffu);
        }
      }
    }
  }
  if constexpr (XT != PCB_DTYPE_F32) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      am[2 * w] = C::bits16_to_f32_bits(am2[w] & 0xffffu);
      am[2 * w + 1] = C::bits16_to_f32_bits(am2[w] >> 16);
    }
  }
#pragma unroll
  for (int i = 0; i < VEC; ++i) red[rl][cc * VEC + i] = am[i];
  __syncthreads();
  if (threadIdx.x < SW) {
    uint32_t v = 0;
    for (int l = 0; l < ROW_LANES; ++l) v = max(v, red[l][threadIdx.x]);
    partial[threadIdx.x] = v;
  }
  if constexpr (SLAB) {
    __syncthreads();
  } else {
    cg::this_cluster().sync();
  }
  if (threadIdx.x < SW) {
    uint32_t v = 0;
    if constexpr (SLAB) {
      v = partial[threadIdx.x];
    } else {
      for (int r = 0; r < nranks; ++r) v = max(v, cg::this_cluster().map_shared_rank(partial, r)[threadIdx.x]);
    }
    const float safe = clamp_min_eps(__uint_as_float(v), args.eps);
    const float qs = SLAB ? mode_quant_scale<MODE>(safe, fp8_max) : quant_scale_from_amax(safe, fp8_max);
    qs_s[threadIdx.x] = qs;
    const int64_t c = col0 + threadIdx.x;
    if (SLAB && c < args.n) {
      args.scale[b * args.ssb + slab * args.ss_slab + c * args.ssc] = __frcp_rn(qs);
    } else if (!SLAB && rank == 0 && c < args.n) {
      args.scale[b * args.ssb + c * args.ssc] = __fdiv_rn(safe, fp8_max);
    }
  }
  if constexpr (SLAB) {
    __syncthreads();
  } else {
    cg::this_cluster().sync();  // remote reads of `partial` are done; qs_s visible to the CTA
  }
  // This thread's column scales, read from shared memory once.
  float qreg[VEC];
#pragma unroll
  for (int i = 0; i < VEC; ++i) qreg[i] = qs_s[cc * VEC + i];
  // Chunk::store takes one scale; columns differ, so convert pairwise here.
  auto cast_store = [&](const C& ch, int64_t r) {
    uint8_t out[VEC];
#pragma unroll
    for (int i = 0; i < VEC; i += 2) {
      const uint16_t p = cvt2_fp8<YT>(__fmul_rn(ch.v(i), qreg[i]), __fmul_rn(ch.v(i + 1), qreg[i + 1]));
      out[i] = (uint8_t)(p & 0xff);
      out[i + 1] = (uint8_t)(p >> 8);
    }
    if constexpr (VEC == 8) {
      *reinterpret_cast<uint2*>(yb + r * args.sym + col) = *reinterpret_cast<const uint2*>(out);
    } else {
      *reinterpret_cast<uint32_t*>(yb + r * args.sym + col) = *reinterpret_cast<const uint32_t*>(out);
    }
  };
  if (col_ok) {
    for (int64_t r0 = r_begin + rl; r0 < r_end; r0 += (int64_t)kColUnroll * ROW_LANES) {
      C ch[kColUnroll];
#pragma unroll
      for (int j = 0; j < kColUnroll; ++j) {
        const int64_t r = r0 + (int64_t)j * ROW_LANES;
        if (r < r_end) ch[j].load(xb + r * args.sxm + col);
      }
#pragma unroll
      for (int j = 0; j < kColUnroll; ++j) {
        const int64_t r = r0 + (int64_t)j * ROW_LANES;
        if (r < r_end) cast_store(ch[j], r);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Per-tensor: (1) per-CTA amax partials, (2) every CTA of the cast kernel
// reduces the partials (deterministic), derives the scale in `scale_dtype`
// arithmetic and quantizes its share; CTA 0 writes the two scale outputs.
// ---------------------------------------------------------------------------
struct TensorArgs {
  const void* x;
  int64_t sxb, sxm, sxn;
  void* y;
  int64_t syb, sym, syn;
  int64_t batch, m, n;
  bool vec;  // contiguous along n, aligned, n % VEC == 0
  float* partials;
  int num_partials;
  float* quant_scale;
  float* dequant_scale;
  int scale_dtype;
  float fp8_max;
  float eps;
  // Dynamic float8 cast numerics: quant scale = fp8_max / amax (one fp32
  // IEEE divide, which equals torchAO's float64 divide rounded to fp32).
  int quant_divide;
};

constexpr int kPerTensorMaxPartials = 1024;

__device__ __forceinline__ float round_to(float v, int dt) {
  if (dt == PCB_DTYPE_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dt == PCB_DTYPE_F16) return __half2float(__float2half_rn(v));
  return v;
}

template <int XT>
__global__ void __launch_bounds__(kThreads) tensor_amax_kernel(const TensorArgs args) {
  using C = Chunk<XT>;
  using T = typename C::T;
  constexpr int VEC = C::VEC;
  __shared__ uint32_t red[kThreads / 32];
  const T* xb = static_cast<const T*>(args.x);
  uint32_t amax = 0;
  const int64_t rows = args.batch * args.m;
  const int64_t tid = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  if (args.vec) {
    const int64_t cpr = args.n / VEC;
    const int64_t total = rows * cpr;
    for (int64_t c = tid; c < total; c += stride) {
      const int64_t row = c / cpr;
      const int64_t bi = row / args.m, r = row - bi * args.m;
      C ch;
      ch.load(xb + bi * args.sxb + r * args.sxm + (c - row * cpr) * VEC);
      amax = max(amax, ch.amax_bits());
    }
  } else {
    const int64_t total = rows * args.n;
    for (int64_t e = tid; e < total; e += stride) {
      const int64_t row = e / args.n;
      const int64_t bi = row / args.m, r = row - bi * args.m;
      amax = max(amax, abs_bits(InType<XT>::to_f32(xb[bi * args.sxb + r * args.sxm + (e - row * args.n) * args.sxn])));
    }
  }
  amax = team_max<kThreads>(amax, red);
  if (threadIdx.x == 0) args.partials[blockIdx.x] = __uint_as_float(amax);
}

template <int XT, int YT>
__global__ void __launch_bounds__(kThreads) tensor_cast_kernel(const TensorArgs args) {
  using C = Chunk<XT>;
  using T = typename C::T;
  constexpr int VEC = C::VEC;
  __shared__ uint32_t red[kThreads / 32];
  uint32_t amax = 0;
  for (int i = threadIdx.x; i < args.num_partials; i += kThreads)
    amax = max(amax, __float_as_uint(args.partials[i]));
  amax = team_max<kThreads>(amax, red);
  // x_max_abs.clamp(min=eps) -> fp8_max / x -> reciprocal, all in scale_dtype.
  const int dt = args.scale_dtype;
  const float a = __uint_as_float(amax);
  const float eps_dt = round_to(args.eps, dt);
  const float safe = (a < eps_dt) ? eps_dt : a;
  const float qs = args.quant_divide ? __fdiv_rn(args.fp8_max, safe)
                                     : round_to(__fmul_rn(round_to(__frcp_rn(safe), dt), args.fp8_max), dt);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    if (args.quant_scale) *args.quant_scale = qs;
    if (args.dequant_scale) *args.dequant_scale = round_to(__frcp_rn(qs), dt);
  }
  const T* xb = static_cast<const T*>(args.x);
  uint8_t* yb = static_cast<uint8_t*>(args.y);
  const int64_t rows = args.batch * args.m;
  const int64_t tid = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  if (args.vec) {
    const int64_t cpr = args.n / VEC;
    const int64_t total = rows * cpr;
    for (int64_t c = tid; c < total; c += stride) {
      const int64_t row = c / cpr;
      const int64_t bi = row / args.m, r = row - bi * args.m;
      const int64_t col = (c - row * cpr) * VEC;
      C ch;
      ch.load(xb + bi * args.sxb + r * args.sxm + col);
      ch.template store<YT>(yb + bi * args.syb + r * args.sym + col, qs);
    }
  } else {
    const int64_t total = rows * args.n;
    for (int64_t e = tid; e < total; e += stride) {
      const int64_t row = e / args.n;
      const int64_t bi = row / args.m, r = row - bi * args.m;
      const int64_t col = e - row * args.n;
      const float v = InType<XT>::to_f32(xb[bi * args.sxb + r * args.sxm + col * args.sxn]);
      yb[bi * args.syb + r * args.sym + col * args.syn] = cvt1_fp8<YT>(__fmul_rn(v, qs));
    }
  }
}

// ---------------------------------------------------------------------------
// Byte repack (layout change / zero padding) for fp8 operands.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) pack_u8_kernel(const uint8_t* src, int64_t batch, int64_t rows,
                                                           int64_t cols, int64_t ssb, int64_t ssr, int64_t ssc,
                                                           uint8_t* dst, int64_t dsb, int64_t dsr, int64_t cols_padded) {
  const int64_t total = batch * rows * cols_padded;
  for (int64_t e = (int64_t)blockIdx.x * kThreads + threadIdx.x; e < total; e += (int64_t)gridDim.x * kThreads) {
    const int64_t row = e / cols_padded;
    const int64_t c = e - row * cols_padded;
    const int64_t bi = row / rows, r = row - bi * rows;
    dst[bi * dsb + r * dsr + c] = (c < cols) ? src[bi * ssb + r * ssr + c * ssc] : (uint8_t)0;
  }
}

}  // namespace quant
}  // namespace pcb
