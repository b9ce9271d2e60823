// Per-block quantization of 16-bit inputs in 128x128 tiles staged by TMA:
// GM = 128 quantizes each tile as one group (128x128 blocks), GM = 1 as 128
// row groups of 128 elements (1x128 blocks).
//
// Persistent CTAs (TileCfg::CTAS_PER_SM per SM) walk the 128x128 tiles.  Thread 0
// keeps kTileStages tiles (32 KB each) in flight with one
// cp.async.bulk.tensor load per tile (no multicast); the 256 threads take a
// landed tile from shared memory into registers (8 x 16 bytes each, so a warp
// reads 512 contiguous bytes: no bank conflicts), reduce its amax, hand the
// buffer back to the next load, and write fp8 + the tile's dequant scale.
// 128-192 KB of loads in flight per SM keep HBM busy without a CTA having to
// re-issue loads between its reduction and its stores.
#pragma once

#include "common.cuh"
#include "gemm_sm100.cuh"  // tma_load_3d
#include "quant_kernels.cuh"

namespace pcb {
namespace quant {

constexpr int kTileRows = 128;
// Tile bytes for element size ES (2: bf16 / fp16; 4: fp32, 128x128 groups only).
template <int ES>
__host__ __device__ constexpr int tile_bytes() { return 128 * 128 * ES; }
// Tiles in flight per SM (measured on B200 with bf16 inputs of 0.9-1.9 GB):
// 128x128 groups run two CTAs of 2 stages (128 KB; 0.85 of the HBM copy rate,
// against 0.72 for one CTA of 6 stages, whose per-tile CTA barrier then
// stalls the only resident CTA); 1x128 groups four CTAs of one stage (0.82,
// against 0.78 for three CTAs of 2 stages: while one CTA reduces and stores,
// the others' loads are in flight); fp32 128x128 tiles (64 KB) one CTA of 3.
template <int GM, int ES = 2>
struct TileCfg {
  static constexpr int STAGES = (GM == 1) ? 1 : (ES == 4 ? 3 : 2);
  static constexpr int CTAS_PER_SM = (GM == 1) ? 4 : (ES == 4 ? 1 : 2);
  static constexpr int SMEM = STAGES * tile_bytes<ES>() + 1024 + 64;
};

struct TileArgs {
  void* y;
  int64_t syb, sym;
  float* scale;
  int64_t ssb, ssm, ssn;
  int64_t m, n;
  int64_t groups_m, groups_n;  // groups_n = column tiles; groups_m = row groups (m for 1x128, row tiles for 128x128)
  int64_t num_tiles;
  float eps;
};

template <int XT, int YT, int MODE, int GM, int STAGES_ = TileCfg<GM, sizeof(typename InType<XT>::T)>::STAGES,
          int CTAS_ = TileCfg<GM, sizeof(typename InType<XT>::T)>::CTAS_PER_SM>
__global__ void __launch_bounds__(kThreads, CTAS_)
    quant_tile128_tma_kernel(const __grid_constant__ CUtensorMap tmap, const TileArgs a) {
  static_assert(XT == PCB_DTYPE_BF16 || XT == PCB_DTYPE_F16 || (XT == PCB_DTYPE_F32 && GM == 128),
                "16-bit inputs, or fp32 with 128x128 groups");
  static_assert(GM == 1 || GM == kTileRows, "whole-tile or per-row groups");
  using C = Chunk<XT>;
  constexpr int ES = (int)sizeof(typename C::T);
  constexpr int kTileBytes = tile_bytes<ES>();
  constexpr int kTileStages = STAGES_;
  constexpr int CPT = kTileBytes / 16 / kThreads;  // chunks per thread (8; 16 for fp32)
  constexpr int CPR = 128 * ES / 16;               // 16-byte chunks per 128-column row
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t s_base = smem_u32(smem);
  const uint32_t bar_full = s_base + kTileStages * kTileBytes;  // [kTileStages]
  __shared__ uint32_t red[2][kThreads / 32];
  __shared__ int abort_flag;

  const int t = threadIdx.x;
  const int warp = t >> 5;
  const int64_t first = blockIdx.x;
  const int64_t step = gridDim.x;
  const int64_t mine = first < a.num_tiles ? (a.num_tiles - 1 - first) / step + 1 : 0;
  // Tiles are 128 rows high whatever the group height.
  const int64_t tiles_m = (GM == 1) ? (a.groups_m + kTileRows - 1) / kTileRows : a.groups_m;
  const int64_t per_batch = tiles_m * a.groups_n;
  const float fp8_max = Fp8Max<YT>::value;

  auto issue = [&](int s, int64_t g) {
    const int64_t b = g / per_batch;
    const int64_t rem = g - b * per_batch;
    const int64_t gi = rem / a.groups_n;
    const int64_t gj = rem - gi * a.groups_n;
    const uint32_t fb = bar_full + 8 * s;
    mbar_arrive_expect_tx(fb, kTileBytes);  // out-of-range rows / columns arrive as zeros
    gemm::tma_load_3d(s_base + s * kTileBytes, &tmap, fb, (int)(gj * 128), (int)(gi * kTileRows), (int)b);
  };

  if (t == 0) {
    for (int s = 0; s < kTileStages; ++s) mbar_init(bar_full + 8 * s, 1);
    abort_flag = 0;
    fence_barrier_init();
    gemm::prefetch_tmap(&tmap);
  }
  __syncthreads();
  // A dependent kernel launched with programmatic stream serialization (the
  // scaled BMM) may start its prologue now; it waits for this grid to finish
  // before it reads anything.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (t == 0)
    for (int s = 0; s < kTileStages && s < mine; ++s) issue(s, first + s * step);

  int64_t it = 0;
  for (; it < mine; ++it) {
    const int s = (int)(it % kTileStages);
    if (!mbar_wait_bounded(bar_full + 8 * s, (uint32_t)((it / kTileStages) & 1), &abort_flag, SITE_QUANT_TILE)) break;
    const uint8_t* tile = smem + s * kTileBytes;
    C reg[CPT];
    uint32_t amax = 0;
#pragma unroll
    for (int i = 0; i < CPT; ++i) {
      reg[i].raw = *reinterpret_cast<const uint4*>(tile + (i * kThreads + t) * 16);
      amax = max(amax, reg[i].amax_bits());
    }
    if constexpr (GM == kTileRows) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, off));
      if ((t & 31) == 0) red[it & 1][warp] = amax;
    }
    __syncthreads();  // every thread holds its chunks: the buffer can be refilled
    if (t == 0 && it + kTileStages < mine) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(s, first + (it + kTileStages) * step);
    }

    const int64_t g = first + it * step;
    const int64_t b = g / per_batch;
    const int64_t rem = g - b * per_batch;
    const int64_t gi = rem / a.groups_n;  // tile row
    const int64_t gj = rem - gi * a.groups_n;
    uint8_t* yt = static_cast<uint8_t*>(a.y) + b * a.syb + gi * kTileRows * a.sym + gj * 128;
    if constexpr (GM == kTileRows) {
      uint32_t r = 0;
#pragma unroll
      for (int w = 0; w < kThreads / 32; ++w) r = max(r, red[it & 1][w]);
      const float safe = clamp_min_eps(__uint_as_float(r), a.eps);
      const float qs = mode_quant_scale<MODE>(safe, fp8_max);
      if (t == 0) {
        const float deq = mode_dequant_scale<MODE>(safe, fp8_max, qs);
        a.scale[b * a.ssb + gi * a.ssm + gj * a.ssn] = deq;
      }
#pragma unroll
      for (int i = 0; i < CPT; ++i) {
        const int c = i * kThreads + t;
        const int r_in = c / CPR;
        const int col = (c % CPR) * C::VEC;
        if (gi * kTileRows + r_in < a.m && gj * 128 + col < a.n) reg[i].template store<YT>(yt + r_in * a.sym + col, qs);
      }
    } else {
      // Row groups: register i of thread t is chunk t % 16 of tile row
      // 16 i + t / 16, so each row's amax reduces over 16 consecutive lanes.
      // The 16-bit magnitudes of two registers share one word, so each
      // shuffle step reduces two rows.
      const int col = (t & 15) * 8;
      uint32_t rmax[CPT];
#pragma unroll
      for (int i = 0; i < CPT; i += 2) {
        uint32_t w = reg[i].amax16() | (reg[i + 1].amax16() << 16);
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) w = __vmaxu2(w, __shfl_xor_sync(0xffffffffu, w, off));
        rmax[i] = C::bits16_to_f32_bits(w & 0xffffu);
        rmax[i + 1] = C::bits16_to_f32_bits(w >> 16);
      }
      // The 16 lanes of a row group all hold rmax[0..CPT); lane j < CPT
      // derives the scales of register row j once, and the group reads them
      // back by shuffles (one reciprocal per lane instead of CPT).
      const int j = t & 15;
      uint32_t my_max = rmax[0];
#pragma unroll
      for (int i = 1; i < CPT; ++i) my_max = (j == i) ? rmax[i] : my_max;
      const float my_safe = clamp_min_eps(__uint_as_float(my_max), a.eps);
      const float my_qs = mode_quant_scale<MODE>(my_safe, fp8_max);
      if (j < CPT) {
        const int64_t row = gi * kTileRows + j * 16 + (t >> 4);
        if (row < a.m) a.scale[b * a.ssb + row * a.ssm + gj * a.ssn] = mode_dequant_scale<MODE>(my_safe, fp8_max, my_qs);
      }
#pragma unroll
      for (int i = 0; i < CPT; ++i) {
        const float qs = __shfl_sync(0xffffffffu, my_qs, (t & 16) | i);
        const int64_t row = gi * kTileRows + i * 16 + (t >> 4);
        if (row < a.m && gj * 128 + col < a.n) reg[i].template store<YT>(yt + (i * 16 + (t >> 4)) * a.sym + col, qs);
      }
    }
  }
  if (it < mine && t == 0) {
    // Aborted: let the loads already issued land before the CTA exits (each
    // wait again bounded; the CTA's abort flag is not consulted here).
    volatile int keep_waiting = 0;
    for (int64_t j = it; j < mine && j < it + kTileStages; ++j)
      mbar_wait_bounded(bar_full + 8 * (int)(j % kTileStages), (uint32_t)((j / kTileStages) & 1), &keep_waiting,
                        SITE_QUANT_TILE);
  }
}

}  // namespace quant
}  // namespace pcb
