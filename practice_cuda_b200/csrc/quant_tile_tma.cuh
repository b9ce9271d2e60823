// 128x128 per-block quantization of 16-bit inputs, staged by TMA.
//
// One persistent CTA per SM walks its share of the 128x128 tiles.  Thread 0
// keeps kTileStages tiles (32 KB each) in flight with one
// cp.async.bulk.tensor load per tile (no multicast); the 256 threads take a
// landed tile from shared memory into registers (8 x 16 bytes each, so a warp
// reads 512 contiguous bytes: no bank conflicts), reduce its amax, hand the
// buffer back to the next load, and write fp8 + the tile's dequant scale.
// 192 KB of loads in flight per SM keep HBM busy without the CTA having to
// re-issue loads between its reduction and its stores.
#pragma once

#include "common.cuh"
#include "gemm_sm100.cuh"  // tma_load_3d
#include "quant_kernels.cuh"

namespace pcb {
namespace quant {

constexpr int kTileStages = 6;
constexpr int kTileRows = 128;
constexpr int kTileBytes = 128 * 128 * 2;
constexpr int kTileSmem = kTileStages * kTileBytes + 1024 + 64;

struct TileArgs {
  void* y;
  int64_t syb, sym;
  float* scale;
  int64_t ssb, ssm, ssn;
  int64_t m, n;
  int64_t groups_m, groups_n, num_groups;
  float eps;
};

template <int XT, int YT, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    quant_tile128_tma_kernel(const __grid_constant__ CUtensorMap tmap, const TileArgs a) {
  static_assert(XT == PCB_DTYPE_BF16 || XT == PCB_DTYPE_F16, "16-bit inputs only");
  using C = Chunk<XT>;
  constexpr int CPT = kTileBytes / 16 / kThreads;  // chunks per thread (8)
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
  const int64_t mine = first < a.num_groups ? (a.num_groups - 1 - first) / step + 1 : 0;
  const int64_t per_batch = a.groups_m * a.groups_n;
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
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    if ((t & 31) == 0) red[it & 1][warp] = amax;
    __syncthreads();  // every thread holds its chunks: the buffer can be refilled
    uint32_t r = 0;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) r = max(r, red[it & 1][w]);
    if (t == 0 && it + kTileStages < mine) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(s, first + (it + kTileStages) * step);
    }

    const int64_t g = first + it * step;
    const int64_t b = g / per_batch;
    const int64_t rem = g - b * per_batch;
    const int64_t gi = rem / a.groups_n;
    const int64_t gj = rem - gi * a.groups_n;
    const float safe = clamp_min_eps(__uint_as_float(r), a.eps);
    const float qs = quant_scale_from_amax(safe, fp8_max);
    if (t == 0) {
      const float deq = (MODE == kDeqReciprocal) ? __frcp_rn(qs) : __fdiv_rn(safe, fp8_max);
      a.scale[b * a.ssb + gi * a.ssm + gj * a.ssn] = deq;
    }
    uint8_t* yt = static_cast<uint8_t*>(a.y) + b * a.syb + gi * kTileRows * a.sym + gj * 128;
#pragma unroll
    for (int i = 0; i < CPT; ++i) {
      const int c = i * kThreads + t;
      const int r_in = c >> 4;         // 16 chunks of 8 elements per 128-column row
      const int col = (c & 15) * 8;
      if (gi * kTileRows + r_in < a.m && gj * 128 + col < a.n) reg[i].template store<YT>(yt + r_in * a.sym + col, qs);
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
