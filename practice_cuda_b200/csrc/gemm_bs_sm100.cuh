// Block-scaled FP8 batched GEMM for sm_100a (power-of-two / E8M0 scales).
//
// C[b, m, n] = sum_k A[b, m, k] B[b, k, n] sa[b, m/qbm, k/128] sb[b, k/128, n/qbn]
// where every scale is an exact power of two.  The scales are applied by the
// tensor core itself (tcgen05.mma.kind::mxf8f6f4.block_scale, one 8-bit
// exponent per 32 K elements of each A row / B column), so the accumulator
// stays in TMEM for the whole K loop: no per-K-group promotion in registers.
//
// CTA = 12 warps, persistent over 128x256 output tiles (one CTA per SM):
//   warp 0      producer: per stage one TMA load of A, one (or two) of B and
//               bulk copies of the stage's packed E8M0 scale factors (1.5 KB,
//               prepared by pack_sf_kernel in the 32 x 16-byte layout that
//               tcgen05.cp reads); no multicast
//   warp 1      TMEM allocator + MMA issuer: per stage it copies the scale
//               factors from shared memory into TMEM (tcgen05.cp) and issues
//               four block-scaled MMAs
//   warps 4-11  epilogue (bias / GELU / cast / store), released as soon as the
//               accumulator is in registers so the next tile's MMAs can start.
#pragma once

#include "gemm_sm100.cuh"

namespace pcb {
namespace gemm {

__device__ __forceinline__ void umma_f8_bs(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t tsfa, uint32_t tsfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb)
      : "memory");
}

// Shared -> TMEM copy of one 32-row x 16-byte scale-factor block, replicated
// into all four 32-lane quarters (4 TMEM columns).
__device__ __forceinline__ void tmem_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Descriptor of an unswizzled 32 x 16-byte block: 8-row core matrices of
// 128 contiguous bytes, 128 bytes apart.
__device__ __forceinline__ uint64_t make_sf_desc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)(16u >> 4) << 16;   // leading byte offset (one core matrix along K)
  d |= (uint64_t)(128u >> 4) << 32;  // stride byte offset between 8-row core matrices
  d |= (uint64_t)1 << 46;            // descriptor version for tcgen05
  return d;                          // layout 0: no swizzle
}

// Block-scaled instruction descriptor: fp8 A/B, E8M0 scale factors, M=128,
// N=bn; sf_id picks the byte of each 32-bit scale word (the 32-K block).
__host__ __device__ constexpr uint32_t make_idesc_bs(int bn, int fmt, int a_mn, int b_mn, int sf_id) {
  return ((uint32_t)sf_id << 4) | ((uint32_t)fmt << 7) | ((uint32_t)fmt << 10) | ((uint32_t)a_mn << 15) |
         ((uint32_t)b_mn << 16) | ((uint32_t)(bn >> 3) << 17) | (1u << 23) | ((uint32_t)(BM >> 4) << 24) |
         ((uint32_t)sf_id << 29);
}

struct BsSmem {
  static constexpr int BN = 256;
  static constexpr int STAGES = 4;
  static constexpr int A_BYTES = BM * BK;        // 16 KB
  static constexpr int B_BYTES = BN * BK;        // 32 KB
  static constexpr int SFA_BYTES = 512;          // 128 rows x 4 bytes
  static constexpr int SF_BYTES = 512 + 1024;    // SFA + SFB (256 columns)
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
  static constexpr int OFF_SF = OFF_B + STAGES * B_BYTES;
  static constexpr int OFF_BAR = OFF_SF + STAGES * SF_BYTES;
  static constexpr int NUM_BARS = 2 * STAGES + 2;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int BYTES = OFF_MISC + 16;
  static constexpr int ALLOC = BYTES + 1024;
};
constexpr int kSfCols = 12;        // TMEM columns of scale factors per stage (SFA 4 + SFB 8)
constexpr uint32_t kBsTmemCols = 512;  // accumulator (256) + scale-factor ring

// E8M0 byte of a power-of-two fp32 scale (its biased exponent).
__device__ __forceinline__ uint32_t e8m0_of(float s) { return (__float_as_uint(s) >> 23) & 0xffu; }

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// Packs the power-of-two fp32 scales of one operand into 512-byte blocks,
// one per (batch, 128-row block, 128-deep K stage): line i (16 bytes) holds
// the E8M0 bytes of rows i, i+32, i+64, i+96, each repeated for the four
// 32-K blocks of the stage.  Rows past `rows` get 1.0 (byte 127).
// scale(b, r, s) = scale[b * ssb + (r / qb) * ssr + s * sss].
struct PackSfArgs {
  const float* scale;
  long long ssb, ssr, sss;
  int qb;
  int rows, row_blocks, k_stages, batch;
  uint4* out;  // [batch][row_blocks][k_stages][32] lines
};

__global__ void __launch_bounds__(256) pack_sf_kernel(const PackSfArgs a) {
  const long long total = (long long)a.batch * a.row_blocks * a.k_stages * 32;
  for (long long idx = blockIdx.x * 256ll + threadIdx.x; idx < total; idx += (long long)gridDim.x * 256) {
    const int i = (int)(idx & 31);
    long long rest = idx >> 5;
    const int ks = (int)(rest % a.k_stages);
    rest /= a.k_stages;
    const int rb = (int)(rest % a.row_blocks);
    const int b = (int)(rest / a.row_blocks);
    uint32_t w[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int r = rb * 128 + 32 * q + i;
      const uint32_t e = r < a.rows ? e8m0_of(__ldg(a.scale + b * a.ssb + (long long)(r / a.qb) * a.ssr + ks * a.sss))
                                    : 127u;
      w[q] = e * 0x01010101u;
    }
    a.out[idx] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

template <bool A_MN, bool B_MN, int FMT>
__global__ void __launch_bounds__(kThreads, 1)
    bmm_blockscaled_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                           const Params p) {
  using S = BsSmem;
  constexpr int BN = S::BN;
  constexpr int STAGES = S::STAGES;
  constexpr int EPI_COLS = BN / 2;
  constexpr uint32_t STAGE_TX = S::A_BYTES + S::B_BYTES + S::SF_BYTES;
  static_assert(BN + STAGES * kSfCols <= (int)kBsTmemCols, "TMEM budget");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t s_base = smem_u32(smem);
  const uint32_t bar_full = s_base + S::OFF_BAR;          // [STAGES]: operand + scale-factor bytes
  const uint32_t bar_empty = bar_full + 8 * STAGES;       // [STAGES]
  const uint32_t bar_tfull = bar_empty + 8 * STAGES;
  const uint32_t bar_tempty = bar_tfull + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + S::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    mbar_init(bar_tfull, 1);
    mbar_init(bar_tempty, 8);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), kBsTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (p.inject_error && blockIdx.x == 0 && threadIdx.x == 0) report_error(p.inject_error, SITE_GEMM_INJECTED);

  const int tiles_per_batch = p.m_blocks * p.n_blocks;

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kLowRegs));
    if (warp == 0 && lane == 0) {
      // ------------------------------ TMA producer ------------------------------
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        const int b = tile / tiles_per_batch;
        const int rem = tile - b * tiles_per_batch;
        const int mb = rem / p.n_blocks;
        const int nb = rem - mb * p.n_blocks;
        for (int ks = 0; ks < p.k_stages; ++ks) {
          if (!mbar_wait_bounded(bar_empty + 8 * stage, phase ^ 1, abort_flag, SITE_GEMM_PRODUCER)) {
            ok = false;
            break;
          }
          const uint32_t fb = bar_full + 8 * stage;
          const uint32_t sa_dst = s_base + S::OFF_A + stage * S::A_BYTES;
          const uint32_t sb_dst = s_base + S::OFF_B + stage * S::B_BYTES;
          mbar_arrive_expect_tx(fb, STAGE_TX);
          if constexpr (A_MN) tma_load_3d(sa_dst, &tmap_a, fb, mb * BM, ks * BK, b);
          else tma_load_3d(sa_dst, &tmap_a, fb, ks * BK, mb * BM, b);
          if constexpr (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 128; ++j) tma_load_3d(sb_dst + j * 128 * BK, &tmap_b, fb, nb * BN + j * 128, ks * BK, b);
          } else {
            tma_load_3d(sb_dst, &tmap_b, fb, ks * BK, nb * BN, b);
          }
          const uint32_t sf_dst = s_base + S::OFF_SF + stage * S::SF_BYTES;
          bulk_load(sf_dst, p.sfa + (((long long)b * p.m_blocks + mb) * p.k_stages + ks) * 32, 512, fb);
#pragma unroll
          for (int j = 0; j < 2; ++j)
            bulk_load(sf_dst + 512 + 512 * j,
                      p.sfb + (((long long)b * 2 * p.n_blocks + 2 * nb + j) * p.k_stages + ks) * 32, 512, fb);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        volatile int keep_waiting = 0;
        for (int s = 0; s < STAGES; ++s) mbar_wait_bounded(bar_full + 8 * s, 0, &keep_waiting, SITE_GEMM_PRODUCER);
      }
    } else if (warp == 1 && lane == 0) {
      // ------------------------------- MMA issuer -------------------------------
      int stage = 0;
      uint32_t phase = 0;
      uint32_t tcount = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++tcount) {
        if (!mbar_wait_bounded(bar_tempty, (tcount & 1) ^ 1, abort_flag, SITE_GEMM_MMA)) break;
        tc_fence_after();
        for (int ks = 0; ks < p.k_stages; ++ks) {
          if (!mbar_wait_bounded(bar_full + 8 * stage, phase, abort_flag, SITE_GEMM_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sf_s = s_base + S::OFF_SF + stage * S::SF_BYTES;
          const uint32_t sf_t = tmem_base + BN + stage * kSfCols;
          tmem_cp_sf(sf_t, make_sf_desc(sf_s));
          tmem_cp_sf(sf_t + 4, make_sf_desc(sf_s + 512));
          tmem_cp_sf(sf_t + 8, make_sf_desc(sf_s + 1024));
          const uint32_t sa_addr = s_base + S::OFF_A + stage * S::A_BYTES;
          const uint32_t sb_addr = s_base + S::OFF_B + stage * S::B_BYTES;
          const uint64_t adesc0 = make_sw128_desc(sa_addr, A_MN ? (uint32_t)(128 * BK) : 16u);
          const uint64_t bdesc0 = make_sw128_desc(sb_addr, B_MN ? (uint32_t)(128 * BK) : 16u);
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk) {
            const uint64_t a_off = A_MN ? (uint64_t)(kk * UMMA_K * 128 >> 4) : (uint64_t)(kk * UMMA_K >> 4);
            const uint64_t b_off = B_MN ? (uint64_t)(kk * UMMA_K * 128 >> 4) : (uint64_t)(kk * UMMA_K >> 4);
            umma_f8_bs(tmem_base, adesc0 + a_off, bdesc0 + b_off, make_idesc_bs(BN, FMT, A_MN, B_MN, kk), sf_t,
                       sf_t + 4, (ks > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(bar_empty + 8 * stage);  // smem stage (operands + scale factors) free once these retire
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(bar_tfull);
      }
    }
  } else {
    // -------------------------------- epilogue --------------------------------
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kHighRegs));
    const int ew = warp - kEpiWarp0;
    const int quarter = warp & 3;
    const int half = ew >> 2;
    const int row_in_tile = quarter * 32 + lane;
    uint32_t tcount = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++tcount) {
      const int b = tile / tiles_per_batch;
      const int rem = tile - b * tiles_per_batch;
      const int mb = rem / p.n_blocks;
      const int nb = rem - mb * p.n_blocks;
      if (!mbar_wait_bounded(bar_tfull, tcount & 1, abort_flag, SITE_GEMM_EPILOGUE)) break;
      tc_fence_after();
      uint32_t v[EPI_COLS];
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + half * EPI_COLS;
#pragma unroll
      for (int c = 0; c < EPI_COLS / 32; ++c) {
        uint32_t (&chunk)[32] = *reinterpret_cast<uint32_t(*)[32]>(v + 32 * c);
        tmem_ld32_nowait(taddr + c * 32, chunk);
      }
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_tempty);  // the next tile's MMAs may overwrite the accumulator
      float* accf = reinterpret_cast<float*>(v);
      store_row<EPI_COLS>(p, accf, b, mb * BM + row_in_tile, nb * BN + half * EPI_COLS);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kBsTmemCols);
}

}  // namespace gemm
}  // namespace pcb
