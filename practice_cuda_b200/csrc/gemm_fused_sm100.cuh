// Fused quantize -> scaled FP8 GEMM for sm_100a (BASELINE cfg4 path).
//
// The activation X (bf16/fp16, K contiguous) is quantized on the fly in 1x128
// groups and multiplied by a pre-quantized fp8 B with per-block (or
// per-channel) fp32 scales; 128x128 output tiles, persistent over tiles.
//
// CTA = 16 warps (one CTA per SM):
//   warp 0      TMA producer: a 128x128 bf16 X tile into a staging buffer and
//               the matching fp8 B tile, per 128-deep K stage
//   warp 1      TMEM allocator + MMA issuer
//   warps 2-3   idle
//   warps 4-7   quantizers: per stage, amax / scale / saturating cast of the
//               128 rows of the staged X tile into the 128-byte-swizzled
//               K-major fp8 A operand, plus the row scales into a scale ring;
//               optionally also to global memory (for reuse in a backward pass)
//   warps 8-15  epilogue: as in bmm_scaled_kernel (promotion per K group,
//               bias, activation, cast, store), row scales from the ring
// The quantization arithmetic is that of pcb_quant_per_block (1x128), so the
// fp8 A bytes and scales match the unfused path bit for bit.
#pragma once

#include "gemm_sm100.cuh"
#include "quant_kernels.cuh"

namespace pcb {
namespace gemm {

constexpr int kFusedThreads = 512;
constexpr int kFusedQuantWarp0 = 4;
constexpr int kFusedEpiWarp0 = 8;
constexpr int kScaleRing = 8;
constexpr int kFusedPrefetch = 2;  // K groups of column scales in flight per epilogue thread  // >= STAGES + kNumAcc + 1 groups in flight

struct FusedSmem {
  static constexpr int BN = 128;
  static constexpr int STAGES = 3;
  static constexpr int X_BYTES = BM * BK * 2;  // bf16 staging, 256-byte rows
  static constexpr int A_BYTES = BM * BK;      // fp8, swizzled
  static constexpr int B_BYTES = BN * BK;
  static constexpr int EPI_COLS = BN / 2;
  static constexpr int OFF_X = 0;
  static constexpr int OFF_A = OFF_X + STAGES * X_BYTES;
  static constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
  static constexpr int OFF_RING = OFF_B + STAGES * B_BYTES;  // kScaleRing x 128 floats
  static constexpr int OFF_COLSCALE = OFF_RING + kScaleRing * BM * 4;
  static constexpr int OFF_BAR = OFF_COLSCALE + 8 * EPI_COLS * 4;
  static constexpr int NUM_BARS = 3 * STAGES + 2 * kNumAcc + kScaleRing;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int BYTES = OFF_MISC + 16;
  static constexpr int ALLOC = BYTES + 1024;
};



template <bool B_MN, int XT, bool COL_UNIFORM>
__global__ void __launch_bounds__(kFusedThreads, 1)
    quant_bmm_fused_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_b,
                           const Params p) {
  using S = FusedSmem;
  constexpr int BN = S::BN;
  constexpr int STAGES = S::STAGES;
  constexpr int EPI_COLS = S::EPI_COLS;
  constexpr int NACC = kNumAcc;
  constexpr uint32_t TMEM_COLS = NACC * BN;
  constexpr uint32_t IDESC = make_idesc(BN, 0, 0, 0, B_MN ? 1 : 0);
  constexpr uint32_t STAGE_TX = S::X_BYTES + S::B_BYTES;
  using C = quant::Chunk<XT>;
  static_assert(C::VEC == 8, "16-bit activations");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t s_base = smem_u32(smem);
  const uint32_t bar_raw = s_base + S::OFF_BAR;         // [STAGES] X + B bytes landed
  const uint32_t bar_q = bar_raw + 8 * STAGES;          // [STAGES] A quantized (4 warps)
  const uint32_t bar_empty = bar_q + 8 * STAGES;        // [STAGES] stage consumed by the MMA
  const uint32_t bar_tfull = bar_empty + 8 * STAGES;    // [NACC]
  const uint32_t bar_tempty = bar_tfull + 8 * NACC;     // [NACC]
  const uint32_t bar_ring = bar_tempty + 8 * NACC;      // [kScaleRing] row scales written
  float* ring = reinterpret_cast<float*>(smem + S::OFF_RING);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + S::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_raw + 8 * s, 1);
      mbar_init(bar_q + 8 * s, 4);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int i = 0; i < NACC; ++i) {
      mbar_init(bar_tfull + 8 * i, 1);
      mbar_init(bar_tempty + 8 * i, 8);
    }
    for (int i = 0; i < kScaleRing; ++i) mbar_init(bar_ring + 8 * i, 4);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_b);
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int tiles_per_batch = p.m_blocks * p.n_blocks;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        const int b = tile / tiles_per_batch;
        const int rem = tile - b * tiles_per_batch;
        const int mb = rem / p.n_blocks;
        const int nb = rem - mb * p.n_blocks;
        for (int ks = 0; ks < p.k_stages; ++ks) {
          if (!mbar_wait_bounded(bar_empty + 8 * stage, phase ^ 1, abort_flag, SITE_FUSED_PRODUCER)) {
            ok = false;
            break;
          }
          const uint32_t fb = bar_raw + 8 * stage;
          mbar_arrive_expect_tx(fb, STAGE_TX);
          tma_load_3d(s_base + S::OFF_X + stage * S::X_BYTES, &tmap_x, fb, ks * BK, mb * BM, b);
          const uint32_t sb_dst = s_base + S::OFF_B + stage * S::B_BYTES;
          if constexpr (B_MN) {
            tma_load_3d(sb_dst, &tmap_b, fb, nb * BN, ks * BK, b);
          } else {
            tma_load_3d(sb_dst, &tmap_b, fb, ks * BK, nb * BN, b);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        for (int s = 0; s < STAGES; ++s) mbar_wait_bounded(bar_raw + 8 * s, 0, abort_flag, SITE_FUSED_PRODUCER);
      }
    }
  } else if (warp == 1) {
    // ------------------------------- MMA issuer -------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t acc_cnt = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        for (int g = 0; g < p.num_groups && ok; ++g) {  // one K group per stage (1x128 activation groups)
          const uint32_t abuf = acc_cnt % NACC;
          const uint32_t aphase = (acc_cnt / NACC) & 1;
          if (!mbar_wait_bounded(bar_tempty + 8 * abuf, aphase ^ 1, abort_flag, SITE_FUSED_MMA) ||
              !mbar_wait_bounded(bar_q + 8 * stage, phase, abort_flag, SITE_FUSED_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + abuf * BN;
          const uint64_t adesc0 = make_sw128_desc(s_base + S::OFF_A + stage * S::A_BYTES, 16u);
          const uint64_t bdesc0 =
              make_sw128_desc(s_base + S::OFF_B + stage * S::B_BYTES, B_MN ? (uint32_t)(128 * BK) : 16u);
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk) {
            const uint64_t a_off = (uint64_t)(kk * UMMA_K >> 4);
            const uint64_t b_off = B_MN ? (uint64_t)(kk * UMMA_K * 128 >> 4) : (uint64_t)(kk * UMMA_K >> 4);
            if (!(kProfiling && (p.debug_flags & 2))) umma_f8(d_tmem, adesc0 + a_off, bdesc0 + b_off, IDESC, kk > 0 ? 1u : 0u);
          }
          umma_commit(bar_empty + 8 * stage);
          umma_commit(bar_tfull + 8 * abuf);
          ++acc_cnt;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp >= kFusedQuantWarp0 && warp < kFusedEpiWarp0) {
    // -------------------------------- quantizers --------------------------------
    const int qw = warp - kFusedQuantWarp0;  // rows [32*qw, 32*qw + 32)
    const int half = lane >> 4;             // which of the two rows of a step
    const int c16 = lane & 15;              // 16-byte chunk (8 elements) of the row
    int stage = 0;
    uint32_t phase = 0;
    uint32_t gq = 0;  // K groups quantized so far (same order as the MMA / epilogue)
    bool ok = true;
    const float fp8_max = 448.0f;
    for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
      const int b = tile / tiles_per_batch;
      const int rem = tile - b * tiles_per_batch;
      const int mb = rem / p.n_blocks;
      const int nb = rem - mb * p.n_blocks;
      const bool write_out = nb == 0;  // one tile column writes the quantized X
      for (int ks = 0; ks < p.k_stages; ++ks) {
        if (!mbar_wait_bounded(bar_raw + 8 * stage, phase, abort_flag, SITE_FUSED_PRODUCER)) {
          ok = false;
          break;
        }
        const uint8_t* xs = smem + S::OFF_X + stage * S::X_BYTES;
        uint8_t* aq = smem + S::OFF_A + stage * S::A_BYTES;
        float* slot = ring + (gq % kScaleRing) * BM;
        const int kcol = ks * BK + c16 * 8;
        if (!(kProfiling && (p.debug_flags & 8))) {
        // All 16 row-pair loads first (explicit shared-memory loads), then the
        // reductions and casts, so the loads overlap instead of serialising.
        const uint32_t xs_s = smem_u32(xs) + (uint32_t)(qw * 32 + half) * 256u + (uint32_t)c16 * 16u;
        const uint32_t aq_s = smem_u32(aq);
        C ch[16];
#pragma unroll
        for (int it = 0; it < 16; ++it) {
          asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(ch[it].raw.x), "=r"(ch[it].raw.y), "=r"(ch[it].raw.z), "=r"(ch[it].raw.w)
                       : "r"(xs_s + (uint32_t)it * 512u));
        }
        uint32_t am[16];
#pragma unroll
        for (int it = 0; it < 16; ++it) am[it] = ch[it].amax_bits();
#pragma unroll
        for (int off = 8; off > 0; off >>= 1)
#pragma unroll
          for (int it = 0; it < 16; ++it) am[it] = max(am[it], __shfl_xor_sync(0xffffffffu, am[it], off));
#pragma unroll
        for (int it = 0; it < 16; ++it) {
          const int r = qw * 32 + 2 * it + half;
          const float safe = clamp_min_eps(__uint_as_float(am[it]), p.eps);
          const float qs = quant_scale_from_amax(safe, fp8_max);
          uint2 q;
          q.x = (uint32_t)cvt2_fp8<PCB_DTYPE_E4M3>(__fmul_rn(ch[it].v(0), qs), __fmul_rn(ch[it].v(1), qs)) |
                ((uint32_t)cvt2_fp8<PCB_DTYPE_E4M3>(__fmul_rn(ch[it].v(2), qs), __fmul_rn(ch[it].v(3), qs)) << 16);
          q.y = (uint32_t)cvt2_fp8<PCB_DTYPE_E4M3>(__fmul_rn(ch[it].v(4), qs), __fmul_rn(ch[it].v(5), qs)) |
                ((uint32_t)cvt2_fp8<PCB_DTYPE_E4M3>(__fmul_rn(ch[it].v(6), qs), __fmul_rn(ch[it].v(7), qs)) << 16);
          // 128-byte-swizzled K-major row r: 16-byte chunk (c16/2) XOR (r % 8).
          const uint32_t dst = aq_s + (uint32_t)r * 128u + ((uint32_t)((c16 >> 1) ^ (r & 7)) << 4) + ((c16 & 1) << 3);
          asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(dst), "r"(q.x), "r"(q.y) : "memory");
          const float deq = __frcp_rn(qs);
          if (c16 == 0) slot[r] = deq;
          const int row = mb * BM + r;
          if (write_out && row < p.m) {
            if (p.xq && kcol < p.k)
              *reinterpret_cast<uint2*>(static_cast<uint8_t*>(p.xq) + (long long)b * p.sxqb +
                                        (long long)row * p.sxqm + kcol) = q;
            if (p.xs && c16 == 0) p.xs[(long long)b * p.sxsb + (long long)row * p.sxsm + (long long)ks * p.sxsk] = deq;
          }
        }
        }
        fence_proxy_async_smem();  // generic-proxy smem writes -> visible to the tensor core
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(bar_q + 8 * stage);
          mbar_arrive(bar_ring + 8 * (gq % kScaleRing));
        }
        ++gq;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp >= kFusedEpiWarp0) {
    // -------------------------------- epilogue --------------------------------
    const int ew = warp - kFusedEpiWarp0;  // 0..7
    const int quarter = warp & 3;
    const int half = ew >> 2;
    const int row_in_tile = quarter * 32 + lane;
    float* colscale = reinterpret_cast<float*>(smem + S::OFF_COLSCALE) + ew * EPI_COLS;
    uint32_t acc_cnt = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
      const int b = tile / tiles_per_batch;
      const int rem = tile - b * tiles_per_batch;
      const int mb = rem / p.n_blocks;
      const int nb = rem - mb * p.n_blocks;
      const int row = mb * BM + row_in_tile;
      const int col0 = nb * BN + half * EPI_COLS;
      const float* sb_b = p.sb ? p.sb + (long long)b * p.ssbb : nullptr;
      float2 acc[EPI_COLS / 2];
#pragma unroll
      for (int i = 0; i < EPI_COLS / 2; ++i) acc[i] = make_float2(0.f, 0.f);
      auto col_scale = [&](int g) -> float {
        return (COL_UNIFORM && sb_b && col0 < p.n)
                   ? __ldg(sb_b + (long long)g * p.ssbk + (long long)(col0 / p.qbn) * p.ssbn)
                   : 1.f;
      };
      float s_col_next = col_scale(0);
      for (int g = 0; g < p.num_groups && ok; ++g) {
        const uint32_t abuf = acc_cnt % NACC;
        const uint32_t aphase = (acc_cnt / NACC) & 1;
        const float s_col = s_col_next;
        if (g + 1 < p.num_groups) s_col_next = col_scale(g + 1);  // one group ahead
        if constexpr (!COL_UNIFORM) {
          __syncwarp();
          for (int i = lane; i < EPI_COLS; i += 32) {
            const int c = col0 + i;
            colscale[i] =
                (sb_b && c < p.n) ? __ldg(sb_b + (long long)g * p.ssbk + (long long)(c / p.qbn) * p.ssbn) : 1.f;
          }
          __syncwarp();
        }
        const uint32_t slot = acc_cnt % kScaleRing;
        if (!mbar_wait_bounded(bar_ring + 8 * slot, (acc_cnt / kScaleRing) & 1, abort_flag, SITE_FUSED_EPILOGUE) ||
            !mbar_wait_bounded(bar_tfull + 8 * abuf, aphase, abort_flag, SITE_FUSED_EPILOGUE)) {
          ok = false;
          break;
        }
        const float s_row = ring[slot * BM + row_in_tile];
        tc_fence_after();
        if (kProfiling && (p.debug_flags & 1)) {
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_tempty + 8 * abuf);
          ++acc_cnt;
          continue;
        }
        const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + abuf * BN + half * EPI_COLS;
#pragma unroll
        for (int c = 0; c < EPI_COLS / 32; ++c) {
          uint32_t v[32];
          tmem_ld32_nowait(taddr + c * 32, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float2 s2;
            if constexpr (COL_UNIFORM) {
              s2 = make_float2(s_row * s_col, s_row * s_col);
            } else {
              s2 = make_float2(s_row * colscale[c * 32 + 2 * i], s_row * colscale[c * 32 + 2 * i + 1]);
            }
            acc[c * 16 + i] =
                __ffma2_rn(make_float2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1])), s2, acc[c * 16 + i]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_tempty + 8 * abuf);
        ++acc_cnt;
      }
      if (!ok) break;
      store_row<EPI_COLS>(p, reinterpret_cast<float*>(acc), b, row, col0);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
}

}  // namespace gemm
}  // namespace pcb
