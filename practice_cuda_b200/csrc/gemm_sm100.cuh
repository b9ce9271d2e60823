// Scaled FP8 batched GEMM for sm_100a: TMA -> shared memory ring -> tcgen05.mma
// (kind::f8f6f4, fp32 accumulators in TMEM) -> epilogue warps that promote
// every K quant group with its fp32 scales into register accumulators.
//
// CTA = 12 warps, persistent over output tiles (one CTA per SM):
//   warp 0      TMA producer (one elected lane), no multicast
//   warp 1      TMEM allocator + MMA issuer (warp-uniform loop, elect.sync
//               lane issues)
//   warps 2-3   scale loader: each tile's fp32 scales, W K groups at a time,
//               into a four-slot shared ring read by the epilogue
//   warps 4-11  epilogue: two warpgroups; warpgroup h owns tile columns
//               [h*BN/2, (h+1)*BN/2), warp (w % 4) owns TMEM lanes / rows
//               [32*(w%4), 32*(w%4)+32).
// Tiles are 128 x BN (BN = 128 or 256).  TMEM holds 512 / BN accumulator
// buffers of BN fp32 columns, so the MMA of K-group g+1 runs while the
// epilogue promotes group g.  With PAIR the tile is 256 x BN on a CTA pair
// (cta_group::2): each CTA stages its own 128 A rows and half of the B
// columns, the even CTA issues the MMAs for both and multicasts its commits
// (smem stage free, accumulator full) to both CTAs, and both CTAs' epilogues
// read their own TMEM half and arrive on the leader's accumulator-empty
// barrier (plain remote arrives, no cluster-scope release).
#pragma once

#include <type_traits>

#include "common.cuh"

namespace pcb {
namespace gemm {

constexpr int BM = 128;           // rows per tile (UMMA M)
constexpr int BK = 128;           // K elements per pipeline stage = one 128-byte swizzle atom
constexpr int UMMA_K = 32;        // K per tcgen05.mma for 8-bit inputs
constexpr int kThreads = 384;
constexpr int kEpiWarp0 = 4;
constexpr int kEpiThreads = 256;
// Register split for the 128x256 tile (setmaxnreg): the producer/MMA
// warpgroup drops to kLowRegs so the epilogue warpgroups can hold 128 fp32
// accumulators per thread.  The launch holds kThreads * kLaunchRegs registers
// (checked on the host before every launch) and the split adds up to it.
constexpr int kLaunchRegs = 168;  // 65536 / 384, rounded down to a multiple of 8
#ifdef PCB_GEMM_LOW_REGS
constexpr int kLowRegs = PCB_GEMM_LOW_REGS;
constexpr int kHighRegs = (kThreads * kLaunchRegs - 128 * kLowRegs) / 256;
#else
constexpr int kLowRegs = 56;   // producer, MMA issuer, scale loader
constexpr int kHighRegs = 224;
#endif
static_assert(128 * kLowRegs + 256 * kHighRegs == kThreads * kLaunchRegs, "register split must match the launch");
#ifndef PCB_GEMM_EPI_CW
#define PCB_GEMM_EPI_CW 64  // TMEM columns per epilogue load (16, 32 or 64)
#endif
constexpr int kNumAcc = 4;        // TMEM accumulator buffers of BN fp32 columns
constexpr int kScaleWin = 8;      // K groups of scales per shared-memory window
constexpr int kScaleSlots = 4;    // windows in the shared-memory scale ring
constexpr int kScaleWinCols = 4;  // K groups per window when B scales vary per column
constexpr int kScaleThreads = 64; // scale-loader threads (warps 2-3)

// Profiling switches (Params::debug_flags) exist only in builds compiled with
// -DPCB200_PROFILING; the shipped library compiles every check below to false.
#ifdef PCB200_PROFILING
constexpr bool kProfiling = true;
#else
constexpr bool kProfiling = false;
#endif

// Cycle trace of CTA 0's pipeline hand-offs, compiled only into trace builds
// (-DPCB_GEMM_TRACE) used to find where a K group's time goes.
#ifdef PCB_GEMM_TRACE
__device__ long long g_gemm_trace[16][1024];
#define PCB_TRACE(ev, idx)                                                   \
  do {                                                                       \
    if (blockIdx.x == 0 && (idx) < 1024) g_gemm_trace[ev][idx] = clock64(); \
  } while (0)
__device__ unsigned long long g_cta_span[4][1024];  // per-CTA start / end: globaltimer ns, clock64
#define PCB_CTA_SPAN(i)                                        \
  do {                                                         \
    if (threadIdx.x == 0 && blockIdx.x < 1024) {               \
      g_cta_span[i][blockIdx.x] = global_timer_ns();           \
      g_cta_span[2 + (i)][blockIdx.x] = (unsigned long long)clock64(); \
    }                                                          \
  } while (0)
#else
#define PCB_TRACE(ev, idx) \
  do {                     \
  } while (0)
#define PCB_CTA_SPAN(i) \
  do {                  \
  } while (0)
#endif

struct Params {
  int batch, m, n, k;
  int a_fmt, b_fmt;  // operand formats for the instruction descriptor: 0 = E4M3, 1 = E5M2
  int m_blocks, n_blocks, num_tiles;
  int k_stages;          // ceil(k / BK)
  int stages_per_group;  // qbk / BK (or k_stages for a single group)
  int num_groups;        // ceil(k_stages / stages_per_group)
  // scale_a[b*ssab + (m/qbm)*ssam + g*ssak]; scale_b[b*ssbb + g*ssbk + (n/qbn)*ssbn]
  const float* sa;
  long long ssab, ssam, ssak;
  int qbm;
  const float* sb;
  long long ssbb, ssbk, ssbn;
  int qbn;
  int col_uniform;  // sb constant over each warpgroup's column half
  // Per-column B scales only: 16-byte scale loads.  sa_vec 2 = rows
  // contiguous per K group (qbm == 1); sb_vec = B scales contiguous along N
  // (qbn == 1).  0 = scalar loads.
  int sa_vec, sb_vec;
  // output / bias
  void* c;
  long long scb, scm;
  int c_dtype;
  int c_vec;  // 16-byte vector stores allowed
  int c_tma;  // bf16 / fp16 C written by TMA stores from shared memory (bmm_scaled_kernel on a CTA pair)
  const void* bias;
  long long sbib, sbim, sbin;
  int bias_dtype;
  int activation;
  int inject_error;
  // Fused quantize->GEMM only: optional copies of the quantized activation
  // (fp8 [B, M, K], K contiguous) and its 1x128 scales [B, M, ceil(K/128)].
  void* xq;
  long long sxqb, sxqm;
  float* xs;
  long long sxsb, sxsm, sxsk;
  float eps;
  // Block-scaled GEMM only: packed E8M0 scale factors (pack_sf_kernel layout).
  const uint4* sfa;
  const uint4* sfb;
  int debug_flags;  // PCB200_PROFILING builds only: 1 = epilogue skips its math, 2 = no MMAs issued,
                   // 8 = fused quantizer skipped
};

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// L2 prefetch of one tensor-map box (no shared memory written, nothing to wait on).
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap* map, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void umma_f8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every previously issued tcgen05.mma of this thread completes.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}


// ---- CTA-pair (cta_group::2) helpers -------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// TMA load into this CTA's shared memory that completes its bytes on the
// pair leader's mbarrier (`bar_cluster` is a shared::cluster address).
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar_cluster, int c0,
                                                 int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Arrive on an mbarrier of another CTA of the cluster.  The TMEM reads this
// publishes are ordered by tcgen05.fence::before_thread_sync, so no
// cluster-scope release (a full memory fence) is needed.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}


// Warp-uniform forms: every lane of the warp executes them and the lane
// chosen by elect.sync issues the instruction, so the issuing loop runs as
// convergent warp code instead of a one-lane divergent branch.  Descriptors
// are passed as their low and high 32-bit words (only the low word, start
// address and LBO, changes from stage to stage).  PAIR selects cta_group::2
// (M = 256 over the CTA pair, commits multicast to both CTAs).
template <bool PAIR>
__device__ __forceinline__ void umma_f8_elect(uint32_t d_tmem, uint32_t a_lo, uint32_t a_hi, uint32_t b_lo,
                                              uint32_t b_hi, uint32_t idesc, uint32_t accumulate) {
  if constexpr (PAIR) {
    asm volatile(
        "{\n\t.reg .pred e, p;\n\t.reg .b64 ad, bd;\n\t"
        "mov.b64 ad, {%1, %2};\n\t"
        "mov.b64 bd, {%3, %4};\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %6, 0;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], ad, bd, %5, p;\n\t}" ::"r"(d_tmem),
        "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred e, p;\n\t.reg .b64 ad, bd;\n\t"
        "mov.b64 ad, {%1, %2};\n\t"
        "mov.b64 bd, {%3, %4};\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %6, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], ad, bd, %5, p;\n\t}" ::"r"(d_tmem),
        "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

template <bool PAIR>
__device__ __forceinline__ void umma_commit_elect(uint32_t bar) {
  if constexpr (PAIR) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n\t}" ::"r"(bar),
        "h"((uint16_t)0x3)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(bar)
        : "memory");
  }
}


// 32 consecutive fp32 columns of this thread's TMEM lane (no wait).
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 64 consecutive fp32 columns of this thread's TMEM lane (no wait).
__device__ __forceinline__ void tmem_ld64_nowait(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
      "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr));
}

// 16 consecutive fp32 columns of this thread's TMEM lane (no wait).
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// N (16, 32 or 64) consecutive fp32 columns of this thread's TMEM lane (no wait).
template <int N>
__device__ __forceinline__ void tmem_ld_n(uint32_t taddr, uint32_t (&r)[N]) {
  if constexpr (N == 64) tmem_ld64_nowait(taddr, r);
  else if constexpr (N == 32) tmem_ld32_nowait(taddr, r);
  else tmem_ld16_nowait(taddr, r);
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Ties registers filled by an earlier tcgen05.ld to a point after the
// tcgen05.wait::ld, so the compiler cannot move their uses above the wait.
template <int N>
__device__ __forceinline__ void tmem_regs_ready(uint32_t (&r)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

// UMMA shared-memory descriptor for a 128-byte-swizzled tile.
//   K-major : rows of 128 bytes (BK fp8), 8-row atoms 1024 B apart (SBO).
//   MN-major: 128-element MN slabs, K rows 128 B apart; 8-K-row atoms 1024 B
//             apart (SBO); consecutive 128-wide MN slabs `lbo` bytes apart.
__device__ __forceinline__ uint64_t make_sw128_desc(uint32_t saddr, uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for tcgen05
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor of kind::f8f6f4: fp32 accumulate, A and B formats
// (0 = E4M3, 1 = E5M2; they may differ), majorness, N = bn, M = m.
__host__ __device__ constexpr uint32_t make_idesc(int bn, int a_fmt, int b_fmt, int a_mn, int b_mn, int m = BM) {
  return (1u << 4) | ((uint32_t)a_fmt << 7) | ((uint32_t)b_fmt << 10) | ((uint32_t)a_mn << 15) |
         ((uint32_t)b_mn << 16) | ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

template <int BN, bool PAIR = false, bool COLU = true>
struct Smem {
  // A CTA pair splits the B tile: each CTA stages BN/2 of its N rows.
  static constexpr int B_ROWS = PAIR ? BN / 2 : BN;
  // The CTA pair gives one operand stage (32 KB) to output staging.
  static constexpr int STAGES = (BN == 256 && !PAIR) ? 4 : (PAIR ? 5 : 6);
  static constexpr int A_BYTES = BM * BK;      // 16 KB
  static constexpr int B_BYTES = B_ROWS * BK;  // 32 / 16 KB
  static constexpr int EPI_COLS = BN / 2;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
  static constexpr int OFF_COLSCALE = OFF_B + STAGES * B_BYTES;           // (unused)
  // Scale ring slot of SW K groups: row scales [SW][BM], then the B scales:
  // uniform ones [SW][2] (one per 128-column block) or per column [SW][BN].
  static constexpr int SW = COLU ? kScaleWin : kScaleWinCols;
  static constexpr int SC_SLOT = SW * (BM + (COLU ? 2 : BN));
  static constexpr int OFF_SCALE = OFF_COLSCALE + (COLU ? 8 * EPI_COLS * 4 : 0);
  static constexpr int OFF_BAR = OFF_SCALE + kScaleSlots * SC_SLOT * 4;
  static constexpr int NUM_BARS = 2 * STAGES + 2 * kNumAcc + 2 * kScaleSlots;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;                  // tmem addr, abort flag
  // Output staging for TMA stores (CTA pair only): one 4 KB buffer per
  // epilogue warp, a 32-row x 64-column bf16 / fp16 box in the 128-byte swizzle.
  static constexpr int CSTG_BUF = PAIR ? 4096 : 0;
  static constexpr int OFF_CSTG = (OFF_MISC + 16 + 1023) / 1024 * 1024;
  static constexpr int BYTES = OFF_CSTG + 8 * CSTG_BUF;
  static constexpr int ALLOC = BYTES + 1024;                              // slack for 1 KB alignment
  static_assert(ALLOC <= 232448, "shared memory per CTA");
};

// TMA store of one box from shared memory, tracked in this thread's bulk groups.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until at most N of this thread's bulk store groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Generic-proxy shared-memory writes become visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.7071067811865475f)); }

__device__ __forceinline__ float load_bias(const void* p, int dt, long long off) {
  if (dt == PCB_DTYPE_F32) return __ldg(static_cast<const float*>(p) + off);
  if (dt == PCB_DTYPE_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[off]);
  return __half2float(static_cast<const __half*>(p)[off]);
}

// Bias, activation, cast and store of one thread's EPI_COLS accumulators
// (row `row`, columns [col0, col0 + EPI_COLS)) of batch `b`.
template <int EPI_COLS>
__device__ __forceinline__ void store_row(const Params& p, float* accf, int b, int row, int col0) {
  if (row < p.m) {
    const long long crow = (long long)b * p.scb + (long long)row * p.scm;
    if (p.bias) {
#pragma unroll
      for (int i = 0; i < EPI_COLS; ++i) {
        const int c = col0 + i;
        if (c < p.n)
          accf[i] += load_bias(p.bias, p.bias_dtype, (long long)b * p.sbib + (long long)row * p.sbim + (long long)c * p.sbin);
      }
    }
    if (p.activation == PCB_ACT_GELU) {
#pragma unroll
      for (int i = 0; i < EPI_COLS; ++i) accf[i] = gelu_erf(accf[i]);
    }
    const bool full = p.c_vec && (col0 + EPI_COLS <= p.n);
    if (p.c_dtype == PCB_DTYPE_BF16 || p.c_dtype == PCB_DTYPE_F16) {
      uint16_t* out = static_cast<uint16_t*>(p.c) + crow + col0;
      if (full) {
#pragma unroll
        for (int i = 0; i < EPI_COLS; i += 8) {
          uint4 w;
          uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if (p.c_dtype == PCB_DTYPE_BF16) {
              __nv_bfloat162 h = __floats2bfloat162_rn(accf[i + 2 * q], accf[i + 2 * q + 1]);
              wp[q] = *reinterpret_cast<uint32_t*>(&h);
            } else {
              __half2 h = __floats2half2_rn(accf[i + 2 * q], accf[i + 2 * q + 1]);
              wp[q] = *reinterpret_cast<uint32_t*>(&h);
            }
          }
          *reinterpret_cast<uint4*>(out + i) = w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < EPI_COLS; ++i) {
          if (col0 + i < p.n) {
            if (p.c_dtype == PCB_DTYPE_BF16) {
              __nv_bfloat16 h = __float2bfloat16_rn(accf[i]);
              out[i] = *reinterpret_cast<uint16_t*>(&h);
            } else {
              __half h = __float2half_rn(accf[i]);
              out[i] = *reinterpret_cast<uint16_t*>(&h);
            }
          }
        }
      }
    } else if (p.c_dtype == PCB_DTYPE_F32) {
      float* out = static_cast<float*>(p.c) + crow + col0;
      if (full) {
#pragma unroll
        for (int i = 0; i < EPI_COLS; i += 4)
          *reinterpret_cast<float4*>(out + i) = make_float4(accf[i], accf[i + 1], accf[i + 2], accf[i + 3]);
      } else {
#pragma unroll
        for (int i = 0; i < EPI_COLS; ++i)
          if (col0 + i < p.n) out[i] = accf[i];
      }
    } else {
      uint8_t* out = static_cast<uint8_t*>(p.c) + crow + col0;
#pragma unroll
      for (int i = 0; i < EPI_COLS; ++i) {
        if (col0 + i < p.n)
          out[i] = (p.c_dtype == PCB_DTYPE_E4M3) ? cvt1_fp8<PCB_DTYPE_E4M3>(accf[i]) : cvt1_fp8<PCB_DTYPE_E5M2>(accf[i]);
      }
    }
  }
}

// Bias, activation and a TMA store of one warp's 32 rows x EPI_COLS columns
// of bf16 / fp16 C, 64 columns at a time (fp32 C: 32 at a time): every lane writes its row's 128
// bytes into the warp's 4 KB staging buffer (128-byte swizzle: conflict-free)
// and lane 0 stores the 32 x 64 box.  Whole 128-byte row segments keep the
// store engine's request count low (per-thread 16-byte row stores cost ~9000
// cycles per 256 x 256 tile, during which the MMA stalls).  The buffer is
// rewritten only after the previous box store has read it.  Rows and columns
// outside C are clipped by the tensor map.
template <int EPI_COLS>
__device__ __forceinline__ void store_rows_tma(const Params& p, const CUtensorMap* tmap_c, float* accf, int b,
                                               int row, int warp_row0, int col0, uint32_t stg, int lane) {
  if (row < p.m) {
    if (p.bias) {
#pragma unroll
      for (int i = 0; i < EPI_COLS; ++i) {
        const int c = col0 + i;
        if (c < p.n)
          accf[i] += load_bias(p.bias, p.bias_dtype, (long long)b * p.sbib + (long long)row * p.sbim + (long long)c * p.sbin);
      }
    }
    if (p.activation == PCB_ACT_GELU) {
#pragma unroll
      for (int i = 0; i < EPI_COLS; ++i) accf[i] = gelu_erf(accf[i]);
    }
  }
  const bool bf16 = p.c_dtype == PCB_DTYPE_BF16;
  const uint32_t swz = (uint32_t)(lane & 7);
  if (p.c_dtype == PCB_DTYPE_F32) {
    // fp32: 32-column boxes (128-byte rows), EPI_COLS / 32 per warp.
#pragma unroll
    for (int q = 0; q < EPI_COLS / 32; ++q) {
      if (lane == 0) bulk_wait_read<0>();
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float* f = accf + 32 * q + 4 * c;
        const uint32_t dst = stg + (uint32_t)lane * 128u + (((uint32_t)c ^ swz) << 4);
        asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "f"(f[0]), "f"(f[1]), "f"(f[2]), "f"(f[3])
                     : "memory");
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && warp_row0 < p.m && col0 + 32 * q < p.n) tma_store_3d(tmap_c, stg, col0 + 32 * q, warp_row0, b);
    }
    return;
  }
#pragma unroll
  for (int q = 0; q < EPI_COLS / 64; ++q) {
    if (lane == 0) bulk_wait_read<0>();
    __syncwarp();
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float lo = accf[64 * q + 8 * c + 2 * j], hi = accf[64 * q + 8 * c + 2 * j + 1];
        if (bf16) {
          __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
          w[j] = *reinterpret_cast<uint32_t*>(&h);
        } else {
          __half2 h = __floats2half2_rn(lo, hi);
          w[j] = *reinterpret_cast<uint32_t*>(&h);
        }
      }
      const uint32_t dst = stg + (uint32_t)lane * 128u + (((uint32_t)c ^ swz) << 4);
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3])
                   : "memory");
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0 && warp_row0 < p.m && col0 + 64 * q < p.n) tma_store_3d(tmap_c, stg, col0 + 64 * q, warp_row0, b);
  }
}

template <int BN, bool A_MN, bool B_MN, bool COL_UNIFORM, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    bmm_scaled_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                      const __grid_constant__ CUtensorMap tmap_c, const Params p) {
  static_assert(!PAIR || BN == 256, "the CTA pair runs 256x256 tiles");
  using S = Smem<BN, PAIR, COL_UNIFORM>;
  constexpr int STAGES = S::STAGES;
  constexpr int EPI_COLS = S::EPI_COLS;
  constexpr int NACC = (BN == 256) ? 2 : kNumAcc;  // TMEM accumulator buffers of BN columns
  constexpr uint32_t TMEM_COLS = NACC * BN;
  static_assert(NACC * BN <= 512, "TMEM holds 512 fp32 columns");
  constexpr int W = S::SW;
  const uint32_t IDESC = make_idesc(BN, p.a_fmt, p.b_fmt, A_MN ? 1 : 0, B_MN ? 1 : 0, PAIR ? 2 * BM : BM);
  // Bytes that land on the (leader's) full barrier per stage.
  constexpr uint32_t STAGE_TX = (PAIR ? 2 : 1) * (S::A_BYTES + S::B_BYTES);
  constexpr int TILE_M = PAIR ? 2 * BM : BM;  // output rows per tile

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t s_base = smem_u32(smem);
  const uint32_t bar_full = s_base + S::OFF_BAR;                  // [STAGES]
  const uint32_t bar_empty = bar_full + 8 * STAGES;               // [STAGES]
  const uint32_t bar_tfull = bar_empty + 8 * STAGES;              // [NACC]
  const uint32_t bar_tempty = bar_tfull + 8 * kNumAcc;            // [NACC]
  const uint32_t bar_sfull = bar_tempty + 8 * kNumAcc;            // [kScaleSlots] scale window loaded
  const uint32_t bar_sempty = bar_sfull + 8 * kScaleSlots;        // [kScaleSlots] scale window consumed
  float* sring = reinterpret_cast<float*>(smem + S::OFF_SCALE);   // [kScaleSlots][S::SC_SLOT]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + S::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Pair mode: cluster of two CTAs; rank 0 (leader) issues the MMAs and owns
  // the full / tmem-empty barriers that both CTAs feed.
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int first_tile = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int tile_step = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  // Waits whose arrival may come from the peer CTA poll without suspending.
  auto wait = [&](uint32_t bar, uint32_t parity, int site) -> bool {
    return PAIR ? mbar_spin_bounded(bar, parity, abort_flag, site) : mbar_wait_bounded(bar, parity, abort_flag, site);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int i = 0; i < NACC; ++i) {
      mbar_init(bar_tfull + 8 * i, 1);
      mbar_init(bar_tempty + 8 * i, PAIR ? 16 : 8);  // one arrive per epilogue warp (of both CTAs)
    }
    for (int i = 0; i < kScaleSlots; ++i) {
      mbar_init(bar_sfull + 8 * i, kScaleThreads);  // every scale-loader thread
      mbar_init(bar_sempty + 8 * i, 8);             // every epilogue warp of this CTA
    }
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
  }
  if constexpr (PAIR) {
    if (warp == 1) tmem_alloc_pair(smem_u32(tmem_slot), TMEM_COLS);
    tc_fence_before();
    cluster_sync_all();  // both CTAs' barriers exist before any remote arrive / TMA
  } else {
    if (warp == 1) tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
    tc_fence_before();
    __syncthreads();
  }
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Launched with programmatic stream serialization: barrier set-up, TMEM
  // allocation and tensor-map prefetch overlap the previous kernel's tail;
  // nothing global is read or written before that kernel has completed.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  PCB_CTA_SPAN(0);

  if (p.inject_error && blockIdx.x == 0 && threadIdx.x == 0) report_error(p.inject_error, SITE_GEMM_INJECTED);

  const int tiles_per_batch = p.m_blocks * p.n_blocks;

  if (warp < 4) {
    if constexpr (BN == 256) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kLowRegs));
  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int pcnt = 0;  // stages issued (trace index)
      (void)pcnt;
      for (int tile = first_tile; tile < p.num_tiles && ok; tile += tile_step) {
        const int b = tile / tiles_per_batch;
        const int rem = tile - b * tiles_per_batch;
        const int mb = rem / p.n_blocks;
        const int nb = rem - mb * p.n_blocks;
        const int a_row = mb * TILE_M + (int)rank * BM;           // this CTA's A rows
        const int b_col = nb * BN + (int)rank * S::B_ROWS;        // this CTA's B columns
        for (int ks = 0; ks < p.k_stages; ++ks) {
          PCB_TRACE(8, pcnt);
          if (!wait(bar_empty + 8 * stage, phase ^ 1, SITE_GEMM_PRODUCER)) {
            ok = false;
            break;
          }
          PCB_TRACE(9, pcnt);
          ++pcnt;
          const uint32_t fb = bar_full + 8 * stage;
          const uint32_t sa_dst = s_base + S::OFF_A + stage * S::A_BYTES;
          const uint32_t sb_dst = s_base + S::OFF_B + stage * S::B_BYTES;
          if constexpr (PAIR) {
            if (leader) mbar_arrive_expect_tx(fb, STAGE_TX);
            const uint32_t fbl = mapa_shared(fb, 0);
            if constexpr (A_MN) tma_load_3d_pair(sa_dst, &tmap_a, fbl, a_row, ks * BK, b);
            else tma_load_3d_pair(sa_dst, &tmap_a, fbl, ks * BK, a_row, b);
            if constexpr (B_MN) tma_load_3d_pair(sb_dst, &tmap_b, fbl, b_col, ks * BK, b);
            else tma_load_3d_pair(sb_dst, &tmap_b, fbl, ks * BK, b_col, b);
          } else {
            mbar_arrive_expect_tx(fb, STAGE_TX);
            if constexpr (A_MN) {
              tma_load_3d(sa_dst, &tmap_a, fb, a_row, ks * BK, b);
            } else {
              tma_load_3d(sa_dst, &tmap_a, fb, ks * BK, a_row, b);
            }
            if constexpr (B_MN) {
#pragma unroll
              for (int j = 0; j < BN / 128; ++j)
                tma_load_3d(sb_dst + j * 128 * BK, &tmap_b, fb, b_col + j * 128, ks * BK, b);
            } else {
              tma_load_3d(sb_dst, &tmap_b, fb, ks * BK, b_col, b);
            }
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Let the copies already issued land before the CTA can exit.
        for (int s = 0; s < STAGES; ++s) mbar_wait_bounded(bar_full + 8 * s, 0, abort_flag, SITE_GEMM_PRODUCER);
      }
    }
  } else if (warp == 1) {
    // ------------------------------- MMA issuer -------------------------------
    // Warp-uniform issuer: all lanes run the loop and poll the barriers with
    // collective bounded waits; the elect.sync lane issues the MMAs and
    // commits (a one-lane divergent loop costs hundreds of cycles per group).
    if (leader) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      const uint64_t ad64 = make_sw128_desc(s_base + S::OFF_A, A_MN ? (uint32_t)(128 * BK) : 16u);
      const uint64_t bd64 = make_sw128_desc(s_base + S::OFF_B, B_MN ? (uint32_t)(128 * BK) : 16u);
      const uint32_t a_lo0 = (uint32_t)ad64, a_hi = (uint32_t)(ad64 >> 32);
      const uint32_t b_lo0 = (uint32_t)bd64, b_hi = (uint32_t)(bd64 >> 32);
      auto uwait = [&](uint32_t bar, uint32_t parity) -> bool {
        return mbar_spin_bounded_warp(bar, parity, abort_flag, SITE_GEMM_MMA);
      };
      // The four MMAs of the smem stage in `stage` into accumulator `d_tmem`
      // (the first of them overwrites it when `fresh`).
      auto issue_stage = [&](uint32_t d_tmem, bool fresh) {
        tc_fence_after();
        // Stage offsets go into the descriptors' start-address field (addr >> 4).
        const uint32_t a_lo = a_lo0 + (uint32_t)((stage * S::A_BYTES) >> 4);
        const uint32_t b_lo = b_lo0 + (uint32_t)((stage * S::B_BYTES) >> 4);
#pragma unroll
        for (int kk = 0; kk < BK / UMMA_K; ++kk) {
          // K advance: 32 bytes along a K-major row, or 32 K rows of 128 B of an
          // MN-major tile (encoded >> 4).
          const uint32_t a_off = A_MN ? (uint32_t)(kk * UMMA_K * 128 >> 4) : (uint32_t)(kk * UMMA_K >> 4);
          const uint32_t b_off = B_MN ? (uint32_t)(kk * UMMA_K * 128 >> 4) : (uint32_t)(kk * UMMA_K >> 4);
          if (!(kProfiling && (p.debug_flags & 2)))
            umma_f8_elect<PAIR>(d_tmem, a_lo + a_off, a_hi, b_lo + b_off, b_hi, IDESC, (kk > 0 || !fresh) ? 1u : 0u);
        }
        // smem stage (of both CTAs) free once these MMAs retire
        umma_commit_elect<PAIR>(bar_empty + 8 * stage);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      };
      if (p.stages_per_group == 1 && NACC == 2) {
        // One smem stage per K group (qbk == 128, or K <= 128): a flat loop over
        // this CTA's (tile, group) sequence, two groups per iteration, so the
        // accumulator of group j (buffer j & 1, use (j >> 1) + 1) is a constant.
        const int my_tiles = first_tile < p.num_tiles ? (p.num_tiles - first_tile + tile_step - 1) / tile_step : 0;
        const int total = my_tiles * p.num_groups;
        auto group = [&](auto JB, int j) -> bool {
          constexpr uint32_t buf = decltype(JB)::value;
          PCB_TRACE(0, j);
          if (!uwait(bar_tempty + 8 * buf, ((uint32_t)(j >> 1) & 1u) ^ 1u))
            return false;
          PCB_TRACE(1, j);
          if (!uwait(bar_full + 8 * stage, phase)) return false;
          PCB_TRACE(2, j);
          issue_stage(tmem_base + buf * BN, true);
          umma_commit_elect<PAIR>(bar_tfull + 8 * buf);  // accumulator of group j ready (both CTAs)
          PCB_TRACE(3, j);
          return true;
        };
        for (int j = 0; j < total; j += 2) {
          if (!group(std::integral_constant<uint32_t, 0>{}, j)) {
            ok = false;
            break;
          }
          if (j + 1 < total && !group(std::integral_constant<uint32_t, 1>{}, j + 1)) {
            ok = false;
            break;
          }
        }
      } else {
        uint32_t acc_cnt = 0;
        for (int tile = first_tile; tile < p.num_tiles && ok; tile += tile_step) {
          for (int g = 0; g < p.num_groups && ok; ++g, ++acc_cnt) {
            const uint32_t abuf = acc_cnt % NACC;
            PCB_TRACE(0, acc_cnt);
            if (!uwait(bar_tempty + 8 * abuf, ((acc_cnt / NACC) & 1) ^ 1)) {
              ok = false;
              break;
            }
            PCB_TRACE(1, acc_cnt);
            const int ks0 = g * p.stages_per_group;
            const int ks1 = min(p.k_stages, ks0 + p.stages_per_group);
            for (int ks = ks0; ks < ks1; ++ks) {
              if (!uwait(bar_full + 8 * stage, phase)) {
                ok = false;
                break;
              }
              if (ks == ks0) PCB_TRACE(2, acc_cnt);
              issue_stage(tmem_base + abuf * BN, ks == ks0);
            }
            if (!ok) break;
            umma_commit_elect<PAIR>(bar_tfull + 8 * abuf);  // accumulator of group g ready (both CTAs)
            PCB_TRACE(3, acc_cnt);
          }
        }
      }
    }
  } else {
    // ----------------------------- scale loader --------------------------------
    // Warps 2-3 stage the fp32 scales of the next W K groups of each tile in
    // a four-slot shared ring: row scales [g][row] of this CTA's BM rows and,
    // for uniform B scales, the scale of each epilogue half [g][half].  The
    // epilogue then reads one shared word per group instead of issuing a
    // global load whose latency under the operand stream stalls it.
    const int t = threadIdx.x - 64;
    uint32_t wc = 0;
    bool ok = true;
    for (int tile = first_tile; tile < p.num_tiles && ok; tile += tile_step) {
      const int b = tile / tiles_per_batch;
      const int rem = tile - b * tiles_per_batch;
      const int mb = rem / p.n_blocks;
      const int nb = rem - mb * p.n_blocks;
      const int row0 = mb * TILE_M + (int)rank * BM;
      const float* sa_b = p.sa ? p.sa + (long long)b * p.ssab : nullptr;
      const float* sb_b = p.sb ? p.sb + (long long)b * p.ssbb : nullptr;
      for (int g0 = 0; g0 < p.num_groups; g0 += W, ++wc) {
        const uint32_t slot = wc % kScaleSlots;
        if (!mbar_spin_bounded_warp(bar_sempty + 8 * slot, ((wc / kScaleSlots) & 1) ^ 1, abort_flag,
                                    SITE_GEMM_EPILOGUE)) {
          ok = false;
          break;
        }
        float* dst = sring + slot * S::SC_SLOT;
        // Per-column B scales: one pass of 16-byte loads where the layouts
        // allow (rounds of scalar loads per window were slower than the
        // epilogue consumes windows).
        const bool vec_rows = !COL_UNIFORM && p.sa_vec == 2 && row0 + BM <= p.m;
        if constexpr (!COL_UNIFORM) {
          if (vec_rows) {
            // Rows contiguous per K group: BM / 4 float4 per group.
            constexpr int U = W * (BM / 4) / kScaleThreads;
            float4 v[U];
#pragma unroll
            for (int i = 0; i < U; ++i) {
              const int u = t + i * kScaleThreads, gw = u / (BM / 4), rq = u % (BM / 4);
              v[i] = g0 + gw < p.num_groups
                         ? __ldg(reinterpret_cast<const float4*>(sa_b + row0 + 4 * rq + (long long)(g0 + gw) * p.ssak))
                         : make_float4(1.f, 1.f, 1.f, 1.f);
            }
#pragma unroll
            for (int i = 0; i < U; ++i) {
              const int u = t + i * kScaleThreads, gw = u / (BM / 4), rq = u % (BM / 4);
              *reinterpret_cast<float4*>(dst + gw * BM + 4 * rq) = v[i];
            }
          }
          // Per-column B scales of the tile's BN columns, [gw][col].
          if (p.sb_vec && g0 + W <= p.num_groups && nb * BN + BN <= p.n) {
            constexpr int U = W * (BN / 4) / kScaleThreads;
            float4 v[U];
#pragma unroll
            for (int i = 0; i < U; ++i) {
              const int u = t + i * kScaleThreads, gw = u / (BN / 4), cq = u % (BN / 4);
              v[i] = __ldg(reinterpret_cast<const float4*>(sb_b + (long long)(g0 + gw) * p.ssbk + nb * BN + 4 * cq));
            }
#pragma unroll
            for (int i = 0; i < U; ++i) {
              const int u = t + i * kScaleThreads, gw = u / (BN / 4), cq = u % (BN / 4);
              *reinterpret_cast<float4*>(dst + BM * W + gw * BN + 4 * cq) = v[i];
            }
          } else {
            constexpr int PER_C = W * BN / kScaleThreads, PC = 8;
#pragma unroll 1
            for (int i0 = 0; i0 < PER_C; i0 += PC) {
              float v[PC];
#pragma unroll
              for (int i = 0; i < PC; ++i) {
                const int e = t + (i0 + i) * kScaleThreads;
                const int g = g0 + e / BN, col = nb * BN + e % BN;
                v[i] = (sb_b && col < p.n && g < p.num_groups)
                           ? __ldg(sb_b + (long long)g * p.ssbk + (long long)(col / p.qbn) * p.ssbn)
                           : 1.f;
              }
#pragma unroll
              for (int i = 0; i < PC; ++i) dst[BM * W + t + (i0 + i) * kScaleThreads] = v[i];
            }
          }
        }
        // Element e = r + BM * gw (rows fastest: conflict-free shared stores);
        // thread t takes e = t + 64 i, in passes of 8 loads in flight.
        constexpr int PER_T = BM * W / kScaleThreads, PASS = 8;
#pragma unroll 1
        for (int i0 = vec_rows ? PER_T : 0; i0 < PER_T; i0 += PASS) {
          float v[PASS];
#pragma unroll
          for (int i = 0; i < PASS; ++i) {
            const int e = t + (i0 + i) * kScaleThreads;
            const int row = row0 + e % BM, g = g0 + e / BM;
            v[i] = (sa_b && row < p.m && g < p.num_groups)
                       ? __ldg(sa_b + (long long)(row / p.qbm) * p.ssam + (long long)g * p.ssak)
                       : 1.f;
          }
#pragma unroll
          for (int i = 0; i < PASS; ++i) dst[t + (i0 + i) * kScaleThreads] = v[i];
        }
        if (COL_UNIFORM && t < 2 * W) {
          const int g = g0 + (t >> 1);
          const int col = nb * BN + (t & 1) * EPI_COLS;
          dst[BM * W + t] = (sb_b && col < p.n && g < p.num_groups)
                                ? __ldg(sb_b + (long long)g * p.ssbk + (long long)(col / p.qbn) * p.ssbn)
                                : 1.f;
        }
        mbar_arrive(bar_sfull + 8 * slot);
      }
    }
  }
  } else {
    // -------------------------------- epilogue --------------------------------
    if constexpr (BN == 256) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kHighRegs));
    const int ew = warp - kEpiWarp0;        // 0..7
    const int quarter = warp & 3;           // TMEM lane quarter
    const int half = ew >> 2;               // column half
    const int row_in_tile = quarter * 32 + lane;
    uint32_t acc_cnt = 0;
    uint32_t wc = 0;  // scale windows consumed
    bool ok = true;
    // The tmem-empty barrier lives in the leader; the follower arrives remotely.
    const uint32_t bar_tempty_l = PAIR ? mapa_shared(bar_tempty, 0) : bar_tempty;
    for (int tile = first_tile; tile < p.num_tiles && ok; tile += tile_step) {
      const int b = tile / tiles_per_batch;
      const int rem = tile - b * tiles_per_batch;
      const int mb = rem / p.n_blocks;
      const int nb = rem - mb * p.n_blocks;
      const int row = mb * TILE_M + (int)rank * BM + row_in_tile;
      const int col0 = nb * BN + half * EPI_COLS;

      float2 acc[EPI_COLS / 2];
#pragma unroll
      for (int i = 0; i < EPI_COLS / 2; ++i) acc[i] = make_float2(0.f, 0.f);

      // Pair tiles with uniform B scales: two groups per loop iteration (the
      // loop-back of a single group costs ~200 cycles of the ~750 a group
      // takes on the epilogue's critical path).  The other variants keep one
      // group per iteration, which their registers need.
#pragma unroll(PAIR && COL_UNIFORM ? 2 : 1)
      for (int g = 0; g < p.num_groups && ok; ++g) {
        {
          const uint32_t abuf = acc_cnt % NACC;
          const uint32_t aphase = (acc_cnt / NACC) & 1;
          const int gw = g % W;
          const uint32_t slot = wc % kScaleSlots;
          if (gw == 0 &&
              !mbar_spin_bounded_warp(bar_sfull + 8 * slot, (wc / kScaleSlots) & 1, abort_flag, SITE_GEMM_EPILOGUE)) {
            ok = false;
            break;
          }
          const float* ws = sring + slot * S::SC_SLOT;
          const float s_row = ws[gw * BM + row_in_tile];
          const float s_col = COL_UNIFORM ? ws[BM * W + gw * 2 + half] : 1.f;
          // Per-column B scales of this group and this warp's columns (read
          // from the ring during the promotion, so the slot is handed back
          // after it; uniform scales were read above and free it now).
          const float* colscale = ws + BM * W + gw * BN + half * EPI_COLS;
          const uint32_t colscale_s = smem_u32(colscale);
          const bool win_end = gw == W - 1 || g + 1 == p.num_groups;
          if (COL_UNIFORM && win_end) {
            // This warp has read the window's scales.
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_sempty + 8 * slot);
            ++wc;
          }
          if (threadIdx.x == 128) PCB_TRACE(4, acc_cnt);
          if (!(PAIR ? mbar_spin_bounded_warp(bar_tfull + 8 * abuf, aphase, abort_flag, SITE_GEMM_EPILOGUE)
                     : wait(bar_tfull + 8 * abuf, aphase, SITE_GEMM_EPILOGUE))) {
            ok = false;
            break;
          }
          if (threadIdx.x == 128) PCB_TRACE(5, acc_cnt);
          tc_fence_after();
          if (kProfiling && (p.debug_flags & 1)) {
            __syncwarp();
            if (lane == 0) {
              if constexpr (PAIR) mbar_arrive_cluster(bar_tempty_l + 8 * abuf);
              else mbar_arrive(bar_tempty + 8 * abuf);
            }
            if (!COL_UNIFORM && win_end) {
              __syncwarp();
              if (lane == 0) mbar_arrive(bar_sempty + 8 * slot);
              ++wc;
            }
            ++acc_cnt;
            continue;
          }
          const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + abuf * BN + half * EPI_COLS;
          if constexpr (EPI_COLS <= 64) {
            // Narrow half-tile: load it all, free the buffer, then FMA.
            uint32_t v[EPI_COLS / 32][32];
#pragma unroll
            for (int c = 0; c < EPI_COLS / 32; ++c) tmem_ld32_nowait(taddr + c * 32, v[c]);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < EPI_COLS / 32; ++c) tmem_regs_ready(v[c]);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
              if constexpr (PAIR) mbar_arrive_cluster(bar_tempty_l + 8 * abuf);
              else mbar_arrive(bar_tempty + 8 * abuf);
            }
#pragma unroll
            for (int c = 0; c < EPI_COLS / 32; ++c)
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                float2 s2;
                if constexpr (COL_UNIFORM) {
                  s2 = make_float2(s_row * s_col, s_row * s_col);
                } else {
                  s2 = make_float2(s_row * colscale[c * 32 + 2 * i], s_row * colscale[c * 32 + 2 * i + 1]);
                }
                acc[c * 16 + i] = __ffma2_rn(make_float2(__uint_as_float(v[c][2 * i]), __uint_as_float(v[c][2 * i + 1])),
                                             s2, acc[c * 16 + i]);
              }
          } else {
            // Wide half-tile: 32-column TMEM loads, double-buffered so the
            // load of chunk c + 1 is in flight while chunk c is promoted; the
            // buffer is released as soon as the last load has landed.
            constexpr int CW = 32;
            constexpr int NCH = EPI_COLS / CW;
            uint32_t v[2][CW];
            auto promote = [&](const uint32_t(&vc)[CW], int c) {
              if constexpr (COL_UNIFORM) {
                const float2 s2 = make_float2(s_row * s_col, s_row * s_col);
#pragma unroll
                for (int i = 0; i < CW / 2; ++i)
                  acc[c * (CW / 2) + i] = __ffma2_rn(
                      make_float2(__uint_as_float(vc[2 * i]), __uint_as_float(vc[2 * i + 1])), s2, acc[c * (CW / 2) + i]);
              } else {
                // CW column scales of this chunk: broadcast 16-byte shared loads.
                const float2 r2 = make_float2(s_row, s_row);
#pragma unroll
                for (int q = 0; q < CW / 4; ++q) {
                  float4 cs4;
                  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                               : "=f"(cs4.x), "=f"(cs4.y), "=f"(cs4.z), "=f"(cs4.w)
                               : "r"(colscale_s + (uint32_t)(c * CW + 4 * q) * 4u));
                  const float2 sa = __fmul2_rn(make_float2(cs4.x, cs4.y), r2);
                  const float2 sb2 = __fmul2_rn(make_float2(cs4.z, cs4.w), r2);
                  const int a0 = c * (CW / 2) + 2 * q;
                  acc[a0] = __ffma2_rn(make_float2(__uint_as_float(vc[4 * q]), __uint_as_float(vc[4 * q + 1])), sa,
                                       acc[a0]);
                  acc[a0 + 1] = __ffma2_rn(make_float2(__uint_as_float(vc[4 * q + 2]), __uint_as_float(vc[4 * q + 3])),
                                           sb2, acc[a0 + 1]);
                }
              }
            };
            tmem_ld32_nowait(taddr, v[0]);
            tmem_wait_ld();
            tmem_regs_ready(v[0]);
#pragma unroll
            for (int c = 0; c < NCH; ++c) {
              if (c + 1 < NCH) {
                tmem_ld32_nowait(taddr + (c + 1) * CW, v[(c + 1) & 1]);
              } else {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                  if constexpr (PAIR) mbar_arrive_cluster(bar_tempty_l + 8 * abuf);
                  else mbar_arrive(bar_tempty + 8 * abuf);
                }
                if (threadIdx.x == 128) PCB_TRACE(6, acc_cnt);
              }
              promote(v[c & 1], c);
              if (c + 1 < NCH) {
                tmem_wait_ld();
                tmem_regs_ready(v[(c + 1) & 1]);
              }
            }
          }
          if (!COL_UNIFORM && win_end) {
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_sempty + 8 * slot);
            ++wc;
          }
          if (threadIdx.x == 128) PCB_TRACE(7, acc_cnt);
          ++acc_cnt;
        }
      }
      if (!ok) break;

      // Bias, activation, cast, store.
      float* accf = reinterpret_cast<float*>(acc);
      if (PAIR && p.c_tma)
        store_rows_tma<EPI_COLS>(p, &tmap_c, accf, b, row, mb * TILE_M + (int)rank * BM + quarter * 32, col0,
                                 s_base + S::OFF_CSTG + (uint32_t)(ew * S::CSTG_BUF), lane);
      else
        store_row<EPI_COLS>(p, accf, b, row, col0);
    }
    // The staging buffers stay valid until every issued store has completed.
    if (PAIR && p.c_tma && lane == 0) bulk_wait_all();
  }

  PCB_CTA_SPAN(1);
  tc_fence_before();
  if constexpr (PAIR) {
    cluster_sync_all();  // no CTA leaves while its peer may still touch its smem / barriers
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem_base, TMEM_COLS);
  } else {
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace gemm
}  // namespace pcb
