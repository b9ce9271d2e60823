// libpcb200: the C ABI (include/pcb200.h) over the sm_100a kernels.
// One translation unit so the device error word is a single symbol.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"
#include "gemm_sm100.cuh"
#include "quant_kernels.cuh"
#include "gemm_fused_sm100.cuh"
#include "gemm_bs_sm100.cuh"
#include "quant_tile_tma.cuh"

using namespace pcb;

namespace {

thread_local std::string g_last_error;
std::atomic<int> g_inject_error{0};

int fail(int status, const char* what) {
  g_last_error = what;
  return status;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
    return PCB_ERR_LAUNCH;
  }
  return PCB_OK;
}

struct DeviceInfo {
  int sm_count = 0;
  int major = 0;
};

DeviceInfo device_info() {
  static std::mutex mu;
  static DeviceInfo cache[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev].sm_count == 0) {
    cudaDeviceGetAttribute(&cache[dev].sm_count, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&cache[dev].major, cudaDevAttrComputeCapabilityMajor, dev);
  }
  return cache[dev];
}

bool aligned(const void* p, int64_t a) { return (reinterpret_cast<uintptr_t>(p) % (uintptr_t)a) == 0; }

template <typename K>
void ensure_smem_attr(K kernel, int bytes) {
  // cudaFuncSetAttribute is per function and device; calling it again is cheap
  // and keeps this stateless across devices and threads.
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}


int elem_size(int dt) {
  switch (dt) {
    case PCB_DTYPE_F32: return 4;
    case PCB_DTYPE_F16:
    case PCB_DTYPE_BF16: return 2;
    case PCB_DTYPE_E4M3:
    case PCB_DTYPE_E5M2: return 1;
    default: return 0;
  }
}

bool is_float_in(int dt) { return dt == PCB_DTYPE_F32 || dt == PCB_DTYPE_F16 || dt == PCB_DTYPE_BF16; }
bool is_fp8(int dt) { return dt == PCB_DTYPE_E4M3 || dt == PCB_DTYPE_E5M2; }

// Dispatch a functor over (input dtype, fp8 output dtype) as compile-time ints.
template <typename F>
int dispatch_xy(int xt, int yt, F&& f) {
  auto with_y = [&](auto xc) -> int {
    if (yt == PCB_DTYPE_E4M3) return f(xc, std::integral_constant<int, PCB_DTYPE_E4M3>{});
    if (yt == PCB_DTYPE_E5M2) return f(xc, std::integral_constant<int, PCB_DTYPE_E5M2>{});
    return fail(PCB_ERR_INVALID, "output dtype must be E4M3 or E5M2");
  };
  if (xt == PCB_DTYPE_F32) return with_y(std::integral_constant<int, PCB_DTYPE_F32>{});
  if (xt == PCB_DTYPE_F16) return with_y(std::integral_constant<int, PCB_DTYPE_F16>{});
  if (xt == PCB_DTYPE_BF16) return with_y(std::integral_constant<int, PCB_DTYPE_BF16>{});
  return fail(PCB_ERR_INVALID, "input dtype must be F32, F16 or BF16");
}

// ---------------------------------------------------------------------------
// Grouped quantization (per-block and per-channel rows share this driver).
// ---------------------------------------------------------------------------
bool make_map_x16(CUtensorMap* map, const void* base, int dt, uint64_t inner, uint64_t outer, uint64_t batch,
                  uint64_t outer_stride_bytes, uint64_t batch_stride_bytes);
bool make_map_tile(CUtensorMap* map, const void* base, int dt, uint64_t inner, uint64_t outer, uint64_t batch,
                   uint64_t outer_stride_bytes, uint64_t batch_stride_bytes);

int launch_groups(const void* x, int xt, int64_t batch, int64_t m, int64_t n, int64_t sxb, int64_t sxm, int64_t sxn,
                  void* y, int yt, int64_t syb, int64_t sym, int64_t syn, float* scale, int64_t ssb, int64_t ssm,
                  int64_t ssn, int64_t gm, int64_t gn, int mode, float eps, cudaStream_t stream) {
  const int es = elem_size(xt);
  const int vec = 16 / es;
  const int64_t groups_m = (m + gm - 1) / gm, groups_n = (n + gn - 1) / gn;
  const int64_t num_groups = batch * groups_m * groups_n;
  if (num_groups == 0) return PCB_OK;
  const DeviceInfo di = device_info();
  const bool vec_ok = sxn == 1 && syn == 1 && n % vec == 0 && gn % vec == 0 && aligned(x, 16) &&
                      (sxm * es) % 16 == 0 && (batch == 1 || (sxb * es) % 16 == 0) && aligned(y, vec) &&
                      sym % vec == 0 && (batch == 1 || syb % vec == 0);
  if (gn == 1 && gm > 1 && sxn == 1 && syn == 1 && n % vec == 0 && aligned(x, 16) && (sxm * es) % 16 == 0 &&
      (batch == 1 || (sxb * es) % 16 == 0) && aligned(y, vec) && sym % vec == 0 && (batch == 1 || syb % vec == 0) &&
      gm <= (int64_t)1 << 30) {
    // Column blocks (gm x 1, e.g. 128 x 1) of a row-major tensor: one CTA per
    // (64-or-32-column strip, row slab), coalesced along the row.
    const int sw = 8 * vec;
    quant::ColArgs a{x, sxb, sxm, y, syb, sym, scale, ssb, ssn, m, n, (int)gm, eps, ssm};
    return dispatch_xy(xt, yt, [&](auto xc, auto yc) -> int {
      constexpr int XT = decltype(xc)::value;
      constexpr int YT = decltype(yc)::value;
      const dim3 grid((unsigned)((n + sw - 1) / sw), (unsigned)groups_m, (unsigned)batch);
      if (mode == quant::kDeqReciprocal)
        quant::quant_cols_cluster_kernel<XT, YT, true><<<grid, quant::kThreads, 0, stream>>>(a);
      else if (mode == quant::kDeqPow2)
        quant::quant_cols_cluster_kernel<XT, YT, true, quant::kDeqPow2><<<grid, quant::kThreads, 0, stream>>>(a);
      else
        return fail(PCB_ERR_UNSUPPORTED, "column-slab quantization is per-block only");
      return check_launch("quant_cols_cluster_kernel (slab)");
    });
  }
  const bool tile16 = (xt == PCB_DTYPE_BF16 || xt == PCB_DTYPE_F16) && (gm == 128 || gm == 1);
  const bool tile32 = xt == PCB_DTYPE_F32 && gm == 128;
  const bool quant_divide = mode == quant::kQuantDivide;  // dynamic float8 casts: group kernels only
  if (vec_ok && (tile16 || tile32) && gn == 128 && m <= INT32_MAX && n <= INT32_MAX && batch <= INT32_MAX &&
      !quant_divide) {
    // 128x128 or 1x128 blocks of a 16-bit tensor: TMA-staged persistent kernel
    // over 128x128 tiles.
    CUtensorMap tm;
    const int es = elem_size(xt);
    if (make_map_tile(&tm, x, xt, (uint64_t)n, (uint64_t)m, (uint64_t)batch, (uint64_t)sxm * es, (uint64_t)sxb * es)) {
      const int64_t num_tiles = batch * ((m + 127) / 128) * groups_n;
      quant::TileArgs a{y, syb, sym, scale, ssb, ssm, ssn, m, n, groups_m, groups_n, num_tiles, eps};
      auto go = [&](auto kernel, auto cfg) -> int {
        using Cfg = decltype(cfg);
        const unsigned grid = (unsigned)std::min<int64_t>(num_tiles, (int64_t)di.sm_count * Cfg::CTAS_PER_SM);
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
        kernel<<<grid, quant::kThreads, Cfg::SMEM, stream>>>(tm, a);
        return check_launch("quant_tile128_tma_kernel");
      };
      return dispatch_xy(xt, yt, [&](auto xc, auto yc) -> int {
        constexpr int XT = decltype(xc)::value;
        constexpr int YT = decltype(yc)::value;
        if constexpr (XT == PCB_DTYPE_F32) {
          using Cfg = quant::TileCfg<128, 4>;
          if (mode == quant::kDeqPow2) return go(quant::quant_tile128_tma_kernel<XT, YT, quant::kDeqPow2, 128>, Cfg{});
          if (mode == quant::kDeqReciprocal)
            return go(quant::quant_tile128_tma_kernel<XT, YT, quant::kDeqReciprocal, 128>, Cfg{});
          return go(quant::quant_tile128_tma_kernel<XT, YT, quant::kDeqDivide, 128>, Cfg{});
        } else if constexpr (XT == PCB_DTYPE_BF16 || XT == PCB_DTYPE_F16) {
          constexpr int R = quant::kDeqReciprocal, D = quant::kDeqDivide;
          constexpr int P = quant::kDeqPow2;
          if (mode == P)
            return gm == 1 ? go(quant::quant_tile128_tma_kernel<XT, YT, P, 1>, quant::TileCfg<1>{})
                           : go(quant::quant_tile128_tma_kernel<XT, YT, P, 128>, quant::TileCfg<128>{});
          if (gm == 1)
            return mode == R ? go(quant::quant_tile128_tma_kernel<XT, YT, R, 1>, quant::TileCfg<1>{})
                             : go(quant::quant_tile128_tma_kernel<XT, YT, D, 1>, quant::TileCfg<1>{});
          return mode == R ? go(quant::quant_tile128_tma_kernel<XT, YT, R, 128>, quant::TileCfg<128>{})
                           : go(quant::quant_tile128_tma_kernel<XT, YT, D, 128>, quant::TileCfg<128>{});
        } else {
          return fail(PCB_ERR_UNSUPPORTED, "unreachable");
        }
      });
    }
  }
  const int64_t cpg = gn / vec;
  if (vec_ok && gm == 1 && cpg <= 32 && (32 % cpg) == 0 && mode != quant::kDeqPow2 && !quant_divide) {
    // Row groups of at most one warp (1x128 and narrower): contiguous row spans.
    constexpr int CH = 8;
    const int64_t spans_per_row = (n / vec + 32 * CH - 1) / (32 * CH);
    const int64_t rows = batch * m;
    quant::RowSpanArgs a{x, sxb, sxm, y, syb, sym, scale, ssb, ssm, ssn, m, n, rows, spans_per_row,
                         rows * spans_per_row, eps};
    return dispatch_xy(xt, yt, [&](auto xc, auto yc) -> int {
      constexpr int XT = decltype(xc)::value;
      constexpr int YT = decltype(yc)::value;
      auto go = [&](auto kernel) -> int {
        const int64_t warps_per_cta = quant::kThreads / 32;
        int64_t grid = (a.units + warps_per_cta - 1) / warps_per_cta;
        grid = std::min<int64_t>(grid, (int64_t)di.sm_count * 3);
        kernel<<<(unsigned)grid, quant::kThreads, 0, stream>>>(a);
        return check_launch("quant_rowspan_kernel");
      };
      const bool recip = mode == quant::kDeqReciprocal;
      switch (cpg) {
        case 1: return recip ? go(quant::quant_rowspan_kernel<XT, YT, 1, CH, quant::kDeqReciprocal>)
                             : go(quant::quant_rowspan_kernel<XT, YT, 1, CH, quant::kDeqDivide>);
        case 2: return recip ? go(quant::quant_rowspan_kernel<XT, YT, 2, CH, quant::kDeqReciprocal>)
                             : go(quant::quant_rowspan_kernel<XT, YT, 2, CH, quant::kDeqDivide>);
        case 4: return recip ? go(quant::quant_rowspan_kernel<XT, YT, 4, CH, quant::kDeqReciprocal>)
                             : go(quant::quant_rowspan_kernel<XT, YT, 4, CH, quant::kDeqDivide>);
        case 8: return recip ? go(quant::quant_rowspan_kernel<XT, YT, 8, CH, quant::kDeqReciprocal>)
                             : go(quant::quant_rowspan_kernel<XT, YT, 8, CH, quant::kDeqDivide>);
        case 16: return recip ? go(quant::quant_rowspan_kernel<XT, YT, 16, CH, quant::kDeqReciprocal>)
                              : go(quant::quant_rowspan_kernel<XT, YT, 16, CH, quant::kDeqDivide>);
        default: return recip ? go(quant::quant_rowspan_kernel<XT, YT, 32, CH, quant::kDeqReciprocal>)
                              : go(quant::quant_rowspan_kernel<XT, YT, 32, CH, quant::kDeqDivide>);
      }
    });
  }
  if (vec_ok) {
    quant::GroupArgs a{x, sxb, sxm, y, syb, sym, scale, ssb, ssm, ssn, batch, m, n, gm, gn, groups_m, groups_n,
                       num_groups, eps};
    const int64_t nch = gm * gn / vec;
    return dispatch_xy(xt, yt, [&](auto xc, auto yc) -> int {
      constexpr int XT = decltype(xc)::value;
      constexpr int YT = decltype(yc)::value;
      auto go = [&](auto kernel, int team) -> int {
        const int64_t teams_per_cta = quant::kThreads / team;
        int64_t grid = (num_groups + teams_per_cta - 1) / teams_per_cta;
        grid = std::min<int64_t>(grid, (int64_t)di.sm_count * 8);
        kernel<<<(unsigned)grid, quant::kThreads, 0, stream>>>(a);
        return check_launch("quant_groups_kernel");
      };
      // Team size and 16-byte chunks per thread by group size: groups of up
      // to 512 chunks (4096 bf16, a per-channel row) take one warp with up to
      // 16 loads in flight per lane and a shuffle reduction; larger groups a
      // whole CTA.
      auto by_size = [&](auto mc) -> int {
        constexpr int MODE = decltype(mc)::value;
        if (nch <= 16) return go(quant::quant_groups_kernel<XT, YT, 8, 2, MODE>, 8);
        if (nch <= 32) return go(quant::quant_groups_kernel<XT, YT, 16, 2, MODE>, 16);
        if (nch <= 128) return go(quant::quant_groups_kernel<XT, YT, 32, 4, MODE>, 32);
        if (nch <= 256) return go(quant::quant_groups_kernel<XT, YT, 32, 8, MODE>, 32);
        if (nch <= 512) return go(quant::quant_groups_kernel<XT, YT, 32, 16, MODE>, 32);
        return go(quant::quant_groups_kernel<XT, YT, 256, 8, MODE>, 256);
      };
      if (mode == quant::kDeqPow2) return by_size(std::integral_constant<int, quant::kDeqPow2>{});
      if (quant_divide) return by_size(std::integral_constant<int, quant::kQuantDivide>{});
      if (mode == quant::kDeqReciprocal) return by_size(std::integral_constant<int, quant::kDeqReciprocal>{});
      return by_size(std::integral_constant<int, quant::kDeqDivide>{});
    });
  }
  if (mode == quant::kDeqPow2)
    return fail(PCB_ERR_UNSUPPORTED, "power-of-two scales need x and y contiguous along n with 16-byte aligned rows");
  quant::GenericArgs a{x, sxb, sxm, sxn, y, syb, sym, syn, scale, ssb, ssm, ssn, batch, m, n, gm, gn,
                       groups_m, groups_n, num_groups, eps};
  return dispatch_xy(xt, yt, [&](auto xc, auto yc) -> int {
    constexpr int XT = decltype(xc)::value;
    constexpr int YT = decltype(yc)::value;
    const int64_t grid = std::min<int64_t>(num_groups, (int64_t)di.sm_count * 8);
    if (mode == quant::kDeqReciprocal)
      quant::quant_groups_generic_kernel<XT, YT, quant::kDeqReciprocal><<<(unsigned)grid, quant::kThreads, 0, stream>>>(a);
    else if (quant_divide)
      quant::quant_groups_generic_kernel<XT, YT, quant::kQuantDivide><<<(unsigned)grid, quant::kThreads, 0, stream>>>(a);
    else
      quant::quant_groups_generic_kernel<XT, YT, quant::kDeqDivide><<<(unsigned)grid, quant::kThreads, 0, stream>>>(a);
    return check_launch("quant_groups_generic_kernel");
  });
}

// ---------------------------------------------------------------------------
// TMA descriptors (driver entry point fetched through the runtime, so the
// library does not link libcuda directly).
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 3-D uint8 map (inner, outer, batch) with a 128-byte swizzled box (128, box_outer, 1).
bool make_map_u8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t batch,
                 uint64_t outer_stride, uint64_t batch_stride, uint32_t box_outer) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {inner, outer, batch};
  if (batch <= 1) {
    batch_stride = ((outer * outer_stride + 15) / 16) * 16;
    if (batch_stride == 0) batch_stride = 16;
  }
  cuuint64_t strides[2] = {outer_stride, batch_stride};
  cuuint32_t box[3] = {128, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 3-D map of 16-bit elements (inner, outer, batch), unswizzled box (128, 128, 1):
// one 128x128 activation tile with 256-byte rows.
bool make_map_x16(CUtensorMap* map, const void* base, int dt, uint64_t inner, uint64_t outer, uint64_t batch,
                  uint64_t outer_stride_bytes, uint64_t batch_stride_bytes) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {inner, outer, batch};
  if (batch <= 1) batch_stride_bytes = std::max<uint64_t>(16, ((outer * outer_stride_bytes + 15) / 16) * 16);
  cuuint64_t strides[2] = {outer_stride_bytes, batch_stride_bytes};
  cuuint32_t box[3] = {128, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType t =
      dt == PCB_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return fn(map, t, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 3-D map of a bf16 / fp16 / fp32 output C (n, m, batch) for TMA stores of
// 32-row boxes with 128-byte rows (64 or 32 columns) in the 128-byte swizzle
// (the pair epilogue's staging layout).
bool make_map_c(CUtensorMap* map, void* base, int dt, uint64_t n, uint64_t m, uint64_t batch,
                  uint64_t row_stride_bytes, uint64_t batch_stride_bytes) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {n, m, batch};
  if (batch <= 1) batch_stride_bytes = std::max<uint64_t>(16, ((m * row_stride_bytes + 15) / 16) * 16);
  cuuint64_t strides[2] = {row_stride_bytes, batch_stride_bytes};
  cuuint32_t box[3] = {dt == PCB_DTYPE_F32 ? 32u : 64u, 32, 1};  // 128-byte box rows
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType t = dt == PCB_DTYPE_BF16  ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                : dt == PCB_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  return fn(map, t, 3, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Unswizzled (128, 128, 1) box of bf16 / fp16 / fp32 elements: one quantizer tile.
bool make_map_tile(CUtensorMap* map, const void* base, int dt, uint64_t inner, uint64_t outer, uint64_t batch,
                   uint64_t outer_stride_bytes, uint64_t batch_stride_bytes) {
  if (dt != PCB_DTYPE_F32) return make_map_x16(map, base, dt, inner, outer, batch, outer_stride_bytes, batch_stride_bytes);
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {inner, outer, batch};
  if (batch <= 1) batch_stride_bytes = std::max<uint64_t>(16, ((outer * outer_stride_bytes + 15) / 16) * 16);
  cuuint64_t strides[2] = {outer_stride_bytes, batch_stride_bytes};
  cuuint32_t box[3] = {128, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool B_MN, int XT, bool COLU>
int launch_fused(const CUtensorMap& tx, const CUtensorMap& tb, const gemm::Params& p, int sm_count,
                 cudaStream_t stream) {
  auto kernel = gemm::quant_bmm_fused_kernel<B_MN, XT, COLU>;
  ensure_smem_attr(kernel, gemm::FusedSmem::ALLOC);
  const int grid = std::min(p.num_tiles, sm_count);
  kernel<<<grid, gemm::kFusedThreads, gemm::FusedSmem::ALLOC, stream>>>(tx, tb, p);
  return check_launch("quant_bmm_fused_kernel");
}


template <int BN, bool A_MN, bool B_MN, bool COLU, bool PAIR>
int launch_bmm(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const gemm::Params& p,
               int sm_count, cudaStream_t stream) {
  using S = gemm::Smem<BN, PAIR, COLU>;
  auto kernel = gemm::bmm_scaled_kernel<BN, A_MN, B_MN, COLU, PAIR>;
  if constexpr (BN == 256) {
    // This instantiation re-splits its registers with setmaxnreg; the split
    // is only valid when the launch holds exactly kLaunchRegs per thread
    // (otherwise setmaxnreg.inc could never be satisfied), so never launch a
    // build where ptxas chose another count.
    static const int num_regs = [&] {
      cudaFuncAttributes fa{};
      return cudaFuncGetAttributes(&fa, kernel) == cudaSuccess ? fa.numRegs : -1;
    }();
    if (num_regs != gemm::kLaunchRegs)
      return fail(PCB_ERR_UNSUPPORTED, "bmm kernel register count differs from its setmaxnreg split");
  }
  ensure_smem_attr(kernel, S::ALLOC);
  if constexpr (PAIR) {
    // Clusters of two CTAs (one tile of 256 rows each), one CTA per SM.
    const int clusters = std::min(p.num_tiles, sm_count / 2);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(2 * clusters), 1, 1);
    cfg.blockDim = dim3(gemm::kThreads, 1, 1);
    cfg.dynamicSmemBytes = S::ALLOC;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    // The kernel's prologue may overlap the previous kernel (griddepcontrol.wait
    // precedes every global access).
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaLaunchKernelEx(&cfg, kernel, ta, tb, tc, p);
  } else {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)std::min(p.num_tiles, sm_count), 1, 1);
    cfg.blockDim = dim3(gemm::kThreads, 1, 1);
    cfg.dynamicSmemBytes = S::ALLOC;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kernel, ta, tb, tc, p);
  }
  return check_launch("bmm_scaled_kernel");
}

template <int BN, bool A_MN, bool B_MN, bool PAIR>
int launch_bmm_cols(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const gemm::Params& p, int sm,
                    cudaStream_t s) {
  if (p.col_uniform) return launch_bmm<BN, A_MN, B_MN, true, PAIR>(ta, tb, tc, p, sm, s);
  return launch_bmm<BN, A_MN, B_MN, false, PAIR>(ta, tb, tc, p, sm, s);
}

template <bool A_MN, bool B_MN, int FMT>
int launch_bmm_bs(const CUtensorMap& ta, const CUtensorMap& tb, const gemm::Params& p, int sm_count,
                  cudaStream_t stream) {
  auto kernel = gemm::bmm_blockscaled_kernel<A_MN, B_MN, FMT>;
  // Same setmaxnreg split as the 128x256 scaled kernel: launch only when
  // ptxas allocated exactly the registers the split assumes.
  static const int num_regs = [&] {
    cudaFuncAttributes fa{};
    return cudaFuncGetAttributes(&fa, kernel) == cudaSuccess ? fa.numRegs : -1;
  }();
  if (num_regs != gemm::kLaunchRegs)
    return fail(PCB_ERR_UNSUPPORTED, "block-scaled bmm kernel register count differs from its setmaxnreg split");
  ensure_smem_attr(kernel, gemm::BsSmem::ALLOC);
  const int grid = std::min(p.num_tiles, sm_count);
  kernel<<<grid, gemm::kThreads, gemm::BsSmem::ALLOC, stream>>>(ta, tb, p);
  return check_launch("bmm_blockscaled_kernel");
}

int dispatch_bmm_bs(bool a_mn, bool b_mn, int fmt, const CUtensorMap& ta, const CUtensorMap& tb,
                    const gemm::Params& p, int sm, cudaStream_t s) {
  if (fmt == 0) {
    if (!a_mn && !b_mn) return launch_bmm_bs<false, false, 0>(ta, tb, p, sm, s);
    if (!a_mn && b_mn) return launch_bmm_bs<false, true, 0>(ta, tb, p, sm, s);
    if (a_mn && !b_mn) return launch_bmm_bs<true, false, 0>(ta, tb, p, sm, s);
    return launch_bmm_bs<true, true, 0>(ta, tb, p, sm, s);
  }
  if (!a_mn && !b_mn) return launch_bmm_bs<false, false, 1>(ta, tb, p, sm, s);
  if (!a_mn && b_mn) return launch_bmm_bs<false, true, 1>(ta, tb, p, sm, s);
  if (a_mn && !b_mn) return launch_bmm_bs<true, false, 1>(ta, tb, p, sm, s);
  return launch_bmm_bs<true, true, 1>(ta, tb, p, sm, s);
}

template <int BN, bool PAIR>
int dispatch_bmm_layout(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                        const gemm::Params& p, int sm, cudaStream_t s) {
  if (!a_mn && !b_mn) return launch_bmm_cols<BN, false, false, PAIR>(ta, tb, tc, p, sm, s);
  if (!a_mn && b_mn) return launch_bmm_cols<BN, false, true, PAIR>(ta, tb, tc, p, sm, s);
  if (a_mn && !b_mn) return launch_bmm_cols<BN, true, false, PAIR>(ta, tb, tc, p, sm, s);
  return launch_bmm_cols<BN, true, true, PAIR>(ta, tb, tc, p, sm, s);
}

// ---------------------------------------------------------------------------
// Scratch for pcb_quant_per_tensor_noalloc.  The per-tensor quantizer reduces
// the amax in two launches and parks one partial per amax CTA in between;
// this variant keeps those partials in a fixed array that is part of the
// library image instead of in caller-provided memory.  Every GPU that loads
// the library holds these 4 KiB until the process exits.
// ---------------------------------------------------------------------------
constexpr int kNoAllocPartials = 1024;  // fp32 slots = the most amax CTAs ever launched
static __device__ __align__(256) float g_noalloc_partials[kNoAllocPartials];

// Device address of g_noalloc_partials on the current device.  The name is a
// host-side stand-in in host code, so it must be translated once per device
// (with that device current) before a kernel may be given it.
float* noalloc_partials_on_current_device() {
  static std::mutex mu;
  static float* addr[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    fail(PCB_ERR_DEVICE, "pcb_quant_per_tensor_noalloc: no current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_partials);
    if (e != cudaSuccess || p == nullptr) {
      // Clear the pending (non-sticky) error so the next entry point's launch check
      // does not report it as its own.
      (void)cudaGetLastError();
      fail(PCB_ERR_DEVICE, (std::string("pcb_quant_per_tensor_noalloc: cudaGetSymbolAddress failed: ") +
                            cudaGetErrorString(e)).c_str());
      return nullptr;
    }
    addr[dev] = static_cast<float*>(p);
  }
  return addr[dev];
}

}  // namespace

extern "C" {

int pcb_version(void) { return PCB200_ABI_VERSION; }

const char* pcb_status_name(int status) {
  switch (status) {
    case PCB_OK: return "PCB_OK";
    case PCB_ERR_INVALID: return "PCB_ERR_INVALID";
    case PCB_ERR_UNSUPPORTED: return "PCB_ERR_UNSUPPORTED";
    case PCB_ERR_LAYOUT: return "PCB_ERR_LAYOUT";
    case PCB_ERR_LAUNCH: return "PCB_ERR_LAUNCH";
    case PCB_ERR_DEVICE: return "PCB_ERR_DEVICE";
    case PCB_ERR_TIMEOUT: return "PCB_ERR_TIMEOUT";
    default: return "PCB_ERR_UNKNOWN";
  }
}

const char* pcb_last_error_text(void) { return g_last_error.c_str(); }

int pcb_get_device_error(int* code, int* site, int* info) {
  unsigned int h[3] = {0, 0, 0};
  if (cudaDeviceSynchronize() != cudaSuccess) return check_launch("pcb_get_device_error sync");
  if (cudaMemcpyFromSymbol(h, pcb::g_device_error, sizeof(h)) != cudaSuccess)
    return check_launch("pcb_get_device_error read");
  const unsigned int zero[3] = {0, 0, 0};
  if (cudaMemcpyToSymbol(pcb::g_device_error, zero, sizeof(zero)) != cudaSuccess)
    return check_launch("pcb_get_device_error clear");
  if (code) *code = (int)h[0];
  if (site) *site = (int)h[1];
  if (info) *info = (int)h[2];
  return PCB_OK;
}

int pcb_debug_inject_error(int code) {
  g_inject_error.store(code);
  return PCB_OK;
}

int pcb_quant_per_block(const void* x, int x_dtype, int64_t batch, int64_t m, int64_t n, int64_t sxb, int64_t sxm,
                        int64_t sxn, void* y, int y_dtype, int64_t syb, int64_t sym, int64_t syn, float* scale,
                        int64_t ssb, int64_t ssm, int64_t ssn, int64_t block_m, int64_t block_n, float eps,
                        void* stream) {
  if (batch < 0 || m < 0 || n < 0) return fail(PCB_ERR_INVALID, "negative size");
  if (block_m <= 0 || block_n <= 0) return fail(PCB_ERR_INVALID, "block sizes must be positive");
  if (batch * m * n == 0) return PCB_OK;
  if (!x || !y || !scale) return fail(PCB_ERR_INVALID, "null pointer");
  if (!is_float_in(x_dtype) || !is_fp8(y_dtype)) return fail(PCB_ERR_INVALID, "bad dtype");
  return launch_groups(x, x_dtype, batch, m, n, sxb, sxm, sxn, y, y_dtype, syb, sym, syn, scale, ssb, ssm, ssn,
                       block_m, block_n, quant::kDeqReciprocal, eps, (cudaStream_t)stream);
}

int pcb_quant_per_block_pow2(const void* x, int x_dtype, int64_t batch, int64_t m, int64_t n, int64_t sxb,
                             int64_t sxm, int64_t sxn, void* y, int y_dtype, int64_t syb, int64_t sym, int64_t syn,
                             float* scale, int64_t ssb, int64_t ssm, int64_t ssn, int64_t block_m, int64_t block_n,
                             float eps, void* stream) {
  if (batch < 0 || m < 0 || n < 0) return fail(PCB_ERR_INVALID, "negative size");
  if (block_m <= 0 || block_n <= 0) return fail(PCB_ERR_INVALID, "block sizes must be positive");
  if (batch * m * n == 0) return PCB_OK;
  if (!x || !y || !scale) return fail(PCB_ERR_INVALID, "null pointer");
  if (!is_float_in(x_dtype) || !is_fp8(y_dtype)) return fail(PCB_ERR_INVALID, "bad dtype");
  return launch_groups(x, x_dtype, batch, m, n, sxb, sxm, sxn, y, y_dtype, syb, sym, syn, scale, ssb, ssm, ssn,
                       block_m, block_n, quant::kDeqPow2, eps, (cudaStream_t)stream);
}

int pcb_quant_per_channel(const void* x, int x_dtype, int64_t batch, int64_t m, int64_t n, int64_t sxb, int64_t sxm,
                          int64_t sxn, void* y, int y_dtype, int64_t syb, int64_t sym, int64_t syn, float* scale,
                          int64_t ssb, int64_t ssc, int channel_axis, float eps, void* stream) {
  if (batch < 0 || m < 0 || n < 0) return fail(PCB_ERR_INVALID, "negative size");
  if (channel_axis != -1 && channel_axis != -2) return fail(PCB_ERR_INVALID, "channel_axis must be -1 or -2");
  if (batch * m * n == 0) return PCB_OK;
  if (!x || !y || !scale) return fail(PCB_ERR_INVALID, "null pointer");
  if (!is_float_in(x_dtype) || !is_fp8(y_dtype)) return fail(PCB_ERR_INVALID, "bad dtype");
  cudaStream_t s = (cudaStream_t)stream;
  if (channel_axis == -2) {
    // One group per row: (1 x n), scale index (b, row).
    return launch_groups(x, x_dtype, batch, m, n, sxb, sxm, sxn, y, y_dtype, syb, sym, syn, scale, ssb, ssc, 0, 1, n,
                         quant::kDeqDivide, eps, s);
  }
  // One scale per column.
  if (sxm == 1 && sym == 1 && !(sxn == 1 && m > 1)) {
    // Column-contiguous storage: a column is a contiguous run -> rows of x^T.
    return launch_groups(x, x_dtype, batch, n, m, sxb, sxn, sxm, y, y_dtype, syb, syn, sym, scale, ssb, ssc, 0, 1, m,
                         quant::kDeqDivide, eps, s);
  }
  const int es = elem_size(x_dtype);
  const int vec = 16 / es;
  const bool vec_ok = sxn == 1 && syn == 1 && n % vec == 0 && aligned(x, 16) && (sxm * es) % 16 == 0 &&
                      (batch == 1 || (sxb * es) % 16 == 0) && aligned(y, vec) && sym % vec == 0 &&
                      (batch == 1 || syb % vec == 0);
  if (!vec_ok) {
    return launch_groups(x, x_dtype, batch, m, n, sxb, sxm, sxn, y, y_dtype, syb, sym, syn, scale, ssb, 0, ssc, m, 1,
                         quant::kDeqDivide, eps, s);
  }
  const int sw = 8 * vec;
  const int cl = (int)std::min<int64_t>(8, std::max<int64_t>(1, (m + 255) / 256));
  quant::ColArgs a{x, sxb, sxm, y, syb, sym, scale, ssb, ssc, m, n, (int)((m + cl - 1) / cl), eps, 0};
  return dispatch_xy(x_dtype, y_dtype, [&](auto xc, auto yc) -> int {
    constexpr int XT = decltype(xc)::value;
    constexpr int YT = decltype(yc)::value;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((n + sw - 1) / sw), (unsigned)cl, (unsigned)batch);
    cfg.blockDim = dim3(quant::kThreads, 1, 1);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = (unsigned)cl;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, quant::quant_cols_cluster_kernel<XT, YT>, a);
    return check_launch("quant_cols_cluster_kernel");
  });
}

int64_t pcb_quant_per_tensor_workspace_floats(void) { return quant::kPerTensorMaxPartials; }

int pcb_quant_per_tensor(const void* x, int x_dtype, int64_t batch, int64_t m, int64_t n, int64_t sxb, int64_t sxm,
                         int64_t sxn, void* y, int y_dtype, int64_t syb, int64_t sym, int64_t syn, float* quant_scale,
                         float* dequant_scale, int scale_dtype, float fp8_max, float eps, float* workspace,
                         void* stream) {
  if (batch < 0 || m < 0 || n < 0) return fail(PCB_ERR_INVALID, "negative size");
  if (!x || !y || !workspace) return fail(PCB_ERR_INVALID, "null pointer");
  if (!is_float_in(x_dtype) || !is_fp8(y_dtype) || !is_float_in(scale_dtype)) return fail(PCB_ERR_INVALID, "bad dtype");
  cudaStream_t s = (cudaStream_t)stream;
  const DeviceInfo di = device_info();
  const int es = elem_size(x_dtype);
  const int vec = 16 / es;
  const bool vec_ok = sxn == 1 && syn == 1 && n % vec == 0 && aligned(x, 16) && (sxm * es) % 16 == 0 &&
                      (batch == 1 || (sxb * es) % 16 == 0) && aligned(y, vec) && sym % vec == 0 &&
                      (batch == 1 || syb % vec == 0);
  const int64_t total = batch * m * n;
  const int64_t per_cta = (int64_t)quant::kThreads * (vec_ok ? vec : 1);
  int amax_grid = (int)std::min<int64_t>(std::max<int64_t>(1, (total + per_cta - 1) / per_cta),
                                         std::min<int64_t>(quant::kPerTensorMaxPartials, (int64_t)di.sm_count * 4));
  quant::TensorArgs a{x, sxb, sxm, sxn, y, syb, sym, syn, batch, m, n, vec_ok, workspace, amax_grid,
                      quant_scale, dequant_scale, scale_dtype, fp8_max, eps};
  return dispatch_xy(x_dtype, y_dtype, [&](auto xc, auto yc) -> int {
    constexpr int XT = decltype(xc)::value;
    constexpr int YT = decltype(yc)::value;
    quant::tensor_amax_kernel<XT><<<amax_grid, quant::kThreads, 0, s>>>(a);
    int st = check_launch("tensor_amax_kernel");
    if (st != PCB_OK) return st;
    const int cast_grid = (int)std::min<int64_t>(std::max<int64_t>(1, (total + per_cta - 1) / per_cta),
                                                 (int64_t)di.sm_count * 8);
    quant::tensor_cast_kernel<XT, YT><<<cast_grid, quant::kThreads, 0, s>>>(a);
    return check_launch("tensor_cast_kernel");
  });
}

int pcb_quant_float8_dynamic(const void* x, int x_dtype, int64_t batch, int64_t m, int64_t n, int64_t sxb,
                             int64_t sxm, int64_t sxn, void* y, int y_dtype, int64_t syb, int64_t sym, int64_t syn,
                             float* scale, int64_t ssb, int64_t ssm, int axiswise, float eps, float* workspace,
                             void* stream) {
  if (batch < 0 || m < 0 || n < 0) return fail(PCB_ERR_INVALID, "negative size");
  if (axiswise != 0 && axiswise != 1) return fail(PCB_ERR_INVALID, "axiswise must be 0 (tensorwise) or 1 (rows)");
  if (!is_float_in(x_dtype) || !is_fp8(y_dtype)) return fail(PCB_ERR_INVALID, "bad dtype");
  cudaStream_t s = (cudaStream_t)stream;
  const float fp8_max = y_dtype == PCB_DTYPE_E4M3 ? 448.0f : 57344.0f;
  if (axiswise) {
    if (batch * m * n == 0) return PCB_OK;
    if (!x || !y || !scale) return fail(PCB_ERR_INVALID, "null pointer");
    return launch_groups(x, x_dtype, batch, m, n, sxb, sxm, sxn, y, y_dtype, syb, sym, syn, scale, ssb, ssm, 0, 1, n,
                         quant::kQuantDivide, eps, s);
  }
  if (!x || !y || !scale || !workspace) return fail(PCB_ERR_INVALID, "null pointer");
  const DeviceInfo di = device_info();
  const int es = elem_size(x_dtype);
  const int vec = 16 / es;
  const bool vec_ok = sxn == 1 && syn == 1 && n % vec == 0 && aligned(x, 16) && (sxm * es) % 16 == 0 &&
                      (batch == 1 || (sxb * es) % 16 == 0) && aligned(y, vec) && sym % vec == 0 &&
                      (batch == 1 || syb % vec == 0);
  const int64_t total = batch * m * n;
  const int64_t per_cta = (int64_t)quant::kThreads * (vec_ok ? vec : 1);
  const int amax_grid = (int)std::min<int64_t>(std::max<int64_t>(1, (total + per_cta - 1) / per_cta),
                                               std::min<int64_t>((int64_t)di.sm_count * 4, quant::kPerTensorMaxPartials));
  quant::TensorArgs a{x, sxb, sxm, sxn, y, syb, sym, syn, batch, m, n, vec_ok, workspace, amax_grid,
                      scale, nullptr, PCB_DTYPE_F32, fp8_max, eps, 1};
  return dispatch_xy(x_dtype, y_dtype, [&](auto xc, auto yc) -> int {
    constexpr int XT = decltype(xc)::value;
    constexpr int YT = decltype(yc)::value;
    quant::tensor_amax_kernel<XT><<<amax_grid, quant::kThreads, 0, s>>>(a);
    int st = check_launch("tensor_amax_kernel");
    if (st != PCB_OK) return st;
    const int cast_grid = (int)std::min<int64_t>(std::max<int64_t>(1, (total + per_cta - 1) / per_cta),
                                                 (int64_t)di.sm_count * 8);
    quant::tensor_cast_kernel<XT, YT><<<cast_grid, quant::kThreads, 0, s>>>(a);
    return check_launch("tensor_cast_kernel");
  });
}

int pcb_quant_per_tensor_noalloc(const void* x, int x_dtype, int64_t batch, int64_t m, int64_t n, int64_t sxb,
                                 int64_t sxm, int64_t sxn, void* y, int y_dtype, int64_t syb, int64_t sym,
                                 int64_t syn, float* quant_scale, float* dequant_scale, int scale_dtype,
                                 float fp8_max, float eps, void* stream) {
  if (batch < 0 || m < 0 || n < 0) return fail(PCB_ERR_INVALID, "negative size");
  if (!x || !y) return fail(PCB_ERR_INVALID, "null pointer");
  if (!is_float_in(x_dtype) || !is_fp8(y_dtype) || !is_float_in(scale_dtype)) return fail(PCB_ERR_INVALID, "bad dtype");
  float* partials = noalloc_partials_on_current_device();
  if (!partials) return PCB_ERR_DEVICE;
  cudaStream_t s = (cudaStream_t)stream;
  const DeviceInfo di = device_info();
  const int es = elem_size(x_dtype);
  const int vec = 16 / es;
  const bool vec_ok = sxn == 1 && syn == 1 && n % vec == 0 && aligned(x, 16) && (sxm * es) % 16 == 0 &&
                      (batch == 1 || (sxb * es) % 16 == 0) && aligned(y, vec) && sym % vec == 0 &&
                      (batch == 1 || syb % vec == 0);
  const int64_t total = batch * m * n;
  const int64_t per_cta = (int64_t)quant::kThreads * (vec_ok ? vec : 1);
  const int64_t wanted = std::min<int64_t>(std::max<int64_t>(1, (total + per_cta - 1) / per_cta),
                                           (int64_t)di.sm_count * 4);
  if (wanted > kNoAllocPartials)
    return fail(PCB_ERR_INVALID,
                "pcb_quant_per_tensor_noalloc: the launch needs more amax partial slots than the "
                "1024-slot static scratch holds");
  const int amax_grid = (int)wanted;
  // Every partial slot the cast kernel reads (0 .. amax_grid-1) is written by
  // the amax kernel of this same call, so nothing needs clearing first.
  quant::TensorArgs a{x, sxb, sxm, sxn, y, syb, sym, syn, batch, m, n, vec_ok, partials, amax_grid,
                      quant_scale, dequant_scale, scale_dtype, fp8_max, eps};
  return dispatch_xy(x_dtype, y_dtype, [&](auto xc, auto yc) -> int {
    constexpr int XT = decltype(xc)::value;
    constexpr int YT = decltype(yc)::value;
    quant::tensor_amax_kernel<XT><<<amax_grid, quant::kThreads, 0, s>>>(a);
    int st = check_launch("tensor_amax_kernel (noalloc)");
    if (st != PCB_OK) return st;
    const int cast_grid = (int)std::min<int64_t>(std::max<int64_t>(1, (total + per_cta - 1) / per_cta),
                                                 (int64_t)di.sm_count * 8);
    quant::tensor_cast_kernel<XT, YT><<<cast_grid, quant::kThreads, 0, s>>>(a);
    return check_launch("tensor_cast_kernel (noalloc)");
  });
}

int pcb_quant_bmm_fused(const void* x, int x_dtype, int64_t sxb, int64_t sxm, int64_t sxk, const void* b,
                        int64_t sbb, int64_t sbk, int64_t sbn, int b_dtype, int64_t batch, int64_t m, int64_t n,
                        int64_t k, const float* scale_b, int64_t ssbb, int64_t ssbk, int64_t ssbn, int64_t qbn,
                        const void* bias, int bias_dtype, int64_t sbib, int64_t sbim, int64_t sbin, void* c,
                        int c_dtype, int64_t scb, int64_t scm, int64_t scn, void* xq, int64_t sxqb, int64_t sxqm,
                        float* xs, int64_t sxsb, int64_t sxsm, int64_t sxsk, int activation, float eps,
                        void* stream) {
  if (batch < 0 || m < 0 || n < 0 || k < 0) return fail(PCB_ERR_INVALID, "negative size");
  if (x_dtype != PCB_DTYPE_BF16 && x_dtype != PCB_DTYPE_F16) return fail(PCB_ERR_INVALID, "x must be BF16 or F16");
  if (b_dtype != PCB_DTYPE_E4M3) return fail(PCB_ERR_INVALID, "B must be E4M3");
  if (elem_size(c_dtype) == 0) return fail(PCB_ERR_INVALID, "bad output dtype");
  if (bias && !is_float_in(bias_dtype)) return fail(PCB_ERR_INVALID, "bias dtype must be F32/F16/BF16");
  if (activation != PCB_ACT_NONE && activation != PCB_ACT_GELU) return fail(PCB_ERR_INVALID, "bad activation");
  if (qbn <= 0) return fail(PCB_ERR_INVALID, "qbn must be positive");
  if (batch == 0 || m == 0 || n == 0) return PCB_OK;
  if (k == 0) return fail(PCB_ERR_UNSUPPORTED, "K must be positive for the fused path");
  if (!x || !b || !c) return fail(PCB_ERR_INVALID, "null pointer");
  if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX || batch > 65535)
    return fail(PCB_ERR_UNSUPPORTED, "dimension too large");
  if (scn != 1) return fail(PCB_ERR_LAYOUT, "output must be contiguous along N");
  if (sxk != 1 || (sxm * 2) % 16 != 0 || (batch > 1 && (sxb * 2) % 16 != 0) || !aligned(x, 16) || k % 8 != 0)
    return fail(PCB_ERR_LAYOUT, "x must be K-contiguous with 16-byte aligned rows");
  if (xq && (sxqm % 8 != 0 || !aligned(xq, 8))) return fail(PCB_ERR_LAYOUT, "quantized x output rows must be 8-byte aligned");
  const DeviceInfo di = device_info();
  if (di.major != 10) return fail(PCB_ERR_DEVICE, "pcb_quant_bmm_fused needs an sm_100 device");
  bool b_mn;
  if (sbk == 1) {
    b_mn = false;
    if (sbn % 16 != 0) return fail(PCB_ERR_LAYOUT, "K-major B stride must be a multiple of 16 bytes");
  } else if (sbn == 1) {
    b_mn = true;
    if (sbk % 16 != 0) return fail(PCB_ERR_LAYOUT, "N-major B stride must be a multiple of 16 bytes");
  } else {
    return fail(PCB_ERR_LAYOUT, "B must be contiguous along K or N");
  }
  if ((batch > 1 && sbb % 16 != 0) || !aligned(b, 16)) return fail(PCB_ERR_LAYOUT, "B batch stride / base alignment");
  CUtensorMap tx, tb;
  if (!make_map_x16(&tx, x, x_dtype, (uint64_t)k, (uint64_t)m, (uint64_t)batch, (uint64_t)sxm * 2,
                    (uint64_t)sxb * 2))
    return fail(PCB_ERR_LAYOUT, "cuTensorMapEncodeTiled rejected x");
  const bool okB = b_mn ? make_map_u8(&tb, b, (uint64_t)n, (uint64_t)k, (uint64_t)batch, (uint64_t)sbk, (uint64_t)sbb, 128)
                        : make_map_u8(&tb, b, (uint64_t)k, (uint64_t)n, (uint64_t)batch, (uint64_t)sbn, (uint64_t)sbb, 128);
  if (!okB) return fail(PCB_ERR_LAYOUT, "cuTensorMapEncodeTiled rejected B");
  constexpr int bn = gemm::FusedSmem::BN;
  gemm::Params p{};
  p.batch = (int)batch;
  p.m = (int)m;
  p.n = (int)n;
  p.k = (int)k;
  p.m_blocks = (int)((m + gemm::BM - 1) / gemm::BM);
  p.n_blocks = (int)((n + bn - 1) / bn);
  p.num_tiles = (int)(batch * p.m_blocks * p.n_blocks);
  p.k_stages = (int)((k + gemm::BK - 1) / gemm::BK);
  p.stages_per_group = 1;
  p.num_groups = p.k_stages;
  p.sb = scale_b;
  p.ssbb = ssbb;
  p.ssbk = ssbk;
  p.ssbn = ssbn;
  p.qbn = (int)std::min<int64_t>(qbn, INT32_MAX);
  p.col_uniform = (!scale_b || ssbn == 0 || qbn % gemm::FusedSmem::EPI_COLS == 0 || qbn >= n) ? 1 : 0;
  p.c = c;
  p.scb = scb;
  p.scm = scm;
  const int ces = elem_size(c_dtype);
  p.c_dtype = c_dtype;
  p.c_vec = (aligned(c, 16) && (scm * ces) % 16 == 0 && (batch == 1 || (scb * ces) % 16 == 0)) ? 1 : 0;
  p.bias = bias;
  p.sbib = sbib;
  p.sbim = sbim;
  p.sbin = sbin;
  p.bias_dtype = bias_dtype;
  p.activation = activation;
  p.xq = xq;
  p.sxqb = sxqb;
  p.sxqm = sxqm;
  p.xs = xs;
  p.sxsb = sxsb;
  p.sxsm = sxsm;
  p.sxsk = sxsk;
  p.eps = eps;
#ifdef PCB200_PROFILING
  // Profiling builds only: PCB200_BMM_DEBUG (1 epilogue math, 2 MMAs, 8 quantizer work skipped).
  if (const char* dbg = std::getenv("PCB200_BMM_DEBUG")) p.debug_flags = std::atoi(dbg);
#endif
  cudaStream_t s = (cudaStream_t)stream;
  const int sm = di.sm_count;
  if (x_dtype == PCB_DTYPE_BF16) {
    if (b_mn) return p.col_uniform ? launch_fused<true, PCB_DTYPE_BF16, true>(tx, tb, p, sm, s)
                                   : launch_fused<true, PCB_DTYPE_BF16, false>(tx, tb, p, sm, s);
    return p.col_uniform ? launch_fused<false, PCB_DTYPE_BF16, true>(tx, tb, p, sm, s)
                         : launch_fused<false, PCB_DTYPE_BF16, false>(tx, tb, p, sm, s);
  }
  if (b_mn) return p.col_uniform ? launch_fused<true, PCB_DTYPE_F16, true>(tx, tb, p, sm, s)
                                 : launch_fused<true, PCB_DTYPE_F16, false>(tx, tb, p, sm, s);
  return p.col_uniform ? launch_fused<false, PCB_DTYPE_F16, true>(tx, tb, p, sm, s)
                       : launch_fused<false, PCB_DTYPE_F16, false>(tx, tb, p, sm, s);
}

int pcb_pack_u8(const void* src, int64_t batch, int64_t rows, int64_t cols, int64_t ssb, int64_t ssr, int64_t ssc,
                void* dst, int64_t dsb, int64_t dsr, int64_t cols_padded, void* stream) {
  if (batch < 0 || rows < 0 || cols < 0 || cols_padded < cols) return fail(PCB_ERR_INVALID, "bad pack sizes");
  const int64_t total = batch * rows * cols_padded;
  if (total == 0) return PCB_OK;
  if (!src || !dst) return fail(PCB_ERR_INVALID, "null pointer");
  const DeviceInfo di = device_info();
  const int64_t grid = std::min<int64_t>((total + quant::kThreads - 1) / quant::kThreads, (int64_t)di.sm_count * 8);
  quant::pack_u8_kernel<<<(unsigned)grid, quant::kThreads, 0, (cudaStream_t)stream>>>(
      static_cast<const uint8_t*>(src), batch, rows, cols, ssb, ssr, ssc, static_cast<uint8_t*>(dst), dsb, dsr,
      cols_padded);
  return check_launch("pack_u8_kernel");
}

int64_t pcb_bmm_block_scaled_workspace_bytes(int64_t batch, int64_t m, int64_t n, int64_t k) {
  if (batch <= 0 || m <= 0 || n <= 0 || k <= 0) return 0;
  const int64_t k_stages = (k + gemm::BK - 1) / gemm::BK;
  const int64_t m_blocks = (m + gemm::BM - 1) / gemm::BM;
  const int64_t n_blocks128 = 2 * ((n + 255) / 256);
  return 512 * k_stages * batch * (m_blocks + n_blocks128);
}

static int bmm_entry(const void* a, int64_t sab, int64_t sam, int64_t sak, const void* b, int64_t sbb, int64_t sbk,
                   int64_t sbn, int ab_dtype, int b_dtype, int64_t batch, int64_t m, int64_t n, int64_t k,
                   const float* scale_a,
                   int64_t ssab, int64_t ssam, int64_t ssak, int64_t qbm, const float* scale_b, int64_t ssbb,
                   int64_t ssbk, int64_t ssbn, int64_t qbn, int64_t qbk, const void* bias, int bias_dtype,
                   int64_t sbib, int64_t sbim, int64_t sbin, void* c, int c_dtype, int64_t scb, int64_t scm,
                   int64_t scn, int activation, void* stream, bool block_scaled, void* workspace = nullptr,
                     int64_t workspace_bytes = 0) {
  if (batch < 0 || m < 0 || n < 0 || k < 0) return fail(PCB_ERR_INVALID, "negative size");
  // ab_dtype is A's format; B's is b_dtype (the same unless the mixed entry point is used).
  if (!is_fp8(ab_dtype) || !is_fp8(b_dtype)) return fail(PCB_ERR_INVALID, "A/B dtype must be E4M3 or E5M2");
  if (block_scaled && ab_dtype != b_dtype) return fail(PCB_ERR_UNSUPPORTED, "block-scaled bmm needs one fp8 format");
  if (elem_size(c_dtype) == 0) return fail(PCB_ERR_INVALID, "bad output dtype");
  if (bias && !is_float_in(bias_dtype)) return fail(PCB_ERR_INVALID, "bias dtype must be F32/F16/BF16");
  if (activation != PCB_ACT_NONE && activation != PCB_ACT_GELU) return fail(PCB_ERR_INVALID, "bad activation");
  if (qbm <= 0 || qbn <= 0 || qbk <= 0) return fail(PCB_ERR_INVALID, "quant block sizes must be positive");
  if (batch == 0 || m == 0 || n == 0) return PCB_OK;
  if (!c || (k > 0 && (!a || !b))) return fail(PCB_ERR_INVALID, "null pointer");
  if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX || batch > 65535)
    return fail(PCB_ERR_UNSUPPORTED, "dimension too large");
  if (scn != 1) return fail(PCB_ERR_LAYOUT, "output must be contiguous along N");
  const DeviceInfo di = device_info();
  if (di.major != 10) return fail(PCB_ERR_DEVICE, "pcb_bmm_scaled needs an sm_100 device");

  const int64_t k_stages = (k + gemm::BK - 1) / gemm::BK;
  int64_t spg;
  if (qbk >= k) {
    spg = std::max<int64_t>(1, k_stages);
  } else {
    if (qbk % gemm::BK != 0) return fail(PCB_ERR_UNSUPPORTED, "qbk must be a multiple of 128 or >= K");
    spg = qbk / gemm::BK;
  }

  // Operand layouts (bytes == elements for fp8).
  bool a_mn = false, b_mn = false;
  CUtensorMap ta, tb;
  // 128x256 tiles (128x128 when N <= 128): 32 KB of fp8 operands per
  // 128-deep K stage feed 8.4 MFLOP, which keeps L2 traffic per FLOP low.
  const int bn = (block_scaled || n > 128) ? 256 : 128;
  if (block_scaled) {
    if (!scale_a || !scale_b) return fail(PCB_ERR_INVALID, "block-scaled bmm needs both scale tensors");
    if (qbk != gemm::BK) return fail(PCB_ERR_UNSUPPORTED, "block-scaled bmm needs qbk == 128");
  }
  // 256x256 tiles on a CTA pair (cta_group::2) whenever M spans two 128-row
  // halves: each CTA stages its own 128 A rows and half of the B tile, so an
  // SM moves 32 KB of operands per 128-deep K stage instead of 48 KB.  Per-K-
  // group promotion runs on both CTAs' epilogues, which hand each TMEM
  // accumulator back to the leader's MMA issuer.
  bool pair = !block_scaled && bn == 256 && m > 128;
#ifdef PCB200_PROFILING
  // Profiling builds only: PCB200_BMM_PAIR=0 keeps every tile on one CTA.
  if (const char* e = std::getenv("PCB200_BMM_PAIR")) pair = pair && std::atoi(e) != 0;
#endif
  if (k == 0) {
    // No K stages: the kernel only writes bias/zeros; the maps are never read.
    std::memset(&ta, 0, sizeof(ta));
    std::memset(&tb, 0, sizeof(tb));
  } else {
  if (sak == 1) {
    a_mn = false;
    if (sam % 16 != 0) return fail(PCB_ERR_LAYOUT, "K-major A row stride must be a multiple of 16 bytes");
  } else if (sam == 1) {
    a_mn = true;
    if (sak % 16 != 0) return fail(PCB_ERR_LAYOUT, "M-major A stride must be a multiple of 16 bytes");
  } else {
    return fail(PCB_ERR_LAYOUT, "A must be contiguous along K or M");
  }
  if (sbk == 1) {
    b_mn = false;
    if (sbn % 16 != 0) return fail(PCB_ERR_LAYOUT, "K-major B stride must be a multiple of 16 bytes");
  } else if (sbn == 1) {
    b_mn = true;
    if (sbk % 16 != 0) return fail(PCB_ERR_LAYOUT, "N-major B stride must be a multiple of 16 bytes");
  } else {
    return fail(PCB_ERR_LAYOUT, "B must be contiguous along K or N");
  }
  if (batch > 1 && (sab % 16 != 0 || sbb % 16 != 0)) return fail(PCB_ERR_LAYOUT, "batch strides must be multiples of 16 bytes");
  if (k > 0 && (!aligned(a, 16) || !aligned(b, 16))) return fail(PCB_ERR_LAYOUT, "A/B must be 16-byte aligned");

  const uint64_t kk = (uint64_t)k;
  bool okA = a_mn ? make_map_u8(&ta, a, (uint64_t)m, kk, (uint64_t)batch, (uint64_t)sak, (uint64_t)sab, 128)
                  : make_map_u8(&ta, a, kk, (uint64_t)m, (uint64_t)batch, (uint64_t)sam, (uint64_t)sab, 128);
  bool okB = b_mn ? make_map_u8(&tb, b, (uint64_t)n, kk, (uint64_t)batch, (uint64_t)sbk, (uint64_t)sbb, 128)
                  : make_map_u8(&tb, b, kk, (uint64_t)n, (uint64_t)batch, (uint64_t)sbn, (uint64_t)sbb,
                                (uint32_t)(pair ? bn / 2 : bn));
  if (!okA || !okB) return fail(PCB_ERR_LAYOUT, "cuTensorMapEncodeTiled rejected the operand layout");
  }
  // Each epilogue thread holds BN/2 fp32 accumulators of its row.
  const int epi_cols = bn / 2;

  gemm::Params p{};
  p.batch = (int)batch;
  p.m = (int)m;
  p.n = (int)n;
  p.k = (int)k;
  const int tile_m = pair ? 2 * gemm::BM : gemm::BM;
  p.m_blocks = (int)((m + tile_m - 1) / tile_m);
  p.n_blocks = (int)((n + bn - 1) / bn);
  p.num_tiles = (int)(batch * p.m_blocks * p.n_blocks);
  p.k_stages = (int)k_stages;
  p.stages_per_group = (int)spg;
  p.num_groups = (int)((k_stages + spg - 1) / spg);
  p.sa = scale_a;
  p.ssab = ssab;
  p.ssam = ssam;
  p.ssak = ssak;
  p.qbm = (int)std::min<int64_t>(qbm, INT32_MAX);
  p.sb = scale_b;
  p.ssbb = ssbb;
  p.ssbk = ssbk;
  p.ssbn = ssbn;
  p.qbn = (int)std::min<int64_t>(qbn, INT32_MAX);
  p.col_uniform = (!scale_b || ssbn == 0 || qbn % epi_cols == 0 || qbn >= n) ? 1 : 0;
  p.sa_vec = (scale_a && aligned(scale_a, 16) && (batch == 1 || ssab % 4 == 0) && qbm == 1 && ssam == 1 &&
              ssak % 4 == 0) ? 2 : 0;
  p.sb_vec = (scale_b && aligned(scale_b, 16) && (batch == 1 || ssbb % 4 == 0) && qbn == 1 && ssbn == 1 &&
              ssbk % 4 == 0) ? 1 : 0;
  p.c = c;
  p.scb = scb;
  p.scm = scm;
  const int ces = elem_size(c_dtype);
  p.c_dtype = c_dtype;
  p.c_vec = (aligned(c, 16) && (scm * ces) % 16 == 0 && (batch == 1 || (scb * ces) % 16 == 0)) ? 1 : 0;
  p.bias = bias;
  p.sbib = sbib;
  p.sbim = sbim;
  p.sbin = sbin;
  p.bias_dtype = bias_dtype;
  p.activation = activation;
  p.inject_error = g_inject_error.exchange(0);
#ifdef PCB200_PROFILING
  // Profiling builds only: PCB200_BMM_DEBUG=1 skips the epilogue math, =2
  // skips the MMAs; results are then meaningless.
  if (const char* dbg = std::getenv("PCB200_BMM_DEBUG")) p.debug_flags = std::atoi(dbg);
#endif
  const int fmt = (ab_dtype == PCB_DTYPE_E4M3) ? 0 : 1;
  p.a_fmt = fmt;
  p.b_fmt = (b_dtype == PCB_DTYPE_E4M3) ? 0 : 1;
  cudaStream_t s = (cudaStream_t)stream;
  if (block_scaled) {
    if (k == 0) return fail(PCB_ERR_UNSUPPORTED, "block-scaled bmm needs K > 0");
    const int64_t need = pcb_bmm_block_scaled_workspace_bytes(batch, m, n, k);
    if (!workspace || workspace_bytes < need) return fail(PCB_ERR_INVALID, "block-scaled bmm workspace too small");
    if (!aligned(workspace, 16)) return fail(PCB_ERR_INVALID, "block-scaled bmm workspace must be 16-byte aligned");
    uint4* sfa = static_cast<uint4*>(workspace);
    uint4* sfb = sfa + (int64_t)batch * p.m_blocks * p.k_stages * 32;
    gemm::PackSfArgs pa{scale_a, ssab, ssam, ssak, p.qbm, (int)m, p.m_blocks, p.k_stages, (int)batch, sfa};
    gemm::PackSfArgs pb{scale_b, ssbb, ssbn, ssbk, p.qbn, (int)n, 2 * p.n_blocks, p.k_stages, (int)batch, sfb};
    for (const gemm::PackSfArgs& pk : {pa, pb}) {
      const int64_t lines = (int64_t)pk.batch * pk.row_blocks * pk.k_stages * 32;
      const unsigned grid = (unsigned)std::min<int64_t>((lines + 255) / 256, (int64_t)di.sm_count * 8);
      gemm::pack_sf_kernel<<<grid, 256, 0, s>>>(pk);
      if (int st = check_launch("pack_sf_kernel")) return st;
    }
    p.sfa = sfa;
    p.sfb = sfb;
    return dispatch_bmm_bs(a_mn, b_mn, fmt, ta, tb, p, di.sm_count, s);
  }
  // On the CTA pair, bf16 / fp16 C leaves through TMA stores of swizzled
  // 32 x 64 boxes staged in shared memory (per-thread row stores stall the
  // epilogue, and with it the MMA, for thousands of cycles per tile).
  CUtensorMap tc;
  std::memset(&tc, 0, sizeof(tc));
  if (pair && (c_dtype == PCB_DTYPE_BF16 || c_dtype == PCB_DTYPE_F16 || c_dtype == PCB_DTYPE_F32) && p.c_vec)
    p.c_tma = make_map_c(&tc, c, c_dtype, (uint64_t)n, (uint64_t)m, (uint64_t)batch, (uint64_t)(scm * ces),
                           (uint64_t)(scb * ces)) ? 1 : 0;
  if (pair) return dispatch_bmm_layout<256, true>(a_mn, b_mn, ta, tb, tc, p, di.sm_count, s);
  if (bn == 256) return dispatch_bmm_layout<256, false>(a_mn, b_mn, ta, tb, tc, p, di.sm_count, s);
  return dispatch_bmm_layout<128, false>(a_mn, b_mn, ta, tb, tc, p, di.sm_count, s);
}
int pcb_bmm_scaled(const void* a, int64_t sab, int64_t sam, int64_t sak, const void* b, int64_t sbb, int64_t sbk,
                   int64_t sbn, int ab_dtype, int64_t batch, int64_t m, int64_t n, int64_t k, const float* scale_a,
                   int64_t ssab, int64_t ssam, int64_t ssak, int64_t qbm, const float* scale_b, int64_t ssbb,
                   int64_t ssbk, int64_t ssbn, int64_t qbn, int64_t qbk, const void* bias, int bias_dtype,
                   int64_t sbib, int64_t sbim, int64_t sbin, void* c, int c_dtype, int64_t scb, int64_t scm,
                   int64_t scn, int activation, void* stream) {
  return bmm_entry(a, sab, sam, sak, b, sbb, sbk, sbn, ab_dtype, ab_dtype, batch, m, n, k, scale_a, ssab, ssam, ssak,
                   qbm, scale_b, ssbb, ssbk, ssbn, qbn, qbk, bias, bias_dtype, sbib, sbim, sbin, c, c_dtype, scb, scm,
                   scn, activation, stream, false);
}

int pcb_bmm_scaled_mixed(const void* a, int64_t sab, int64_t sam, int64_t sak, int a_dtype, const void* b,
                         int64_t sbb, int64_t sbk, int64_t sbn, int b_dtype, int64_t batch, int64_t m, int64_t n,
                         int64_t k, const float* scale_a, int64_t ssab, int64_t ssam, int64_t ssak, int64_t qbm,
                         const float* scale_b, int64_t ssbb, int64_t ssbk, int64_t ssbn, int64_t qbn, int64_t qbk,
                         const void* bias, int bias_dtype, int64_t sbib, int64_t sbim, int64_t sbin, void* c,
                         int c_dtype, int64_t scb, int64_t scm, int64_t scn, int activation, void* stream) {
  return bmm_entry(a, sab, sam, sak, b, sbb, sbk, sbn, a_dtype, b_dtype, batch, m, n, k, scale_a, ssab, ssam, ssak,
                   qbm, scale_b, ssbb, ssbk, ssbn, qbn, qbk, bias, bias_dtype, sbib, sbim, sbin, c, c_dtype, scb, scm,
                   scn, activation, stream, false);
}

int pcb_bmm_block_scaled(const void* a, int64_t sab, int64_t sam, int64_t sak, const void* b, int64_t sbb, int64_t sbk,
                         int64_t sbn, int ab_dtype, int64_t batch, int64_t m, int64_t n, int64_t k, const float* scale_a,
                         int64_t ssab, int64_t ssam, int64_t ssak, int64_t qbm, const float* scale_b, int64_t ssbb,
                         int64_t ssbk, int64_t ssbn, int64_t qbn, int64_t qbk, const void* bias, int bias_dtype,
                         int64_t sbib, int64_t sbim, int64_t sbin, void* c, int c_dtype, int64_t scb, int64_t scm,
                         int64_t scn, int activation, void* workspace,
                         int64_t workspace_bytes, void* stream) {
  return bmm_entry(a, sab, sam, sak, b, sbb, sbk, sbn, ab_dtype, ab_dtype, batch, m, n, k, scale_a, ssab, ssam, ssak,
                   qbm, scale_b, ssbb, ssbk, ssbn, qbn, qbk, bias, bias_dtype, sbib, sbim, sbin, c, c_dtype, scb, scm,
                   scn, activation, stream, true, workspace, workspace_bytes);
}


#ifdef PCB_GEMM_TRACE
// Trace builds only: copy CTA 0's cycle stamps (16 x 1024 long long) to host.
int pcb_trace_read(long long* host) {
  return cudaMemcpyFromSymbol(host, gemm::g_gemm_trace, sizeof(gemm::g_gemm_trace)) == cudaSuccess ? PCB_OK
                                                                                                   : PCB_ERR_DEVICE;
}
#endif

}  // extern "C"
