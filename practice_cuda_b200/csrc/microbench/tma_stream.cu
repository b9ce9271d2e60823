// Diagnostic microbenchmark (not part of libpcb200): per-SM TMA streaming throughput for operand-tile box shapes.
// One CTA per SM, a ring of S stages; thread 0 issues loads, thread 32 waits
// "full" and hands the stage back immediately (no consumer work).
#include <cudaTypedefs.h>
#include <cstdio>
#include <cstdint>
#include <vector>
#include <cuda_runtime.h>
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ bool try_wait(uint32_t bar, uint32_t ph) {
  uint32_t ok;
  asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}" : "=r"(ok) : "r"(bar), "r"(ph) : "memory");
  return ok;
}
struct Args { int mode; int stages; int stage_bytes; int iters; int rows; int kchunks; int batch; };
__global__ void __launch_bounds__(64, 1) k(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, Args a, long long* out) {
  extern __shared__ __align__(1024) uint8_t sm[];
  __shared__ __align__(8) uint64_t full[8], empty[8];
  uint8_t* s = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(s);
  if (threadIdx.x == 0) {
    for (int i = 0; i < a.stages; ++i) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&full[i])) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&empty[i])) : "memory");
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  long long t0 = clock64();
  if (threadIdx.x == 0) {
    int st = 0; uint32_t ph = 0;
    for (int it = 0; it < a.iters; ++it) {
      long long g = 0;
      while (!try_wait(smem_u32(&empty[st]), ph ^ 1) && ++g < 100000000LL) {}
      const uint32_t fb = smem_u32(&full[st]);
      const uint32_t dst = sb + st * a.stage_bytes;
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(fb), "r"(a.stage_bytes) : "memory");
      // walk K for this CTA's row block; wrap inside the tensor
      const int kc = (it * (a.mode == 1 || a.mode == 3 ? 2 : 1)) % a.kchunks;
      const int row = (blockIdx.x % 16) * 128;
      const int bz = (blockIdx.x / 16) % a.batch;
      if (a.mode == 0) {  // A-like 3D box (128 K bytes, 128 rows) + B-like 3D box (128 N, 128 K rows)
        asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
                     ::"r"(dst), "l"(&ta), "r"(fb), "r"(kc * 128), "r"(row), "r"(bz) : "memory");
        asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
                     ::"r"(dst + 16384), "l"(&tb), "r"(fb), "r"((blockIdx.x % 8) * 256), "r"(kc * 128), "r"(bz) : "memory");
      } else if (a.mode == 1) {  // 2 K-chunks per box: A 4D (128, 128, 2), B 3D (128 N, 256 K rows)
        asm volatile("cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];"
                     ::"r"(dst), "l"(&ta), "r"(fb), "r"(0), "r"(row), "r"(kc), "r"(bz) : "memory");
        asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
                     ::"r"(dst + 32768), "l"(&tb), "r"(fb), "r"((blockIdx.x % 8) * 256), "r"(kc * 128), "r"(bz) : "memory");
      } else if (a.mode == 2) {  // A only, 3D
        asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
                     ::"r"(dst), "l"(&ta), "r"(fb), "r"(kc * 128), "r"(row), "r"(bz) : "memory");
      } else {  // B only, 256 K rows
        asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
                     ::"r"(dst), "l"(&tb), "r"(fb), "r"((blockIdx.x % 8) * 256), "r"(kc * 128), "r"(bz) : "memory");
      }
      if (++st == a.stages) { st = 0; ph ^= 1; }
    }
  } else if (threadIdx.x == 32) {
    int st = 0; uint32_t ph = 0;
    for (int it = 0; it < a.iters; ++it) {
      long long g = 0;
      while (!try_wait(smem_u32(&full[st]), ph) && ++g < 100000000LL) {}
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&empty[st])) : "memory");
      if (++st == a.stages) { st = 0; ph ^= 1; }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) out[blockIdx.x] = clock64() - t0;
}
int main() {
  PFN_cuTensorMapEncodeTiled_v12000 enc; cudaDriverEntryPointQueryResult q;
  cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", (void**)&enc, cudaEnableDefault, &q);
  const int B = 4, M = 4096, K = 7168, N = 2048;
  uint8_t *A, *Bm; cudaMalloc(&A, (size_t)B * M * K); cudaMalloc(&Bm, (size_t)B * K * N);
  cudaMemset(A, 0x38, (size_t)B * M * K); cudaMemset(Bm, 0x38, (size_t)B * K * N);
  long long* d; cudaMalloc(&d, 148 * 8);
  int sms; cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  for (int mode = 0; mode < 4; ++mode) {
    CUtensorMap ta, tb;
    cuuint32_t e3[3] = {1, 1, 1}, e4[4] = {1, 1, 1, 1};
    if (mode == 1) {
      cuuint64_t dims[4] = {128, (cuuint64_t)M, (cuuint64_t)K / 128, (cuuint64_t)B};
      cuuint64_t str[3] = {(cuuint64_t)K, 128, (cuuint64_t)M * K};
      cuuint32_t box[4] = {128, 128, 2, 1};
      CUresult r = enc(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, A, dims, str, box, e4, CU_TENSOR_MAP_INTERLEAVE_NONE,
                       CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r != CUDA_SUCCESS) { printf("4d map failed %d\n", (int)r); continue; }
    } else {
      cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)M, (cuuint64_t)B};
      cuuint64_t str[2] = {(cuuint64_t)K, (cuuint64_t)M * K};
      cuuint32_t box[3] = {128, 128, 1};
      enc(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, A, dims, str, box, e3, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    {
      cuuint64_t dims[3] = {(cuuint64_t)N, (cuuint64_t)K, (cuuint64_t)B};
      cuuint64_t str[2] = {(cuuint64_t)N, (cuuint64_t)K * N};
      cuuint32_t box[3] = {128, (cuuint32_t)((mode == 1 || mode == 3) ? 256 : 128), 1};
      enc(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, Bm, dims, str, box, e3, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    const int stage_bytes = mode == 0 ? 32768 : mode == 1 ? 65536 : mode == 2 ? 16384 : 32768;
    for (int stages : {2, 3, 6}) {
      if (stages * stage_bytes > 196608) continue;
      Args a{mode, stages, stage_bytes, 2000, M, K / 128, B};
      a.iters = 64 * 1024 * 1024 / stage_bytes;
      k<<<sms, 64, stages * stage_bytes + 1024>>>(ta, tb, a, d);
      cudaError_t e = cudaDeviceSynchronize();
      std::vector<long long> h(sms); cudaMemcpy(h.data(), d, sms * 8, cudaMemcpyDeviceToHost);
      long long mx = 0; for (auto v : h) mx = v > mx ? v : mx;
      printf("mode=%d stages=%d stage_kb=%d err=%s bytes/clk/SM=%.1f\n", mode, stages, stage_bytes / 1024,
             cudaGetErrorString(e), (double)a.iters * stage_bytes / mx);
    }
  }
  return 0;
}
