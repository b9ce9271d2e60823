// Diagnostic microbenchmark (not part of libpcb200): cycle cost of mbarrier waits and tcgen05.commit for one thread.
#include <cstdio>
#include <cstdint>
#include <cuda_runtime.h>
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__global__ void k(long long* out) {
  __shared__ __align__(8) uint64_t bar[4];
  __shared__ uint32_t tslot;
  __shared__ volatile int flag;
  const uint32_t b0 = smem_u32(&bar[0]);
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(b0), "r"(1) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    flag = 1;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tslot)), "r"(32) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // complete phase 0
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(b0) : "memory");
    long long t0 = clock64();
    uint32_t ok = 0, acc = 0;
    for (int i = 0; i < 1000; ++i) {
      asm volatile("{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}" : "=r"(ok) : "r"(b0), "r"(0) : "memory");
      acc += ok;
    }
    long long t1 = clock64();
    for (int i = 0; i < 1000; ++i) {
      asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}" : "=r"(ok) : "r"(b0), "r"(0) : "memory");
      acc += ok;
    }
    long long t2 = clock64();
    for (int i = 0; i < 1000; ++i) { acc += flag; }
    long long t3 = clock64();
    for (int i = 0; i < 1000; ++i) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    }
    long long t4 = clock64();
    // commit + wait on a fresh barrier per iteration (arrive count 1)
    const uint32_t b1 = smem_u32(&bar[1]);
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(b1), "r"(1) : "memory");
    uint32_t ph = 0;
    long long t5 = clock64();
    for (int i = 0; i < 1000; ++i) {
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(b1) : "memory");
      long long guard = 0;
      do {
        asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}" : "=r"(ok) : "r"(b1), "r"(ph) : "memory");
      } while (!ok && ++guard < 100000000LL);
      ph ^= 1;
    }
    long long t6 = clock64();
    for (int i = 0; i < 1000; ++i) {
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(b1) : "memory");
    }
    long long t7 = clock64();
    out[0] = t1 - t0; out[1] = t2 - t1; out[2] = t3 - t2; out[3] = t4 - t3; out[4] = t6 - t5; out[5] = t7 - t6; out[6] = acc;
  }
  __syncthreads();
  if (threadIdx.x < 32) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tslot), "r"(32) : "memory");
}
int main() {
  long long* d; cudaMalloc(&d, 64); long long h[8] = {};
  k<<<1, 128>>>(d); cudaError_t e = cudaDeviceSynchronize();
  cudaMemcpy(h, d, 64, cudaMemcpyDeviceToHost);
  printf("err=%s per-iteration cycles: test_wait(done)=%.1f try_wait(done)=%.1f volatile smem ld=%.1f tcgen05.fence=%.1f commit+wait=%.1f commit only=%.1f\n",
         cudaGetErrorString(e), h[0]/1000.0, h[1]/1000.0, h[2]/1000.0, h[3]/1000.0, h[4]/1000.0, h[5]/1000.0);
  return 0;
}
