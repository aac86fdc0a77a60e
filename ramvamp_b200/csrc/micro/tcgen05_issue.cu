// Microbenchmark: how fast one thread can issue tcgen05.mma (kind::f16,
// M = 128, K = 16, f32 accumulator in tensor memory) for N = 16..256, and
// what a stage's commit / wait / fence adds; and the int8 rate (kind::i8,
// signed 8-bit A and B, s32 accumulator, K = 32 per instruction) that the
// tensor-peak roofline of an int8 design would use.  This is the rate that bounds
// the tensor-core prefill path when an expert holds few tokens.
// Modes: back-to-back MMAs; commit + wait after every 4; two commits per 4
// (one per ring, as the GEMM's MMA thread does); two commits, two waits on
// completed barriers and a fence per 4.  Operands are constant f16 data in
// shared memory; results are not read.  Every wait is bounded.
//   make -C ramvamp_b200/csrc micro && ramvamp_b200/csrc/micro/bin/tcgen05_issue
#include <cstdio>
#include <cstdint>
#include <cuda_runtime.h>
__device__ __forceinline__ uint32_t sa(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
template <bool I8>
__global__ void k(int n, int reps, int mode, long long *out) {
  extern __shared__ __align__(1024) uint8_t sm[];
  __shared__ uint32_t tm;
  __shared__ __align__(8) uint64_t bar, bar2[2], bar3;
  const int warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < 64 * 1024 / 4; i += blockDim.x) ((uint32_t *)sm)[i] = 0x3c003c00u;
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sa(&bar)));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 100000;" ::"r"(sa(&bar2[0])));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 100000;" ::"r"(sa(&bar2[1])));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sa(&bar3)));
    asm volatile("fence.mbarrier_init.release.cluster;");
  }
  asm volatile("fence.proxy.async.shared::cta;");
  __syncwarp();
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(sa(&tm)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t t = tm;
  if (threadIdx.x == 0) {
    // c_format bits [4,6): F32 = 1 / S32 = 2; a/b format bits [7,10) and
    // [10,13): F16 = 0 / signed 8-bit = 1; N >> 3 at bit 17; M >> 4 at bit 24.
    const uint32_t idesc = (I8 ? (2u << 4) | (1u << 7) | (1u << 10) : (1u << 4)) | ((uint32_t)(n >> 3) << 17) |
                           (8u << 24);
    const uint32_t lo = (8u << 16) | (sa(sm) >> 4), hi = 64u | (1u << 14);
    uint32_t ph = 0;
    long long t0 = clock64();
    for (int r = 0; r < reps; r++) {
      for (int kk = 0; kk < 4; kk++) {
        const uint64_t a = ((uint64_t)hi << 32) | (lo + 16 * kk), b = ((uint64_t)hi << 32) | (lo + 1024 + 16 * kk);
        if constexpr (I8)
          asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n"
                       ::"r"(t), "l"(a), "l"(b), "r"(idesc), "r"(1) : "memory");
        else
          asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
                       ::"r"(t), "l"(a), "l"(b), "r"(idesc), "r"(1) : "memory");
      }
      if (mode >= 2) {
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(sa(&bar2[0])) : "memory");
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(sa(&bar2[1])) : "memory");
      }
      if (mode == 3) {
        // waits on barriers that are already complete (count 0 phases), plus the fence
        uint32_t ok;
        asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n" : "=r"(ok) : "r"(sa(&bar3)), "r"(1u) : "memory");
        asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n" : "=r"(ok) : "r"(sa(&bar3)), "r"(1u) : "memory");
        asm volatile("tcgen05.fence::after_thread_sync;");
        if (!ok) out[1] = 1;
      }
      if (mode == 1) {
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(sa(&bar)) : "memory");
        uint32_t ok = 0;
        long long w0 = clock64();
        while (!ok && clock64() - w0 < 100000000LL) {
          asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n" : "=r"(ok) : "r"(sa(&bar)), "r"(ph) : "memory");
        }
        ph ^= 1;
      }
    }
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(sa(&bar)) : "memory");
    uint32_t ok = 0;
    long long w0 = clock64();
    while (!ok && clock64() - w0 < 100000000LL) {
      asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n" : "=r"(ok) : "r"(sa(&bar)), "r"(ph) : "memory");
    }
    out[blockIdx.x] = clock64() - t0;
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(t));
  }
}
int main() {
  long long *out;
  cudaMalloc(&out, 1024 * 8);
  cudaFuncSetAttribute(k<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
  cudaFuncSetAttribute(k<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
  for (int mode = 0; mode < 4; mode++)
    for (int n : {16, 32, 64, 128, 256}) {
      const int reps = 256;
      k<false><<<1, 128, 64 * 1024>>>(n, reps, mode, out);
      long long c;
      cudaMemcpy(&c, out, 8, cudaMemcpyDeviceToHost);
      const double per = (double)c / (reps * 4);
      printf("f16  mode %s N=%3d: %.1f cycles per MMA (128x%dx16), %.0f MAC/clk\n", mode == 0 ? "back-to-back " : mode == 1 ? "commit+wait/4" : mode == 2 ? "2 commits/4  " : "2cm+2wait+f/4", n, per, n,
             128.0 * n * 16 / per);
    }
  int sms = 0, clk_khz = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  cudaDeviceGetAttribute(&clk_khz, cudaDevAttrClockRate, 0);
  for (int n : {64, 128, 256}) {
    const int reps = 256;
    k<true><<<1, 128, 64 * 1024>>>(n, reps, 0, out);
    long long c;
    cudaMemcpy(&c, out, 8, cudaMemcpyDeviceToHost);
    const double per = (double)c / (reps * 4), mac = 128.0 * n * 32 / per;
    printf("i8   back-to-back N=%3d: %.1f cycles per MMA (128x%dx32), %.0f MAC/clk per SM = %.2f POPS at %d SMs x %.0f MHz\n",
           n, per, n, mac, 2.0 * mac * sms * clk_khz * 1e3 / 1e15, sms, clk_khz / 1e3);
  }
  printf("status: %s\n", cudaGetErrorString(cudaDeviceSynchronize()));
  return 0;
}
