// Microbenchmark: time for one kernel to stream a decode layer's worth of
// expert bytes (14 MB) that are cold in L2 (windows drawn from a 2 GB
// buffer), with 1-D bulk copies (cp.async.bulk into shared memory on an
// mbarrier; one or many copies per CTA) and with plain 128-bit loads.  The
// floor it shows (~12 us per cold 14 MB launch) bounds the decode expert
// kernels.  Every wait is bounded.
//   make -C ramvamp_b200/csrc micro && ramvamp_b200/csrc/micro/bin/hbm_stream
#include <cstdio>
#include <cstdint>
#include <cuda_runtime.h>

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t c) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(c) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void expect_tx(uint64_t *bar, uint32_t b) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(b) : "memory");
}
__device__ __forceinline__ void bulk(void *dst, const void *src, uint32_t b, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(dst)), "l"(src), "r"(b), "r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool try_wait(uint64_t *bar, uint32_t ph) {
  uint32_t ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0,1,0,p;\n}\n"
               : "=r"(ok) : "r"(smem_addr(bar)), "r"(ph) : "memory");
  return ok;
}

// chunk = bytes per copy, ncopy copies per CTA
__global__ void k_bulk(const uint8_t *src, size_t cta_bytes, int chunk, unsigned *sink) {
  extern __shared__ __align__(16) uint8_t sm[];
  uint64_t *bar = (uint64_t *)sm;
  uint8_t *buf = sm + 16;
  const uint8_t *s = src + (size_t)blockIdx.x * cta_bytes;
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    expect_tx(bar, (uint32_t)cta_bytes);
    for (size_t o = 0; o < cta_bytes; o += chunk) bulk(buf + o, s + o, chunk, bar);
  }
  __syncthreads();
  long long t0 = clock64();
  while (!try_wait(bar, 0)) {
    if (clock64() - t0 > 2000000000LL) break;
  }
  unsigned acc = 0;
  for (size_t i = threadIdx.x * 4; i < cta_bytes; i += blockDim.x * 4) acc ^= *(const unsigned *)(buf + i);
  if (acc == 0x12345678u) sink[0] = acc;
}

__global__ void k_ldg(const uint4 *src, size_t cta_bytes, unsigned *sink) {
  const uint4 *s = src + (size_t)blockIdx.x * (cta_bytes / 16);
  unsigned acc = 0;
  for (size_t i = threadIdx.x; i < cta_bytes / 16; i += blockDim.x) {
    uint4 v = __ldg(s + i);
    acc ^= v.x ^ v.y ^ v.z ^ v.w;
  }
  if (acc == 0x12345678u) sink[0] = acc;
}

int main() {
  const size_t total = 2ull << 30, work = 14155776;
  uint8_t *buf;
  unsigned *sink;
  cudaMalloc(&buf, total);
  cudaMalloc(&sink, 64);
  cudaMemset(buf, 1, total);
  cudaFuncSetAttribute(k_bulk, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  struct Cfg { const char *name; int mode; size_t cta_bytes; int chunk; int threads; };
  Cfg cfgs[] = {
      {"bulk 18432B/CTA as 16x1152", 0, 18432, 1152, 64},
      {"bulk 18432B/CTA as 1x18432", 0, 18432, 18432, 64},
      {"bulk 73728B/CTA as 64x1152", 0, 73728, 1152, 256},
      {"bulk 73728B/CTA as 4x18432", 0, 73728, 18432, 256},
      {"bulk 36864B/CTA as 2x18432", 0, 36864, 18432, 128},
      {"bulk 5040B/CTA 1 copy", 0, 5040, 5040, 32},
      {"ldg 18432B/CTA 64 thr", 1, 18432, 0, 64},
      {"ldg 18432B/CTA 256 thr", 1, 18432, 0, 256},
      {"ldg 73728B/CTA 256 thr", 1, 73728, 0, 256},
      {"ldg 98304B/CTA 512 thr", 1, 98304, 0, 512},
  };
  for (auto &c : cfgs) {
    const int ctas = (int)(work / c.cta_bytes);
    float best = 1e9, sum = 0;
    int reps = 20;
    for (int r = 0; r < reps; r++) {
      const uint8_t *src = buf + ((size_t)(r * 97 % 120) * (16 << 20));  // 16 MB-spaced windows
      cudaEventRecord(a);
      if (c.mode == 0)
        k_bulk<<<ctas, c.threads, c.cta_bytes + 16>>>(src, c.cta_bytes, c.chunk, sink);
      else
        k_ldg<<<ctas, c.threads>>>((const uint4 *)src, c.cta_bytes, sink);
      cudaEventRecord(b);
      cudaEventSynchronize(b);
      float ms;
      cudaEventElapsedTime(&ms, a, b);
      if (r >= 3) { best = ms < best ? ms : best; sum += ms; }
    }
    const double bytes = (double)ctas * c.cta_bytes;
    printf("%-32s ctas=%5d  best %.2f us (%.0f GB/s)  mean %.2f us\n", c.name, ctas, best * 1e3,
           bytes / (best * 1e-3) / 1e9, sum / (reps - 3) * 1e3);
  }
  cudaError_t e = cudaGetLastError();
  printf("status: %s\n", cudaGetErrorString(e));
  return 0;
}
