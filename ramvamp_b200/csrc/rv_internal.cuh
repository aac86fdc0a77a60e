// rv_internal.cuh -- shared device/host helpers of the ramvamp_b200 library.
//
// Everything here is sm_100a code: 32-wide warps, cp.async.bulk (the TMA
// engine's 1-D bulk copy) into shared memory completed on an mbarrier, and
// IEEE-exact intrinsics (__fmul_rn, __fadd_rn, __fmaf_rn, __fdiv_rn,
// __dadd_rn, ...) wherever the reference's float order must be reproduced.
// The library is built without --use_fast_math.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "../../include/ramvamp_b200.h"

#define RV_DEVFN __device__ __forceinline__
#define RV_FULL 0xffffffffu

// ----------------------------------------------------------------- errors
// Thread-local detail of the last failure (rv_last_error).
void rv_set_error(int status, const char *fmt, ...);
#define RV_FAIL(status, ...)            \
  do {                                  \
    rv_set_error((status), __VA_ARGS__); \
    return (status);                    \
  } while (0)
#define RV_CUDA(call)                                                                        \
  do {                                                                                       \
    cudaError_t e_ = (call);                                                                 \
    if (e_ != cudaSuccess)                                                                   \
      RV_FAIL(RV_ERR_CUDA, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, \
              __LINE__);                                                                     \
  } while (0)
#define RV_LAUNCH_CHECK()                                                                \
  do {                                                                                   \
    cudaError_t e_ = cudaGetLastError();                                                 \
    if (e_ != cudaSuccess)                                                               \
      RV_FAIL(RV_ERR_CUDA, "kernel launch failed: %s (%s:%d)", cudaGetErrorString(e_), \
              __FILE__, __LINE__);                                                       \
  } while (0)

// Device-side error word: set (first writer wins) when a bounded wait runs
// out or a device check fails; read and cleared by rv_device_status.
__device__ int g_rv_dev_error;

// A bounded wait gives up after this many SM cycles (~1 s at 1.9 GHz).
#define RV_WAIT_CYCLES 2000000000LL

RV_DEVFN void rv_dev_fail(int code) { atomicCAS(&g_rv_dev_error, 0, code); }

// ------------------------------------------------------------ formats
__host__ __device__ inline int rv_fmt_block_bytes(int f) {
  return f == RV_Q4_K ? 144 : f == RV_Q5_K ? 176 : f == RV_Q6_K ? 210 : f == RV_Q8_0 ? 34
         : f == RV_Q8_K ? 292 : 0;
}
__host__ __device__ inline bool rv_fmt_is_kquant(int f) {
  return f == RV_Q4_K || f == RV_Q5_K || f == RV_Q6_K;
}

// --------------------------------------------------------- memory helpers
RV_DEVFN uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

RV_DEVFN float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// 16-bit little-endian load at any even address (shared or global).
RV_DEVFN uint16_t ld16(const uint8_t *p) { return *(const uint16_t *)p; }

// 32-bit little-endian load at any byte address inside shared memory:
// two aligned words and a funnel shift.  Reads up to 7 bytes past p, so
// every shared buffer read through it carries 16 bytes of slack.
RV_DEVFN uint32_t ld32u(const uint8_t *p) {
  uintptr_t a = (uintptr_t)p;
  const uint32_t *w = (const uint32_t *)(a & ~(uintptr_t)3);
  return __funnelshift_r(w[0], w[1], (uint32_t)(a & 3) * 8u);
}
RV_DEVFN int ld32a(const uint8_t *p) { return *(const int *)p; }

// ----------------------------------------------- mbarrier + bulk copies
RV_DEVFN void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
RV_DEVFN void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}
// Orders earlier generic-proxy shared-memory accesses before later
// async-proxy (bulk copy) writes to the same buffer.
RV_DEVFN void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// 1-D bulk copy global -> shared (no multicast): both addresses 16-byte
// aligned, bytes a multiple of 16.
RV_DEVFN void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}
RV_DEVFN bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, "
      "0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false (and the device error word set) if the phase did not
// complete within `limit` SM cycles.  The clock is read only every 32nd
// probe, and waiters off the critical path pass sleep_ns > 0 to back off
// between probes, so spinning warps leave the issue slots to warps with work.
RV_DEVFN bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, uint32_t sleep_ns = 0,
                                long long limit = RV_WAIT_CYCLES) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t i = 1;; i++) {
    if (sleep_ns) __nanosleep(sleep_ns);
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 31) == 0 && clock64() - t0 > limit) {
      rv_dev_fail(RV_ERR_TIMEOUT);
      return false;
    }
  }
}

// ------------------------------------- flags shared with other GPUs
// A 32-bit flag another GPU (or this one) sets with a release store at
// system scope; waiters read it with acquire loads, so everything the
// setter wrote before its release is visible to the waiter after it.
// Flags count upwards: a wait for `target` is satisfied by any value at or
// past it (compared modulo 2^32).
RV_DEVFN uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
RV_DEVFN void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
RV_DEVFN bool flag_reached(uint32_t v, uint32_t target) { return (int32_t)(v - target) >= 0; }
// Bounded: false (and the device error word set) if the flag did not reach
// target within `limit` SM cycles.
RV_DEVFN bool flag_wait_bounded(const uint32_t *flag, uint32_t target, long long limit = RV_WAIT_CYCLES) {
  if (flag_reached(ld_acquire_sys(flag), target)) return true;
  const long long t0 = clock64();
  for (uint32_t i = 1;; i++) {
    __nanosleep(32);
    if (flag_reached(ld_acquire_sys(flag), target)) return true;
    if ((i & 15) == 0 && clock64() - t0 > limit) {
      rv_dev_fail(RV_ERR_TIMEOUT);
      return false;
    }
  }
}

// ------------------------------------------------- thread-block clusters
RV_DEVFN uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Every thread of every CTA of the cluster arrives, then waits for all.  The
// CTAs of a cluster are scheduled together, so each of them reaches it.
RV_DEVFN void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The shared::cluster address of this CTA's shared variable `p` in CTA `rank`.
RV_DEVFN uint32_t dsmem_addr(const void *p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(p)), "r"(rank));
  return r;
}
RV_DEVFN void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
// Arrive (release, cluster scope) on an mbarrier of another CTA of the cluster.
RV_DEVFN void mbar_arrive_cluster(uint32_t addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
}
// Bounded wait (acquire, cluster scope) on this CTA's mbarrier.
RV_DEVFN bool mbar_wait_cluster_bounded(uint64_t *bar, uint32_t parity) {
  const long long t0 = clock64();
  for (uint32_t i = 0;; i++) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n selp.u32 "
        "%0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((i & 31) == 31 && clock64() - t0 > RV_WAIT_CYCLES) {
      rv_dev_fail(RV_ERR_TIMEOUT);
      return false;
    }
  }
}

// Barrier over the first NT threads of the block (named barrier 1), or the
// whole block (__syncthreads) when NT == 0; the _and form also returns
// whether the predicate held in every participating thread.
template <int NT>
RV_DEVFN void cta_sync() {
  if constexpr (NT == 0) __syncthreads();
  else asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory");
}
template <int NT>
RV_DEVFN bool cta_sync_and(bool p) {
  if constexpr (NT == 0) {
    return __syncthreads_and(p);
  } else {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred a, b;\n setp.ne.u32 a, %1, 0;\n bar.red.and.pred b, 1, %2, a;\n selp.u32 %0, 1, 0, b;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)p), "n"(NT)
        : "memory");
    return r != 0;
  }
}

// Stage `bytes` from global `src` into shared `dst`.  Aligned ranges go
// through the bulk-copy engine (issued by the calling thread, completion
// counted on `bar`); returns the bytes it put in flight.  Unaligned ranges
// are copied by the whole block with byte loads (all threads must call, and
// a __syncthreads must follow before reading).
RV_DEVFN bool rv_bulk_ok(const void *src, const void *dst, size_t bytes) {
  return ((((uintptr_t)src) | ((uintptr_t)dst) | bytes) & 15) == 0;
}
RV_DEVFN void rv_copy_bytes_block(uint8_t *dst, const uint8_t *src, size_t bytes) {
  for (size_t i = threadIdx.x; i < bytes; i += blockDim.x) dst[i] = src[i];
}

// ------------------------------------------------------ phase clocks
// Compiled out unless RV_PHASE_CLOCK is defined: thread 0 of each CTA stamps
// %globaltimer (ns, common to all SMs) at the phases of a kernel (the GPU analogue of the reference's
// PhaseClock, model/prefill.rs:414-520), read back by rv_debug_phase_clock.
#ifdef RV_PHASE_CLOCK
#define RV_PHASE_KERNELS 6  // 3, 4: per-stage traces of one tensor-GEMM CTA; 5: exact router chains
#define RV_PHASE_CTAS 8192
#define RV_PHASES 10
__device__ long long g_rv_phase[RV_PHASE_KERNELS][RV_PHASE_CTAS][RV_PHASES];
RV_DEVFN long long rv_globaltimer() {
  long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
#define RV_PHASE(k, i)                                                                       \
  do {                                                                                      \
    const unsigned cta_ = blockIdx.x + gridDim.x * blockIdx.y;                              \
    if (threadIdx.x == 0 && cta_ < RV_PHASE_CTAS) g_rv_phase[k][cta_][i] = rv_globaltimer(); \
  } while (0)
// Stamp from whichever thread calls it (one thread per CTA by construction).
#define RV_PHASE_ANY(k, i)                                                        \
  do {                                                                           \
    const unsigned cta_ = blockIdx.x + gridDim.x * blockIdx.y;                   \
    if (cta_ < RV_PHASE_CTAS) g_rv_phase[k][cta_][i] = rv_globaltimer();         \
  } while (0)
// %globaltimer of thread 0 in slot i, from a helper shared by several
// kernels (slot k only meaningful for the kernel that owns it).
#define RV_PHASE_ANY_T0(k, i)                                                              \
  do {                                                                                    \
    const unsigned cta_ = blockIdx.x + gridDim.x * blockIdx.y;                            \
    if (threadIdx.x == 0 && cta_ < RV_PHASE_CTAS) g_rv_phase[k][cta_][i] = rv_globaltimer(); \
  } while (0)
// clock64 of thread 0 in slot i (pairs with a %globaltimer stamp to give
// the SM clock rate during a phase).
#define RV_PHASE_CLK(k, i)                                                                    \
  do {                                                                                       \
    const unsigned cta_ = blockIdx.x + gridDim.x * blockIdx.y;                               \
    if (threadIdx.x == 0 && cta_ < RV_PHASE_CTAS) g_rv_phase[k][cta_][i] = (long long)clock64(); \
  } while (0)
// Per-stage event trace of one CTA of a one-dimensional grid (blockIdx.x ==
// 20): row `stage` of kernel slot k.
#define RV_TRACE(k, stage, ev)                                                          \
  do {                                                                                 \
    if (blockIdx.x == 20 && blockIdx.y == 0 && (stage) < RV_PHASE_CTAS)                \
      g_rv_phase[k][stage][ev] = rv_globaltimer();                                     \
  } while (0)
// Event ev of the decode routing tail (the last routing CTA, thread 0).
#define RV_TRACE_TAIL(ev)                                                      \
  do {                                                                        \
    if (threadIdx.x == 0) g_rv_phase[3][0][ev] = rv_globaltimer();            \
  } while (0)
#else
#define RV_TRACE_TAIL(ev) \
  do {                    \
  } while (0)
#define RV_TRACE(k, stage, ev) \
  do {                         \
  } while (0)
#define RV_PHASE_ANY(k, i) \
  do {                   \
  } while (0)
#define RV_PHASE_CLK(k, i) \
  do {                   \
  } while (0)
#define RV_PHASE_ANY_T0(k, i) \
  do {                      \
  } while (0)
#define RV_PHASE(k, i) \
  do {                 \
  } while (0)
#endif

// -------------------------------------------- programmatic dependent launch
// A kernel launched with programmatic stream serialization may start while
// the previous kernel in the stream is still running; it must call
// pdl_wait() before touching anything that kernel writes.  pdl_trigger()
// lets the next such kernel start early.  Both are no-ops for ordinary
// launches.
RV_DEVFN void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
RV_DEVFN void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// 16-byte asynchronous global -> shared copy (both addresses 16-byte aligned).
RV_DEVFN void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
RV_DEVFN void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
RV_DEVFN void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Copies `bytes` from global to shared memory with every thread of the CTA,
// all copies in flight at once: 16-byte cp.async pieces when both ends and
// the size are 16-byte aligned, else 4-byte words (both ends 4-byte aligned)
// loaded four at a time.  The caller synchronizes the CTA before reading.
RV_DEVFN void stage_to_smem(void *dst, const void *src, size_t bytes) {
  if ((((uintptr_t)dst | (uintptr_t)src | bytes) & 15) == 0) {
    for (size_t k = threadIdx.x; k < bytes / 16; k += blockDim.x)
      cp_async16((uint8_t *)dst + 16 * k, (const uint8_t *)src + 16 * k);
    cp_async_commit();
    cp_async_wait<0>();
  } else {
    const uint32_t *s = (const uint32_t *)src;
    uint32_t *d = (uint32_t *)dst;
    const size_t words = bytes / 4;
#pragma unroll 4
    for (size_t k = threadIdx.x; k < words; k += blockDim.x) d[k] = s[k];
  }
}

// True when every double within 2^-k * |r| of r (k in 30..52) rounds to the
// same float as r, so the f32 result of a double computation does not
// depend on how the double was summed within that bound.  Decided from the
// 29 mantissa bits the float rounding drops: the rounding boundaries (the
// midpoints between floats) are where they equal 2^28, and 2^-k * |r| is
// less than 2^(53-k) units of r's last place.  False outside the normal
// float range.
RV_DEVFN bool f32_rounding_stable(double r, int k) {
  const uint64_t b = (uint64_t)__double_as_longlong(r);
  const int ex = (int)((b >> 52) & 0x7ff) - 1023;
  if (ex < -125 || ex > 126) return false;
  const long long low = (long long)(b & ((1ull << 29) - 1));
  return llabs(low - (1ll << 28)) > (1ll << (53 - k));
}

// ------------------------------------------------ Q8_K warp quantizer
// Quantizes 256 floats held 8 per lane (lane l holds elements 8l..8l+7)
// into one packed 292-byte Q8_K block at `out` (4-byte aligned), exactly as
// quantize_row_q8_k (kernels/quants/quantize.rs:68-103): the signed value of
// the first element with the largest magnitude is anchored at -127
// (iscale = -127/max), q = clamp(round-half-even(iscale*v), -128, 127),
// bsums of 16-element groups, d = 1/iscale; an all-zero block is all zeros.
RV_DEVFN void q8k_quantize_warp(const float (&v)[8], int lane, uint8_t *out) {
  float amax = 0.0f;
#pragma unroll
  for (int e = 0; e < 8; e++) amax = fmaxf(amax, fabsf(v[e]));
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(RV_FULL, amax, o));
  uint32_t *w32 = (uint32_t *)out;
  if (amax == 0.0f) {
    // d, qs[8l..8l+8), bsums: 73 words; lane l clears words l, l+32, l+64.
    for (int k = lane; k < 73; k += 32) w32[k] = 0u;
    return;
  }
  int idx = 256;
#pragma unroll
  for (int e = 7; e >= 0; e--)
    if (fabsf(v[e]) == amax) idx = 8 * lane + e;
#pragma unroll
  for (int o = 16; o; o >>= 1) idx = min(idx, __shfl_xor_sync(RV_FULL, idx, o));
  float mine = v[0];
#pragma unroll
  for (int e = 1; e < 8; e++)
    if ((idx & 7) == e) mine = v[e];
  const float maxv = __shfl_sync(RV_FULL, mine, idx >> 3);
  const float iscale = __fdiv_rn(-127.0f, maxv);
  int q[8], s = 0;
#pragma unroll
  for (int e = 0; e < 8; e++) {
    int n = __float2int_rn(__fmul_rn(iscale, v[e]));
    n = max(-128, min(127, n));
    q[e] = n;
    s += n;
  }
  s += __shfl_xor_sync(RV_FULL, s, 1);
  uint32_t lo = (q[0] & 0xff) | ((q[1] & 0xff) << 8) | ((q[2] & 0xff) << 16) | ((uint32_t)q[3] << 24);
  uint32_t hi = (q[4] & 0xff) | ((q[5] & 0xff) << 8) | ((q[6] & 0xff) << 16) | ((uint32_t)q[7] << 24);
  w32[1 + 2 * lane] = lo;
  w32[2 + 2 * lane] = hi;
  if ((lane & 1) == 0) ((int16_t *)(out + 260))[lane >> 1] = (int16_t)s;
  if (lane == 0) *(float *)out = __fdiv_rn(1.0f, iscale);
}

// ---------------------------------------------- lane-exact k-quant dots
// The reference's production dot (kernels/quants/avx2.rs:554-838) keeps
// eight i32 lanes per super-block: lane i sums, over every 32-byte weight
// vector, the products of bytes 4i..4i+3 scaled by that vector's sub-block
// scale (maddubs + madd_epi16); Q4_K/Q5_K also keep four min lanes
// (mins_dot, avx2.rs:536-548).  Per block: acc[i] = fma(d*y.d, lane[i],
// acc[i]).  A GPU thread owns lane i of one weight row: it forms exactly
// lane i's integer sum with dp4a (four int8 products = one lane's bytes of
// one vector) and runs lane i's FMA chain over the row's blocks in order,
// so the float result is bit-identical to the AVX2 dot.

// Weight-side state of one block for lane i (depends only on the weight).
struct WBlock {
  uint32_t q[8];  // Q4_K/Q5_K: lo[0..3], hi[0..3]; Q6_K: (q-32) vectors [h*4+k]
  int sc[8];      // Q4_K/Q5_K: eight 6-bit scales; Q6_K: scale of vector [h*4+k]
  int m0, m1;     // min-lane multipliers (Q4_K/Q5_K, lane < 4)
  float d, dmin;
};

// get_scale_min_k4 (kernels/quants/blocks.rs:127-141) over the 12 bytes.
RV_DEVFN void unpack_k4_scales(const uint8_t *s12, int lane, WBlock &w) {
  uint32_t a = ld32u(s12), b = ld32u(s12 + 4), c = ld32u(s12 + 8);
  uint32_t s[12] = {a & 255, (a >> 8) & 255, (a >> 16) & 255, a >> 24,
                    b & 255, (b >> 8) & 255, (b >> 16) & 255, b >> 24,
                    c & 255, (c >> 8) & 255, (c >> 16) & 255, c >> 24};
  int mn[8];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    if (j < 4) {
      w.sc[j] = (int)(s[j] & 63);
      mn[j] = (int)(s[j + 4] & 63);
    } else {
      w.sc[j] = (int)((s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4));
      mn[j] = (int)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
  }
  // Min lane i (< 4) pairs sub-blocks 2i and 2i+1; selects keep mn in registers.
  const int i = lane & 3;
  w.m0 = i == 0 ? mn[0] : i == 1 ? mn[2] : i == 2 ? mn[4] : mn[6];
  w.m1 = i == 0 ? mn[1] : i == 1 ? mn[3] : i == 2 ? mn[5] : mn[7];
}

template <int FMT>
RV_DEVFN void load_wblock(const uint8_t *blk, int lane, WBlock &w) {
  if constexpr (FMT == RV_Q4_K || FMT == RV_Q5_K) {
    w.d = h2f(ld16(blk));
    w.dmin = h2f(ld16(blk + 2));
    unpack_k4_scales(blk + 4, lane, w);
    if constexpr (FMT == RV_Q4_K) {
#pragma unroll
      for (int j = 0; j < 4; j++) {
        uint32_t q = ld32u(blk + 16 + 32 * j + 4 * lane);
        w.q[j] = q & 0x0F0F0F0Fu;
        w.q[4 + j] = (q >> 4) & 0x0F0F0F0Fu;
      }
    } else {
      const uint32_t qh = ld32u(blk + 16 + 4 * lane);
#pragma unroll
      for (int j = 0; j < 4; j++) {
        uint32_t q = ld32u(blk + 48 + 32 * j + 4 * lane);
        w.q[j] = (q & 0x0F0F0F0Fu) + (((qh >> (2 * j)) & 0x01010101u) << 4);
        w.q[4 + j] = ((q >> 4) & 0x0F0F0F0Fu) + (((qh >> (2 * j + 1)) & 0x01010101u) << 4);
      }
    }
  } else {  // Q6_K
    w.d = h2f(ld16(blk + 208));
    w.dmin = 0.0f;
    w.m0 = w.m1 = 0;
#pragma unroll
    for (int h = 0; h < 2; h++) {
      uint32_t ql0 = ld32u(blk + 64 * h + 4 * lane);
      uint32_t ql1 = ld32u(blk + 64 * h + 32 + 4 * lane);
      uint32_t qh = ld32u(blk + 128 + 32 * h + 4 * lane);
      uint32_t v0 = (ql0 & 0x0F0F0F0Fu) | ((qh & 0x03030303u) << 4);
      uint32_t v1 = (ql1 & 0x0F0F0F0Fu) | (((qh >> 2) & 0x03030303u) << 4);
      uint32_t v2 = ((ql0 >> 4) & 0x0F0F0F0Fu) | (((qh >> 4) & 0x03030303u) << 4);
      uint32_t v3 = ((ql1 >> 4) & 0x0F0F0F0Fu) | (((qh >> 6) & 0x03030303u) << 4);
      w.q[4 * h + 0] = __vsub4(v0, 0x20202020u);
      w.q[4 * h + 1] = __vsub4(v1, 0x20202020u);
      w.q[4 * h + 2] = __vsub4(v2, 0x20202020u);
      w.q[4 * h + 3] = __vsub4(v3, 0x20202020u);
      const int hi = lane >= 4 ? 1 : 0;
#pragma unroll
      for (int k = 0; k < 4; k++) w.sc[4 * h + k] = (int)(int8_t)blk[192 + 8 * h + 2 * k + hi];
    }
  }
}

// Lane sums of one weight block against one packed Q8_K activation block
// `act` (4-byte aligned): S = lane i's scaled integer sum, Mn = min lane
// (valid for lane < 4, Q4_K/Q5_K).
template <int FMT>
RV_DEVFN void lane_sums(const WBlock &w, const uint8_t *act, int lane, int &S, int &Mn) {
  const uint8_t *qs = act + 4;
  int s = 0;
  if constexpr (FMT == RV_Q4_K || FMT == RV_Q5_K) {
#pragma unroll
    for (int j = 0; j < 4; j++) {
      s += w.sc[2 * j] * __dp4a((int)w.q[j], ld32a(qs + 64 * j + 4 * lane), 0);
      s += w.sc[2 * j + 1] * __dp4a((int)w.q[4 + j], ld32a(qs + 64 * j + 32 + 4 * lane), 0);
    }
    const int16_t *bs = (const int16_t *)(act + 260);
    const int i = lane & 3;
    Mn = w.m0 * ((int)bs[4 * i] + (int)bs[4 * i + 1]) +
         w.m1 * ((int)bs[4 * i + 2] + (int)bs[4 * i + 3]);
  } else {
#pragma unroll
    for (int h = 0; h < 2; h++)
#pragma unroll
      for (int k = 0; k < 4; k++)
        s += w.sc[4 * h + k] * __dp4a((int)w.q[4 * h + k], ld32a(qs + 128 * h + 32 * k + 4 * lane), 0);
    Mn = 0;
  }
  S = s;
}

// Horizontal sum of the eight lanes held by 8 consecutive threads, in the
// order of hsum_ps_8 (avx2.rs:494-500): ((v0+v4)+(v2+v6)) + ((v1+v5)+(v3+v7)),
// minus hsum_ps_4 of the min lanes ((m0+m2)+(m1+m3)) for Q4_K/Q5_K.
// All 32 threads of the warp must call; the result is valid on lane 0 of
// each group of eight.
template <int FMT>
RV_DEVFN float lane_reduce(float acc, float accm) {
  float s = __fadd_rn(acc, __shfl_xor_sync(RV_FULL, acc, 4));
  float t = __fadd_rn(s, __shfl_xor_sync(RV_FULL, s, 2));
  float u = __fadd_rn(t, __shfl_xor_sync(RV_FULL, t, 1));
  if constexpr (FMT == RV_Q6_K) {
    return u;
  } else {
    float a = __fadd_rn(accm, __shfl_xor_sync(RV_FULL, accm, 2));
    float b = __fadd_rn(a, __shfl_xor_sync(RV_FULL, a, 1));
    return __fsub_rn(u, b);
  }
}

// One block's float step for lane i (avx2.rs:557-562, 598; 747, 836).
template <int FMT>
RV_DEVFN void lane_step(const WBlock &w, const uint8_t *act, int lane, float &acc, float &accm) {
  int S, Mn;
  lane_sums<FMT>(w, act, lane, S, Mn);
  const float yd = *(const float *)act;
  if constexpr (FMT != RV_Q6_K) {
    if (lane < 4) accm = __fmaf_rn(__fmul_rn(w.dmin, yd), __int2float_rn(Mn), accm);
  }
  acc = __fmaf_rn(__fmul_rn(w.d, yd), __int2float_rn(S), acc);
}
