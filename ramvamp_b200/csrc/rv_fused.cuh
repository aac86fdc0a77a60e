// rv_fused.cuh -- one-token decode: the expert half of the speculative
// pipeline in a single cooperative launch.
//
// k_route_chain (the exact router chains and routing) runs beside it; this
// kernel does everything else of the layer, in three phases separated by
// counters instead of kernel boundaries:
//   A  CTAs 0..E/4-1: RMSNorm, the logit bounds of four experts, the Q8_K
//      of the normed row (route_spec_cta); each then bumps fz[0].
//   B  every CTA waits for fz[0] == E/4, rebuilds the speculated set
//      (spec_build), asks L2 for the down rows its warps will need, and
//      runs one gate/up tile of 16 rows (gate_up_unit); the last tile of
//      each 256-row block quantizes it and bumps fz[2 + unit].
//   C  each warp takes one down tile of 8 rows, waits until its unit's
//      SwiGLU rows are all quantized, computes them and stores the rows of
//      the pairs the exact routing selected; the last tile of each row
//      group adds the combine.  The exact routing is the chain kernel's
//      output: the first read of it waits for that grid (PDL).
// A cooperative launch keeps every CTA resident, so the waits always end;
// each is bounded anyway.  The last CTA out clears the counters.
#pragma once
#include "rv_moe.cuh"

#define RV_FUSED_THREADS 128
// Counters in B.fz, each on its own 128-byte line so that polling CTAs do
// not queue behind one another: bounds CTAs done, CTAs done, the bounds-
// ready flag in RV_FZ_REPL copies (CTA c polls copy c mod RV_FZ_REPL),
// then the quantized SwiGLU blocks of each unit.
#define RV_FZ_LINE 32
#define RV_FZ_REPL 16
#define RV_FZ_BOUNDS 0
#define RV_FZ_EXIT RV_FZ_LINE
#define RV_FZ_FLAG(r) ((2 + (r)) * RV_FZ_LINE)
#define RV_FZ_UNIT(u) ((2 + RV_FZ_REPL + (u)) * RV_FZ_LINE)
#define RV_FZ_INTS RV_FZ_UNIT(256)
#define RV_FUSED_GU_R 16   // gate/up rows per tile (128 threads: 16 rows x 2 parts x 4 lanes)
#define RV_FUSED_DN_ROWS 8  // down rows per warp tile

// Bounded wait until *p >= target (acquire), backing off from 32 ns to
// 256 ns between polls.  False on timeout.
RV_DEVFN bool wait_count_geq(const int *p, int target) {
  const long long t0 = clock64();
  uint32_t sleep_ns = 32;
  for (uint32_t i = 0;; i++) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    if (v >= target) return true;
    __nanosleep(sleep_ns);
    if (sleep_ns < 256) sleep_ns <<= 1;
    if ((i & 15) == 15 && clock64() - t0 > RV_WAIT_CYCLES) {
      rv_dev_fail(RV_ERR_TIMEOUT);
      return false;
    }
  }
}

// Shared memory of the fused kernel: the largest of the three phases.
struct FusedLayout {
  size_t a, b, c_warp, total;
};
template <int FGU, int FDN>
__host__ __device__ inline FusedLayout fused_layout(const MoeDims &d, size_t gu_row_bytes, size_t down_row_bytes) {
  FusedLayout L;
  const size_t r16 = 15;
  L.a = 16 + (size_t)(RV_SPEC_EPC + 1) * d.H * 4 + (size_t)(d.H + 4) * 4;
  const size_t gst = FGU == RV_Q6_K ? gu_row_bytes : gu_row_bytes + 16;
  L.b = 16 + ((2 * (size_t)RV_FUSED_GU_R * gst + r16) & ~r16) + 16 + d.act_stride +
        (FGU == RV_Q6_K ? (size_t)d.hb * 64 * 4 : 0) + 2 * RV_FUSED_GU_R * RV_MOE_MT * 4;
  const size_t dst = FDN == RV_Q6_K ? down_row_bytes : down_row_bytes + 16;
  L.c_warp = ((16 + ((RV_FUSED_DN_ROWS * dst + r16) & ~r16) + 16 + d.amoe_stride +
               (FDN == RV_Q6_K ? (size_t)d.mb * 64 * 4 : 0) + 16) + r16) & ~r16;
  // Phase A's mbarriers sit at offset 0, phase B's at 16, phase C's from
  // 32: no phase re-initializes another's barrier.
  L.total = L.a;
  if (16 + L.b > L.total) L.total = 16 + L.b;
  if (32 + 4 * L.c_warp > L.total) L.total = 32 + 4 * L.c_warp;
  return L;
}

// One down tile (RV_FUSED_DN_ROWS rows of unit u's expert e) by one warp,
// for the unit's positions [p0, p1) (tokens = set bits of msk), into
// B.staged at the exact pairs.  smw: the warp's shared memory (two
// mbarriers, then the weight rows, the activations, the Q6_K word sums).
// ACTS_AFTER_WAIT: the activations are the previous kernel's output (copy
// them after the PDL wait); otherwise they are already final (only the
// routing read waits).
template <int FMT, int G, int NBG, bool ACTS_AFTER_WAIT = false>
RV_DEVFN bool down_tile_warp(const MoeDims &d, const MoeBufs &B, const MoeWeights &W, uint8_t *smw, int e, int p0,
                             int p1, uint32_t msk, int tile, uint32_t *s_pair, uint32_t &wphase, uint32_t &aphase) {
  constexpr int ROWS = RV_FUSED_DN_ROWS, MT = RV_MOE_MT;
  const int lane = threadIdx.x & 31;
  const int row0 = tile * ROWS, nrows = min(ROWS, d.H - row0);
  uint64_t *bar = (uint64_t *)smw;
  const size_t st = tile_stride<FMT>(W.down_row_bytes);
  uint8_t *wsm = smw + 16;
  uint8_t *asm_ = wsm + (((size_t)ROWS * st + 15) & ~(size_t)15) + 16;
  int *asum = (int *)(asm_ + (size_t)(p1 - p0) * d.amoe_stride);
  const uint8_t *dsrc = W.base + (size_t)e * W.stride + W.down_off + (size_t)row0 * W.down_row_bytes;
  // Weights: one warp stages its own rows (the bulk copy is issued by lane 0).
  const size_t wbytes = (size_t)nrows * W.down_row_bytes;
  bool wbulk;
  if constexpr (FMT == RV_Q6_K) wbulk = rv_bulk_ok(dsrc, wsm, wbytes);
  else wbulk = rv_bulk_ok(dsrc, wsm, W.down_row_bytes);
  const uint8_t *asrc = B.acts_moe + (size_t)p0 * d.amoe_stride;
  const uint32_t abytes = (uint32_t)((p1 - p0) * d.amoe_stride);
  const bool abulk = rv_bulk_ok(asrc, asm_, abytes);
  __syncwarp();
  if (lane == 0) {
    fence_proxy_async();
    if (wbulk) {
      mbar_arrive_expect_tx(bar, (uint32_t)wbytes);
      if constexpr (FMT == RV_Q6_K) {
        bulk_g2s(wsm, dsrc, (uint32_t)wbytes, bar);
      } else {
        for (int r = 0; r < nrows; r++)
          bulk_g2s(wsm + r * st, dsrc + (size_t)r * W.down_row_bytes, (uint32_t)W.down_row_bytes, bar);
      }
    }
    if (abulk && !ACTS_AFTER_WAIT) {
      mbar_arrive_expect_tx(bar + 1, abytes);
      bulk_g2s(asm_, asrc, abytes, bar + 1);
    }
  }
  if (!wbulk)
    for (size_t i = lane; i < wbytes; i += 32) wsm[(i / W.down_row_bytes) * st + i % W.down_row_bytes] = dsrc[i];
  if (!abulk && !ACTS_AFTER_WAIT)
    for (uint32_t i = lane; i < abytes; i += 32) asm_[i] = asrc[i];
  // The exact pair of each position (the chain kernel's routing).
  pdl_wait();
  if constexpr (ACTS_AFTER_WAIT) {
    if (abulk) {
      if (lane == 0) {
        mbar_arrive_expect_tx(bar + 1, abytes);
        bulk_g2s(asm_, asrc, abytes, bar + 1);
      }
    } else {
      for (uint32_t i = lane; i < abytes; i += 32) asm_[i] = asrc[i];
    }
  }
  if (lane < p1 - p0) {
    const int t = spec_nth_bit(msk, lane);
    uint32_t pair = ~0u;
    for (int k = 0; k < d.K; k++)
      if (B.ids[(size_t)t * d.K + k] == (uint32_t)e) pair = (uint32_t)(t * d.K + k);
    s_pair[lane] = pair;
  }
  const bool any = __any_sync(RV_FULL, lane < p1 - p0 && s_pair[lane] != ~0u);
  bool ok = true;
  if (wbulk) {
    ok = mbar_wait_bounded(bar, wphase);
    wphase ^= 1;
  }
  if (abulk) {
    ok = mbar_wait_bounded(bar + 1, aphase) && ok;
    aphase ^= 1;
  }
  __syncwarp();
  if (!__all_sync(RV_FULL, ok)) return false;
  if (!any) return true;
  const int rsub = lane / G, g = lane % G;
  const bool live = rsub < ROWS && rsub < nrows;
  const uint8_t *wrow = wsm + (size_t)(live ? rsub : 0) * st;
  const int mt = p1 - p0;
  if constexpr (FMT == RV_Q6_K) {
    for (int m = 0; m < mt; m++) act_word_sums(asm_ + (size_t)m * d.amoe_stride, d.mb, asum + m * d.mb * 64, lane, 32);
    __syncwarp();
  }
  for (int m0 = 0; m0 < mt; m0 += MT) {
    const int mm = min(MT, mt - m0);
    if constexpr (G > 1) {
      for (int m = 0; m < mm; m++) {
        const float res = row_dot_split<FMT, G, NBG>(wrow, asm_ + (size_t)(m0 + m) * d.amoe_stride,
                                                      asum + (m0 + m) * d.mb * 64, g);
        const uint32_t pair = s_pair[m0 + m];
        if (g == G - 1 && live && pair != ~0u) B.staged[(size_t)pair * d.H + row0 + rsub] = res;
      }
    } else {
      float res[MT];
      row_dot_tokens<FMT, MT>(wrow, d.mb, asm_ + (size_t)m0 * d.amoe_stride, d.amoe_stride, asum + m0 * d.mb * 64,
                              (size_t)d.mb * 64, mm, res);
#pragma unroll
      for (int m = 0; m < MT; m++)
        if (m < mm && live) {
          const uint32_t pair = s_pair[m0 + m];
          if (pair != ~0u) B.staged[(size_t)pair * d.H + row0 + rsub] = res[m];
        }
    }
  }
  return true;
}

template <int FGU, int FDN, int GEO>
__global__ void __launch_bounds__(RV_FUSED_THREADS, 4) k_decode_fused(MoeDims dd, MoeBufs B, MoeWeights W) {
  const MoeDims d = geo_dims<GEO>(dd);
  extern __shared__ __align__(16) uint8_t sm[];
  __shared__ SpecSmem ss;
  __shared__ uint32_t s_pair[4][RV_SPEC_MAX_T];
  __shared__ int s_last[1];
  __shared__ int s_wlast[4];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cta = blockIdx.x, ncta = gridDim.x;
  const int nb = (d.E + RV_SPEC_EPC - 1) / RV_SPEC_EPC;
  RV_PHASE(1, 0);
  if (cta < nb) RV_PHASE(0, 0);
  // ---- A: norm, bounds, Q8_K (the residual is final: the chain kernel
  // launched this grid only after the previous layer completed).  The last
  // bounds CTA raises the ready flag.
  if (cta < nb) {
    route_spec_cta<false>(d, B, sm, cta, nb);
    __syncthreads();
    if (tid == 0) {
      __threadfence();
      if (atomicAdd(&B.fz[RV_FZ_BOUNDS], 1) == nb - 1) {
        __threadfence();
        for (int r = 0; r < RV_FZ_REPL; r++) atomicExch(&B.fz[RV_FZ_FLAG(r)], 1);
      }
    }
  }
  if (tid == 0) s_last[0] = wait_count_geq(&B.fz[RV_FZ_FLAG(cta % RV_FZ_REPL)], 1) ? 0 : -1;
  __syncthreads();
  if (s_last[0] < 0) return;
  // The bounds and Q8_K rows were written by other CTAs (generic stores);
  // the gate/up tiles read the Q8_K rows through the bulk-copy engine.
  asm volatile("fence.proxy.async.global;" ::: "memory");
  RV_PHASE(1, 1);
  // ---- B: the speculated units, then this CTA's gate/up tiles.
  spec_build(d.E, d.K, B.T, B.spec, ss);
  const int nu = ss.n_units;
  const int dtiles = d.H / RV_FUSED_DN_ROWS;  // a multiple of 4: a CTA's four warps share a unit
  const int gtiles = d.M / RV_FUSED_GU_R;
  uint8_t *smb = sm + 16;
  uint32_t phase = 0;
  if (tid == 0) mbar_init((uint64_t *)smb, 1);
  __syncthreads();
  for (int task = cta; task < nu * gtiles; task += ncta) {
    const int u = task / gtiles, tile = task % gtiles;
    const int e = ss.uexp[u], p0 = ss.start[e];
    const uint32_t msk = ss.mask[e];
    if (!gate_up_unit<FGU, 4, 2, RV_FUSED_GU_R>(d, B, W, smb, u, e, p0, p0 + __popc(msk), tile,
                                                [&](int c) { return (uint32_t)spec_nth_bit(msk, c - p0); }, phase,
                                                B.fz + RV_FZ_UNIT(0), RV_FZ_LINE))
      return;
  }
  // The down rows this CTA's warps will need, into L2 (after the gate/up
  // weights, which are on the critical path, have streamed in).
  if (lane == 0)
    for (int task = cta * 4 + warp; task < nu * dtiles; task += ncta * 4) {
      const int e = ss.uexp[task / dtiles], tile = task % dtiles;
      const uint8_t *src =
          W.base + (size_t)e * W.stride + W.down_off + (size_t)tile * RV_FUSED_DN_ROWS * W.down_row_bytes;
      const uint32_t bytes = (uint32_t)(RV_FUSED_DN_ROWS * W.down_row_bytes);
      if ((((uintptr_t)src | bytes) & 15) == 0) prefetch_l2(src, bytes);
    }
  __syncthreads();  // gate/up's shared memory is free for the down tiles
  // The next layer's chain kernel may launch now: it waits for this grid
  // before reading the residual, and this grid needs no more CTAs.
  pdl_trigger();
  // ---- C: down tiles.  Round k: warp w takes tile (cta*4 + k*ncta*4 + w);
  // the four share a unit, whose readiness thread 0 polls for all.
  const FusedLayout L = fused_layout<FGU, FDN>(d, W.gu_row_bytes, W.down_row_bytes);
  uint8_t *smw = sm + 32 + (size_t)warp * L.c_warp;
  if (lane == 0) {
    mbar_init((uint64_t *)smw, 1);
    mbar_init((uint64_t *)smw + 1, 1);
  }
  __syncwarp();
  uint32_t wphase = 0, aphase = 0;
  bool first = true;
  for (int base = cta * 4; base < nu * dtiles; base += ncta * 4) {
    const int u = base / dtiles;
    if (first) RV_PHASE_ANY_T0(2, 0);
    if (tid == 0) s_last[0] = wait_count_geq(&B.fz[RV_FZ_UNIT(u)], d.mb) ? 0 : -1;
    __syncthreads();
    if (s_last[0] < 0) return;
    asm volatile("fence.proxy.async.global;" ::: "memory");  // acts_moe: other CTAs' stores, read by bulk copy
    if (first) RV_PHASE_ANY_T0(2, 2);
    const int task = base + warp, tile = task % dtiles;
    const int e = ss.uexp[u], p0 = ss.start[e];
    const uint32_t msk = ss.mask[e];
    bool ok;
    if (d.mb == 3) ok = down_tile_warp<FDN, 3, 1>(d, B, W, smw, e, p0, p0 + __popc(msk), msk, tile, s_pair[warp],
                                                   wphase, aphase);
    else ok = down_tile_warp<FDN, 1, 1>(d, B, W, smw, e, p0, p0 + __popc(msk), msk, tile, s_pair[warp], wphase,
                                        aphase);
    if (!ok) return;
    if (first) RV_PHASE_ANY_T0(2, 4);
    first = false;
    // The last unit to finish this row tile adds the combine.
    __threadfence();
    __syncwarp();
    if (lane == 0) {
      int *cnt = &B.down_cnt[tile];
      const int old = atomicAdd(cnt, 1);
      s_wlast[warp] = old == nu - 1;
      if (old == nu - 1) *cnt = 0;
    }
    __syncwarp();
    if (s_wlast[warp]) {
      __threadfence();
      const int row0 = tile * RV_FUSED_DN_ROWS, nrows = min(RV_FUSED_DN_ROWS, d.H - row0);
      // acc = 0; acc += w_k * d_k in top-k order; residual += acc (forward.rs:2744-2753).
      for (int i = lane; i < B.T * nrows; i += 32) {
        const int t = i / nrows, h = row0 + i % nrows;
        float acc = 0.0f;
        for (int k = 0; k < d.K; k++) {
          const size_t pair = (size_t)t * d.K + k;
          acc = __fadd_rn(acc, __fmul_rn(B.w[pair], __ldcg(B.staged + pair * d.H + h)));
        }
        float *res = B.residual + (size_t)t * d.H + h;
        *res = __fadd_rn(*res, acc);
      }
    }
    __syncthreads();  // s_last[0] is reused by the next round's poll
  }
  RV_PHASE(1, 5);
  // CTA 0: check that the speculated set held the exact routing and write
  // the dispatch taps (position -> token-major pair, ~0 where unselected).
  if (cta == 0) {
    pdl_wait();
    for (int p = tid; p < B.T * d.K; p += blockDim.x) {
      const uint32_t e = B.ids[p];
      // Cannot happen: the speculated set holds the exact top-k.
      if (e >= (uint32_t)d.E || !((ss.mask[e] >> (p / d.K)) & 1u)) rv_dev_fail(RV_ERR_ROUTED_OUT_OF_RANGE);
    }
    for (int e = tid; e < d.E; e += blockDim.x) {
      uint32_t m = ss.mask[e];
      int pos = ss.start[e];
      while (m) {
        const int t = __ffs(m) - 1;
        m &= m - 1;
        uint32_t pair = ~0u;
        for (int k = 0; k < d.K; k++)
          if (B.ids[(size_t)t * d.K + k] == (uint32_t)e) pair = (uint32_t)(t * d.K + k);
        B.index[pos++] = pair;
      }
    }
    for (int e = tid; e <= d.E; e += blockDim.x) B.index_start[e] = ss.start[e];
  }
  // The last CTA out clears the counters for the next call.
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(&B.fz[RV_FZ_EXIT], 1) == ncta - 1) {
      B.fz[RV_FZ_BOUNDS] = 0;
      B.fz[RV_FZ_EXIT] = 0;
      for (int r = 0; r < RV_FZ_REPL; r++) B.fz[RV_FZ_FLAG(r)] = 0;
      for (int u = 0; u < d.E; u++) B.fz[RV_FZ_UNIT(u)] = 0;
      __threadfence();
    }
  }
}

