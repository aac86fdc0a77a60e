// rv_moe.cuh -- the routed-expert FFN pipeline for T tokens of one layer.
//
// Stages (one launch each, all on the caller's stream):
//   k_prologue      ffn RMSNorm (f64, norm.rs:38-60) + Q8_K of the normed rows
//   k_router_logits one serial f32 chain per (token, expert) (forward.rs:1231-1237)
//   k_route         f64 softmax, top-k by repeated argmax, renormalization
//                   (forward.rs:2669-2705), per-expert counts
//   k_index         CSR inverse index by expert (prefill.rs:2536-2580) and the
//                   work list of (expert, token range) units
//   k_gate_up       gate and up rows of one expert for its tokens, SwiGLU with
//                   the host-libm exponential, and (last tile of each 256-row
//                   block) the Q8_K of the SwiGLU output (forward.rs:2235-2246)
//   k_down          down rows of one expert for its tokens, staged by (token, slot)
//   k_combine       fixed top-k-order reduction plus residual add
//                   (forward.rs:2744-2753, prefill.rs:2749-2778)
// Every float step is the reference's, so the result is bit-identical to its
// AVX2 CPU path.
#pragma once
#include "rv_expf.cuh"
#include "rv_internal.cuh"
#include "rv_kernels.cuh"

#define RV_MOE_MT 8          // tokens staged per pass
#define RV_MOE_TOK_CHUNK 64  // tokens per work unit
#define RV_GU_ROWS 16        // gate (and up) rows per k_gate_up CTA
#define RV_DOWN_ROWS 32      // down rows per k_down CTA

struct MoeDims {
  int H, M, E, K;
  int hb, mb;              // blocks per hidden / moe row
  size_t act_stride;       // bytes per token row of Q8_K(normed), 16-multiple
  size_t amoe_stride;      // bytes per pair row of Q8_K(swiglu), 16-multiple
  float eps;
  int norm_topk;
};

struct MoeBufs {
  const float *ffn_norm, *router;
  float *residual;
  float *normed;           // [T][H]
  uint8_t *acts;           // [T][act_stride]
  float *logits;           // [T][E]
  uint32_t *ids;           // [T][K]
  float *w;                // [T][K]
  int *counts;             // [E], zero between calls
  uint32_t *index_start;   // [E+1]
  uint32_t *index;         // [T*K] pair ids, grouped by expert
  int4 *units;             // [max_units] (expert, pos0, pos1, 0)
  int *n_units;            // [1]
  float *hbuf;             // [T*K][M] SwiGLU output, CSR order
  uint8_t *acts_moe;       // [T*K][amoe_stride]
  float *staged;           // [T][K][H]
  int *tile_cnt;           // [max_units][M/256], zero between calls
  int T;
  int max_units;
};

struct MoeWeights {
  const uint8_t *base;     // layer blob 0
  uint64_t stride, gate_off, up_off, down_off;
  size_t gu_row_bytes, down_row_bytes;
};

// ------------------------------------------------------------ prologue
__global__ void __launch_bounds__(256) k_prologue(MoeDims d, MoeBufs B) {
  extern __shared__ __align__(16) uint8_t sm[];
  double *red = (double *)sm;
  float *xs = (float *)(sm + 34 * sizeof(double));
  const int t = blockIdx.x;
  const float *x = B.residual + (size_t)t * d.H;
  for (int k = threadIdx.x; k < d.H; k += blockDim.x) xs[k] = x[k];
  __syncthreads();
  const float inv = rms_inv_block(xs, (size_t)d.H, d.eps, red);
  for (int k = threadIdx.x; k < d.H; k += blockDim.x) {
    const float v = __fmul_rn(__fmul_rn(xs[k], inv), B.ffn_norm[k]);
    xs[k] = v;
    B.normed[(size_t)t * d.H + k] = v;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int b = warp; b < d.hb; b += blockDim.x >> 5) {
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; e++) v[e] = xs[b * 256 + 8 * lane + e];
    q8k_quantize_warp(v, lane, B.acts + (size_t)t * d.act_stride + (size_t)b * 292);
  }
}

// ------------------------------------------------------- router logits
// Warp w of the CTA owns expert blockIdx.y*4+w; lane l owns token
// blockIdx.x*32+l.  Each logit is the reference's serial f32 chain:
// acc = acc + router[e][k] * normed[t][k] for k = 0..H-1, no FMA.
__global__ void __launch_bounds__(128) k_router_logits(MoeDims d, MoeBufs B) {
  const int e = blockIdx.y * 4 + (threadIdx.x >> 5);
  const int t = blockIdx.x * 32 + (threadIdx.x & 31);
  if (e >= d.E || t >= B.T) return;
  const float4 *r4 = (const float4 *)(B.router + (size_t)e * d.H);
  const float4 *x4 = (const float4 *)(B.normed + (size_t)t * d.H);
  float acc = 0.0f;
  const int n4 = d.H >> 2;
#pragma unroll 4
  for (int k = 0; k < n4; k++) {
    const float4 r = __ldg(r4 + k), x = x4[k];
    acc = __fadd_rn(acc, __fmul_rn(r.x, x.x));
    acc = __fadd_rn(acc, __fmul_rn(r.y, x.y));
    acc = __fadd_rn(acc, __fmul_rn(r.z, x.z));
    acc = __fadd_rn(acc, __fmul_rn(r.w, x.w));
  }
  B.logits[(size_t)t * d.E + e] = acc;
}

// ----------------------------------------------------------- top-k route
// One warp per token, E <= 256 (8 per lane), K <= 16.
__global__ void __launch_bounds__(128) k_route(MoeDims d, MoeBufs B) {
  __shared__ double es[4][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 4 + warp;
  if (t >= B.T) return;
  const float *lg = B.logits + (size_t)t * d.E;
  float p[8];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int e = lane + 32 * j;
    p[j] = e < d.E ? lg[e] : -INFINITY;
    if (e < d.E) mx = fmaxf(mx, p[j]);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(RV_FULL, mx, o));
  const double dmx = (double)mx;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int e = lane + 32 * j;
    if (e < d.E) {
      const double ex = exp(__dsub_rn((double)p[j], dmx));
      es[warp][e] = ex;
      p[j] = __double2float_rn(ex);
    }
  }
  __syncwarp();
  double sum = 0.0;
  if (lane == 0)
    for (int e = 0; e < d.E; e++) sum = __dadd_rn(sum, es[warp][e]);
  sum = __shfl_sync(RV_FULL, sum, 0);
  const float inv = __double2float_rn(__drcp_rn(sum));
#pragma unroll
  for (int j = 0; j < 8; j++) p[j] = (lane + 32 * j) < d.E ? __fmul_rn(p[j], inv) : -INFINITY;
  // Top-k by repeated argmax: strict '>' scan from expert 0, so the lowest
  // index wins a tie; the winner is blanked with -inf (forward.rs:2688-2699).
  uint32_t ids[16];
  float ws[16];
  for (int k = 0; k < d.K; k++) {
    float bp = -INFINITY;
    int be = 1 << 30;
#pragma unroll
    for (int j = 0; j < 8; j++)
      if (p[j] > bp) {
        bp = p[j];
        be = lane + 32 * j;
      }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float op = __shfl_xor_sync(RV_FULL, bp, o);
      const int oe = __shfl_xor_sync(RV_FULL, be, o);
      if (op > bp || (op == bp && oe < be)) {
        bp = op;
        be = oe;
      }
    }
    if (be == (1 << 30)) be = 0;  // nothing beat -inf: the scan keeps expert 0
    ids[k] = (uint32_t)be;
    ws[k] = bp;
#pragma unroll
    for (int j = 0; j < 8; j++)
      if (lane + 32 * j == be) p[j] = -INFINITY;
  }
  if (d.norm_topk) {
    float s = -0.0f;
    for (int k = 0; k < d.K; k++) s = __fadd_rn(s, ws[k]);
    for (int k = 0; k < d.K; k++) ws[k] = __fdiv_rn(ws[k], s);
  }
  if (lane < d.K) {
    uint32_t id = 0;
    float wv = 0.0f;
    for (int k = 0; k < d.K; k++)
      if (k == lane) {
        id = ids[k];
        wv = ws[k];
      }
    B.ids[(size_t)t * d.K + lane] = id;
    B.w[(size_t)t * d.K + lane] = wv;
    atomicAdd(&B.counts[id], 1);
  }
}

// ----------------------------------------------------------- dispatch
__global__ void __launch_bounds__(1024) k_index(MoeDims d, MoeBufs B) {
  __shared__ uint32_t start[257];
  __shared__ uint32_t cursor[256];
  if (threadIdx.x == 0) {
    uint32_t s = 0;
    int n = 0;
    for (int e = 0; e < d.E; e++) {
      const uint32_t c = (uint32_t)B.counts[e];
      start[e] = s;
      for (uint32_t p = 0; p < c; p += RV_MOE_TOK_CHUNK) {
        if (n < B.max_units)
          B.units[n] = make_int4(e, (int)(s + p), (int)(s + min(c, p + RV_MOE_TOK_CHUNK)), 0);
        n++;
      }
      s += c;
    }
    start[d.E] = s;
    if (n > B.max_units) rv_dev_fail(RV_ERR_LENGTH_MISMATCH);
    *B.n_units = min(n, B.max_units);
  }
  __syncthreads();
  for (int e = threadIdx.x; e <= d.E; e += blockDim.x) {
    B.index_start[e] = start[e];
    if (e < d.E) {
      cursor[e] = start[e];
      B.counts[e] = 0;  // ready for the next call
    }
  }
  __syncthreads();
  const int pairs = B.T * d.K;
  if (start[d.E] != (uint32_t)pairs) rv_dev_fail(RV_ERR_LENGTH_MISMATCH);  // stale counts
  for (int p = threadIdx.x; p < pairs; p += blockDim.x) {
    const uint32_t e = B.ids[p];
    if (e >= (uint32_t)d.E) {
      rv_dev_fail(RV_ERR_ROUTED_OUT_OF_RANGE);
      continue;
    }
    const uint32_t pos = atomicAdd(&cursor[e], 1u);
    if (pos < (uint32_t)pairs) B.index[pos] = (uint32_t)p;
    else rv_dev_fail(RV_ERR_LENGTH_MISMATCH);
  }
}

// ------------------------------------------------- gate/up + SwiGLU + Q8_K
// grid = (max_units, M / RV_GU_ROWS), block = 256 threads:
// thread (part, row, lane) = (tid/128, (tid/8)%16, tid%8).
template <int FMT>
__global__ void __launch_bounds__(256) k_gate_up(MoeDims d, MoeBufs B, MoeWeights W) {
  extern __shared__ __align__(16) uint8_t sm[];
  constexpr int R = RV_GU_ROWS, MT = RV_MOE_MT;
  constexpr int BB = FMT == RV_Q4_K ? 144 : FMT == RV_Q5_K ? 176 : 210;
  const int u = blockIdx.x, tile = blockIdx.y;
  if (u >= *B.n_units) return;
  const int4 unit = B.units[u];
  const int e = unit.x, p0 = unit.y, p1 = unit.z;
  uint64_t *bar = (uint64_t *)sm;
  __shared__ int s_last;
  const size_t wtile = (size_t)R * W.gu_row_bytes;
  uint8_t *wsm = sm + 16;                              // [2][R][row]
  uint8_t *asm_ = wsm + ((2 * wtile + 15) & ~(size_t)15) + 16;  // [MT][act_stride]
  float *gu = (float *)(asm_ + MT * d.act_stride + 16);        // [2][R][MT]
  const uint8_t *blob = W.base + (size_t)e * W.stride;
  const uint8_t *gsrc = blob + W.gate_off + (size_t)tile * wtile;
  const uint8_t *usrc = blob + W.up_off + (size_t)tile * wtile;
  const bool wbulk = rv_bulk_ok(gsrc, wsm, wtile) && rv_bulk_ok(usrc, wsm + wtile, wtile);
  const bool abulk = rv_bulk_ok(B.acts, asm_, d.act_stride);
  if (threadIdx.x == 0) mbar_init(bar, 1);
  __syncthreads();
  if (!wbulk) {
    rv_copy_bytes_block(wsm, gsrc, wtile);
    rv_copy_bytes_block(wsm + wtile, usrc, wtile);
  }
  const int part = threadIdx.x >> 7, r = (threadIdx.x >> 3) & 15, lane = threadIdx.x & 7;
  const uint8_t *wrow = wsm + (size_t)part * wtile + (size_t)r * W.gu_row_bytes;
  uint32_t phase = 0;
  bool ok = true;
  for (int c0 = p0; c0 < p1; c0 += MT) {
    const int mt = min(MT, p1 - c0);
    __syncthreads();
    if (threadIdx.x == 0 && (abulk || (c0 == p0 && wbulk))) {
      fence_proxy_async();
      uint32_t tx = 0;
      if (c0 == p0 && wbulk) tx += (uint32_t)(2 * wtile);
      if (abulk) tx += (uint32_t)(mt * d.act_stride);
      mbar_arrive_expect_tx(bar, tx);
      if (c0 == p0 && wbulk) {
        bulk_g2s(wsm, gsrc, (uint32_t)wtile, bar);
        bulk_g2s(wsm + wtile, usrc, (uint32_t)wtile, bar);
      }
      if (abulk)
        for (int m = 0; m < mt; m++) {
          const uint32_t tok = B.index[c0 + m] / (uint32_t)d.K;
          bulk_g2s(asm_ + (size_t)m * d.act_stride, B.acts + (size_t)tok * d.act_stride,
                   (uint32_t)d.act_stride, bar);
        }
    }
    if (!abulk)
      for (int m = 0; m < mt; m++) {
        const uint32_t tok = B.index[c0 + m] / (uint32_t)d.K;
        rv_copy_bytes_block(asm_ + (size_t)m * d.act_stride, B.acts + (size_t)tok * d.act_stride,
                            d.act_stride);
      }
    if (abulk || (c0 == p0 && wbulk)) {
      ok = mbar_wait_bounded(bar, phase);
      phase ^= 1;
    }
    __syncthreads();
    if (!ok) return;
    float acc[MT], accm[MT];
#pragma unroll
    for (int m = 0; m < MT; m++) acc[m] = accm[m] = 0.0f;
    for (int b = 0; b < d.hb; b++) {
      WBlock w;
      load_wblock<FMT>(wrow + (size_t)b * BB, lane, w);
#pragma unroll
      for (int m = 0; m < MT; m++)
        if (m < mt) lane_step<FMT>(w, asm_ + (size_t)m * d.act_stride + (size_t)b * 292, lane, acc[m], accm[m]);
    }
#pragma unroll
    for (int m = 0; m < MT; m++) {
      const float res = lane_reduce<FMT>(acc[m], accm[m]);
      if (lane == 0) gu[(part * R + r) * MT + m] = res;
    }
    __syncthreads();
    if (threadIdx.x < R * MT) {
      const int rr = threadIdx.x / MT, m = threadIdx.x % MT;
      if (m < mt) {
        const float h = swiglu_ref(gu[rr * MT + m], gu[(R + rr) * MT + m]);
        B.hbuf[(size_t)(c0 + m) * d.M + (size_t)tile * R + rr] = h;
      }
    }
  }
  // The last of the 256/R tiles of this 256-row block quantizes it.
  __threadfence();
  __syncthreads();
  const int qb = tile * R / 256;
  if (threadIdx.x == 0) {
    int *cnt = &B.tile_cnt[(size_t)u * d.mb + qb];
    const int old = atomicAdd(cnt, 1);
    s_last = (old == 256 / R - 1);
    if (s_last) *cnt = 0;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int warp = threadIdx.x >> 5, wl = threadIdx.x & 31;
  for (int pos = p0 + warp; pos < p1; pos += 8) {
    float v[8];
    const float *src = B.hbuf + (size_t)pos * d.M + (size_t)qb * 256 + 8 * wl;
#pragma unroll
    for (int k = 0; k < 8; k++) v[k] = __ldcg(src + k);
    q8k_quantize_warp(v, wl, B.acts_moe + (size_t)pos * d.amoe_stride + (size_t)qb * 292);
  }
}

// ------------------------------------------------------------- down
// grid = (max_units, H / RV_DOWN_ROWS), block = 256 = 32 rows x 8 lanes.
template <int FMT>
__global__ void __launch_bounds__(256) k_down(MoeDims d, MoeBufs B, MoeWeights W) {
  extern __shared__ __align__(16) uint8_t sm[];
  constexpr int R = RV_DOWN_ROWS, MT = RV_MOE_MT;
  constexpr int BB = FMT == RV_Q4_K ? 144 : FMT == RV_Q5_K ? 176 : 210;
  const int u = blockIdx.x, tile = blockIdx.y;
  if (u >= *B.n_units) return;
  const int4 unit = B.units[u];
  const int e = unit.x, p0 = unit.y, p1 = unit.z;
  uint64_t *bar = (uint64_t *)sm;
  const size_t wtile = (size_t)R * W.down_row_bytes;
  uint8_t *wsm = sm + 16;
  uint8_t *asm_ = wsm + ((wtile + 15) & ~(size_t)15) + 16;
  const uint8_t *dsrc = W.base + (size_t)e * W.stride + W.down_off + (size_t)tile * wtile;
  const bool wbulk = rv_bulk_ok(dsrc, wsm, wtile);
  const bool abulk = rv_bulk_ok(B.acts_moe, asm_, d.amoe_stride);
  if (threadIdx.x == 0) mbar_init(bar, 1);
  __syncthreads();
  if (!wbulk) rv_copy_bytes_block(wsm, dsrc, wtile);
  const int r = threadIdx.x >> 3, lane = threadIdx.x & 7;
  const uint8_t *wrow = wsm + (size_t)r * W.down_row_bytes;
  uint32_t phase = 0;
  bool ok = true;
  for (int c0 = p0; c0 < p1; c0 += MT) {
    const int mt = min(MT, p1 - c0);
    __syncthreads();
    const uint8_t *asrc = B.acts_moe + (size_t)c0 * d.amoe_stride;
    if (threadIdx.x == 0 && (abulk || (c0 == p0 && wbulk))) {
      fence_proxy_async();
      uint32_t tx = 0;
      if (c0 == p0 && wbulk) tx += (uint32_t)wtile;
      if (abulk) tx += (uint32_t)(mt * d.amoe_stride);
      mbar_arrive_expect_tx(bar, tx);
      if (c0 == p0 && wbulk) bulk_g2s(wsm, dsrc, (uint32_t)wtile, bar);
      if (abulk) bulk_g2s(asm_, asrc, (uint32_t)(mt * d.amoe_stride), bar);
    }
    if (!abulk) rv_copy_bytes_block(asm_, asrc, (size_t)mt * d.amoe_stride);
    if (abulk || (c0 == p0 && wbulk)) {
      ok = mbar_wait_bounded(bar, phase);
      phase ^= 1;
    }
    __syncthreads();
    if (!ok) return;
    float acc[MT], accm[MT];
#pragma unroll
    for (int m = 0; m < MT; m++) acc[m] = accm[m] = 0.0f;
    for (int b = 0; b < d.mb; b++) {
      WBlock w;
      load_wblock<FMT>(wrow + (size_t)b * BB, lane, w);
#pragma unroll
      for (int m = 0; m < MT; m++)
        if (m < mt) lane_step<FMT>(w, asm_ + (size_t)m * d.amoe_stride + (size_t)b * 292, lane, acc[m], accm[m]);
    }
#pragma unroll
    for (int m = 0; m < MT; m++) {
      const float res = lane_reduce<FMT>(acc[m], accm[m]);
      if (lane == 0 && m < mt) {
        const uint32_t pair = B.index[c0 + m];
        B.staged[(size_t)pair * d.H + (size_t)tile * R + r] = res;
      }
    }
  }
}

// ------------------------------------------------------------ combine
__global__ void k_combine(MoeDims d, MoeBufs B) {
  const int t = blockIdx.x;
  const int h = blockIdx.y * blockDim.x + threadIdx.x;
  if (h >= d.H) return;
  float acc = 0.0f;
  for (int k = 0; k < d.K; k++) {
    const size_t pair = (size_t)t * d.K + k;
    acc = __fadd_rn(acc, __fmul_rn(B.w[pair], B.staged[pair * d.H + h]));
  }
  float *res = B.residual + (size_t)t * d.H + h;
  *res = __fadd_rn(*res, acc);
}
