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
#include "rv_rowdot.cuh"
#include "rv_spec.cuh"

#define RV_MOE_MT 8          // tokens staged per pass
#define RV_MOE_TOK_CHUNK 64  // tokens per work unit

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
  int *route_cnt;          // [1] CTAs done in k_route_decode, zero between calls
  int *down_cnt;           // [H/8] units done per down row tile, zero between calls
  float2 *spec;            // [T][E] (lo, hi) bounds of the router logits (speculative decode)
  int T;
  int ms;                  // activation slots per CTA pass: min(T, RV_MOE_MT)
  int max_units;
  // tensor-core path (RV_MOE_TENSOR); null when the engine has none
  __half *xq, *xm;         // gate/up operand B: [padded rows][H] Q8_K levels, [..][hb*16] mins operand (f16, core-matrix order)
  float *xd;               // [padded rows][hb] Q8_K scales
  __half *hq, *hm;         // down operand B, the same for the Q8_K of the SwiGLU rows
  float *hdsc;             // [padded rows][mb]
  float *gu;               // [T*K][2M] gate | up outputs, CSR order
  int tc_groups;           // 8-row groups of the operand matrices (padded rows / 8)
  int4 *tc_units;          // [max_tc] (expert, pos0, pos1, padded pos0)
  int *n_tc;               // [1]
  uint32_t *tc_pstart;     // [E] padded first row of each expert
  int max_tc;
  uint8_t *tc_a;           // dequantized weight stages per expert (k_tc_predeq), null when the engine has none
  int *tc_apre;            // [E] 1: this call's k_tc_predeq wrote the expert's stages
  // Expert-parallel output (null otherwise): the down projection of
  // dispatch slot p goes to row ep_home[p] of the output buffer of the rank
  // that sent it, ep_out[p / ep_cap] (that rank's memory, mapped here).
  float *const *ep_out;
  const uint32_t *ep_home;
  uint32_t ep_cap;
};

// The row the down projection of dispatch slot `pair` is stored to: the
// engine's staged rows, or (expert parallel) the home rank's output row.
RV_DEVFN float *down_out_row(const MoeBufs &B, uint32_t pair, int H) {
  if (B.ep_out) return B.ep_out[pair / B.ep_cap] + (size_t)B.ep_home[pair] * H;
  return B.staged + (size_t)pair * H;
}

struct MoeWeights {
  const uint8_t *base;     // layer blob 0
  uint64_t stride, gate_off, up_off, down_off;
  size_t gu_row_bytes, down_row_bytes;
};

// The geometry as compile-time constants when GEO == 1 (Qwen3-30B-A3B:
// hidden 2048, moe 768, 128 experts, top-8), so the decode kernels' loops
// and index arithmetic fold; GEO == 0 keeps the engine's runtime values.
#define RV_GEO_QWEN3 1
template <int GEO>
RV_DEVFN MoeDims geo_dims(const MoeDims &d) {
  MoeDims g = d;
  if constexpr (GEO == RV_GEO_QWEN3) {
    g.H = 2048;
    g.M = 768;
    g.E = 128;
    g.K = 8;
    g.hb = 8;
    g.mb = 3;
    g.act_stride = 2336;
    g.amoe_stride = 880;
  }
  return g;
}

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

// ----------------------------------------------------------- top-k route
// Softmax, top-k and renormalization of token t's logits by one warp
// (forward.rs:2669-2705): f32 max, f64 exp of (x - max), f32 copy of each
// exponential, serial f64 sum in index order, f32 reciprocal scale; top-k by
// repeated argmax with a strict '>' scan (the lowest index wins a tie, the
// winner is blanked with -inf); renormalization by the in-order f32 sum.
// E <= 256 (8 per lane), K <= 16.  Writes ids/w and counts (any address
// space: global in k_route, shared in k_route_decode).
RV_DEVFN float ld_logit(const float *p) { return __isShared(p) ? *p : __ldcg(p); }

// lg: token t's E logits (global, written by other CTAs, or shared).
RV_DEVFN void route_token_warp(const MoeDims &d, const MoeBufs &B, int t, const float *lg, int lane, double *es,
                               int *counts) {
  float p[8];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int e = lane + 32 * j;
    p[j] = e < d.E ? ld_logit(lg + e) : -INFINITY;
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
      es[e] = ex;
      p[j] = __double2float_rn(ex);
    }
  }
  __syncwarp();
  // The reference sums the exponentials serially in index order.  A tree sum
  // of these <= 256 non-negative terms differs from it by < 2^-44 relative,
  // so unless 1/sum lies that close to a float rounding midpoint the f32
  // reciprocal is the same; otherwise lane 0 redoes the serial sum.
  double part = 0.0;
#pragma unroll
  for (int j = 0; j < 8; j++)
    if (lane + 32 * j < d.E) part = __dadd_rn(part, es[lane + 32 * j]);
#pragma unroll
  for (int o = 16; o; o >>= 1) part = __dadd_rn(part, __shfl_xor_sync(RV_FULL, part, o));
  double rinv = __drcp_rn(part);
  if (!f32_rounding_stable(rinv, 42)) {
    double sum = 0.0;
    if (lane == 0)
      for (int e = 0; e < d.E; e++) sum = __dadd_rn(sum, es[e]);
    rinv = __drcp_rn(__shfl_sync(RV_FULL, sum, 0));
  }
  const float inv = __double2float_rn(rinv);
#pragma unroll
  for (int j = 0; j < 8; j++) p[j] = (lane + 32 * j) < d.E ? __fmul_rn(p[j], inv) : -INFINITY;
  uint32_t my_id = 0;
  float my_w = 0.0f, wsum = -0.0f;
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
    if (lane == k) {
      my_id = (uint32_t)be;
      my_w = bp;
    }
    wsum = __fadd_rn(wsum, bp);  // the in-order sum of the selected weights
#pragma unroll
    for (int j = 0; j < 8; j++)
      if (lane + 32 * j == be) p[j] = -INFINITY;
  }
  if (lane < d.K) {
    if (d.norm_topk) my_w = __fdiv_rn(my_w, wsum);
    B.ids[(size_t)t * d.K + lane] = my_id;
    B.w[(size_t)t * d.K + lane] = my_w;
    atomicAdd(&counts[my_id], 1);
  }
}

// The same routing for one token by a whole CTA of 128 threads, thread i
// owning experts i and i+128: block max, one f64 exponential per thread,
// tree sum with the serial fallback, then top-k by rank (the number of
// probabilities greater than p_e, or equal at a lower index) -- the order
// the repeated strict-'>' argmax produces whenever every probability is a
// number; otherwise warp 0 runs the warp version.  Scratch: es [256]
// doubles, ps [256] floats, sel [16] floats, red [8] doubles, flag.
template <int NT = 0>
RV_DEVFN void route_token_block(const MoeDims &d, const MoeBufs &B, int t, const float *lg, double *es, float *ps,
                                float *sel, double *red, int *counts, uint32_t *sids, const uint8_t *cand = nullptr,
                                int ncand = 0, const uint32_t *cmask = nullptr) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float x[2];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < 2; j++) {
    const int e = tid + 128 * j;
    x[j] = e < d.E ? ld_logit(lg + e) : -INFINITY;
    if (e < d.E) mx = fmaxf(mx, x[j]);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(RV_FULL, mx, o));
  RV_TRACE_TAIL(0);
  float *redf = (float *)(red + 4);
  if (lane == 0) redf[warp] = mx;
  cta_sync<NT>();
  mx = fmaxf(fmaxf(redf[0], redf[1]), fmaxf(redf[2], redf[3]));
  RV_TRACE_TAIL(1);
  const double dmx = (double)mx;
  double part = 0.0;
  float pf[2];
#pragma unroll
  for (int j = 0; j < 2; j++) {
    const int e = tid + 128 * j;
    pf[j] = -INFINITY;
    if (e < d.E) {
      const double ex = exp(__dsub_rn((double)x[j], dmx));
      es[e] = ex;
      pf[j] = __double2float_rn(ex);
      part = __dadd_rn(part, ex);
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) part = __dadd_rn(part, __shfl_xor_sync(RV_FULL, part, o));
  RV_TRACE_TAIL(2);
  cta_sync<NT>();  // redf reads done, es complete
  if (lane == 0) red[warp] = part;
  cta_sync<NT>();
  RV_TRACE_TAIL(3);
  // Any order of these <= 256 non-negative terms is within 2^-44 relative of
  // the reference's serial sum; recompute serially when 1/sum is that close
  // to a float rounding midpoint.
  double rinv = __drcp_rn(__dadd_rn(__dadd_rn(red[0], red[1]), __dadd_rn(red[2], red[3])));
  if (!f32_rounding_stable(rinv, 42)) {
    double sum = 0.0;
    for (int e = 0; e < d.E; e++) sum = __dadd_rn(sum, es[e]);
    rinv = __drcp_rn(sum);
  }
  const float inv = __double2float_rn(rinv);
  bool finite = true;
#pragma unroll
  for (int j = 0; j < 2; j++) {
    const int e = tid + 128 * j;
    if (e < 256) {
      const float p = e < d.E ? __fmul_rn(pf[j], inv) : -INFINITY;
      ps[e] = p;
      if (e < d.E && !(p == p && p != INFINITY && p != -INFINITY)) finite = false;
    }
  }
  const bool all_finite = cta_sync_and<NT>(finite);
  RV_TRACE_TAIL(4);
  if (!all_finite) {
    if (warp == 0) route_token_warp(d, B, t, lg, lane, es, counts);
    cta_sync<NT>();
    if (tid < d.K) sids[t * d.K + tid] = __ldcg(B.ids + (size_t)t * d.K + tid);
    cta_sync<NT>();
    return;
  }
  if (cand) {
    // Only the listed experts can be in the top-k, so ranking them among
    // themselves gives the same order (checked below).
    for (int ci = tid; ci < ncand; ci += 128) {
      const int e = cand[ci];
      const float p = ps[e];
      int rank = 0;
      for (int i = 0; i < ncand; i++) {
        const int f = cand[i];
        const float q = ps[f];
        rank += (q > p) | ((q == p) & (f < e));
      }
      if (rank < d.K) {
        B.ids[(size_t)t * d.K + rank] = (uint32_t)e;
        sids[t * d.K + rank] = (uint32_t)e;
        sel[rank] = p;
        atomicAdd(&counts[e], 1);
      }
    }
  } else
#pragma unroll
  for (int j = 0; j < 2; j++) {
    const int e = tid + 128 * j;
    if (e < d.E) {
      const float p = ps[e];
      // ps is padded with -inf to a multiple of 16 entries: 16 independent
      // compares per step, four vector loads.
      int r0 = 0, r1 = 0, r2 = 0, r3 = 0;
      for (int i = 0; i < d.E; i += 16) {
        const float4 a = *(const float4 *)(ps + i), b = *(const float4 *)(ps + i + 4);
        const float4 c = *(const float4 *)(ps + i + 8), f = *(const float4 *)(ps + i + 12);
        r0 += (a.x > p) + ((a.x == p) & (i + 0 < e)) + (a.y > p) + ((a.y == p) & (i + 1 < e)) + (a.z > p) +
              ((a.z == p) & (i + 2 < e)) + (a.w > p) + ((a.w == p) & (i + 3 < e));
        r1 += (b.x > p) + ((b.x == p) & (i + 4 < e)) + (b.y > p) + ((b.y == p) & (i + 5 < e)) + (b.z > p) +
              ((b.z == p) & (i + 6 < e)) + (b.w > p) + ((b.w == p) & (i + 7 < e));
        r2 += (c.x > p) + ((c.x == p) & (i + 8 < e)) + (c.y > p) + ((c.y == p) & (i + 9 < e)) + (c.z > p) +
              ((c.z == p) & (i + 10 < e)) + (c.w > p) + ((c.w == p) & (i + 11 < e));
        r3 += (f.x > p) + ((f.x == p) & (i + 12 < e)) + (f.y > p) + ((f.y == p) & (i + 13 < e)) + (f.z > p) +
              ((f.z == p) & (i + 14 < e)) + (f.w > p) + ((f.w == p) & (i + 15 < e));
      }
      const int rank = r0 + r1 + r2 + r3;
      if (rank < d.K) {
        B.ids[(size_t)t * d.K + rank] = (uint32_t)e;
        sids[t * d.K + rank] = (uint32_t)e;
        sel[rank] = p;
        atomicAdd(&counts[e], 1);
      }
    }
  }
  RV_TRACE_TAIL(5);
  cta_sync<NT>();
  RV_TRACE_TAIL(6);
  if (cand) {
    // No unlisted expert beats the k-th selected one.
    const float pk = sel[d.K - 1];
    const uint32_t ek = sids[t * d.K + d.K - 1];
#pragma unroll
    for (int j = 0; j < 2; j++) {
      const int e = tid + 128 * j;
      if (e < d.E && !((cmask[e >> 5] >> (e & 31)) & 1u) && (ps[e] > pk || (ps[e] == pk && (uint32_t)e < ek)))
        rv_dev_fail(RV_ERR_ROUTED_OUT_OF_RANGE);
    }
  }
  if (tid < d.K) {
    float wsum = -0.0f;  // the in-order sum of the selected weights
    for (int k = 0; k < d.K; k++) wsum = __fadd_rn(wsum, sel[k]);
    const float w = d.norm_topk ? __fdiv_rn(sel[tid], wsum) : sel[tid];
    B.w[(size_t)t * d.K + tid] = w;
  }
  cta_sync<NT>();
  RV_TRACE_TAIL(7);
}

__global__ void __launch_bounds__(128) k_route(MoeDims d, MoeBufs B) {
  __shared__ double es[4][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 4 + warp;
  if (t >= B.T) return;
  route_token_warp(d, B, t, B.logits + (size_t)t * d.E, lane, es[warp], B.counts);
}

// ----------------------------------------------------------- dispatch
// CSR inverse index (prefill.rs:2536-2580) and the work units, built by one
// CTA from per-expert counts in shared memory: warp 0 scans the counts and
// the unit counts, every thread writes units, then the (token, slot) pairs
// are placed by expert.  s_cnt/s_cur: [256] ints, s_st/s_us: [257].
// sparse: dispatch slots whose expert id is ~0 are empty and skipped.
// slot_n (shared memory, or null): the pairs form n_sources ranges of
// slot_cap slots of which the first slot_n[s] are filled; only those are
// placed.
RV_DEVFN void build_index_cta(const MoeDims &d, const MoeBufs &B, int *s_cnt, uint32_t *s_st,
                              uint32_t *s_cur, int *s_us, bool sparse = false, const uint32_t *slot_n = nullptr,
                              int n_sources = 0, int slot_cap = 0) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pairs = B.T * d.K;
  if (warp == 0) {
    int c[8], u[8], sc = 0, su = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const int e = lane * 8 + i;
      c[i] = e < d.E ? s_cnt[e] : 0;
      u[i] = (c[i] + RV_MOE_TOK_CHUNK - 1) / RV_MOE_TOK_CHUNK;
      sc += c[i];
      su += u[i];
    }
    int xc = sc, xu = su;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int yc = __shfl_up_sync(RV_FULL, xc, o), yu = __shfl_up_sync(RV_FULL, xu, o);
      if (lane >= o) {
        xc += yc;
        xu += yu;
      }
    }
    const int tc = __shfl_sync(RV_FULL, xc, 31), tu = __shfl_sync(RV_FULL, xu, 31);
    xc -= sc;
    xu -= su;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const int e = lane * 8 + i;
      if (e < d.E) {
        s_st[e] = (uint32_t)xc;
        s_cur[e] = (uint32_t)xc;
        s_us[e] = xu;
      }
      xc += c[i];
      xu += u[i];
    }
    if (lane == 0) {
      s_st[d.E] = (uint32_t)tc;
      s_us[d.E] = tu;
      if ((sparse ? tc > pairs : tc != pairs) || tu > B.max_units) rv_dev_fail(RV_ERR_LENGTH_MISMATCH);
      *B.n_units = min(tu, B.max_units);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e <= d.E; e += blockDim.x) B.index_start[e] = s_st[e];
  for (int e = threadIdx.x; e < d.E; e += blockDim.x) {
    const int c = s_cnt[e];
    int u = s_us[e];
    for (int p = 0; p < c; p += RV_MOE_TOK_CHUNK, u++)
      if (u < B.max_units)
        B.units[u] = make_int4(e, (int)s_st[e] + p, (int)s_st[e] + min(c, p + RV_MOE_TOK_CHUNK), 0);
  }
  if (slot_n) {  // only the filled slots of each source's range
    __syncthreads();
    for (int s = 0; s < n_sources; s++)
      for (int i = threadIdx.x; i < (int)slot_n[s]; i += blockDim.x) {
        const int p = s * slot_cap + i;
        const uint32_t e = B.ids[p];
        if (e >= (uint32_t)d.E) continue;  // dropped when laid out
        const uint32_t pos = atomicAdd(&s_cur[e], 1u);
        if (pos < (uint32_t)pairs) B.index[pos] = (uint32_t)p;
        else rv_dev_fail(RV_ERR_LENGTH_MISMATCH);
      }
    return;
  }
  for (int p = threadIdx.x; p < pairs; p += blockDim.x) {
    const uint32_t e = B.ids[p];
    if (e >= (uint32_t)d.E) {
      if (!(sparse && e == ~0u)) rv_dev_fail(RV_ERR_ROUTED_OUT_OF_RANGE);
      continue;
    }
    const uint32_t pos = atomicAdd(&s_cur[e], 1u);
    if (pos < (uint32_t)pairs) B.index[pos] = (uint32_t)p;
    else rv_dev_fail(RV_ERR_LENGTH_MISMATCH);
  }
}

// The dispatch index for at most 32 pairs (decode): positions in expert
// order (pairs of one expert in pair order), per-expert CSR starts, one
// work unit per distinct expert.  sids: the pairs' expert ids in shared
// memory.
RV_DEVFN void build_index_small(const MoeDims &d, const MoeBufs &B, const uint32_t *sids) {
  const int P = B.T * d.K;
  const int tid = threadIdx.x;
  for (int e = tid; e <= d.E; e += blockDim.x) {
    int below = 0;
    for (int q = 0; q < P; q++) below += sids[q] < (uint32_t)e;
    B.index_start[e] = (uint32_t)below;
  }
  if (tid < 32) {
    const int p = tid;
    const uint32_t e = p < P ? sids[p] : 0xFFFFFFFFu;
    int pos = 0, cnt = 0;
    bool first = true;
    for (int q = 0; q < P; q++) {
      const uint32_t eq = __shfl_sync(RV_FULL, e, q);
      pos += (eq < e) | ((eq == e) & (q < p));
      cnt += eq == e;
      first = first && !((eq == e) & (q < p));
    }
    const unsigned firsts = __ballot_sync(RV_FULL, p < P && first);
    int u = 0;  // distinct experts below e
    for (int q = 0; q < P; q++) {
      const uint32_t eq = __shfl_sync(RV_FULL, e, q);
      u += ((firsts >> q) & 1u) && eq < e;
    }
    if (p < P) {
      B.index[pos] = (uint32_t)p;
      if (first) B.units[u] = make_int4((int)e, pos, pos + cnt, 0);
    }
    if (p == 0) *B.n_units = __popc(firsts);
  }
}

// Large-T dispatch: counts come from k_route's global atomics and are
// cleared here for the next call.
__global__ void __launch_bounds__(1024) k_index(MoeDims d, MoeBufs B) {
  __shared__ int s_cnt[256];
  __shared__ uint32_t s_st[257], s_cur[256];
  __shared__ int s_us[257];
  for (int e = threadIdx.x; e < 256; e += blockDim.x) s_cnt[e] = e < d.E ? B.counts[e] : 0;
  __syncthreads();
  for (int e = threadIdx.x; e < d.E; e += blockDim.x) B.counts[e] = 0;
  build_index_cta(d, B, s_cnt, s_st, s_cur, s_us);
}

// ------------------------------------------------------- decode routing
// Everything before the experts for T <= RV_SMALL_T tokens in one launch:
// grid = E CTAs of four warps; CTA e owns expert e (one serial chain per SM,
// so no two chains compete for an SM's issue slots).  Each CTA stages its
// router row and the norm weight (before waiting on the previous kernel:
// they do not depend on it) and the T residual rows with bulk copies, the
// four warps compute the RMSNorm of every token, and lane t of warp 0 runs
// the serial f32 chain of logit (t, e) from shared memory.  The last CTA to finish writes normed
// and its Q8_K, routes every token and builds the dispatch index.
#define RV_SMALL_T 8
// dot_f32 (forward.rs:1231-1237): acc = acc + a[k]*b[k] for k in order, no
// FMA.  The adds form one dependent chain; the products of the next 32
// elements are formed between the adds of the current 32 (and their
// operands loaded one block earlier), so the chain runs near the add
// latency.  n4 (float4 count) must be a multiple of 8.
RV_DEVFN float serial_dot_f32(const float4 *a, const float4 *b, int n4) {
  float acc = 0.0f;
  float p[32];
  float4 ra[8], rb[8];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    ra[j] = a[j];
    rb[j] = b[j];
  }
#pragma unroll
  for (int j = 0; j < 8; j++) {
    p[4 * j + 0] = __fmul_rn(ra[j].x, rb[j].x);
    p[4 * j + 1] = __fmul_rn(ra[j].y, rb[j].y);
    p[4 * j + 2] = __fmul_rn(ra[j].z, rb[j].z);
    p[4 * j + 3] = __fmul_rn(ra[j].w, rb[j].w);
  }
  const int k1 = 8 < n4 ? 8 : 0;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    ra[j] = a[k1 + j];
    rb[j] = b[k1 + j];
  }
  for (int k = 8; k <= n4; k += 8) {
    const int kn = k + 8 < n4 ? k + 8 : 0;
    float4 na[8], nb[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
      na[j] = a[kn + j];
      nb[j] = b[kn + j];
    }
    float q[32];
#pragma unroll
    for (int j = 0; j < 8; j++) {
      acc = __fadd_rn(acc, p[4 * j + 0]);
      q[4 * j + 0] = __fmul_rn(ra[j].x, rb[j].x);
      acc = __fadd_rn(acc, p[4 * j + 1]);
      q[4 * j + 1] = __fmul_rn(ra[j].y, rb[j].y);
      acc = __fadd_rn(acc, p[4 * j + 2]);
      q[4 * j + 2] = __fmul_rn(ra[j].z, rb[j].z);
      acc = __fadd_rn(acc, p[4 * j + 3]);
      q[4 * j + 3] = __fmul_rn(ra[j].w, rb[j].w);
    }
#pragma unroll
    for (int j = 0; j < 32; j++) p[j] = q[j];
#pragma unroll
    for (int j = 0; j < 8; j++) {
      ra[j] = na[j];
      rb[j] = nb[j];
    }
  }
  return acc;
}

// RMSNorm (norm.rs:17-60) of T rows held in shared memory at stride
// xstride, in place, by a 128-thread CTA.  The f64 sum of squares is split
// over the four warps (each row in four quarters); any summation order lies
// within the 2^-38 bound f32_rounding_stable checks, and the serial order
// is recomputed when the f32 result is not stable.  Then x = (x * inv) * w.
// red: [T][4] doubles, s_inv: [T] floats, both shared.
template <int NT = 0>
RV_DEVFN void norm_rows_cta(const MoeDims &d, int T, float *xs, int xstride, const float *nw, double *red,
                            float *s_inv) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = d.H / 4;  // elements per warp per token
  for (int t = 0; t < T; t++) {
    const float *x = xs + t * xstride + warp * q;
    double p0 = 0.0, p1 = 0.0, p2 = 0.0, p3 = 0.0;
    for (int k = 4 * lane; k < q; k += 128) {
      const float4 v = *(const float4 *)(x + k);
      // (double)v * (double)v is exact, so the fused form adds the same value.
      p0 = __fma_rn((double)v.x, (double)v.x, p0);
      p1 = __fma_rn((double)v.y, (double)v.y, p1);
      p2 = __fma_rn((double)v.z, (double)v.z, p2);
      p3 = __fma_rn((double)v.w, (double)v.w, p3);
    }
    double part = __dadd_rn(__dadd_rn(p0, p1), __dadd_rn(p2, p3));
#pragma unroll
    for (int o = 16; o; o >>= 1) part = __dadd_rn(part, __shfl_xor_sync(RV_FULL, part, o));
    if (lane == 0) red[4 * t + warp] = part;
  }
  RV_PHASE_ANY_T0(0, 6);
  cta_sync<NT>();
  if (threadIdx.x < T) {
    const int t = threadIdx.x;
    const double sum = __dadd_rn(__dadd_rn(red[4 * t], red[4 * t + 1]), __dadd_rn(red[4 * t + 2], red[4 * t + 3]));
    // The reference rounds sum/n, + eps, sqrt and 1/x one by one in f64;
    // the f64 reciprocal square root of the mean lies within a few ulps
    // (2^-50 relative) of that, far inside the 2^-38 the check allows.
    const double r = rsqrt(__dadd_rn(__dmul_rn(sum, 1.0 / (double)d.H), (double)d.eps));
    float inv = __double2float_rn(r);
    if (!f32_rounding_stable(r, 38)) {
      const float *x = xs + t * xstride;
      double ser = 0.0;  // the reference's serial order
      for (int k = 0; k < d.H; k++) {
        const double v = (double)x[k];
        ser = __dadd_rn(ser, __dmul_rn(v, v));
      }
      inv = rms_inv_from_sum(ser, (size_t)d.H, d.eps);
    }
    s_inv[t] = inv;
  }
  RV_PHASE_ANY_T0(0, 9);
  cta_sync<NT>();
  for (int t = 0; t < T; t++) {
    float4 *x = (float4 *)(xs + t * xstride);
    const float inv = s_inv[t];
    for (int k = threadIdx.x; k < d.H / 4; k += (NT ? NT : (int)blockDim.x)) {
      float4 v = x[k];
      const float4 w = ((const float4 *)nw)[k];
      v.x = __fmul_rn(__fmul_rn(v.x, inv), w.x);
      v.y = __fmul_rn(__fmul_rn(v.y, inv), w.y);
      v.z = __fmul_rn(__fmul_rn(v.z, inv), w.z);
      v.w = __fmul_rn(__fmul_rn(v.w, inv), w.w);
      x[k] = v;
    }
  }
  cta_sync<NT>();
}

__global__ void __launch_bounds__(128) k_route_decode(MoeDims d, MoeBufs B) {
  extern __shared__ __align__(16) uint8_t sm[];
  __shared__ double es[4][256];
  __shared__ int s_cnt[256];
  __shared__ uint32_t s_st[257], s_cur[256];
  __shared__ int s_us[257];
  __shared__ int s_last;
  __shared__ float s_inv[RV_SMALL_T];
  RV_PHASE(0, 0);
  const int T = B.T, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e0 = blockIdx.x;
  const int xstride = d.H + 4;  // padded rows: conflict-free per-lane reads
  uint64_t *bar = (uint64_t *)sm;                // [2]: router rows + norm weight, residual rows
  float *rows = (float *)(sm + 16);              // [H] router row e
  float *nw = rows + d.H;                        // [H] ffn_norm weight
  float *xs = nw + d.H;                          // [T][H + 4]
  double *red = (double *)(xs + T * xstride);    // [T][4] per-warp partial sums
  const int n_rows = 1;
  const float *rsrc = B.router + (size_t)e0 * d.H;
  const size_t rbytes = (size_t)n_rows * d.H * 4;
  const bool rbulk = rv_bulk_ok(rsrc, rows, rbytes) && rv_bulk_ok(B.ffn_norm, nw, (size_t)d.H * 4);
  const bool xbulk = rv_bulk_ok(B.residual, xs, (size_t)d.H * 4);
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    mbar_init(bar + 1, 1);
    if (rbulk) {
      mbar_arrive_expect_tx(bar, (uint32_t)(rbytes + (size_t)d.H * 4));
      bulk_g2s(rows, rsrc, (uint32_t)rbytes, bar);
      bulk_g2s(nw, B.ffn_norm, (uint32_t)(d.H * 4), bar);
    }
  }
  if (!rbulk) {
    for (size_t k = threadIdx.x; k < (size_t)n_rows * d.H; k += blockDim.x) rows[k] = rsrc[k];
    for (int k = threadIdx.x; k < d.H; k += blockDim.x) nw[k] = B.ffn_norm[k];
  }
  pdl_wait();  // the residual is the previous kernel's output
  RV_PHASE(0, 1);
  if (threadIdx.x == 0 && xbulk) {
    mbar_arrive_expect_tx(bar + 1, (uint32_t)(T * d.H * 4));
    for (int t = 0; t < T; t++)
      bulk_g2s(xs + t * xstride, B.residual + (size_t)t * d.H, (uint32_t)(d.H * 4), bar + 1);
  }
  if (!xbulk)
    for (int t = 0; t < T; t++)
      for (int k = threadIdx.x; k < d.H; k += blockDim.x) xs[t * xstride + k] = B.residual[(size_t)t * d.H + k];
  __syncthreads();
  if (xbulk && !mbar_wait_bounded(bar + 1, 0)) return;
  if (rbulk && !mbar_wait_bounded(bar, 0)) return;
  RV_PHASE(0, 2);
  norm_rows_cta(d, T, xs, xstride, nw, red, s_inv);
  // The Q8_K rows of the normed tokens and the normed tap do not depend on
  // the routing: CTA e's warps 1-3 write block e (of T*hb) while warp 0
  // runs the router chain.
  if (warp > 0) {
    for (int tb = e0 + (int)gridDim.x * (warp - 1); tb < T * d.hb; tb += 3 * (int)gridDim.x) {
      const int t = tb / d.hb, b = tb % d.hb;
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; e++) v[e] = xs[t * xstride + b * 256 + 8 * lane + e];
      q8k_quantize_warp(v, lane, B.acts + (size_t)t * d.act_stride + (size_t)b * 292);
#pragma unroll
      for (int e = 0; e < 8; e++) B.normed[(size_t)t * d.H + b * 256 + 8 * lane + e] = v[e];
    }
  }
  RV_PHASE(0, 3);
  RV_PHASE(0, 4);
  // Router logits: acc = acc + router[e][k] * normed[t][k], k = 0..H-1.
  if (warp < n_rows && lane < T)
    B.logits[(size_t)lane * d.E + e0 + warp] =
        serial_dot_f32((const float4 *)(rows + warp * d.H), (const float4 *)(xs + lane * xstride), d.H / 4);
  RV_PHASE(0, 5);
  // The expert kernel may launch now (it waits for this grid's completion
  // before reading the routing): its CTAs are resident when routing ends.
  pdl_trigger();
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int old = atomicAdd(B.route_cnt, 1);
    s_last = old == (int)gridDim.x - 1;
    if (s_last) *B.route_cnt = 0;
  }
  __syncthreads();
  if (!s_last) return;
  RV_PHASE(0, 6);
  __threadfence();
  for (int e = threadIdx.x; e < 256; e += blockDim.x) s_cnt[e] = 0;
  __syncthreads();
  // Routing: one or two tokens by the whole CTA, more by one warp each.
  __shared__ uint32_t s_ids[32];
  if (T <= 2) {
    __shared__ __align__(16) float s_ps[256];
    __shared__ float s_sel[16];
    __shared__ double s_red[8];
    for (int t = 0; t < T; t++)
      route_token_block(d, B, t, B.logits + (size_t)t * d.E, es[0], s_ps, s_sel, s_red, s_cnt, s_ids);
  } else {
    for (int t = warp; t < T; t += 4) route_token_warp(d, B, t, B.logits + (size_t)t * d.E, lane, es[warp], s_cnt);
    __syncthreads();
    for (int i = threadIdx.x; i < T * d.K && i < 32; i += blockDim.x) s_ids[i] = __ldcg(B.ids + i);
  }
  __syncthreads();
  RV_PHASE(0, 7);
  if (T * d.K <= 32) build_index_small(d, B, s_ids);
  else build_index_cta(d, B, s_cnt, s_st, s_cur, s_us);
  RV_PHASE(0, 8);
}

// ------------------------------------------- speculative decode routing
// k_route_spec: grid = ceil(E / 4) + ceil(T * hb / 4) CTAs of four warps;
// warp w of CTA c < ceil(E / 4) owns expert 4c + w, the later CTAs the Q8_K
// blocks.  Stages the CTA's four router rows and the norm weight
// (before waiting on the previous kernel), then the T residual rows;
// RMSNorm of every token; the f32 interval of logit (t, e) for every token
// (spec_bounds_warp); the Q8_K rows and the normed tap, block b of token t
// by warp (t*hb + b) of the quantizing CTAs (measured: gate/up starts
// 1.2 us sooner, 895 against 867 tok/s, than when two of the expert CTAs
// also quantized).  Everything the expert kernels need before the exact
// router chains have run.
#define RV_SPEC_EPC 4  // experts per k_route_spec CTA
// The body of k_route_spec for CTA `cta` of `ncta` (128 threads, shared
// memory `sm`).  PDL: wait for the previous kernel before reading the
// residual and then let the next kernel launch (a kernel whose residual is
// already final passes false).  Returns false when a copy timed out.
template <bool PDL>
RV_DEVFN bool route_spec_cta(const MoeDims &d, const MoeBufs &B, uint8_t *sm, int cta, int ncta) {
  __shared__ float s_inv[RV_SMALL_T];
  __shared__ double s_red[4 * RV_SMALL_T];
  const int T = B.T, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // CTAs [0, nbc) bound RV_SPEC_EPC experts' logits each; any CTAs past
  // them only quantize the normed rows (so the grid's last CTA is not one
  // that does both).
  const int nbc = (d.E + RV_SPEC_EPC - 1) / RV_SPEC_EPC;
  const int e0 = cta * RV_SPEC_EPC, ne = cta < nbc ? min(RV_SPEC_EPC, d.E - e0) : 0;
  const int xstride = d.H + 4;
  uint64_t *bar = (uint64_t *)sm;                // [2]: router rows + norm weight, residual rows
  float *rows = (float *)(sm + 16);              // [4][H]
  float *nw = rows + RV_SPEC_EPC * d.H;          // [H] ffn_norm weight
  float *xs = nw + d.H;                          // [T][H + 4]
  const float *rsrc = B.router + (size_t)e0 * d.H;
  const bool rbulk = rv_bulk_ok(rsrc, rows, (size_t)ne * d.H * 4) && rv_bulk_ok(B.ffn_norm, nw, (size_t)d.H * 4);
  const bool xbulk = rv_bulk_ok(B.residual, xs, (size_t)d.H * 4);
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    mbar_init(bar + 1, 1);
    if (rbulk) {
      mbar_arrive_expect_tx(bar, (uint32_t)((ne + 1) * d.H * 4));
      if (ne > 0) bulk_g2s(rows, rsrc, (uint32_t)(ne * d.H * 4), bar);
      bulk_g2s(nw, B.ffn_norm, (uint32_t)(d.H * 4), bar);
    }
  }
  if (!rbulk) {
    for (int k = threadIdx.x; k < ne * d.H; k += blockDim.x) rows[k] = rsrc[k];
    for (int k = threadIdx.x; k < d.H; k += blockDim.x) nw[k] = B.ffn_norm[k];
  }
  if constexpr (PDL) {
    pdl_wait();  // the residual is the previous kernel's output
    // The exact-chain kernel reads the residual without waiting: it may
    // launch only now.
    pdl_trigger();
  }
  RV_PHASE(0, 1);
  if (threadIdx.x == 0 && xbulk) {
    mbar_arrive_expect_tx(bar + 1, (uint32_t)(T * d.H * 4));
    for (int t = 0; t < T; t++)
      bulk_g2s(xs + t * xstride, B.residual + (size_t)t * d.H, (uint32_t)(d.H * 4), bar + 1);
  }
  if (!xbulk)
    for (int t = 0; t < T; t++)
      for (int k = threadIdx.x; k < d.H; k += blockDim.x) xs[t * xstride + k] = B.residual[(size_t)t * d.H + k];
  __syncthreads();
  bool ok = true;
  if (xbulk) ok = mbar_wait_bounded(bar + 1, 0);
  if (rbulk) ok = mbar_wait_bounded(bar, 0) && ok;
  if (!__syncthreads_and(ok)) return false;
  RV_PHASE(0, 2);
  RV_PHASE_CLK(0, 7);
  norm_rows_cta(d, T, xs, xstride, nw, s_red, s_inv);
  RV_PHASE(0, 3);
  RV_PHASE_CLK(0, 8);
  if (warp < ne)
    for (int t = 0; t < T; t++) {
      const float2 b = spec_bounds_warp(rows + (size_t)warp * d.H, xs + t * xstride, d.H, lane);
      if (lane == 0) B.spec[(size_t)t * d.E + e0 + warp] = b;
    }
  RV_PHASE(0, 4);
  const bool qcta = ncta > nbc;  // quantizing CTAs of their own
  if (qcta && cta < nbc) {
    RV_PHASE(0, 5);
    return true;
  }
  const int gw = (qcta ? cta - nbc : cta) * 4 + warp, nwg = (qcta ? ncta - nbc : ncta) * 4;
  for (int tb = gw; tb < T * d.hb; tb += nwg) {
    const int t = tb / d.hb, b = tb % d.hb;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; e++) v[e] = xs[t * xstride + b * 256 + 8 * lane + e];
    q8k_quantize_warp(v, lane, B.acts + (size_t)t * d.act_stride + (size_t)b * 292);
#pragma unroll
    for (int e = 0; e < 8; e++) B.normed[(size_t)t * d.H + b * 256 + 8 * lane + e] = v[e];
  }
  RV_PHASE(0, 5);
  return true;
}

template <int GEO>
__global__ void __launch_bounds__(128) k_route_spec(MoeDims dd, MoeBufs B) {
  const MoeDims d = geo_dims<GEO>(dd);
  extern __shared__ __align__(16) uint8_t sm[];
  RV_PHASE(0, 0);
  route_spec_cta<true>(d, B, sm, blockIdx.x, gridDim.x);
}

// k_route_chain: the exact router chains, CH experts per CTA (grid =
// ceil(E / CH), one cluster when CLUSTER), 160 threads.  Warps 0-3 stage
// the CTA's router rows, the residual rows and the norm weight, compute
// the RMSNorm themselves (the same arithmetic as k_route_spec, so the same
// bits) and run one serial f32 chain per (token, expert): thread i < T*CH
// owns logit (i / CH, blockIdx.x*CH + i % CH).  The logits are gathered in
// CTA 0 of the cluster through distributed shared memory (or, without a
// cluster, by the last CTA through global memory), which routes every token
// (f64 softmax, top-k, renormalization).  Warp 4 only gates the launch of
// the next (speculative gate/up) kernel: that kernel reads k_route_spec's
// output without waiting, so this grid triggers once k_route_spec has
// completed.  The residual was written by the previous layer, complete
// before k_route_spec triggered this launch.
#define RV_CHAIN_THREADS 160
template <bool CLUSTER, int GEO>
__global__ void __launch_bounds__(RV_CHAIN_THREADS) k_route_chain(MoeDims dd, MoeBufs B, int CH, MoeWeights W) {
  (void)W;  // the layer's expert slabs (unused: L2 prefetches from here delayed the pipeline)
  const MoeDims d = geo_dims<GEO>(dd);
  extern __shared__ __align__(16) uint8_t sm[];
  __shared__ double es[4][256];
  __shared__ int s_cnt[256];
  __shared__ uint32_t s_ids[32];
  __shared__ __align__(16) float s_ps[256];
  __shared__ float s_sel[16];
  __shared__ double s_red[8];
  __shared__ float s_inv[RV_SMALL_T];
  __shared__ double s_nred[4 * RV_SMALL_T];
  __shared__ __align__(16) float s_lg[CLUSTER ? RV_SPEC_MAX_T * 256 : 1];  // CTA 0: the gathered logits
  __shared__ __align__(8) uint64_t s_gbar;                                  // CTA 0: one arrival per logit
  __shared__ uint8_t s_cand[CLUSTER ? RV_SPEC_MAX_T * 256 : 1];             // CTA 0: speculated experts per token
  __shared__ int s_ncand[RV_SPEC_MAX_T];
  __shared__ uint32_t s_cmask[RV_SPEC_MAX_T * 8];
  __shared__ int s_last;
  RV_PHASE(5, 0);
  const int T = B.T, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int xstride = d.H + 4;
  const int ef = blockIdx.x * CH, ne = min(CH, d.E - ef);
  const bool lead = CLUSTER ? cluster_ctarank() == 0 : true;
  uint64_t *bar = (uint64_t *)sm;           // [2]: router rows, residual rows + norm weight
  float *rows = (float *)(sm + 16);         // [CH][H + 4]
  float *xs = rows + (size_t)CH * xstride;  // [T][H + 4]
  float *nw = xs + (size_t)T * xstride;     // [H]
  const bool rbulk = rv_bulk_ok(B.router + (size_t)ef * d.H, rows, (size_t)d.H * 4);
  const bool xbulk = rv_bulk_ok(B.residual, xs, (size_t)d.H * 4) && rv_bulk_ok(B.ffn_norm, nw, (size_t)d.H * 4);
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_init(bar + 1, 1);
    if (CLUSTER && lead) mbar_init(&s_gbar, (uint32_t)(T * d.E));
  }
  if constexpr (CLUSTER) cluster_sync_all();  // CTA 0's gather barrier exists before any arrival
  else __syncthreads();
  if (warp == 4) {
    pdl_wait();
    pdl_trigger();
    if (CLUSTER && lead) {
      // While the chains run: the speculated experts of every token, so
      // the routing below ranks only those (named barrier 2 hands them over).
      spec_candidates_warp(d.E, d.K, T, B.spec, s_cand, s_ncand, s_cmask, lane);
      __syncwarp();
      asm volatile("bar.arrive 2, %0;" ::"n"(RV_CHAIN_THREADS) : "memory");    }
    return;
  }
  if (tid == 0) {  // the residual and norm weight first: the norm needs them before the chains need the rows
    if (xbulk) {
      mbar_arrive_expect_tx(bar + 1, (uint32_t)((T + 1) * d.H * 4));
      for (int t = 0; t < T; t++)
        bulk_g2s(xs + (size_t)t * xstride, B.residual + (size_t)t * d.H, (uint32_t)(d.H * 4), bar + 1);
      bulk_g2s(nw, B.ffn_norm, (uint32_t)(d.H * 4), bar + 1);
    }
    if (rbulk) {
      mbar_arrive_expect_tx(bar, (uint32_t)(ne * d.H * 4));
      for (int r = 0; r < ne; r++)
        bulk_g2s(rows + (size_t)r * xstride, B.router + (size_t)(ef + r) * d.H, (uint32_t)(d.H * 4), bar);
    }
  }
  if (!rbulk)
    for (int r = 0; r < ne; r++)
      for (int k = tid; k < d.H; k += 128) rows[(size_t)r * xstride + k] = B.router[(size_t)(ef + r) * d.H + k];
  if (!xbulk) {
    for (int t = 0; t < T; t++)
      for (int k = tid; k < d.H; k += 128) xs[(size_t)t * xstride + k] = B.residual[(size_t)t * d.H + k];
    for (int k = tid; k < d.H; k += 128) nw[k] = B.ffn_norm[k];
  }
  cta_sync<128>();
  // Every compute thread takes the same exit, so no named barrier below
  // is left waiting for a thread that returned.
  bool ok = true;
  if (xbulk) ok = mbar_wait_bounded(bar + 1, 0);
  RV_PHASE(5, 1);
  if (!cta_sync_and<128>(ok)) return;
  norm_rows_cta<128>(d, T, xs, xstride, nw, s_nred, s_inv);
  if (rbulk) ok = mbar_wait_bounded(bar, 0);
  RV_PHASE(5, 2);
  if (!cta_sync_and<128>(ok)) return;
  float lg = 0.0f;
  int e_mine = -1, t_mine = 0;
  if (tid < T * CH) {
    const int t = tid / CH, el = tid % CH;
    if (el < ne) {
      e_mine = ef + el;
      t_mine = t;
      lg = serial_dot_f32((const float4 *)(rows + (size_t)el * xstride), (const float4 *)(xs + (size_t)t * xstride),
                          d.H / 4);
    }
  }
  if (e_mine >= 0) {
    B.logits[(size_t)t_mine * d.E + e_mine] = lg;
    if constexpr (CLUSTER) {
      st_cluster_f32(dsmem_addr(&s_lg[t_mine * d.E + e_mine], 0), lg);
      mbar_arrive_cluster(dsmem_addr(&s_gbar, 0));
    }
  }
  RV_PHASE(5, 3);
  const float *lgs;
  if constexpr (CLUSTER) {
    if (!lead) return;
    ok = mbar_wait_cluster_bounded(&s_gbar, 0);
    if (!cta_sync_and<128>(ok)) return;
    lgs = s_lg;
  } else {
    __threadfence();
    cta_sync<128>();
    if (tid == 0) {
      const int old = atomicAdd(B.route_cnt, 1);
      s_last = old == (int)gridDim.x - 1;
      if (s_last) *B.route_cnt = 0;
    }
    cta_sync<128>();
    if (!s_last) return;
    __threadfence();
    lgs = B.logits;
  }
  RV_PHASE(5, 4);
  for (int e = tid; e < 256; e += 128) s_cnt[e] = 0;
  if constexpr (CLUSTER) asm volatile("bar.sync 2, %0;" ::"n"(RV_CHAIN_THREADS) : "memory");
  else cta_sync<128>();
  if (T <= 2) {
    for (int t = 0; t < T; t++) {
      if constexpr (CLUSTER)
        route_token_block<128>(d, B, t, lgs + (size_t)t * d.E, es[0], s_ps, s_sel, s_red, s_cnt, s_ids,
                               s_cand + t * 256, s_ncand[t], s_cmask + t * 8);
      else
        route_token_block<128>(d, B, t, lgs + (size_t)t * d.E, es[0], s_ps, s_sel, s_red, s_cnt, s_ids);
    }
  } else {
    for (int t = warp; t < T; t += 4) route_token_warp(d, B, t, lgs + (size_t)t * d.E, lane, es[warp], s_cnt);
  }
  RV_PHASE(5, 5);
}

// Large-T router logits: CTA = 16 experts x 32 tokens; lane t of warp w
// runs the chains of token blockIdx.x*32+t with the four experts
// blockIdx.y*16+4w .. +3, so each token value read from shared memory feeds
// four chains (the router values are warp-wide broadcasts).  Router rows
// and normed rows are staged RV_RCHUNK floats at a time (bulk copies,
// double-buffered; token rows padded so the lanes' 16-byte reads hit
// distinct banks).  Each chain is dot_f32's (forward.rs:1231-1237): acc =
// acc + r[k]*x[k] for k ascending, separate multiply and add.
#define RV_RCHUNK 128
#define RV_REXP 16
__host__ __device__ constexpr size_t router_logits_smem() {
  return 16 + 2 * (size_t)(RV_REXP * RV_RCHUNK + 32 * (RV_RCHUNK + 4)) * 4;
}
__global__ void __launch_bounds__(128) k_router_logits(MoeDims d, MoeBufs B) {
  extern __shared__ __align__(16) uint8_t sm[];
  uint64_t *bar = (uint64_t *)sm;  // [2]
  const int xs_stride = RV_RCHUNK + 4;
  float *buf = (float *)(sm + 16);
  const int stage_floats = RV_REXP * RV_RCHUNK + 32 * xs_stride;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e0 = blockIdx.y * RV_REXP, t0 = blockIdx.x * 32;
  const int ne = min(RV_REXP, d.E - e0), nt = min(32, B.T - t0);
  const int nchunks = d.H / RV_RCHUNK;
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    mbar_init(bar + 1, 1);
  }
  __syncthreads();
  auto issue = [&](int c) {
    float *st = buf + (c & 1) * stage_floats;
    mbar_arrive_expect_tx(bar + (c & 1), (uint32_t)((ne + nt) * RV_RCHUNK * 4));
    for (int i = 0; i < ne; i++)
      bulk_g2s(st + i * RV_RCHUNK, B.router + (size_t)(e0 + i) * d.H + (size_t)c * RV_RCHUNK, RV_RCHUNK * 4,
               bar + (c & 1));
    for (int i = 0; i < nt; i++)
      bulk_g2s(st + RV_REXP * RV_RCHUNK + i * xs_stride, B.normed + (size_t)(t0 + i) * d.H + (size_t)c * RV_RCHUNK,
               RV_RCHUNK * 4, bar + (c & 1));
  };
  if (threadIdx.x == 0) {
    issue(0);
    if (nchunks > 1) issue(1);
  }
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  const bool live = lane < nt && 4 * warp < ne;
  for (int c = 0; c < nchunks; c++) {
    if (!mbar_wait_bounded(bar + (c & 1), (uint32_t)((c >> 1) & 1))) return;
    const float *st = buf + (c & 1) * stage_floats;
    if (live) {
      // Rows past ne were not staged: their chains compute on stale values
      // and are not stored.
      const float4 *r4 = (const float4 *)(st + 4 * warp * RV_RCHUNK);
      const float4 *x4 = (const float4 *)(st + RV_REXP * RV_RCHUNK + lane * xs_stride);
#pragma unroll 4
      for (int k = 0; k < RV_RCHUNK / 4; k++) {
        const float4 x = x4[k];
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const float4 r = r4[i * (RV_RCHUNK / 4) + k];
          acc[i] = __fadd_rn(acc[i], __fmul_rn(r.x, x.x));
          acc[i] = __fadd_rn(acc[i], __fmul_rn(r.y, x.y));
          acc[i] = __fadd_rn(acc[i], __fmul_rn(r.z, x.z));
          acc[i] = __fadd_rn(acc[i], __fmul_rn(r.w, x.w));
        }
      }
    }
    __syncthreads();  // stage (c & 1) consumed
    if (threadIdx.x == 0 && c + 2 < nchunks) {
      fence_proxy_async();
      issue(c + 2);
    }
  }
  if (lane < nt)
#pragma unroll
    for (int i = 0; i < 4; i++)
      if (4 * warp + i < ne) B.logits[(size_t)(t0 + lane) * d.E + e0 + 4 * warp + i] = acc[i];
}

// ------------------------------------------------- weight-tile staging
// Rows [r0, r0+n) of a matrix with `row_bytes` per row go to shared memory.
// Q4_K/Q5_K rows land at a padded stride (row_bytes + 16: 16-byte aligned
// blocks, conflict-free 128-bit reads), one bulk copy per row; Q6_K rows
// (630 bytes, only 2-byte aligned) land densely in one bulk copy when the
// range is 16-byte aligned.  Misaligned sources fall back to a cooperative
// byte copy into the same layout.  Returns the bytes that go through the
// bulk-copy engine on `bar` (issued by thread 0 when `issue`); 0 means the
// cooperative copy ran and a __syncthreads must follow.
template <int FMT>
RV_DEVFN size_t tile_stride(size_t row_bytes) {
  return FMT == RV_Q6_K ? row_bytes : row_bytes + 16;
}
template <int FMT>
RV_DEVFN uint32_t stage_rows(uint8_t *dst, const uint8_t *src, size_t row_bytes, int n, uint64_t *bar,
                             bool issue) {
  const size_t st = tile_stride<FMT>(row_bytes);
  if constexpr (FMT == RV_Q6_K) {
    if (rv_bulk_ok(src, dst, (size_t)n * row_bytes)) {
      if (issue && threadIdx.x == 0) bulk_g2s(dst, src, (uint32_t)(n * row_bytes), bar);
      return (uint32_t)(n * row_bytes);
    }
    if (issue) rv_copy_bytes_block(dst, src, (size_t)n * row_bytes);
    return 0;
  } else {
    if (rv_bulk_ok(src, dst, row_bytes)) {
      if (issue && threadIdx.x == 0)
        for (int r = 0; r < n; r++) bulk_g2s(dst + r * st, src + r * row_bytes, (uint32_t)row_bytes, bar);
      return (uint32_t)(n * row_bytes);
    }
    if (issue)
      for (size_t i = threadIdx.x; i < (size_t)n * row_bytes; i += blockDim.x)
        dst[(i / row_bytes) * st + i % row_bytes] = src[i];
    return 0;
  }
}

// ------------------------------------------------- gate/up + SwiGLU + Q8_K
// A CTA computes rows [tile*R, tile*R+R) of both gate and up of one unit's
// expert for all of the unit's positions, staged B.ms at a time.  G > 1:
// split mode (one token at a time, G lanes per row, NBG blocks each);
// G == 1: token mode (a thread per row, up to 8 tokens in flight).
// 2*R*G/32 warps.  Then SwiGLU with the host-libm exponential, and the last
// of the tiles of each 256-row block quantizes that block of every
// position.  tok(c): the token of position c.  phase: parity of the CTA's
// mbarrier, carried from unit to unit.  Returns false when a wait ran out.
template <int FMT, int G, int NBG, int R, typename TokOf>
RV_DEVFN bool gate_up_unit(const MoeDims &d, const MoeBufs &B, const MoeWeights &W, uint8_t *sm, int u, int e,
                           int p0, int p1, int tile, TokOf tok, uint32_t &phase, int *ready = nullptr,
                           int ready_stride = 1) {
  constexpr int MT = RV_MOE_MT, RPW = 32 / G, NW = 2 * R * G / 32;
  const int ms = B.ms;
  __shared__ int s_last;
  uint64_t *bar = (uint64_t *)sm;
  const size_t st = tile_stride<FMT>(W.gu_row_bytes);
  const size_t wtile = (size_t)R * st;
  uint8_t *wsm = sm + 16;                                       // [2][R][st]
  uint8_t *asm_ = wsm + ((2 * wtile + 15) & ~(size_t)15) + 16;  // [ms][act_stride]
  float *gu = (float *)(asm_ + ms * d.act_stride);              // [2][R][MT]
  const uint8_t *blob = W.base + (size_t)e * W.stride;
  const uint8_t *gsrc = blob + W.gate_off + (size_t)tile * R * W.gu_row_bytes;
  const uint8_t *usrc = blob + W.up_off + (size_t)tile * R * W.gu_row_bytes;
  const bool abulk = rv_bulk_ok(B.acts, asm_, d.act_stride);
  const uint32_t wtx = stage_rows<FMT>(wsm, gsrc, W.gu_row_bytes, R, bar, false) +
                       stage_rows<FMT>(wsm + wtile, usrc, W.gu_row_bytes, R, bar, false);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int part = warp / (NW / 2);  // warps [0, NW/2) gate, [NW/2, NW) up
  const int rsub = lane / G, g = lane % G;
  const int r = (warp % (NW / 2)) * RPW + rsub;  // row within the part
  const uint8_t *wrow = wsm + (size_t)part * wtile + (size_t)r * st;
  bool ok = true;
  for (int c0 = p0; c0 < p1; c0 += ms) {
    const int mt = min(ms, p1 - c0);
    __syncthreads();
    const bool first = c0 == p0;
    const uint32_t tx = (first ? wtx : 0u) + (abulk ? (uint32_t)(mt * d.act_stride) : 0u);
    if (threadIdx.x == 0 && tx) {
      fence_proxy_async();
      mbar_arrive_expect_tx(bar, tx);
    }
    if (first) {
      stage_rows<FMT>(wsm, gsrc, W.gu_row_bytes, R, bar, true);
      stage_rows<FMT>(wsm + wtile, usrc, W.gu_row_bytes, R, bar, true);
    }
    for (int m = 0; m < mt; m++) {
      const uint32_t t = tok(c0 + m);
      if (abulk) {
        if (threadIdx.x == 0)
          bulk_g2s(asm_ + (size_t)m * d.act_stride, B.acts + (size_t)t * d.act_stride, (uint32_t)d.act_stride,
                   bar);
      } else {
        rv_copy_bytes_block(asm_ + (size_t)m * d.act_stride, B.acts + (size_t)t * d.act_stride, d.act_stride);
      }
    }
    if (tx) {
      ok = mbar_wait_bounded(bar, phase);
      phase ^= 1;
    }
    __syncthreads();
    if (!ok) return false;
    RV_PHASE(1, 2);
    for (int m0 = 0; m0 < mt; m0 += MT) {
      const int mm = min(MT, mt - m0);
      if constexpr (G > 1) {
        for (int m = 0; m < mm; m++) {
          const float res = row_dot_split<FMT, G, NBG>(wrow, asm_ + (size_t)(m0 + m) * d.act_stride, g);
          if (g == G - 1) gu[(part * R + r) * MT + m] = res;
        }
      } else {
        float res[MT];
        row_dot_tokens<FMT, MT>(wrow, d.hb, asm_ + (size_t)m0 * d.act_stride, d.act_stride, mm, res);
#pragma unroll
        for (int m = 0; m < MT; m++)
          if (m < mm) gu[(part * R + r) * MT + m] = res[m];
      }
      RV_PHASE(1, 5);
      __syncthreads();
      for (int i = threadIdx.x; i < R * mm; i += blockDim.x) {
        const int rr = i / mm, m = i % mm;
        const float h = swiglu_ref(gu[rr * MT + m], gu[(R + rr) * MT + m]);
        B.hbuf[(size_t)(c0 + m0 + m) * d.M + (size_t)tile * R + rr] = h;
      }
      __syncthreads();
    }
  }
  RV_PHASE(1, 3);
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
  if (!s_last) return true;
  RV_PHASE(1, 4);
  __threadfence();
  const int nwarps = blockDim.x >> 5;
  for (int pos = p0 + warp; pos < p1; pos += nwarps) {
    float v[8];
    const float *src = B.hbuf + (size_t)pos * d.M + (size_t)qb * 256 + 8 * lane;
#pragma unroll
    for (int k = 0; k < 8; k++) v[k] = __ldcg(src + k);
    q8k_quantize_warp(v, lane, B.acts_moe + (size_t)pos * d.amoe_stride + (size_t)qb * 292);
  }
  if (ready) {  // one more 256-row block of this unit's SwiGLU rows is quantized
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) atomicAdd(&ready[(size_t)u * ready_stride], 1);
  }
  return true;
}

// grid = (units, M / R).  Dispatch from the index (SPEC false: launched as a
// programmatic dependent of the routing kernel) or from the speculated
// pairs (SPEC true: every CTA rebuilds them from the logit bounds and
// strides over the units).
template <int FMT, int G, int NBG, int R, bool SPEC, int GEO>
__global__ void __launch_bounds__(2 * R * G, 4) k_gate_up(MoeDims dd, MoeBufs B, MoeWeights W) {
  const MoeDims d = geo_dims<GEO>(dd);
  extern __shared__ __align__(16) uint8_t sm[];
  RV_PHASE(1, 0);
  const int tile = blockIdx.y;
  uint32_t phase = 0;
  if (threadIdx.x == 0) mbar_init((uint64_t *)sm, 1);
  if constexpr (SPEC) {
    // Reads only the bounds and activations of the routing kernel, which
    // completed before the exact-chain kernel ahead of this one passed its
    // wait, i.e. before this grid launched.  The down kernel may launch once
    // the set is rebuilt (before its own wait it too reads only the bounds):
    // measured 864 against 858 tok/s when it launched at this grid's start
    // (its early CTAs competed with the set rebuild), 814 when it launched
    // after the gate/up rows (too late to stage its weights).
    __shared__ SpecSmem ss;
    spec_build(d.E, d.K, B.T, B.spec, ss);
    pdl_trigger();
    RV_PHASE(1, 1);
    for (int u = blockIdx.x; u < ss.n_units; u += gridDim.x) {
      const int e = ss.uexp[u], p0 = ss.start[e];
      const uint32_t msk = ss.mask[e];
      if (!gate_up_unit<FMT, G, NBG, R>(d, B, W, sm, u, e, p0, p0 + __popc(msk), tile,
                                        [&](int c) { return (uint32_t)spec_nth_bit(msk, c - p0); }, phase))
        break;
    }
    // The down kernel waits for this grid only; one CTA waiting for the
    // exact-chain kernel makes this grid's completion imply that one's.
    if (blockIdx.x == 0 && blockIdx.y == 0) pdl_wait();
  } else {
    // The dispatch index and activations are the routing kernel's output.
    // The down kernel reads the index before its own wait, so it may launch
    // only once the routing grid has completed: trigger after the wait.
    pdl_wait();
    pdl_trigger();
    __syncthreads();
    const int u = blockIdx.x;
    if (u >= *B.n_units) return;
    RV_PHASE(1, 1);
    const int4 unit = B.units[u];
    gate_up_unit<FMT, G, NBG, R>(d, B, W, sm, u, unit.x, unit.y, unit.z, tile,
                                 [&](int c) { return B.index[c] / (uint32_t)d.K; }, phase);
  }
}

// ------------------------------------------------------------- down
// grid = (units, ceil(H / ROWS)), one warp per CTA (ROWS * G <= 32): ROWS
// rows of one unit's expert for all its positions.  Launched as a
// programmatic dependent of k_gate_up: the weight tile (which depends only
// on the dispatch) is requested before waiting for gate/up to finish.
// SPEC: the units are the speculated pairs (rebuilt from the logit bounds
// by every CTA), and only the positions the exact routing selected are
// stored.  With COMBINE, the last unit to finish a row tile also performs
// the fixed top-k-order reduction and residual add for those rows of every
// token (forward.rs:2744-2753); otherwise k_combine does it.
template <int FMT, int G, int NBG, int ROWS, bool COMBINE, bool SPEC, int GEO>
__global__ void __launch_bounds__(32, 16) k_down(MoeDims dd, MoeBufs B, MoeWeights W) {
  const MoeDims d = geo_dims<GEO>(dd);
  extern __shared__ __align__(16) uint8_t sm[];
  constexpr int MT = RV_MOE_MT;
  static_assert(ROWS * G <= 32, "one warp per CTA");
  RV_PHASE(2, 0);
  pdl_trigger();
  const int tile = blockIdx.y;
  const int ms = B.ms;
  const int row0 = tile * ROWS, nrows = min(ROWS, d.H - row0);
  __shared__ int s_last;
  __shared__ uint32_t s_pair[RV_SPEC_MAX_T];
  uint64_t *bar = (uint64_t *)sm;  // [2]: weights, activations
  const size_t st = tile_stride<FMT>(W.down_row_bytes);
  uint8_t *wsm = sm + 16;
  uint8_t *asm_ = wsm + (((size_t)ROWS * st + 15) & ~(size_t)15) + 16;
  uint8_t *arp = asm_ + ms * d.amoe_stride;  // split mode: [ms][mb][RV_ACT_AL] aligned copies
  const bool abulk = rv_bulk_ok(B.acts_moe, asm_, d.amoe_stride);
  const int lane = threadIdx.x;
  if (lane == 0) {
    mbar_init(bar, 1);
    mbar_init(bar + 1, 1);
  }
  __syncwarp();
  int nu;
  const SpecSmem *ssp = nullptr;
  if constexpr (SPEC) {
    __shared__ SpecSmem ss;
    spec_build(d.E, d.K, B.T, B.spec, ss);
    nu = ss.n_units;
    ssp = &ss;
  } else {
    nu = *B.n_units;
  }
  const int rsub = lane / G, g = lane % G;
  const bool live = rsub < ROWS && rsub < nrows;
  uint32_t wphase = 0, aphase = 0;
  for (int u = blockIdx.x; u < nu; u += gridDim.x) {
    int e, p0, p1;
    uint32_t msk = 0;
    if constexpr (SPEC) {
      e = ssp->uexp[u];
      p0 = ssp->start[e];
      msk = ssp->mask[e];
      p1 = p0 + __popc(msk);
    } else {
      const int4 unit = B.units[u];
      e = unit.x;
      p0 = unit.y;
      p1 = unit.z;
    }
    const uint8_t *dsrc = W.base + (size_t)e * W.stride + W.down_off + (size_t)row0 * W.down_row_bytes;
    __syncwarp();
    const uint32_t wtx = stage_rows<FMT>(wsm, dsrc, W.down_row_bytes, nrows, bar, false);
    if (lane == 0 && wtx) {
      fence_proxy_async();
      mbar_arrive_expect_tx(bar, wtx);
    }
    stage_rows<FMT>(wsm, dsrc, W.down_row_bytes, nrows, bar, true);
    RV_PHASE(2, 1);
    pdl_wait();  // acts_moe is k_gate_up's output (and the exact routing, SPEC)
    RV_PHASE(2, 2);
    bool any = true;
    if constexpr (SPEC) {
      // The token-major pair of each position, ~0 where the exact routing
      // did not select the expert.
      if (lane < p1 - p0) {
        const int t = spec_nth_bit(msk, lane);
        uint32_t pair = ~0u;
        for (int k = 0; k < d.K; k++)
          if (B.ids[(size_t)t * d.K + k] == (uint32_t)e) pair = (uint32_t)(t * d.K + k);
        s_pair[lane] = pair;
      }
      any = __any_sync(RV_FULL, lane < p1 - p0 && s_pair[lane] != ~0u);
      __syncwarp();
    }
    const uint8_t *wrow = wsm + (size_t)(live ? rsub : 0) * st;
    bool ok = true, wdone = wtx == 0;
    for (int c0 = p0; c0 < p1 && any; c0 += ms) {
      const int mt = min(ms, p1 - c0);
      __syncwarp();
      const uint8_t *asrc = B.acts_moe + (size_t)c0 * d.amoe_stride;
      if (abulk) {
        if (lane == 0) {
          fence_proxy_async();
          mbar_arrive_expect_tx(bar + 1, (uint32_t)(mt * d.amoe_stride));
          bulk_g2s(asm_, asrc, (uint32_t)(mt * d.amoe_stride), bar + 1);
        }
      } else {
        rv_copy_bytes_block(asm_, asrc, (size_t)mt * d.amoe_stride);
      }
      if (!wdone) {
        ok = mbar_wait_bounded(bar, wphase);
        wphase ^= 1;
        wdone = true;
      }
      if (abulk) {
        ok = mbar_wait_bounded(bar + 1, aphase) && ok;
        aphase ^= 1;
      }
      __syncwarp();
      if (!ok) return;
      RV_PHASE(2, 3);
      if constexpr (G > 1) {  // the row dots read aligned copies (measured: 2.6 -> 2.15 us at decode)
        for (int m = 0; m < mt; m++)
          act_align_row(asm_ + (size_t)m * d.amoe_stride, d.mb, arp + (size_t)m * d.mb * RV_ACT_AL, lane, 32);
        __syncwarp();
      }
      auto pair_of = [&](int c) -> uint32_t {
        if constexpr (SPEC) return s_pair[c - p0];
        else return B.index[c];
      };
      for (int m0 = 0; m0 < mt; m0 += MT) {
        const int mm = min(MT, mt - m0);
        if constexpr (G > 1) {
          for (int m = 0; m < mm; m++) {
            const float res =
                row_dot_split<FMT, G, NBG, true>(wrow, arp + (size_t)(m0 + m) * d.mb * RV_ACT_AL, g);
            const uint32_t pair = pair_of(c0 + m0 + m);
            if (g == G - 1 && live && pair != ~0u) down_out_row(B, pair, d.H)[row0 + rsub] = res;
          }
        } else {
          float res[MT];
          row_dot_tokens<FMT, MT>(wrow, d.mb, asm_ + (size_t)m0 * d.amoe_stride, d.amoe_stride, mm, res);
#pragma unroll
          for (int m = 0; m < MT; m++)
            if (m < mm && live) {
              const uint32_t pair = pair_of(c0 + m0 + m);
              if (pair != ~0u) down_out_row(B, pair, d.H)[row0 + rsub] = res[m];
            }
        }
      }
    }
    if (!wdone) {  // no selected position: the weight copy still has to land
      ok = mbar_wait_bounded(bar, wphase);
      wphase ^= 1;
      __syncwarp();
      if (!ok) return;
    }
    RV_PHASE(2, 4);
    if constexpr (COMBINE) {
      __threadfence();
      __syncwarp();
      if (lane == 0) {
        int *cnt = &B.down_cnt[tile];
        const int old = atomicAdd(cnt, 1);
        s_last = old == nu - 1;
        if (s_last) *cnt = 0;
      }
      __syncwarp();
      if (!s_last) continue;
      RV_PHASE(2, 5);
      __threadfence();
      // acc = 0; acc += w_k * d_k in top-k order; residual += acc.
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
  }
  if (B.ep_out) {  // rows stored into other ranks' memory: one fence after the warp's stores
    __syncwarp();
    if (lane == 0) __threadfence_system();
  }
  if constexpr (SPEC) {
    if (blockIdx.x == 0 && blockIdx.y == 0) {
      // After the wait above (every CTA has a unit): the exact routing is
      // final.  Check that the speculated set held it, and write the
      // dispatch taps (position -> token-major pair, ~0 where unselected).
      for (int p = lane; p < B.T * d.K; p += 32) {
        const uint32_t e = B.ids[p];
        // Cannot happen: the speculated set holds the exact top-k.
        if (e >= (uint32_t)d.E || !((ssp->mask[e] >> (p / d.K)) & 1u)) rv_dev_fail(RV_ERR_ROUTED_OUT_OF_RANGE);
      }
      for (int e = lane; e < d.E; e += 32) {
        uint32_t msk = ssp->mask[e];
        int pos = ssp->start[e];
        while (msk) {
          const int t = __ffs(msk) - 1;
          msk &= msk - 1;
          uint32_t pair = ~0u;
          for (int k = 0; k < d.K; k++)
            if (B.ids[(size_t)t * d.K + k] == (uint32_t)e) pair = (uint32_t)(t * d.K + k);
          B.index[pos++] = pair;
        }
      }
      for (int e = lane; e <= d.E; e += 32) B.index_start[e] = ssp->start[e];
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
