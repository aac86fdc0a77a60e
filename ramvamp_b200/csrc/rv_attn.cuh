// rv_attn.cuh -- the attention half of a decode step on the GPU: per-head
// QK-RMSNorm, NeoX RoPE, the f16 KV append and grouped-query attention over
// the cached positions, each with the reference's float order
// (model/forward.rs:2614-2631, kernels/primitives/{norm,rope,softmax}.rs,
// kernels/attention.rs:1075-1303, kv/mod.rs:336-373).
//
// Rotation factors: the reference forms cos/sin of position * inv_freq in
// f64 with the host libm (pow, sin, cos) and rounds them to f32.  The
// engine builds that table once on the host with the same calls (the
// frequency cache the reference's rope.rs describes) and the kernels read
// row `position` of it, so the rotation is bit-identical.
#pragma once
#include "rv_kernels.cuh"

// Positions of V staged per chunk by k_attn_softmax_out (two chunks of
// RV_ATTN_VCHUNK * head_dim halves plus their probabilities in shared memory).
#define RV_ATTN_VCHUNK 64
__host__ __device__ inline size_t attn_out_smem(int hd, int hpc = 1) {
  return 2 * (size_t)RV_ATTN_VCHUNK * (2 * hd + 4 * hpc);
}

struct AttnArgs {
  float *q;              // [n_heads][hd], normed + rotated in place
  float *k;              // [n_kv][hd], normed + rotated in place
  const float *v;        // [n_kv][hd]
  const float *q_norm;   // [hd]
  const float *k_norm;   // [hd]
  uint16_t *k_cache;     // this layer: [max_positions][n_kv * hd] f16 bits
  uint16_t *v_cache;
  const float2 *rot;     // [max_positions][hd / 2] (cos, sin)
  float *scores;         // [n_heads][positions]
  float *probs;          // [n_heads][positions]
  float *out;            // [n_heads][hd]
  uint8_t *q8k_out;      // when set (2 heads of 128 per CTA): Q8_K of out, one block per CTA
  int n_heads, n_kv, hd;
  int position;          // the row appended; attention covers 0..position
  const int *pos_dev;    // when set, the position is read here when the kernels run
  int max_positions;
  float eps, scale;
};

// The step's position: from device memory in graph-driven decoding.  Past
// the cache (device mode only: the host checks its own) every kernel
// writes nothing and the device error word says CapacityExceeded.
RV_DEVFN int attn_position(const AttnArgs &a) {
  if (!a.pos_dev) return a.position;
  const int p = *a.pos_dev;
  if (p < 0 || p >= a.max_positions) {
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) rv_dev_fail(RV_ERR_CAPACITY_EXCEEDED);
    return -1;
  }
  return p;
}

// One CTA (hd threads) per head: CTAs 0..n_heads-1 take q heads, the rest
// k heads (which also append k and v to the cache).  rmsnorm_in_place
// (norm.rs:72-90): v * inv * w with inv from rms_inv_block (exact); then
// rotate_head (rope.rs:30-45): x0*cos - x1*sin, x0*sin + x1*cos in f32.
__global__ void __launch_bounds__(256) k_attn_prep(AttnArgs a) {
  extern __shared__ __align__(16) uint8_t sm[];
  double *red = (double *)sm;
  float *xs = (float *)(sm + 34 * sizeof(double));
  const int position = attn_position(a);
  if (position < 0) return;  // uniform over the CTA
  const bool is_q = (int)blockIdx.x < a.n_heads;
  const int head = is_q ? (int)blockIdx.x : (int)blockIdx.x - a.n_heads;
  float *x = (is_q ? a.q : a.k) + (size_t)head * a.hd;
  const float *w = is_q ? a.q_norm : a.k_norm;
  const int i = threadIdx.x, half = a.hd >> 1;
  for (int k = i; k < a.hd; k += blockDim.x) xs[k] = x[k];
  __syncthreads();
  const float inv = rms_inv_block(xs, (size_t)a.hd, a.eps, red);
  for (int k = i; k < a.hd; k += blockDim.x) xs[k] = __fmul_rn(__fmul_rn(xs[k], inv), w[k]);
  __syncthreads();
  const float2 *rot = a.rot + (size_t)position * half;
  const size_t kv_dim = (size_t)a.n_kv * a.hd;
  for (int k = i; k < half; k += blockDim.x) {
    const float2 cs = rot[k];
    const float x0 = xs[k], x1 = xs[k + half];
    const float y0 = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
    const float y1 = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
    x[k] = y0;
    x[k + half] = y1;
    if (!is_q) {
      uint16_t *kc = a.k_cache + (size_t)position * kv_dim + (size_t)head * a.hd;
      kc[k] = f32_to_f16_bits(y0);
      kc[k + half] = f32_to_f16_bits(y1);
    }
  }
  if (!is_q) {
    uint16_t *vc = a.v_cache + (size_t)position * kv_dim + (size_t)head * a.hd;
    const float *vh = a.v + (size_t)head * a.hd;
    for (int k = i; k < a.hd; k += blockDim.x) vc[k] = f32_to_f16_bits(vh[k]);
  }
}

// q . K[t] with one f32 accumulator over i ascending (separate multiply and
// add).  For head_dim 128 the whole 256-byte row is loaded before the chain
// starts, so the loads overlap instead of each waiting on the adds.
RV_DEVFN float attn_dot_row(const float *qs, const uint16_t *krow, int hd) {
  const uint4 *kr = (const uint4 *)krow;
  float acc = 0.0f;
  if (hd == 128) {
    uint4 u[16];
#pragma unroll
    for (int c = 0; c < 16; c++) u[c] = kr[c];
#pragma unroll
    for (int c = 0; c < 16; c++) {
      const uint32_t wds[4] = {u[c].x, u[c].y, u[c].z, u[c].w};
#pragma unroll
      for (int j = 0; j < 4; j++) {
        acc = __fadd_rn(acc, __fmul_rn(qs[8 * c + 2 * j], h2f((uint16_t)(wds[j] & 0xFFFFu))));
        acc = __fadd_rn(acc, __fmul_rn(qs[8 * c + 2 * j + 1], h2f((uint16_t)(wds[j] >> 16))));
      }
    }
    return acc;
  }
  for (int c = 0; c < hd / 8; c++) {
    const uint4 u = kr[c];
    const uint32_t wds[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      acc = __fadd_rn(acc, __fmul_rn(qs[8 * c + 2 * j], h2f((uint16_t)(wds[j] & 0xFFFFu))));
      acc = __fadd_rn(acc, __fmul_rn(qs[8 * c + 2 * j + 1], h2f((uint16_t)(wds[j] >> 16))));
    }
  }
  return acc;
}

// qk_scores_scalar (attention.rs): scores[h][t] = scale * (q_h . K[t]) with
// one f32 accumulator over i ascending, separate multiply and add.  Grid
// (n_heads, tiles); thread = position, CTAs striding over 128-position
// tiles; q_h in shared memory; the K row read 8 halves at a time.
__global__ void __launch_bounds__(128) k_attn_scores(AttnArgs a) {
  extern __shared__ __align__(16) uint8_t sm[];
  float *qs = (float *)sm;
  const int position = attn_position(a);
  if (position < 0) return;
  const int h = blockIdx.x, group = a.n_heads / a.n_kv, kvh = h / group;
  for (int k = threadIdx.x; k < a.hd; k += blockDim.x) qs[k] = a.q[(size_t)h * a.hd + k];
  __syncthreads();
  const int positions = position + 1;
  const size_t kv_dim = (size_t)a.n_kv * a.hd;
  for (int t = blockIdx.y * blockDim.x + threadIdx.x; t < positions; t += gridDim.y * blockDim.x) {
    const float acc = attn_dot_row(qs, a.k_cache + (size_t)t * kv_dim + (size_t)kvh * a.hd, a.hd);
    a.scores[(size_t)h * positions + t] = __fmul_rn(a.scale, acc);
  }
}

// k_attn_prep folded into k_attn_scores (rv_attn_block): CTA (h, y) forms
// its own normed and rotated query head (rmsnorm_in_place + rotate_head, as
// k_attn_prep), and the CTA whose tile holds the current position also
// forms this step's key for its kv head, rounded through f16 as the cache
// holds it, and uses it for that position; the first query head of each kv
// head (h % group == 0) writes that position's K and V cache rows.  No CTA
// of this launch reads the current cache row; the next kernel reads V after
// the launch boundary.
// rmsnorm_in_place then rotate_head (as k_attn_prep) of one 128-value head
// by one warp: lane l holds x[l + 32i], i = 0..3, so the rotation pairs
// (k, k + 64) are elements (i, i + 2) of one lane.  The sum of squares is a
// lane sum of four and a shuffle tree; rms_inv_tail makes the inverse RMS
// the serial sum's (the tree sum of 128 squares differs from it by far less
// than the 2^-38 its check allows).  xs (smem[128]) holds the input for
// that check's serial redo, then the result.
RV_DEVFN void norm_rope_warp128(const float *x, const float *w, const float2 *rot, float eps, float *xs, int lane) {
  float v[4], wv[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    v[i] = x[lane + 32 * i];
    wv[i] = w[lane + 32 * i];
  }
  const float2 c0 = rot[lane], c1 = rot[lane + 32];
  double part = 0.0;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    xs[lane + 32 * i] = v[i];
    const double d = (double)v[i];
    part = __dadd_rn(part, __dmul_rn(d, d));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) part = __dadd_rn(part, __shfl_xor_sync(RV_FULL, part, o));
  __syncwarp();
  float inv = 0.0f;
  if (lane == 0) inv = rms_inv_tail(part, xs, 128, eps);
  inv = __shfl_sync(RV_FULL, inv, 0);
  float n[4];
#pragma unroll
  for (int i = 0; i < 4; i++) n[i] = __fmul_rn(__fmul_rn(v[i], inv), wv[i]);
  xs[lane] = __fsub_rn(__fmul_rn(n[0], c0.x), __fmul_rn(n[2], c0.y));
  xs[lane + 64] = __fadd_rn(__fmul_rn(n[0], c0.y), __fmul_rn(n[2], c0.x));
  xs[lane + 32] = __fsub_rn(__fmul_rn(n[1], c1.x), __fmul_rn(n[3], c1.y));
  xs[lane + 96] = __fadd_rn(__fmul_rn(n[1], c1.y), __fmul_rn(n[3], c1.x));
}

// One head's inputs for attn_norm_rope, held in registers: thread k < hd/2
// owns the rotation pair (k, k + hd/2) of x and of the norm weights and the
// pair's cos/sin.  Loaded at kernel entry so that every global load of the
// launch is in flight at once.
struct HeadPair {
  float x0, x1, w0, w1;
  float2 cs;
};
RV_DEVFN HeadPair head_pair_load(const float *x, const float *w, const float2 *rot, int hd) {
  HeadPair r{0.0f, 0.0f, 0.0f, 0.0f, make_float2(0.0f, 0.0f)};
  const int k = threadIdx.x, half = hd >> 1;
  if (k < half) {
    r.x0 = x[k];
    r.x1 = x[k + half];
    r.w0 = w[k];
    r.w1 = w[k + half];
    r.cs = rot[k];
  }
  return r;
}

// rmsnorm_in_place then rotate_head (as k_attn_prep) of one head whose
// pairs the threads hold; the result lands in xs (smem[hd]).
RV_DEVFN void attn_norm_rope(const HeadPair &r, int hd, float eps, float *xs, double *red) {
  const int k = threadIdx.x, half = hd >> 1;
  if (k < half) {
    xs[k] = r.x0;
    xs[k + half] = r.x1;
  }
  __syncthreads();
  const float inv = rms_inv_block(xs, (size_t)hd, eps, red);  // ends with a CTA barrier: xs is free
  if (k < half) {
    const float x0 = __fmul_rn(__fmul_rn(r.x0, inv), r.w0), x1 = __fmul_rn(__fmul_rn(r.x1, inv), r.w1);
    xs[k] = __fsub_rn(__fmul_rn(x0, r.cs.x), __fmul_rn(x1, r.cs.y));
    xs[k + half] = __fadd_rn(__fmul_rn(x0, r.cs.y), __fmul_rn(x1, r.cs.x));
  }
  __syncthreads();
}

// The scores of this CTA's positions (blockIdx.y's tiles) for query head
// blockIdx.x: one serial f32 chain per position, separate multiply and
// add; the current position uses this CTA's own key (ks).
RV_DEVFN void attn_scores_tile(const AttnArgs &a, const float *qs, const float *ks, int position, int kvh,
                               size_t kv_dim) {
  const int h = blockIdx.x, positions = position + 1;
  for (int t = blockIdx.y * blockDim.x + threadIdx.x; t < positions; t += gridDim.y * blockDim.x) {
    float acc = 0.0f;
    if (t == position) {
      for (int i = 0; i < a.hd; i++) acc = __fadd_rn(acc, __fmul_rn(qs[i], ks[i]));
    } else {
      acc = attn_dot_row(qs, a.k_cache + (size_t)t * kv_dim + (size_t)kvh * a.hd, a.hd);
    }
    a.scores[(size_t)h * positions + t] = __fmul_rn(a.scale, acc);
  }
}

__global__ void __launch_bounds__(128) k_attn_scores_prep(AttnArgs a) {
  extern __shared__ __align__(16) uint8_t sm[];
  double *red = (double *)sm;
  float *qs = (float *)(sm + 34 * sizeof(double));
  float *ks = qs + a.hd;
  const int position = attn_position(a);
  if (position < 0) return;
  const int h = blockIdx.x, group = a.n_heads / a.n_kv, kvh = h / group, half = a.hd >> 1;
  const float2 *rot = a.rot + (size_t)position * half;
  const size_t kv_dim = (size_t)a.n_kv * a.hd;
  const bool holds_pos = (int)blockIdx.y == (position / (int)blockDim.x) % (int)gridDim.y;
  const bool writer = holds_pos && h % group == 0;
  if (a.hd == 128) {
    // Warp 0 forms the query head, warp 1 the key, warp 2 appends the V
    // row, all at once (norm_rope_warp128: the same values as below).
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == 0) {
      norm_rope_warp128(a.q + (size_t)h * 128, a.q_norm, rot, a.eps, qs, lane);
    } else if (warp == 1 && holds_pos) {
      norm_rope_warp128(a.k + (size_t)kvh * 128, a.k_norm, rot, a.eps, ks, lane);
      uint16_t *kc = a.k_cache + (size_t)position * kv_dim + (size_t)kvh * 128;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int k = lane + 32 * i;
        const uint16_t kb = f32_to_f16_bits(ks[k]);
        ks[k] = h2f(kb);  // the value attention reads back from the cache
        if (writer) kc[k] = kb;
      }
    } else if (warp == 2 && writer) {
      uint16_t *vc = a.v_cache + (size_t)position * kv_dim + (size_t)kvh * 128;
      const float *vh = a.v + (size_t)kvh * 128;
#pragma unroll
      for (int i = 0; i < 4; i++) vc[lane + 32 * i] = f32_to_f16_bits(vh[lane + 32 * i]);
    }
    __syncthreads();
    attn_scores_tile(a, qs, ks, position, kvh, kv_dim);
    return;
  }
  const HeadPair qp = head_pair_load(a.q + (size_t)h * a.hd, a.q_norm, rot, a.hd);
  HeadPair kp{0.0f, 0.0f, 0.0f, 0.0f, make_float2(0.0f, 0.0f)};
  float v0 = 0.0f, v1 = 0.0f;
  const float *vh = a.v + (size_t)kvh * a.hd;
  if (holds_pos) kp = head_pair_load(a.k + (size_t)kvh * a.hd, a.k_norm, rot, a.hd);
  if (writer && (int)threadIdx.x < half) {
    v0 = vh[threadIdx.x];
    v1 = vh[threadIdx.x + half];
  }
  attn_norm_rope(qp, a.hd, a.eps, qs, red);
  if (holds_pos) {
    attn_norm_rope(kp, a.hd, a.eps, ks, red);
    uint16_t *kc = a.k_cache + (size_t)position * kv_dim + (size_t)kvh * a.hd;
    uint16_t *vc = a.v_cache + (size_t)position * kv_dim + (size_t)kvh * a.hd;
    const int k = threadIdx.x;
    if (k < half) {
      const uint16_t kb0 = f32_to_f16_bits(ks[k]), kb1 = f32_to_f16_bits(ks[k + half]);
      ks[k] = h2f(kb0);  // the value attention reads back from the cache
      ks[k + half] = h2f(kb1);
      if (writer) {
        kc[k] = kb0;
        kc[k + half] = kb1;
        vc[k] = f32_to_f16_bits(v0);
        vc[k + half] = f32_to_f16_bits(v1);
      }
    }
    __syncthreads();
  }
  attn_scores_tile(a, qs, ks, position, kvh, kv_dim);
}

// HPC query heads per CTA (threads split into HPC segments, segment j
// owning head blockIdx.x * HPC + j; the heads share one kv head): softmax
// over the positions (softmax.rs:18-40: f32 max, e = exp(f64(s) - max) in
// f64, f32 copies, the f64 sum in position order, f32 reciprocal), then
// v_reduce_scalar: out[i] = sum over t ascending of p_t * V[t][i], separate
// multiply and add.  The f64 sum is taken in blocks; summation in any order
// of P positive terms errs by at most (P-1)u of the sum, so block and serial
// sums differ by at most 2(P-1)u: when f32(1/sum) is the same for every sum
// within that bound, the blocked sum gives the serial result; otherwise the
// segment's first thread redoes the serial sum.  With q8k_out set and
// HPC * hd == 256 the CTA's outputs are one Q8_K block, quantized here
// (quantize_row_q8_k, the input of attn_output).
template <int HPC>
__global__ void __launch_bounds__(256) k_attn_softmax_out(AttnArgs a) {
  __shared__ double red[34];
  __shared__ float s_max[HPC], s_inv[HPC];
  const int position = attn_position(a);
  if (position < 0) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int seg = blockDim.x / HPC, j = tid / seg, st = tid % seg, wps = seg >> 5, w0 = j * wps;
  const int h = blockIdx.x * HPC + j, group = a.n_heads / a.n_kv, kvh = (blockIdx.x * HPC) / group;
  const int positions = position + 1;
  const float *sc = a.scores + (size_t)h * positions;
  float *pr = a.probs + (size_t)h * positions;
  float mx = -INFINITY;
  for (int t = st; t < positions; t += seg) mx = fmaxf(mx, sc[t]);
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(RV_FULL, mx, o));
  if (lane == 0) red[warp] = (double)mx;
  __syncthreads();
  if (st == 0) {
    float m = -INFINITY;
    for (int w = w0; w < w0 + wps; w++) m = fmaxf(m, (float)red[w]);
    s_max[j] = m;
  }
  __syncthreads();
  const double dmx = (double)s_max[j];
  double part = 0.0;
  for (int t = st; t < positions; t += seg) {
    const double e = exp(__dsub_rn((double)sc[t], dmx));
    pr[t] = __double2float_rn(e);
    part = __dadd_rn(part, e);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) part = __dadd_rn(part, __shfl_xor_sync(RV_FULL, part, o));
  __syncthreads();
  if (lane == 0) red[warp] = part;
  __syncthreads();
  if (st == 0) {
    double sum = 0.0;
    for (int w = w0; w < w0 + wps; w++) sum = __dadd_rn(sum, red[w]);
    const double r = __drcp_rn(sum);
    const unsigned long long bound = 2ull * (unsigned long long)positions + 2ull;
    const int k = 52 - (64 - __clzll((long long)bound));
    float inv = __double2float_rn(r);
    if (!(k >= 30 && isfinite(r) && f32_rounding_stable(r, k))) {
      double ser = 0.0;
      for (int t = 0; t < positions; t++) ser = __dadd_rn(ser, exp(__dsub_rn((double)sc[t], dmx)));
      inv = __double2float_rn(__drcp_rn(ser));
    }
    s_inv[j] = inv;
  }
  __syncthreads();
  const float inv = s_inv[j];
  for (int t = st; t < positions; t += seg) pr[t] = __fmul_rn(pr[t], inv);
  __syncthreads();
  // Values: one serial chain per output element over t ascending.  The kv
  // head's V rows (hd halves each) and each head's probabilities are staged
  // in shared memory RV_ATTN_VCHUNK positions at a time, double-buffered
  // with 16-byte cp.async copies, so the chains read on-chip memory while
  // the next chunk streams in.  Thread st (< hd) of segment j owns element st
  // of head j.
  extern __shared__ __align__(16) uint8_t vsm[];
  const size_t kv_dim = (size_t)a.n_kv * a.hd;
  const uint16_t *vc = a.v_cache + (size_t)kvh * a.hd;
  const int row_bytes = 2 * a.hd, pieces = a.hd / 8;
  float *pbuf0 = (float *)(vsm + 2 * RV_ATTN_VCHUNK * row_bytes);
  // buffer b of the V rows and of the probabilities
  auto vbuf = [&](int b) { return vsm + b * RV_ATTN_VCHUNK * row_bytes; };
  auto pbuf = [&](int b) { return pbuf0 + b * HPC * RV_ATTN_VCHUNK; };
  const int nchunks = (positions + RV_ATTN_VCHUNK - 1) / RV_ATTN_VCHUNK;
  auto stage = [&](int ch) {
    const int t0 = ch * RV_ATTN_VCHUNK, n = min(RV_ATTN_VCHUNK, positions - t0);
    uint8_t *dst = vbuf(ch & 1);
    for (int k = tid; k < n * pieces; k += blockDim.x) {
      const int r = k / pieces, c = k % pieces;
      cp_async16(dst + r * row_bytes + 16 * c, (const uint8_t *)(vc + (size_t)(t0 + r) * kv_dim) + 16 * c);
    }
    for (int r = st; r < n; r += seg) pbuf(ch & 1)[j * RV_ATTN_VCHUNK + r] = pr[t0 + r];
    cp_async_commit();
  };
  float acc = 0.0f;
  stage(0);
  for (int ch = 0; ch < nchunks; ch++) {
    if (ch + 1 < nchunks) {
      stage(ch + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint16_t *vs = (const uint16_t *)vbuf(ch & 1);
    const float *ps = pbuf(ch & 1) + j * RV_ATTN_VCHUNK;
    const int n = min(RV_ATTN_VCHUNK, positions - ch * RV_ATTN_VCHUNK);
    if (st < a.hd) {
#pragma unroll 8
      for (int r = 0; r < n; r++) acc = __fadd_rn(acc, __fmul_rn(ps[r], h2f(vs[r * a.hd + st])));
    }
    __syncthreads();  // this buffer is restaged for chunk ch + 2
  }
  if (st < a.hd) a.out[(size_t)h * a.hd + st] = acc;
  if (HPC == 2 && a.q8k_out && a.hd == 128) {
    float *ys = (float *)vsm;  // the staging buffers are free now
    if (st < a.hd) ys[j * a.hd + st] = acc;
    __syncthreads();
    if (warp == 0) {
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; e++) v[e] = ys[8 * lane + e];
      q8k_quantize_warp(v, lane, a.q8k_out + (size_t)blockIdx.x * 292);
    }
  }
}

// k_attn_scores_prep and k_attn_softmax_out<2> (with the Q8_K epilogue) as
// one launch: CTA p (256 threads) owns query heads 2p and 2p + 1, which
// share one kv head (hd 128).  Warps 0 and 1 form the two normed, rotated
// query heads, warp 2 this step's key (rounded through f16 as the cache
// holds it) and warp 3 this step's V row in f16; the first pair of each kv
// head also appends both rows to the caches.  No CTA reads the cache rows
// of the current position: it uses its own copies of them.  Thread st of
// head j (tid = 128j + st) then forms the scores of positions st, st + 128,
// ... (the scores kernel's chains), and the softmax, the value chains and
// the Q8_K of the pair's outputs follow as in k_attn_softmax_out<2>, with
// scores and probabilities in shared memory.
#define RV_ATTN_FUSED_MAX 256
__host__ __device__ inline size_t attn_fused_smem(int positions) {
  // red[34] f64 | q 2x128 f32 | k 128 f32 | v row 128 f16 | V staging 2 x 64 x 256 B | scores, probs 2 x P f32 each
  return 34 * 8 + 3 * 128 * 4 + 128 * 2 + 2 * (size_t)RV_ATTN_VCHUNK * 256 + 4 * (size_t)positions * sizeof(float);
}
__global__ void __launch_bounds__(256) k_attn_fused(AttnArgs a) {
  extern __shared__ __align__(16) uint8_t sm[];
  __shared__ float s_max[2], s_inv[2];
  double *red = (double *)sm;
  float *qs = (float *)(sm + 34 * 8);
  float *ks = qs + 256;
  uint16_t *vrow = (uint16_t *)(ks + 128);
  uint8_t *vstage = (uint8_t *)(vrow + 128);
  float *sbase = (float *)(vstage + 2 * RV_ATTN_VCHUNK * 256);
  const int position = attn_position(a);
  if (position < 0) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int p = blockIdx.x, group = a.n_heads / a.n_kv, kvh = (2 * p) / group;
  const size_t kv_dim = (size_t)a.n_kv * 128;
  const bool writer = (2 * p) % group == 0;
  const float2 *rot = a.rot + (size_t)position * 64;
  if (warp < 2) {
    norm_rope_warp128(a.q + (size_t)(2 * p + warp) * 128, a.q_norm, rot, a.eps, qs + warp * 128, lane);
  } else if (warp == 2) {
    norm_rope_warp128(a.k + (size_t)kvh * 128, a.k_norm, rot, a.eps, ks, lane);
    uint16_t *kc = a.k_cache + (size_t)position * kv_dim + (size_t)kvh * 128;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int k = lane + 32 * i;
      const uint16_t kb = f32_to_f16_bits(ks[k]);
      ks[k] = h2f(kb);  // the value attention reads back from the cache
      if (writer) kc[k] = kb;
    }
  } else if (warp == 3) {
    uint16_t *vc = a.v_cache + (size_t)position * kv_dim + (size_t)kvh * 128;
    const float *vh = a.v + (size_t)kvh * 128;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int k = lane + 32 * i;
      const uint16_t vb = f32_to_f16_bits(vh[k]);
      vrow[k] = vb;
      if (writer) vc[k] = vb;
    }
  }
  __syncthreads();
  // Scores: acc = sum over i ascending of q[i] * k[i], separate multiply and add.
  const int j = tid >> 7, st = tid & 127, h = 2 * p + j, positions = position + 1;
  const float *qj = qs + j * 128;
  float *sc = sbase + (size_t)j * positions;
  float *pr = sbase + (size_t)(2 + j) * positions;
  for (int t = st; t < positions; t += 128) {
    float acc = 0.0f;
    if (t == position) {
      for (int i = 0; i < 128; i++) acc = __fadd_rn(acc, __fmul_rn(qj[i], ks[i]));
    } else {
      acc = attn_dot_row(qj, a.k_cache + (size_t)t * kv_dim + (size_t)kvh * 128, 128);
    }
    sc[t] = __fmul_rn(a.scale, acc);
  }
  // Softmax (softmax.rs:18-40), as k_attn_softmax_out: segment j = warps 4j..4j+3.
  float mx = -INFINITY;
  for (int t = st; t < positions; t += 128) mx = fmaxf(mx, sc[t]);
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(RV_FULL, mx, o));
  if (lane == 0) red[warp] = (double)mx;
  __syncthreads();
  if (st == 0) {
    float m = -INFINITY;
    for (int w = 4 * j; w < 4 * j + 4; w++) m = fmaxf(m, (float)red[w]);
    s_max[j] = m;
  }
  __syncthreads();
  const double dmx = (double)s_max[j];
  double part = 0.0;
  for (int t = st; t < positions; t += 128) {
    const double e = exp(__dsub_rn((double)sc[t], dmx));
    pr[t] = __double2float_rn(e);
    part = __dadd_rn(part, e);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) part = __dadd_rn(part, __shfl_xor_sync(RV_FULL, part, o));
  __syncthreads();
  if (lane == 0) red[warp] = part;
  __syncthreads();
  if (st == 0) {
    double sum = 0.0;
    for (int w = 4 * j; w < 4 * j + 4; w++) sum = __dadd_rn(sum, red[w]);
    const double r = __drcp_rn(sum);
    const unsigned long long bound = 2ull * (unsigned long long)positions + 2ull;
    const int k = 52 - (64 - __clzll((long long)bound));
    float inv = __double2float_rn(r);
    if (!(k >= 30 && isfinite(r) && f32_rounding_stable(r, k))) {
      double ser = 0.0;
      for (int t = 0; t < positions; t++) ser = __dadd_rn(ser, exp(__dsub_rn((double)sc[t], dmx)));
      inv = __double2float_rn(__drcp_rn(ser));
    }
    s_inv[j] = inv;
  }
  __syncthreads();
  const float inv = s_inv[j];
  for (int t = st; t < positions; t += 128) pr[t] = __fmul_rn(pr[t], inv);
  // Values: one serial chain per output element over t ascending, the V
  // rows staged 64 positions at a time (double-buffered cp.async); the
  // current position's row comes from this CTA's own copy.
  const uint16_t *vcg = a.v_cache + (size_t)kvh * 128;
  auto vbuf = [&](int b) { return vstage + b * RV_ATTN_VCHUNK * 256; };
  const int nchunks = (positions + RV_ATTN_VCHUNK - 1) / RV_ATTN_VCHUNK;
  auto stage = [&](int ch) {
    const int t0 = ch * RV_ATTN_VCHUNK, n = min(RV_ATTN_VCHUNK, positions - t0);
    uint8_t *dst = vbuf(ch & 1);
    for (int k = tid; k < n * 16; k += blockDim.x) {
      const int r = k >> 4, c = k & 15;
      if (t0 + r == position)
        ((uint4 *)(dst + r * 256))[c] = ((const uint4 *)vrow)[c];
      else
        cp_async16(dst + r * 256 + 16 * c, (const uint8_t *)(vcg + (size_t)(t0 + r) * kv_dim) + 16 * c);
    }
    cp_async_commit();
  };
  float acc = 0.0f;
  stage(0);
  for (int ch = 0; ch < nchunks; ch++) {
    if (ch + 1 < nchunks) {
      stage(ch + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // this chunk's rows (and, the first time, every probability) are in place
    const uint16_t *vs = (const uint16_t *)vbuf(ch & 1);
    const float *pc = pr + ch * RV_ATTN_VCHUNK;
    const int n = min(RV_ATTN_VCHUNK, positions - ch * RV_ATTN_VCHUNK);
#pragma unroll 8
    for (int r = 0; r < n; r++) acc = __fadd_rn(acc, __fmul_rn(pc[r], h2f(vs[r * 128 + st])));
    __syncthreads();  // this buffer is restaged for chunk ch + 2
  }
  a.out[(size_t)h * 128 + st] = acc;
  if (a.q8k_out) {
    float *ys = (float *)vstage;  // the staging buffers are free now
    ys[j * 128 + st] = acc;
    __syncthreads();
    if (warp == 0) {
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; e++) v[e] = ys[8 * lane + e];
      q8k_quantize_warp(v, lane, a.q8k_out + (size_t)p * 292);
    }
  }
}

// rope_neox_heads (rope.rs:80-111) for one position, the factors passed by
// value (formed on the host with the reference's f64 libm calls).
#define RV_ROPE_MAX_HALF 256
struct RopeFactors {
  float2 cs[RV_ROPE_MAX_HALF];
};
__global__ void k_rope_heads(float *x, int n_heads, int hd, RopeFactors f) {
  const int half = hd >> 1;
  const size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= (size_t)n_heads * half) return;
  const size_t h = e / half;
  const int k = (int)(e % half);
  float *xh = x + h * hd;
  const float x0 = xh[k], x1 = xh[k + half];
  const float2 cs = f.cs[k];
  xh[k] = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
  xh[k + half] = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
}

// End of a graph-driven decode step: record the sampled id at the step's
// position, feed it back as the next input token, advance the position.
__global__ void k_decode_advance(int *pos, const uint32_t *next, int *token, uint32_t *ids, int ids_cap) {
  const int p = pos[0];
  if (next) {
    if (ids && p >= 0 && p < ids_cap) ids[p] = next[0];
    if (token) token[0] = (int)next[0];
  }
  pos[0] = p + 1;
}

// Sampler::argmax (generate/mod.rs:321-331): the first index of the
// largest value; NaN never wins and an all -inf/NaN row gives 0.  One CTA;
// each thread scans its 16-byte chunks (and the unaligned head and tail) in
// index order with eight loads in flight, then a (value, index) reduction
// that prefers the smaller index on equal values.
RV_DEVFN void argmax_take(float v, uint32_t i, float &bv, uint32_t &bi) {
  if (v > bv) {  // strict: the earlier index keeps a tie; NaN never passes
    bv = v;
    bi = i;
  }
}
__global__ void __launch_bounds__(1024) k_argmax(const float *__restrict__ x, size_t n, uint32_t *out) {
  __shared__ float sv[32];
  __shared__ uint32_t si[32];
  float bv = -INFINITY;
  uint32_t bi = 0xFFFFFFFFu;
  const size_t head = (16 - ((uintptr_t)x & 15)) / 4 % 4;  // floats before the first 16-byte boundary
  const size_t h = head < n ? head : n;
  const size_t n4 = (n - h) / 4;
  const float4 *x4 = (const float4 *)(x + h);
  if (threadIdx.x == 0)
    for (size_t k = 0; k < h; k++) argmax_take(x[k], (uint32_t)k, bv, bi);
  const size_t T = blockDim.x;
  size_t c = threadIdx.x;
  for (; c + 7 * T < n4; c += 8 * T) {
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; u++) v[u] = x4[c + u * T];
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const uint32_t i0 = (uint32_t)(h + 4 * (c + u * T));
      argmax_take(v[u].x, i0, bv, bi);
      argmax_take(v[u].y, i0 + 1, bv, bi);
      argmax_take(v[u].z, i0 + 2, bv, bi);
      argmax_take(v[u].w, i0 + 3, bv, bi);
    }
  }
  for (; c < n4; c += T) {
    const float4 v = x4[c];
    const uint32_t i0 = (uint32_t)(h + 4 * c);
    argmax_take(v.x, i0, bv, bi);
    argmax_take(v.y, i0 + 1, bv, bi);
    argmax_take(v.z, i0 + 2, bv, bi);
    argmax_take(v.w, i0 + 3, bv, bi);
  }
  for (size_t k = h + 4 * n4 + threadIdx.x; k < n; k += T) argmax_take(x[k], (uint32_t)k, bv, bi);
  auto better = [](float v, uint32_t i, float bv_, uint32_t bi_) {
    return i != 0xFFFFFFFFu && (bi_ == 0xFFFFFFFFu || v > bv_ || (v == bv_ && i < bi_));
  };
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float v = __shfl_xor_sync(RV_FULL, bv, o);
    const uint32_t i = __shfl_xor_sync(RV_FULL, bi, o);
    if (better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = -INFINITY;
    uint32_t i = 0xFFFFFFFFu;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++)
      if (better(sv[w], si[w], v, i)) {
        v = sv[w];
        i = si[w];
      }
    out[0] = i == 0xFFFFFFFFu ? 0u : i;
  }
}

// vec_add (primitives/vec.rs:10-22): a[i] += b[i] in f32.
__global__ void k_vec_add(float *a, const float *b, size_t n) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) a[i] = __fadd_rn(a[i], b[i]);
}
