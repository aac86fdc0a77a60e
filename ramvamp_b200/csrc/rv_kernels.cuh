// rv_kernels.cuh -- stand-alone kernels behind the rv_ kernel-level entry
// points: Q8_K quantization, the lane-exact k-quant GEMV (rows / batched),
// RMSNorm, softmax, SwiGLU, integer taps, and the synthetic-weight
// generator with the GPU restatement of the reference's weight quantizers.
#pragma once
#include "rv_expf.cuh"
#include "rv_internal.cuh"

// ------------------------------------------------------------ Q8_K
// One warp per 256-float block; x may have any 4-byte alignment.
__global__ void k_quantize_q8k(const float *__restrict__ x, uint8_t *__restrict__ out,
                               size_t n_blocks) {
  const int lane = threadIdx.x & 31;
  const size_t b = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (b >= n_blocks) return;  // warp-uniform
  float v[8];
  const float *src = x + b * 256 + 8 * lane;
#pragma unroll
  for (int e = 0; e < 8; e++) v[e] = src[e];
  q8k_quantize_warp(v, lane, out + b * 292);
}

// ------------------------------------------------------------ GEMV
// out[(r - r0) * n_acts + a] = row(r) . act_a for r in [r0, r0 + nrows).
// Block = R rows x 8 lanes.  The weight tile is staged once into shared
// memory (bulk copy when 16-byte aligned, else a cooperative byte copy);
// activations are staged MT rows at a time.
struct GemvArgs {
  const uint8_t *w;   // whole matrix
  size_t row_bytes;
  int nb;             // blocks per row
  size_t r0, nrows;   // rows to compute
  const uint8_t *acts;  // packed Q8_K rows, nb*292 bytes each
  size_t n_acts;
  float *out;
  int R;              // rows per CTA
  int accumulate;     // out[...] = out[...] + dot (a fused residual add, vec.rs:10-22)
};

RV_DEVFN void gemv_store(const GemvArgs &g, size_t idx, float v) {
  g.out[idx] = g.accumulate ? __fadd_rn(g.out[idx], v) : v;
}

// One R-row tile `tile` of a k-quant GEMV (the body of k_gemv).
template <int FMT, int MT>
RV_DEVFN void gemv_tile(const GemvArgs &g, size_t tile, uint8_t *sm) {
  uint64_t *bar = (uint64_t *)sm;
  const int R = g.R;
  const size_t act_row = (size_t)g.nb * 292;
  uint8_t *wsm = sm + 16;
  uint8_t *asm_ = wsm + ((R * g.row_bytes + 15) & ~(size_t)15) + 16;
  const size_t tile0 = tile * R;
  const int rows_here = (int)min((size_t)R, g.nrows - tile0);
  const uint8_t *wsrc = g.w + (g.r0 + tile0) * g.row_bytes;
  const size_t wbytes = (size_t)rows_here * g.row_bytes;
  const bool bulk = rv_bulk_ok(wsrc, wsm, wbytes);
  if (threadIdx.x == 0) mbar_init(bar, 1);
  __syncthreads();
  if (bulk) {
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(bar, (uint32_t)wbytes);
      bulk_g2s(wsm, wsrc, (uint32_t)wbytes, bar);
    }
  } else {
    rv_copy_bytes_block(wsm, wsrc, wbytes);
  }
  const int r = threadIdx.x >> 3, lane = threadIdx.x & 7;
  const int rr = r < rows_here ? r : 0;  // idle rows compute row 0, never store
  const uint8_t *wrow = wsm + (size_t)rr * g.row_bytes;
  constexpr int BB = FMT == RV_Q4_K ? 144 : FMT == RV_Q5_K ? 176 : 210;
  bool ok = true;
  for (size_t a0 = 0; a0 < g.n_acts; a0 += MT) {
    const int mt = (int)min((size_t)MT, g.n_acts - a0);
    __syncthreads();  // previous chunk fully consumed
    stage_to_smem(asm_, g.acts + a0 * act_row, (size_t)mt * act_row);
    if (a0 == 0 && bulk) ok = mbar_wait_bounded(bar, 0);
    __syncthreads();
    if (!ok) return;
    float acc[MT], accm[MT];
#pragma unroll
    for (int m = 0; m < MT; m++) acc[m] = accm[m] = 0.0f;
    for (int b = 0; b < g.nb; b++) {
      WBlock w;
      load_wblock<FMT>(wrow + (size_t)b * BB, lane, w);
#pragma unroll
      for (int m = 0; m < MT; m++)
        if (m < mt) lane_step<FMT>(w, asm_ + m * act_row + (size_t)b * 292, lane, acc[m], accm[m]);
    }
#pragma unroll
    for (int m = 0; m < MT; m++) {
      const float res = lane_reduce<FMT>(acc[m], accm[m]);
      if (lane == 0 && r < rows_here && m < mt) gemv_store(g, (tile0 + r) * g.n_acts + a0 + m, res);
    }
  }
}

template <int FMT, int MT>
__global__ void __launch_bounds__(256) k_gemv(GemvArgs g) {
  extern __shared__ __align__(16) uint8_t sm[];
  gemv_tile<FMT, MT>(g, blockIdx.x, sm);
}

// ------------------------------------------------------- lm_head GEMV
// Streaming Q6_K GEMV for one activation row, 8 blocks per row (hidden
// 2048) and many rows: output.weight, 151,936 rows of 1,680 bytes, the
// largest weight read of a decode step.  Same integer lane sums and float
// order as k_gemv (lane_step, lane_reduce), hence bit-identical, but laid
// out to stream HBM:
// - a persistent grid walks 16-row tiles blockIdx.x, + gridDim.x, ...;
//   each CTA keeps RV_LMH_STAGES tiles in flight (one bulk copy per tile,
//   an mbarrier per stage) and refills a stage once every thread is done
//   with it;
// - thread (p, lane) computes lane `lane` of one row; the lane's 64
//   activation words and 8 block scales stay in registers for the whole
//   kernel (they are the same for every row);
// - blocks are 210 bytes, so in a 4-byte-aligned row block b starts 2
//   bytes past a word boundary exactly when b is odd: the unrolled loop
//   knows each block's alignment at compile time (one load per aligned
//   word, two and a funnel shift otherwise);
// - rows are 420 words (4 mod 8), so the four rows a warp reads at once
//   are taken two apart (8 banks apart): no bank conflicts;
// - Q6_K's (q - 32) a is dp4a(q, a, dp4a(-32 x 4, a, 0)), an exact
//   integer identity, so the 6-bit values need no per-byte subtraction.
#define RV_LMH_ROWS 16
#define RV_LMH_STAGES 3

// prmt.b32 in its default mode: a selector nibble with bit 3 set fills the
// byte with the sign of the byte its low bits select.
RV_DEVFN uint32_t prmt_sext(uint32_t x, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(x), "r"(sel));
  return r;
}

// The word at p (shared memory); MIS: p is 2 bytes past a word boundary.
template <bool MIS>
RV_DEVFN uint32_t ld32c(const uint8_t *p) {
  if constexpr (MIS) {
    const uint32_t *a = (const uint32_t *)(p - 2);
    return __funnelshift_r(a[0], a[1], 16);
  } else {
    return *(const uint32_t *)p;
  }
}

// Lane `lane`'s view of one Q6_K block: the eight 6-bit vectors (without
// the -32), their signed scales, d.
struct W6 {
  uint32_t q[8];
  int sc[8];
  float d;
};
template <bool MIS>
RV_DEVFN void load_w6(const uint8_t *blk, int lane, uint32_t sel_lo, uint32_t sel_hi, W6 &w) {
  w.d = h2f(*(const uint16_t *)(blk + 208));
#pragma unroll
  for (int h = 0; h < 2; h++) {
    const uint32_t ql0 = ld32c<MIS>(blk + 64 * h + 4 * lane);
    const uint32_t ql1 = ld32c<MIS>(blk + 64 * h + 32 + 4 * lane);
    const uint32_t qh = ld32c<MIS>(blk + 128 + 32 * h + 4 * lane);
    w.q[4 * h + 0] = (ql0 & 0x0F0F0F0Fu) | ((qh << 4) & 0x30303030u);
    w.q[4 * h + 1] = (ql1 & 0x0F0F0F0Fu) | ((qh << 2) & 0x30303030u);
    w.q[4 * h + 2] = ((ql0 >> 4) & 0x0F0F0F0Fu) | (qh & 0x30303030u);
    w.q[4 * h + 3] = ((ql1 >> 4) & 0x0F0F0F0Fu) | ((qh >> 2) & 0x30303030u);
  }
  // Vector (h, k)'s scale is byte 192 + 8h + 2k + (lane >= 4): byte
  // 2(k & 1) + hi of word 2h + (k >> 1) of the 16 scale bytes.
#pragma unroll
  for (int m = 0; m < 4; m++) {
    const uint32_t word = ld32c<MIS>(blk + 192 + 4 * m);
    w.sc[2 * m] = (int)prmt_sext(word, sel_lo);
    w.sc[2 * m + 1] = (int)prmt_sext(word, sel_hi);
  }
}

__global__ void __launch_bounds__(RV_LMH_ROWS * 8, 2) k_gemv_lm_head(GemvArgs g) {
  extern __shared__ __align__(16) uint8_t sm[];
  uint64_t *bar = (uint64_t *)sm;  // one per stage
  constexpr int R = RV_LMH_ROWS, S = RV_LMH_STAGES;
  constexpr size_t RB = 8 * 210, SB = (size_t)R * RB;
  uint8_t *stage0 = sm + 64;
  const size_t n_tiles = (g.nrows + R - 1) / R;
  const uint8_t *w = g.w + g.r0 * RB;
  auto issue = [&](size_t tile, int st) {
    const uint32_t bytes = (uint32_t)(min((size_t)R, g.nrows - tile * R) * RB);
    mbar_arrive_expect_tx(&bar[st], bytes);
    bulk_g2s(stage0 + st * SB, w + tile * SB, bytes, &bar[st]);
  };
  if (threadIdx.x == 0) {
#pragma unroll
    for (int i = 0; i < S; i++) mbar_init(&bar[i], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
#pragma unroll
    for (int i = 0; i < S; i++)
      if (blockIdx.x + (size_t)i * gridDim.x < n_tiles) issue(blockIdx.x + (size_t)i * gridDim.x, i);
  }
  const int p = threadIdx.x >> 3, lane = threadIdx.x & 7;
  int ax[8][8];
  float yd[8];
#pragma unroll
  for (int b = 0; b < 8; b++) {
    const uint8_t *act = g.acts + 292 * b;
    yd[b] = *(const float *)act;
#pragma unroll
    for (int v = 0; v < 8; v++) ax[b][v] = *(const int *)(act + 4 + 128 * (v >> 2) + 32 * (v & 3) + 4 * lane);
  }
  const int wq = p >> 2, rt = 8 * (wq >> 1) + 2 * (p & 3) + (wq & 1);  // rows two apart within a warp
  const uint32_t jlo = lane >= 4 ? 1u : 0u, jhi = jlo + 2u;
  const uint32_t sel_lo = jlo | ((8u + jlo) * 0x1110u), sel_hi = jhi | ((8u + jhi) * 0x1110u);
  uint32_t phase = 0;  // bit st = parity of stage st's next completion
  int st = 0;
  for (size_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, st = st + 1 == S ? 0 : st + 1) {
    const bool ok = mbar_wait_bounded(&bar[st], (phase >> st) & 1);
    phase ^= 1u << st;
    if (!__syncthreads_and(ok)) return;
    const int rows_here = (int)min((size_t)R, g.nrows - tile * R);
    // Rows past the matrix compute row 0 of the tile and are never stored.
    const uint8_t *wrow = stage0 + st * SB + (size_t)(rt < rows_here ? rt : 0) * RB;
    float acc = 0.0f;
#pragma unroll
    for (int b = 0; b < 8; b++) {
      W6 x;
      if (b & 1) load_w6<true>(wrow + 210 * b, lane, sel_lo, sel_hi, x);
      else load_w6<false>(wrow + 210 * b, lane, sel_lo, sel_hi, x);
      int s = 0;
#pragma unroll
      for (int v = 0; v < 8; v++) s += x.sc[v] * __dp4a((int)x.q[v], ax[b][v], __dp4a((int)0xE0E0E0E0u, ax[b][v], 0));
      acc = __fmaf_rn(__fmul_rn(x.d, yd[b]), __int2float_rn(s), acc);
    }
    const float r = lane_reduce<RV_Q6_K>(acc, 0.0f);
    if (lane == 0 && rt < rows_here) g.out[tile * R + rt] = r;
    __syncthreads();  // every thread is done with this stage
    if (threadIdx.x == 0 && tile + (size_t)S * gridDim.x < n_tiles) {
      fence_proxy_async();  // the reads above happen before the copy overwrites the stage
      issue(tile + (size_t)S * gridDim.x, st);
    }
  }
}

// ------------------------------------------------------- integer taps
// One warp per block: lanes 0..7 write the eight lane sums, 0..3 the mins.
template <int FMT>
__global__ void k_block_sums(const uint8_t *w, const uint8_t *acts, int nb, int32_t *lanes_out,
                             int32_t *mins_out) {
  extern __shared__ __align__(16) uint8_t sm[];
  constexpr int BB = FMT == RV_Q4_K ? 144 : FMT == RV_Q5_K ? 176 : 210;
  const int b = blockIdx.x;
  if (b >= nb) return;
  for (int k = threadIdx.x; k < BB; k += blockDim.x) sm[k] = w[(size_t)b * BB + k];
  uint32_t *as = (uint32_t *)(sm + 256);
  const uint32_t *src = (const uint32_t *)(acts + (size_t)b * 292);
  for (int k = threadIdx.x; k < 73; k += blockDim.x) as[k] = src[k];
  __syncthreads();
  const int lane = threadIdx.x;
  if (lane < 8) {
    WBlock wb;
    load_wblock<FMT>(sm, lane, wb);
    int S, Mn;
    lane_sums<FMT>(wb, (const uint8_t *)as, lane, S, Mn);
    lanes_out[b * 8 + lane] = S;
    if (lane < 4) mins_out[b * 4 + lane] = FMT == RV_Q6_K ? 0 : Mn;
  }
}

// ------------------------------------------------------------ RMSNorm
// One CTA of 256 threads per row; n <= 256 * RV_NORM_MAXE.
#define RV_NORM_MAXE 16

// inv = (float)(1/sqrt(sum/n + eps)) with every double step correctly
// rounded, as norm.rs:51-60 computes it.
RV_DEVFN float rms_inv_from_sum(double sum, size_t n, float eps) {
  const double mean = __ddiv_rn(sum, (double)n);
  return __double2float_rn(__drcp_rn(__dsqrt_rn(__dadd_rn(mean, (double)eps))));
}

// The inverse RMS from a sum of squares `s` taken in some order other than
// the reference's: the correctly rounded f64 steps, and, when the result
// lies within 2^-38 of an f32 rounding midpoint (or is not finite), the
// serial sum over xs[0..n) redone here.
RV_DEVFN float rms_inv_tail(double s, const float *xs, size_t n, float eps) {
  const double mean = __ddiv_rn(s, (double)n);
  const double r = __drcp_rn(__dsqrt_rn(__dadd_rn(mean, (double)eps)));
  const float f = __double2float_rn(r);
  const double df = (double)f;
  const double up = (double)nextafterf(f, INFINITY), dn = (double)nextafterf(f, -INFINITY);
  const double mh = 0.5 * (df + up), ml = 0.5 * (df + dn);
  const double tol = fabs(r) * 0x1p-38;
  if (fabs(mh - r) <= tol || fabs(r - ml) <= tol || !isfinite(r)) {
    double ser = 0.0;
    for (size_t k = 0; k < n; k++) {
      const double v = (double)xs[k];
      ser = __dadd_rn(ser, __dmul_rn(v, v));
    }
    return rms_inv_from_sum(ser, n, eps);
  }
  return f;
}

// The reference sums v*v serially in f64 (norm.rs:38-60).  The tree sum
// used here differs from it by at most 2^-41 relative; when the resulting
// inverse RMS lies that close to a float rounding midpoint, thread 0 redoes
// the sum serially, so the float result is always the reference's.
RV_DEVFN float rms_inv_block(const float *xs /*smem*/, size_t n, float eps, double *red /*smem[33]*/) {
  double part = 0.0;
  for (size_t k = threadIdx.x; k < n; k += blockDim.x) {
    const double v = (double)xs[k];
    part = __dadd_rn(part, __dmul_rn(v, v));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) part = __dadd_rn(part, __shfl_xor_sync(RV_FULL, part, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = part;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) s = __dadd_rn(s, red[w]);
    red[32] = (double)rms_inv_tail(s, xs, n, eps);
  }
  __syncthreads();
  return (float)red[32];
}

__global__ void __launch_bounds__(256) k_rmsnorm(const float *x, const float *w, size_t n, float eps,
                                                 float *out) {
  extern __shared__ __align__(16) uint8_t sm[];
  double *red = (double *)sm;
  float *xs = (float *)(sm + 34 * sizeof(double));
  const size_t row = blockIdx.x;
  for (size_t k = threadIdx.x; k < n; k += blockDim.x) xs[k] = x[row * n + k];
  __syncthreads();
  const float inv = rms_inv_block(xs, n, eps, red);
  for (size_t k = threadIdx.x; k < n; k += blockDim.x)
    out[row * n + k] = __fmul_rn(__fmul_rn(xs[k], inv), w[k]);
}

// ------------------------------------------------------------ softmax
// One warp per row (softmax.rs:18-40): f32 max, f64 exp of (x - max), f32
// copy of each exponential, serial f64 sum in index order, f32 reciprocal.
__global__ void k_softmax(float *x, size_t n, size_t n_rows) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t row = (size_t)blockIdx.x * (blockDim.x >> 5) + warp;
  double *e = (double *)sm + (size_t)warp * n;
  if (row >= n_rows) return;
  float *xr = x + row * n;
  float mx = -INFINITY;
  for (size_t k = lane; k < n; k += 32) mx = fmaxf(mx, xr[k]);
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(RV_FULL, mx, o));
  const double dmx = (double)mx;
  for (size_t k = lane; k < n; k += 32) e[k] = exp(__dsub_rn((double)xr[k], dmx));
  __syncwarp();
  double sum = 0.0;
  if (lane == 0)
    for (size_t k = 0; k < n; k++) sum = __dadd_rn(sum, e[k]);
  sum = __shfl_sync(RV_FULL, sum, 0);
  const float inv = __double2float_rn(__drcp_rn(sum));
  for (size_t k = lane; k < n; k += 32) xr[k] = __fmul_rn(__double2float_rn(e[k]), inv);
}

// ------------------------------------------------------------ SwiGLU
__global__ void k_swiglu(float *gate, const float *up, size_t n) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) gate[i] = swiglu_ref(gate[i], up[i]);
}

// --------------------------------------------------- synthetic weights
// SplitMix64 output function (Steele, Lea, Flood 2014).
RV_DEVFN uint64_t splitmix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Irwin-Hall(12): sum of twelve 24-bit uniforms, centred, scaled.  Exact
// integer arithmetic up to one float rounding and one multiply by sigma,
// so hosts and devices agree bit for bit.
__global__ void k_synth_normal(uint64_t seed, uint64_t offset, float sigma, float *out, size_t n) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint64_t j = offset + i;
  int64_t s = 0;
#pragma unroll
  for (int k = 0; k < 6; k++) {
    const uint64_t z = splitmix64(seed + (j * 6 + (uint64_t)k + 1) * 0x9E3779B97F4A7C15ull);
    s += (int64_t)(z >> 40) + (int64_t)((z >> 16) & 0xFFFFFFull);
  }
  s -= (int64_t)6 << 24;
  const float v = __fmul_rn((float)s, 0x1p-24f);
  out[i] = __fmul_rn(v, sigma);
}

// ----------------------------------------- the reference's weight quantizers
// kernels/quants/test_support.rs:59-219, one thread per 256-weight block,
// every float step with the reference's rounding (IEEE division, roundf =
// half away from zero, ceil, f16 round-to-nearest-even).
// f32 -> f16 bits, round to nearest even, as kernels/quants/f16.rs:39-91
// computes it (overflow to infinity, subnormals, quiet NaN).
RV_DEVFN uint16_t f32_to_f16_bits(float x) {
  const uint32_t bits = __float_as_uint(x);
  const uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
  const int exp = (int)((bits >> 23) & 0xFFu);
  const uint32_t frac = bits & 0x007FFFFFu;
  if (exp == 0xFF) return frac == 0 ? (uint16_t)(sign | 0x7C00u)
                                    : (uint16_t)(sign | 0x7C00u | 0x0200u | ((frac >> 13) & 0x03FFu));
  const int e16 = exp - 112;
  if (e16 >= 0x1F) return (uint16_t)(sign | 0x7C00u);
  if (e16 <= 0) {
    if (e16 < -10) return sign;
    const uint32_t mant = exp == 0 ? frac : (frac | 0x00800000u);
    const uint32_t shift = (uint32_t)(14 - e16);
    const uint32_t ulp = 1u << shift, half = ulp >> 1;
    uint32_t v = mant >> shift;
    const uint32_t rem = mant & (ulp - 1);
    if (rem > half || (rem == half && (v & 1u))) v += 1;
    return (uint16_t)(sign | v);
  }
  uint32_t v = ((uint32_t)e16 << 10) | (frac >> 13);
  const uint32_t rem = frac & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (v & 1u))) v += 1;
  return (uint16_t)(sign | v);
}
RV_DEVFN float f16_round(float v) { return h2f(f32_to_f16_bits(v)); }
RV_DEVFN uint8_t clamp_u8(float v, float lo, float hi) {
  if (v < lo) v = lo;
  else if (v > hi) v = hi;
  if (v != v) return 0;
  return (uint8_t)v;
}
// Both f16 fields of every weight block sit at even offsets.
RV_DEVFN void put_f16(uint8_t *p, float v) { *(uint16_t *)p = f32_to_f16_bits(v); }

template <int LEVELS>
RV_DEVFN void affine_scales_dev(const float *xs, uint8_t *scales, float &d, float &dmin,
                                float *step, float *minv) {
  float scale_f[8], min_f[8];
  for (int j = 0; j < 8; j++) {
    float vmin = INFINITY, vmax = -INFINITY;
    for (int l = 0; l < 32; l++) {
      const float v = xs[32 * j + l];
      vmin = fminf(vmin, v);
      vmax = fmaxf(vmax, v);
    }
    min_f[j] = fmaxf(-vmin, 0.0f);
    scale_f[j] = fmaxf(__fdiv_rn(__fadd_rn(vmax, min_f[j]), (float)LEVELS), 0.0f);
  }
  float max_scale = 0.0f, max_min = 0.0f;
  for (int j = 0; j < 8; j++) {
    max_scale = fmaxf(max_scale, scale_f[j]);
    max_min = fmaxf(max_min, min_f[j]);
  }
  d = f16_round(__fdiv_rn(max_scale, 63.0f));
  dmin = f16_round(__fdiv_rn(max_min, 63.0f));
  uint8_t ls[8], lm[8];
  for (int j = 0; j < 8; j++) {
    ls[j] = d > 0.0f ? clamp_u8(ceilf(__fdiv_rn(scale_f[j], d)), 0.0f, 63.0f) : 0;
    lm[j] = dmin > 0.0f ? clamp_u8(roundf(__fdiv_rn(min_f[j], dmin)), 0.0f, 63.0f) : 0;
    step[j] = __fmul_rn(d, (float)ls[j]);
    minv[j] = __fmul_rn(dmin, (float)lm[j]);
  }
  for (int k = 0; k < 12; k++) scales[k] = 0;
  for (int j = 0; j < 8; j++) {  // pack_scales_k4, test_support.rs:45-58
    if (j < 4) {
      scales[j] = ls[j] & 63;
      scales[j + 4] = lm[j] & 63;
    } else {
      scales[j + 4] = (uint8_t)((ls[j] & 0xF) | ((lm[j] & 0xF) << 4));
      scales[j - 4] |= (uint8_t)((ls[j] >> 4) << 6);
      scales[j] |= (uint8_t)((lm[j] >> 4) << 6);
    }
  }
}

RV_DEVFN uint8_t affine_q_dev(float v, float step, float min, float levels) {
  if (step <= 0.0f) return 0;
  return clamp_u8(roundf(__fdiv_rn(__fadd_rn(v, min), step)), 0.0f, levels);
}

template <int FMT>
__global__ void k_quantize_weights(const float *__restrict__ x, uint8_t *__restrict__ out,
                                   size_t n_blocks) {
  const size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= n_blocks) return;
  const float *xs = x + b * 256;
  if constexpr (FMT == RV_Q4_K || FMT == RV_Q5_K) {
    constexpr int L = FMT == RV_Q4_K ? 15 : 31;
    constexpr int BB = FMT == RV_Q4_K ? 144 : 176;
    uint8_t *o = out + b * BB;
    uint8_t scales[12];
    float d, dmin, step[8], minv[8];
    affine_scales_dev<L>(xs, scales, d, dmin, step, minv);
    put_f16(o, d);
    put_f16(o + 2, dmin);
    for (int k = 0; k < 12; k++) o[4 + k] = scales[k];
    if constexpr (FMT == RV_Q4_K) {
      for (int span = 0; span < 4; span++)
        for (int l = 0; l < 32; l++) {
          const int j0 = 2 * span, j1 = 2 * span + 1;
          const uint8_t q0 = affine_q_dev(xs[64 * span + l], step[j0], minv[j0], 15.0f);
          const uint8_t q1 = affine_q_dev(xs[64 * span + 32 + l], step[j1], minv[j1], 15.0f);
          o[16 + 32 * span + l] = (uint8_t)(q0 | (q1 << 4));
        }
    } else {
      uint8_t qh[32];
      for (int l = 0; l < 32; l++) qh[l] = 0;
      for (int span = 0; span < 4; span++)
        for (int l = 0; l < 32; l++) {
          const int j0 = 2 * span, j1 = 2 * span + 1;
          const uint8_t q0 = affine_q_dev(xs[64 * span + l], step[j0], minv[j0], 31.0f);
          const uint8_t q1 = affine_q_dev(xs[64 * span + 32 + l], step[j1], minv[j1], 31.0f);
          if (q0 >= 16) qh[l] |= (uint8_t)(1u << j0);
          if (q1 >= 16) qh[l] |= (uint8_t)(1u << j1);
          o[48 + 32 * span + l] = (uint8_t)((q0 & 0xF) | ((q1 & 0xF) << 4));
        }
      for (int l = 0; l < 32; l++) o[16 + l] = qh[l];
    }
  } else {
    uint8_t *o = out + b * 210;
    float scale_f[16];
    float max_scale = 0.0f;
    for (int g = 0; g < 16; g++) {
      float amax = 0.0f;
      for (int l = 0; l < 16; l++) amax = fmaxf(amax, fabsf(xs[16 * g + l]));
      scale_f[g] = __fdiv_rn(amax, 31.0f);
      max_scale = fmaxf(max_scale, scale_f[g]);
    }
    const float d = f16_round(__fdiv_rn(max_scale, 127.0f));
    uint8_t ls[16];
    for (int g = 0; g < 16; g++) ls[g] = d > 0.0f ? clamp_u8(ceilf(__fdiv_rn(scale_f[g], d)), 0.0f, 127.0f) : 0;
    for (int k = 0; k < 192; k++) o[k] = 0;
    for (int g = 0; g < 16; g++) {
      const float step = __fmul_rn(d, (float)ls[g]);
      for (int l = 0; l < 16; l++) {
        int v = 0;
        if (step > 0.0f) {
          float q = roundf(__fdiv_rn(xs[16 * g + l], step));
          q = q < -32.0f ? -32.0f : (q > 31.0f ? 31.0f : q);
          v = (int)q;
        }
        const uint8_t qq = (uint8_t)(v + 32);
        const int w = 16 * g + l, half = w >> 7, p = w & 127, quarter = p >> 5, l32 = p & 31;
        // inverse of the ql/qh packing in test_support.rs:197-210
        uint8_t *ql = o + 64 * half + (quarter & 1) * 32 + l32;
        *ql |= (uint8_t)((qq & 0xF) << (quarter >= 2 ? 4 : 0));
        o[128 + 32 * half + l32] |= (uint8_t)((qq >> 4) << (2 * quarter));
      }
    }
    for (int g = 0; g < 16; g++) o[192 + g] = ls[g];
    put_f16(o + 208, d);
  }
}

// ------------------------------------------------------------ Q8_0
// quantize.rs:37-54, one warp per 32-float block (lane = value).  amax
// starts at 0 and fmaxf drops NaN, as f32::max does; the scale math is
// IEEE f32; roundf rounds half away from zero; the cast saturates with
// NaN -> 0 like Rust's `as i8`.
RV_DEVFN int8_t sat_i8(float r) {
  if (r != r) return 0;
  if (r >= 127.0f) return 127;
  if (r <= -128.0f) return -128;
  return (int8_t)r;
}

__global__ void k_quantize_q8_0(const float *__restrict__ x, uint8_t *__restrict__ out, size_t n_blocks) {
  const int lane = threadIdx.x & 31;
  const size_t b = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (b >= n_blocks) return;  // warp-uniform
  const float v = x[b * 32 + lane];
  float amax = fmaxf(0.0f, fabsf(v));
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float d = __fdiv_rn(amax, 127.0f);
  const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
  uint8_t *o = out + b * 36;
  if (lane == 0) *(float *)o = f16_round(d);
  o[4 + lane] = (uint8_t)sat_i8(roundf(__fmul_rn(v, id)));
}

// gemv.rs:296-330 with avx2.rs:942-963 as the dot: out[(r - r0) * n_acts
// + a] = row(r) . act_a.  Block = R rows x 8 lanes; lane i of a row owns
// bytes 4i..4i+3 of every block: s = dp4a (exact), d = f16(w.d) * y.d,
// acc = fma(d, s, acc) in block order, then hsum_ps_8's tree across the
// eight lanes.  Weight tile staged like k_gemv; activations MT rows at a
// time (36-byte blocks).
template <int MT>
RV_DEVFN void gemv_q8_0_tile(const GemvArgs &g, size_t tile, uint8_t *sm) {
  uint64_t *bar = (uint64_t *)sm;
  const int R = g.R;
  const size_t act_row = (size_t)g.nb * 36;
  uint8_t *wsm = sm + 16;
  uint8_t *asm_ = wsm + ((R * g.row_bytes + 15) & ~(size_t)15) + 16;
  const size_t tile0 = tile * R;
  const int rows_here = (int)min((size_t)R, g.nrows - tile0);
  const uint8_t *wsrc = g.w + (g.r0 + tile0) * g.row_bytes;
  const size_t wbytes = (size_t)rows_here * g.row_bytes;
  const bool bulk = rv_bulk_ok(wsrc, wsm, wbytes);
  if (threadIdx.x == 0) mbar_init(bar, 1);
  __syncthreads();
  if (bulk) {
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(bar, (uint32_t)wbytes);
      bulk_g2s(wsm, wsrc, (uint32_t)wbytes, bar);
    }
  } else {
    rv_copy_bytes_block(wsm, wsrc, wbytes);
  }
  const int r = threadIdx.x >> 3, lane = threadIdx.x & 7;
  const int rr = r < rows_here ? r : 0;  // idle rows compute row 0, never store
  const uint8_t *wrow = wsm + (size_t)rr * g.row_bytes;
  bool ok = true;
  for (size_t a0 = 0; a0 < g.n_acts; a0 += MT) {
    const int mt = (int)min((size_t)MT, g.n_acts - a0);
    __syncthreads();  // previous chunk fully consumed
    stage_to_smem(asm_, g.acts + a0 * act_row, (size_t)mt * act_row);
    if (a0 == 0 && bulk) ok = mbar_wait_bounded(bar, 0);
    __syncthreads();
    if (!ok) return;
    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; m++) acc[m] = 0.0f;
    for (int b = 0; b < g.nb; b++) {
      const uint16_t *blk = (const uint16_t *)(wrow + (size_t)b * 34);  // 34-byte blocks: 2-byte aligned
      const float wd = h2f(blk[0]);
      const int w4 = (int)((uint32_t)blk[1 + 2 * lane] | ((uint32_t)blk[2 + 2 * lane] << 16));
#pragma unroll
      for (int m = 0; m < MT; m++)
        if (m < mt) {
          const uint8_t *ab = asm_ + m * act_row + (size_t)b * 36;
          const int s = __dp4a(w4, *(const int *)(ab + 4 + 4 * lane), 0);
          acc[m] = __fmaf_rn(__fmul_rn(wd, *(const float *)ab), (float)s, acc[m]);
        }
    }
#pragma unroll
    for (int m = 0; m < MT; m++) {
      float s = __fadd_rn(acc[m], __shfl_xor_sync(0xffffffffu, acc[m], 4));
      s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 2));
      s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 1));
      if (lane == 0 && r < rows_here && m < mt) gemv_store(g, (tile0 + r) * g.n_acts + a0 + m, s);
    }
  }
}

template <int MT>
__global__ void __launch_bounds__(256) k_gemv_q8_0(GemvArgs g) {
  extern __shared__ __align__(16) uint8_t sm[];
  gemv_q8_0_tile<MT>(g, blockIdx.x, sm);
}

// ----------------------------------------------- one warp per row (decode)
// Single-activation GEMV with a warp per row.  Lane 8g + l (group g, lane l
// of the reference's eight) computes the integer lane sums of blocks g,
// g + 4, g + 8, ... and their scale products (lane_sums, d * yd, dmin * yd);
// then every group runs lane l's float chain over blocks 0..nb-1 in order,
// taking each block's values by shuffle from the group that computed them,
// and reduces as lane_reduce does: the float steps of gemv_tile (lane_step
// per block) in the same order, so the same bits, with four times the warps
// and a quarter of the integer work per thread.  The host picks this tile
// when gemv_wide_nbg(format, nb) > 0 (nb = 4 * NBG) and there is one
// activation row; blockDim = 32 * R.
__host__ __device__ constexpr int gemv_wide_nbg(int fmt, int nb) {
  return fmt == RV_Q8_0 ? (nb == 64 ? 16 : 0) : (nb == 8 ? 2 : nb == 16 ? 4 : 0);
}

// Shared memory of a warp-per-row tile: [16: mbarrier][R rows][16][act_row][16].
__host__ __device__ inline size_t gemv_tile_smem(int R, size_t row_bytes, size_t act_row) {
  return 16 + ((R * row_bytes + 15) & ~(size_t)15) + 16 + ((act_row + 15) & ~(size_t)15) + 16;
}

// Stages an R-row weight tile (bulk copy when aligned) and the activation
// row; false when the copy's wait gave up.
RV_DEVFN bool gemv_stage_row_tile(const GemvArgs &g, size_t tile, uint8_t *sm, size_t act_row, uint8_t *&wsm,
                                  uint8_t *&asm_, int &rows_here) {
  uint64_t *bar = (uint64_t *)sm;
  wsm = sm + 16;
  asm_ = wsm + ((g.R * g.row_bytes + 15) & ~(size_t)15) + 16;
  const size_t tile0 = tile * g.R;
  rows_here = (int)min((size_t)g.R, g.nrows - tile0);
  const uint8_t *wsrc = g.w + (g.r0 + tile0) * g.row_bytes;
  const size_t wbytes = (size_t)rows_here * g.row_bytes;
  const bool bulk = rv_bulk_ok(wsrc, wsm, wbytes);
  if (threadIdx.x == 0) mbar_init(bar, 1);
  __syncthreads();
  if (bulk) {
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(bar, (uint32_t)wbytes);
      bulk_g2s(wsm, wsrc, (uint32_t)wbytes, bar);
    }
  } else {
    rv_copy_bytes_block(wsm, wsrc, wbytes);
  }
  stage_to_smem(asm_, g.acts, act_row);
  bool ok = true;
  if (bulk) ok = mbar_wait_bounded(bar, 0);
  return __syncthreads_and(ok);
}

template <int FMT, int NBG>
RV_DEVFN void gemv_tile_wide(const GemvArgs &g, size_t tile, uint8_t *sm) {
  constexpr int NB = 4 * NBG;
  constexpr int BB = FMT == RV_Q4_K ? 144 : FMT == RV_Q5_K ? 176 : 210;
  uint8_t *wsm, *asm_;
  int rows_here;
  if (!gemv_stage_row_tile(g, tile, sm, (size_t)NB * 292, wsm, asm_, rows_here)) return;
  const int r = threadIdx.x >> 5, lane = threadIdx.x & 31, l = lane & 7, grp = lane >> 3;
  const uint8_t *wrow = wsm + (size_t)(r < rows_here ? r : 0) * g.row_bytes;  // idle rows compute row 0
  int S[NBG], M[NBG];
  float dy[NBG], dmy[NBG];
#pragma unroll
  for (int i = 0; i < NBG; i++) {
    const int b = 4 * i + grp;
    const uint8_t *act = asm_ + (size_t)b * 292;
    WBlock w;
    load_wblock<FMT>(wrow + (size_t)b * BB, l, w);
    M[i] = 0;
    lane_sums<FMT>(w, act, l, S[i], M[i]);
    const float yd = *(const float *)act;
    dy[i] = __fmul_rn(w.d, yd);
    dmy[i] = __fmul_rn(w.dmin, yd);
  }
  float acc = 0.0f, accm = 0.0f;
#pragma unroll
  for (int b = 0; b < NB; b++) {
    const int src = 8 * (b & 3) + l;
    const int Sb = __shfl_sync(RV_FULL, S[b >> 2], src);
    const float d = __shfl_sync(RV_FULL, dy[b >> 2], src);
    if constexpr (FMT != RV_Q6_K) {
      const int Mb = __shfl_sync(RV_FULL, M[b >> 2], src);
      const float dm = __shfl_sync(RV_FULL, dmy[b >> 2], src);
      if (l < 4) accm = __fmaf_rn(dm, __int2float_rn(Mb), accm);
    }
    acc = __fmaf_rn(d, __int2float_rn(Sb), acc);
  }
  const float res = lane_reduce<FMT>(acc, accm);
  if (lane == 0 && r < rows_here) gemv_store(g, tile * g.R + r, res);
}

// The Q8_0 form (34-byte blocks of an f16 scale and 32 int8; 36-byte Q8_0
// activation blocks of an f32 scale and 32 int8): lane l's step per block
// is acc = fma(wd * ad, dp4a(w word l, a word l), acc), then the xor 4, 2,
// 1 reduction, as gemv_q8_0_tile.
template <int NBG>
RV_DEVFN void gemv_q8_0_tile_wide(const GemvArgs &g, size_t tile, uint8_t *sm) {
  constexpr int NB = 4 * NBG;
  uint8_t *wsm, *asm_;
  int rows_here;
  if (!gemv_stage_row_tile(g, tile, sm, (size_t)NB * 36, wsm, asm_, rows_here)) return;
  const int r = threadIdx.x >> 5, lane = threadIdx.x & 31, l = lane & 7, grp = lane >> 3;
  const uint8_t *wrow = wsm + (size_t)(r < rows_here ? r : 0) * g.row_bytes;
  int S[NBG];
  float p[NBG];
#pragma unroll
  for (int i = 0; i < NBG; i++) {
    const int b = 4 * i + grp;
    const uint16_t *blk = (const uint16_t *)(wrow + (size_t)b * 34);  // 34-byte blocks: 2-byte aligned
    const uint8_t *ab = asm_ + (size_t)b * 36;
    const int w4 = (int)((uint32_t)blk[1 + 2 * l] | ((uint32_t)blk[2 + 2 * l] << 16));
    S[i] = __dp4a(w4, *(const int *)(ab + 4 + 4 * l), 0);
    p[i] = __fmul_rn(h2f(blk[0]), *(const float *)ab);
  }
  float acc = 0.0f;
#pragma unroll
  for (int b = 0; b < NB; b++) {
    const int src = 8 * (b & 3) + l;
    const int Sb = __shfl_sync(RV_FULL, S[b >> 2], src);
    const float pb = __shfl_sync(RV_FULL, p[b >> 2], src);
    acc = __fmaf_rn(pb, (float)Sb, acc);
  }
  float v = __fadd_rn(acc, __shfl_xor_sync(RV_FULL, acc, 4));
  v = __fadd_rn(v, __shfl_xor_sync(RV_FULL, v, 2));
  v = __fadd_rn(v, __shfl_xor_sync(RV_FULL, v, 1));
  if (lane == 0 && r < rows_here) gemv_store(g, tile * g.R + r, v);
}

template <int NBG>
__global__ void __launch_bounds__(256) k_gemv_q8_0_wide(GemvArgs g) {
  extern __shared__ __align__(16) uint8_t sm[];
  gemv_q8_0_tile_wide<NBG>(g, blockIdx.x, sm);
}

template <int FMT, int NBG>
__global__ void __launch_bounds__(256) k_gemv_wide(GemvArgs g) {
  extern __shared__ __align__(16) uint8_t sm[];
  gemv_tile_wide<FMT, NBG>(g, blockIdx.x, sm);
}

// Several single-activation GEMVs in one launch (the attention projections
// q, k, v): CTAs [cta0[j], cta0[j+1]) run job j's tiles with job j's format
// (Q4_K / Q5_K / Q6_K against Q8_K activations, Q8_0 against Q8_0).  Every
// job uses the same R (rows per CTA, blockDim = 8R).
#define RV_GEMV_MULTI 4
struct GemvMulti {
  GemvArgs job[RV_GEMV_MULTI];
  int fmt[RV_GEMV_MULTI];
  unsigned cta0[RV_GEMV_MULTI + 1];
  int n;
};
__global__ void __launch_bounds__(256) k_gemv_multi(GemvMulti m) {
  extern __shared__ __align__(16) uint8_t sm[];
  int j = 0;
  while (j + 1 < m.n && blockIdx.x >= m.cta0[j + 1]) j++;
  const size_t tile = blockIdx.x - m.cta0[j];
  // The host sized each job's R for the tile chosen here: blockDim / 32 rows
  // for the warp-per-row tiles, blockDim / 8 for the others.
  const GemvArgs &g = m.job[j];
  switch (m.fmt[j] * 100 + gemv_wide_nbg(m.fmt[j], g.nb)) {
    case RV_Q4_K * 100 + 2: gemv_tile_wide<RV_Q4_K, 2>(g, tile, sm); break;
    case RV_Q4_K * 100 + 4: gemv_tile_wide<RV_Q4_K, 4>(g, tile, sm); break;
    case RV_Q5_K * 100 + 2: gemv_tile_wide<RV_Q5_K, 2>(g, tile, sm); break;
    case RV_Q5_K * 100 + 4: gemv_tile_wide<RV_Q5_K, 4>(g, tile, sm); break;
    case RV_Q6_K * 100 + 2: gemv_tile_wide<RV_Q6_K, 2>(g, tile, sm); break;
    case RV_Q6_K * 100 + 4: gemv_tile_wide<RV_Q6_K, 4>(g, tile, sm); break;
    case RV_Q8_0 * 100 + 16: gemv_q8_0_tile_wide<16>(g, tile, sm); break;
    case RV_Q4_K * 100: gemv_tile<RV_Q4_K, 1>(g, tile, sm); break;
    case RV_Q5_K * 100: gemv_tile<RV_Q5_K, 1>(g, tile, sm); break;
    case RV_Q6_K * 100: gemv_tile<RV_Q6_K, 1>(g, tile, sm); break;
    default: gemv_q8_0_tile<1>(g, tile, sm); break;
  }
}

// ------------------------------------------------------- dequantization
// dequant.rs:28-147, one thread per output value, f32 expressions with the
// reference's roundings (no contraction).  Row i of the output is weight
// row rows[i] (or i when rows is null); an id past out_dim writes zeros
// and sets the device error word.
template <int FMT>
__global__ void k_dequant_rows(const uint8_t *__restrict__ w, size_t row_bytes, size_t in_dim, size_t out_dim,
                               const uint32_t *__restrict__ rows, size_t n_rows, float *__restrict__ out) {
  const size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n_rows * in_dim) return;
  const size_t i = e / in_dim, c = e % in_dim;
  const size_t row = rows ? rows[i] : i;
  if (row >= out_dim) {
    if (c == 0) rv_dev_fail(RV_ERR_TOKEN_OUT_OF_RANGE);
    out[e] = 0.0f;
    return;
  }
  const uint8_t *wr = w + row * row_bytes;
  float v;
  if constexpr (FMT == RV_Q8_0) {
    const uint8_t *blk = wr + (c >> 5) * 34;
    v = __fmul_rn(h2f((uint16_t)(blk[0] | (blk[1] << 8))), (float)(int8_t)blk[2 + (c & 31)]);
  } else if constexpr (FMT == RV_Q6_K) {
    const uint8_t *blk = wr + (c >> 8) * 210;
    const int p = (int)(c & 255), half = p >> 7, quarter = (p & 127) >> 5, l = p & 31;
    const uint8_t *ql = blk + 64 * half, *qh = blk + 128 + 32 * half, *sc = blk + 192 + 8 * half;
    const int lo = (quarter & 1) ? ql[l + 32] : ql[l];
    const int q = (((quarter >= 2) ? (lo >> 4) : (lo & 0xF)) | (((qh[l] >> (2 * quarter)) & 3) << 4)) - 32;
    const float d = h2f((uint16_t)(blk[208] | (blk[209] << 8)));
    v = __fmul_rn(__fmul_rn(d, (float)(int8_t)sc[(l >> 4) + 2 * quarter]), (float)q);
  } else {
    constexpr int BB = FMT == RV_Q4_K ? 144 : 176;
    const uint8_t *blk = wr + (c >> 8) * BB;
    const int p = (int)(c & 255), span = p >> 6, hi = (p >> 5) & 1, l = p & 31, j = 2 * span + hi;
    const uint8_t *s = blk + 4;
    int sc, m;
    if (j < 4) {
      sc = s[j] & 63;
      m = s[j + 4] & 63;
    } else {
      sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
      m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
    const uint8_t qb = blk[(FMT == RV_Q4_K ? 16 : 48) + 32 * span + l];
    int q = hi ? (qb >> 4) : (qb & 0xF);
    if constexpr (FMT == RV_Q5_K) q += ((blk[16 + l] >> j) & 1) ? 16 : 0;
    const float d = h2f((uint16_t)(blk[0] | (blk[1] << 8))), dmin = h2f((uint16_t)(blk[2] | (blk[3] << 8)));
    v = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)m));
  }
  out[e] = v;
}

// rmsnorm (norm.rs:38-60) fused with quantize_row_q8_k and, optionally,
// quantize_row_q8_0 of the normed row: the attention projections' and the
// lm_head's inputs.  One CTA (256 threads) per 256-value block; every CTA
// computes the row's exact inverse RMS (rms_inv_block), normalizes its
// block (x * inv * w, separate f32 multiplies), writes the Q8_K block (warp
// 0) and the block's eight Q8_0 blocks (warps 0..7, lane = value).
__global__ void __launch_bounds__(256) k_norm_quant(const float *__restrict__ x, const float *__restrict__ w, int n,
                                                    float eps, uint8_t *__restrict__ q8k, uint8_t *__restrict__ q80) {
  extern __shared__ __align__(16) uint8_t sm[];
  double *red = (double *)sm;
  float *xs = (float *)(sm + 34 * sizeof(double));
  const int b = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float wk = w[256 * b + threadIdx.x];  // blockDim.x == 256: one weight per thread, loaded up front
  stage_to_smem(xs, x, (size_t)n * sizeof(float));
  __syncthreads();
  const float inv = rms_inv_block(xs, (size_t)n, eps, red);
  float *ys = xs + n;  // this block's normed values
  ys[threadIdx.x] = __fmul_rn(__fmul_rn(xs[256 * b + threadIdx.x], inv), wk);
  __syncthreads();
  if (warp == 0) {
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; e++) v[e] = ys[8 * lane + e];
    q8k_quantize_warp(v, lane, q8k + (size_t)b * 292);
  }
  if (q80 && warp < 8) {
    const float v = ys[32 * warp + lane];
    float amax = fmaxf(0.0f, fabsf(v));
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    uint8_t *o = q80 + (size_t)(8 * b + warp) * 36;
    if (lane == 0) *(float *)o = f16_round(d);
    o[4 + lane] = (uint8_t)sat_i8(roundf(__fmul_rn(v, id)));
  }
}
