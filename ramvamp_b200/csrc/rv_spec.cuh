// rv_spec.cuh -- speculative expert dispatch for decode.
//
// The reference's router logit is a serial f32 chain, acc = acc + r[k]*x[k]
// for k = 0..H-1 (forward.rs:1231-1237): 2048 dependent adds, the longest
// dependent step of a decode layer.  The expert kernels do not need the
// logit values, only which experts are selected, and that can be known
// before the chain has finished:
//
//   * The routing kernel forms the same f32 products and sums them exactly
//     enough in f64 (a tree), together with a rigorous bound on how far the
//     serial f32 chain can land from that sum.  With p_k the f32 products,
//     S_k = p_1 + ... + p_k (real) and u = 2^-24, each add of the chain
//     errs by at most u * |its exact result|, so
//         |chain - S_H| <= u / (1 - H u) * sum_k |S_k|          (running-
//     error bound for recursive summation; Higham, Accuracy and Stability
//     of Numerical Algorithms, 2nd ed., sec. 4.2 and 4.3).  The f64 sums
//     carry their own rounding, bounded by g = 2^-39 times sum |p_k|, and
//     the result is rounded outward to an f32 interval [lo, hi] that holds
//     the chain's value.
//   * Expert e of token t is speculated when hi_e + delta >= L, where L is
//     the K-th largest lo over the experts (with multiplicity) and delta =
//     2^-18.  Every other expert f has at least K experts whose logits
//     exceed its own by more than delta; their softmax probabilities (f64
//     exponential of logit - max, f32 rounding, f32 product with the f32
//     reciprocal of the sum; forward.rs:2669-2705) are then strictly larger
//     as long as none underflows, so the repeated strict-'>' argmax never
//     reaches f.  The underflow guard is L - max(hi) >= -75 (every
//     candidate's probability stays a normal float); when it fails, or a
//     bound is not finite, every expert is speculated.
//
// The speculated set therefore always contains the exact top-k; it is
// usually exactly k experts, and a few more when two logits lie within the
// bound of each other.  The gate/up kernel runs on the speculated pairs
// while the exact chains run beside it, and the down kernel stores only
// the pairs the exact routing selected.  Every stored value is computed by
// the same arithmetic as without speculation, so results are unchanged.
#pragma once
#include "rv_internal.cuh"

#define RV_SPEC_MAX_T 8                  // tokens per speculative call
#define RV_SPEC_DELTA 0x1p-18f           // logit margin for a strict probability order
#define RV_SPEC_UNDERFLOW 75.0f          // exp(-75) * 2^-8 is still a normal float

// Unsigned keys that order floats like the floats (NaN excluded).
RV_DEVFN uint32_t spec_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
RV_DEVFN float spec_unkey(uint32_t k) { return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k); }

// The interval [lo, hi] holding the serial chain acc = acc + row[k]*x[k]
// (k = 0..H-1, f32, no FMA), from the f64 sums of the same f32 products,
// by one warp.  Lane l owns the c = H/32 elements from B = l*c on and
// bounds their share of sum_k |S_k| by c*|S_B| + sum_j (c - j)*|p_{B+j}|
// (|S_{B+j}| <= |S_B| + |p_B| + ... + |p_{B+j}|), so one pass over the
// products and one scan of the lane sums suffice.  Lane l visits its float4
// groups from a rotation by l, which keeps the shared-memory reads free of
// bank conflicts.  The result is valid in lane 0; the pair is (NaN, NaN)
// when a product or the bound is not finite or too large for the chain to
// stay finite.
RV_DEVFN float2 spec_bounds_warp(const float *row, const float *x, int H, int lane) {
  const int c = H >> 5, nq = c >> 2;  // H is a multiple of 256: nq >= 2
  const float4 *r4 = (const float4 *)(row + lane * c), *x4 = (const float4 *)(x + lane * c);
  double s[4] = {0.0, 0.0, 0.0, 0.0}, sa[4] = {0.0, 0.0, 0.0, 0.0}, ws[4] = {0.0, 0.0, 0.0, 0.0};
  for (int q = 0; q < nq; q++) {
    const int qq = (q + lane) % nq;
    const float4 a = r4[qq], b = x4[qq];
    const float pf[4] = {__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y), __fmul_rn(a.z, b.z), __fmul_rn(a.w, b.w)};
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const double p = (double)pf[i], ap = fabs(p);
      s[i] = __dadd_rn(s[i], p);
      sa[i] = __dadd_rn(sa[i], ap);
      ws[i] = __fma_rn((double)(c - 4 * qq - i), ap, ws[i]);
    }
  }
  const double sum = __dadd_rn(__dadd_rn(s[0], s[1]), __dadd_rn(s[2], s[3]));
  double sabs = __dadd_rn(__dadd_rn(sa[0], sa[1]), __dadd_rn(sa[2], sa[3]));
  const double wsum = __dadd_rn(__dadd_rn(ws[0], ws[1]), __dadd_rn(ws[2], ws[3]));
  double inc = sum;  // inclusive scan of the lane sums
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(RV_FULL, inc, o);
    if (lane >= o) inc = __dadd_rn(inc, y);
  }
  const double A = __shfl_sync(RV_FULL, inc, 31);
  double spre = __dadd_rn(__dmul_rn((double)c, fabs(__dsub_rn(inc, sum))), wsum);
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    sabs = __dadd_rn(sabs, __shfl_xor_sync(RV_FULL, sabs, o));
    spre = __dadd_rn(spre, __shfl_xor_sync(RV_FULL, spre, o));
  }
  float2 out = make_float2(0.0f, 0.0f);
  if (lane == 0) {
    // Every f64 sum above has fewer than 2^13 roundings of magnitude at
    // most 2^-53 * sabs each: g = 2^-39 bounds them with room to spare.
    const double g = 0x1p-39, u = 0x1p-24 / (1.0 - (double)H * 0x1p-24);
    const double bd = (u * (spre + (double)H * g * sabs) + g * sabs) * (1.0 + g) * (1.0 + 0x1p-30);
    if (isfinite(sabs) && sabs < 0x1p100 && isfinite(bd)) {
      out.x = __double2float_rd(__dsub_rd(A, bd));
      out.y = __double2float_ru(__dadd_ru(A, bd));
    } else {
      out.x = out.y = __int_as_float(0x7fc00000);
    }
  }
  return out;
}

// The speculated (token, expert) pairs of one call, laid out like the
// dispatch index: positions grouped by expert in expert order, tokens in
// order within an expert; one work unit per expert with a pair.  Built in
// shared memory, identically by every CTA that needs it.
struct SpecSmem {
  uint32_t mask[256];  // tokens speculating expert e
  uint16_t start[257];  // first position of expert e; start[E] = positions
  uint8_t uexp[256];    // expert of unit u
  int n_units;
};

// The j-th (from 0) set bit of m.
RV_DEVFN int spec_nth_bit(uint32_t m, int j) {
  for (int i = 0; i < j; i++) m &= m - 1;
  return __ffs(m) - 1;
}

// Any block size that is a multiple of 32 (all threads call); E <= 256,
// K <= 16, T <= 8.  spec: [T][E] (lo, hi) written by an earlier kernel,
// read once (warp w handles tokens w, w + warps, ...).
RV_DEVFN void spec_build(int E, int K, int T, const float2 *spec, SpecSmem &ss) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
  for (int e = tid; e < 256; e += blockDim.x) ss.mask[e] = 0u;
  __syncthreads();
  for (int t = warp; t < T; t += nw) {
    float2 b[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int e = lane + 32 * j;
      b[j] = e < E ? spec[(size_t)t * E + e] : make_float2(-INFINITY, -INFINITY);
    }
    uint32_t key[8];
    bool bad = false;
    float mhi = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      key[j] = lane + 32 * j < E ? spec_key(b[j].x) : 0u;  // 0 sorts below every float
      bad |= isnan(b[j].x) || isnan(b[j].y);
      mhi = fmaxf(mhi, b[j].y);
    }
    bad = __any_sync(RV_FULL, bad);
#pragma unroll
    for (int o = 16; o; o >>= 1) mhi = fmaxf(mhi, __shfl_xor_sync(RV_FULL, mhi, o));
    uint32_t m = 0u;
    for (int k = 0; k < K; k++) {  // remove the largest key K times
      uint32_t lm = key[0];
#pragma unroll
      for (int j = 1; j < 8; j++) lm = max(lm, key[j]);
      m = __reduce_max_sync(RV_FULL, lm);
      const unsigned win = __ballot_sync(RV_FULL, lm == m);
      if (lane == __ffs(win) - 1) {
        bool done = false;
#pragma unroll
        for (int j = 0; j < 8; j++)
          if (!done && key[j] == m) {
            key[j] = 0u;
            done = true;
          }
      }
    }
    const float thr = spec_unkey(m);
    const bool all = bad || !(__fsub_rd(thr, mhi) >= -RV_SPEC_UNDERFLOW);
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int e = lane + 32 * j;
      if (e < E && (all || __fadd_ru(b[j].y, RV_SPEC_DELTA) >= thr)) atomicOr(&ss.mask[e], 1u << t);
    }
  }
  __syncthreads();
  if (warp == 0) {
    int c[8], sc = 0, su = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const int e = lane * 8 + i;
      c[i] = e < E ? __popc(ss.mask[e]) : 0;
      sc += c[i];
      su += c[i] > 0;
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
      if (e < E) {
        ss.start[e] = (uint16_t)xc;
        if (c[i]) ss.uexp[xu++] = (uint8_t)e;
      }
      xc += c[i];
    }
    if (lane == 0) {
      ss.start[E] = (uint16_t)tc;
      ss.n_units = tu;
    }
  }
  __syncthreads();
}
