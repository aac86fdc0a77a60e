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
// (k = 0..H-1, f32, no FMA), by one warp.  Lane l owns the c = H/32
// elements from B = l*c on.  Its products are summed in f32, four
// interleaved running sums (element 4q+i into sum i) combined pairwise, so
// each product passes through at most c/4 + 2 roundings: the lane sum is
// within gamma = (c/4+2)u/(1-(c/4+2)u) * sum|p| of exact (u = 2^-24).  The
// lane's share of sum_k |S_k| is at most c*|S_B| + sum_j (c - j)*|p_{B+j}|
// (|S_{B+j}| <= |S_B| + |p_B| + ... + |p_{B+j}|); that weighted sum and
// sum |p| are accumulated rounding upward, so they bound their exact
// values from above.  The lane sums are then scanned exactly enough in
// f64, and
//   |chain - A| <= u' * (Spre + H*(gamma + g)*Sa) + (gamma + g)*Sa,
// with u' = u/(1 - H u), g = 2^-39 covering the f64 steps, Spre the bound
// on sum_k |S_k| from the scanned lane starts, Sa = sum |p|.  Lane l visits
// its float4 groups from a rotation by l, which keeps the shared-memory
// reads free of bank conflicts.  The result is valid in lane 0; the pair
// is (NaN, NaN) when a product or the bound is not finite or too large for
// the chain to stay finite.
RV_DEVFN float2 spec_bounds_warp(const float *row, const float *x, int H, int lane) {
  const int c = H >> 5, nq = c >> 2;  // H is a multiple of 256: nq >= 2
  const float4 *r4 = (const float4 *)(row + lane * c), *x4 = (const float4 *)(x + lane * c);
  float s[4] = {0.0f, 0.0f, 0.0f, 0.0f}, sa[4] = {0.0f, 0.0f, 0.0f, 0.0f}, ws[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  int qq = lane % nq;
  for (int q = 0; q < nq; q++) {
    const float4 a = r4[qq], b = x4[qq];
    const float pf[4] = {__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y), __fmul_rn(a.z, b.z), __fmul_rn(a.w, b.w)};
    const float w0 = (float)(c - 4 * qq);  // exact: c <= 128
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float ap = fabsf(pf[i]);
      s[i] = __fadd_rn(s[i], pf[i]);
      sa[i] = __fadd_ru(sa[i], ap);
      ws[i] = __fmaf_ru(w0 - (float)i, ap, ws[i]);
    }
    qq = qq + 1 == nq ? 0 : qq + 1;
  }
  const double sum = (double)__fadd_rn(__fadd_rn(s[0], s[1]), __fadd_rn(s[2], s[3]));
  double sabs = (double)__fadd_ru(__fadd_ru(sa[0], sa[1]), __fadd_ru(sa[2], sa[3]));
  const double wsum = (double)__fadd_ru(__fadd_ru(ws[0], ws[1]), __fadd_ru(ws[2], ws[3]));
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
    // gamma and u' through 1/(1 - x) <= 1 + 2x (x <= 1/2): upper bounds
    // without a division.
    const double u = 0x1p-24, g = 0x1p-39;
    const double gam = (double)(nq + 2) * u * (1.0 + 2.0 * (double)(nq + 2) * u);
    const double up = u * (1.0 + 2.0 * (double)H * u);
    const double sa = sabs * (1.0 + g);
    const double bd = (up * (spre * (1.0 + g) + (double)H * (gam + g) * sa) + (gam + g) * sa) * (1.0 + 0x1p-30);
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

// Token t's speculated experts, by one warp: lane l holds experts l + 32j.
// Loads the token's E bounds once (b), finds the threshold (the K-th
// largest lower bound, or lower) and returns the lane's membership bits
// (bit j: expert l + 32j is speculated).
RV_DEVFN uint32_t spec_token_bits(int E, int K, const float2 *spec_t, int lane) {
  float2 b[8];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int e = lane + 32 * j;
    b[j] = e < E ? spec_t[e] : make_float2(-INFINITY, -INFINITY);
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
  // K rounds, each removing every copy of the current maximum: with tied
  // keys this reaches a lower key than the K-th largest with multiplicity,
  // i.e. a lower threshold and a larger (still safe) set.
  uint32_t m = 0u;
  for (int k = 0; k < K; k++) {
    const uint32_t lm =
        max(max(max(key[0], key[1]), max(key[2], key[3])), max(max(key[4], key[5]), max(key[6], key[7])));
    m = __reduce_max_sync(RV_FULL, lm);
#pragma unroll
    for (int j = 0; j < 8; j++) key[j] = key[j] == m ? 0u : key[j];
  }
  const float thr = spec_unkey(m);
  const bool all = bad || m == 0u || !(__fsub_rd(thr, mhi) >= -RV_SPEC_UNDERFLOW);
  uint32_t bits = 0u;
#pragma unroll
  for (int j = 0; j < 8; j++)
    if (lane + 32 * j < E && (all || __fadd_ru(b[j].y, RV_SPEC_DELTA) >= thr)) bits |= 1u << j;
  return bits;
}

// Any block size that is a multiple of 32 (all threads call); E <= 256,
// K <= 16, T <= 8.  spec: [T][E] (lo, hi) written by an earlier kernel,
// read once (warp w handles tokens w, w + warps, ...).
RV_DEVFN void spec_build(int E, int K, int T, const float2 *spec, SpecSmem &ss) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
  for (int e = tid; e < 256; e += blockDim.x) ss.mask[e] = 0u;
  __syncthreads();
  for (int t = warp; t < T; t += nw) {
    const uint32_t bits = spec_token_bits(E, K, spec + (size_t)t * E, lane);
#pragma unroll
    for (int j = 0; j < 8; j++)
      if ((bits >> j) & 1u) atomicOr(&ss.mask[lane + 32 * j], 1u << t);
  }
  __syncthreads();
  if (warp == 0) {  // experts in rows of 32: unit ranks by ballot, positions by a scan
    int pbase = 0, ubase = 0;
    for (int r = 0; r * 32 < E; r++) {
      const int e = r * 32 + lane;
      const int cnt = e < E ? __popc(ss.mask[e]) : 0;
      const unsigned has = __ballot_sync(RV_FULL, cnt > 0);
      int inc = cnt;
      if (T > 1) {
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(RV_FULL, inc, o);
          if (lane >= o) inc += y;
        }
      } else {
        inc = __popc(has & (0xffffffffu >> (31 - lane)));
      }
      if (e < E) {
        ss.start[e] = (uint16_t)(pbase + inc - cnt);
        if (cnt) ss.uexp[ubase + __popc(has & ((1u << lane) - 1u))] = (uint8_t)e;
      }
      pbase += __shfl_sync(RV_FULL, inc, 31);
      ubase += __popc(has);
    }
    if (lane == 0) {
      ss.start[E] = (uint16_t)pbase;
      ss.n_units = ubase;
    }
  }
  __syncthreads();
}

// The speculated experts of every token, by one warp, as ascending lists
// cand[t * 256 + i], i < ncand[t], and as bit sets cmask[t * 8 + w] (bit
// b: expert 32w + b).  Only listed experts can be in token t's top-k.
RV_DEVFN void spec_candidates_warp(int E, int K, int T, const float2 *spec, uint8_t *cand, int *ncand,
                                   uint32_t *cmask, int lane) {
  for (int t = 0; t < T; t++) {
    const uint32_t bits = spec_token_bits(E, K, spec + (size_t)t * E, lane);
    int n = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const unsigned in = __ballot_sync(RV_FULL, (bits >> j) & 1u);
      if ((bits >> j) & 1u) cand[t * 256 + n + __popc(in & ((1u << lane) - 1u))] = (uint8_t)(lane + 32 * j);
      if (lane == 0) cmask[t * 8 + j] = in;
      n += __popc(in);
    }
    if (lane == 0) ncand[t] = n;
  }
}
