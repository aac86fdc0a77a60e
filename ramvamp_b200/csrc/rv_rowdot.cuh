// rv_rowdot.cuh -- row-per-thread, lane-exact k-quant dots.
//
// The reference's AVX2 dot (kernels/quants/avx2.rs:554-838) keeps eight i32
// lanes per super-block (lane L = bytes 4L..4L+3 of every 32-byte weight
// vector, scaled per vector), folds each block into eight f32 accumulators
// with one FMA per lane, and ends with a fixed horizontal-sum tree; Q4_K and
// Q5_K also carry four min lanes.  Here one thread owns all eight lanes of a
// weight row (so the block's scales are unpacked once, and the activation
// words are broadcast reads shared by every row of the warp), or -- for one
// token -- G threads share a row: each forms the integer lane sums of its
// blocks, and the FMA chain is handed from thread to thread in block order
// with shuffles, so every float operation is the reference's, in its order.
#pragma once
#include "rv_internal.cuh"

// Scales and mins of a Q4_K/Q5_K block via the three-word mask unpack
// (avx2.rs:463-485): sc bytes 0..7 in u0,u1; min bytes 0..7 in u2,u3.
RV_DEVFN void k4_unpack_words(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t &u0, uint32_t &u1,
                              uint32_t &u2, uint32_t &u3) {
  const uint32_t k1 = 0x3f3f3f3fu, k2 = 0x0f0f0f0fu, k3 = 0x03030303u;
  u3 = ((w2 >> 4) & k2) | (((w1 >> 6) & k3) << 4);
  u2 = w1 & k1;
  u1 = (w2 & k2) | (((w0 >> 6) & k3) << 4);
  u0 = w0 & k1;
}
RV_DEVFN int byte_of(uint32_t w, int k) { return (int)((w >> (8 * k)) & 0xFFu); }

// Four Q6_K levels q in [0, 63] (one per byte) -> the signed bytes q - 32:
// each byte's top bit is set before subtracting 32, so no byte borrows from
// the next, and flipping it back leaves q - 32 modulo 256.
RV_DEVFN uint32_t q6_centered(uint32_t v) { return ((v | 0x80808080u) - 0x20202020u) ^ 0x80808080u; }

// Activation blocks in shared memory come in two layouts: the packed Q8_K
// block (292 bytes: d, 256 levels, 16 i16 block sums), and -- AL -- an
// aligned copy (RV_ACT_AL bytes: levels at 0, block sums at 256, d at 288,
// 16-byte aligned), so the levels load four words at a time.
#define RV_ACT_AL 304
template <bool AL>
RV_DEVFN const int *act_levels(const uint8_t *act) { return (const int *)(act + (AL ? 0 : 4)); }
template <bool AL>
RV_DEVFN const int16_t *act_bsums(const uint8_t *act) { return (const int16_t *)(act + (AL ? 256 : 260)); }
template <bool AL>
RV_DEVFN float act_scale(const uint8_t *act) { return *(const float *)(act + (AL ? 288 : 0)); }
// Copies nb packed blocks (src, 4-byte aligned) into the aligned layout at
// dst, 32-bit words, threads t0, t0 + nt, ...
RV_DEVFN void act_align_row(const uint8_t *src, int nb, uint8_t *dst, int t0, int nt) {
  for (int i = t0; i < nb * 73; i += nt) {
    const int b = i / 73, w = i % 73;  // word w of packed block b: 0 = d, 1..64 levels, 65..72 block sums
    const uint32_t v = *(const uint32_t *)(src + (size_t)b * 292 + 4 * w);
    uint8_t *o = dst + (size_t)b * RV_ACT_AL;
    *(uint32_t *)(o + (w == 0 ? 288 : 4 * (w - 1))) = v;
  }
}

// Integer lanes of one block for one activation block `act` (in shared
// memory, packed and 4-byte aligned, or AL: the aligned layout).  `blk` is
// the weight block in shared memory: 16-byte aligned for Q4_K/Q5_K, any
// even address for Q6_K.
template <int FMT, bool AL = false>
RV_DEVFN void block_lanes(const uint8_t *blk, const uint8_t *act, int (&S)[8], int (&Mn)[4], float &dw,
                          float &dmw) {
  const int *aq = act_levels<AL>(act);
  if constexpr (FMT == RV_Q4_K || FMT == RV_Q5_K) {
    const uint4 hdr = *(const uint4 *)blk;
    dw = h2f((uint16_t)(hdr.x & 0xFFFFu));
    dmw = h2f((uint16_t)(hdr.x >> 16));
    uint32_t u0, u1, u2, u3;
    k4_unpack_words(hdr.y, hdr.z, hdr.w, u0, u1, u2, u3);
    uint4 qh0, qh1;
    if constexpr (FMT == RV_Q5_K) {
      qh0 = *(const uint4 *)(blk + 16);
      qh1 = *(const uint4 *)(blk + 32);
    }
    const uint8_t *qs = blk + (FMT == RV_Q4_K ? 16 : 48);
#pragma unroll
    for (int L = 0; L < 8; L++) S[L] = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const uint4 q0 = *(const uint4 *)(qs + 32 * j), q1 = *(const uint4 *)(qs + 32 * j + 16);
      const uint32_t q[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
      int aw[16];  // activation words 16j .. 16j+15
      if constexpr (AL) {
#pragma unroll
        for (int v = 0; v < 4; v++) {
          const int4 a4 = *(const int4 *)(aq + 16 * j + 4 * v);
          aw[4 * v] = a4.x;
          aw[4 * v + 1] = a4.y;
          aw[4 * v + 2] = a4.z;
          aw[4 * v + 3] = a4.w;
        }
      } else {
#pragma unroll
        for (int v = 0; v < 16; v++) aw[v] = aq[16 * j + v];
      }
      const int sl = byte_of(j < 2 ? u0 : u1, (2 * j) & 3), sh = byte_of(j < 2 ? u0 : u1, (2 * j + 1) & 3);
#pragma unroll
      for (int L = 0; L < 8; L++) {
        uint32_t lo = q[L] & 0x0F0F0F0Fu, hi = (q[L] >> 4) & 0x0F0F0F0Fu;
        if constexpr (FMT == RV_Q5_K) {
          const uint32_t h = L < 4 ? (&qh0.x)[L] : (&qh1.x)[L - 4];
          lo += ((h >> (2 * j)) & 0x01010101u) << 4;
          hi += ((h >> (2 * j + 1)) & 0x01010101u) << 4;
        }
        S[L] += sl * __dp4a((int)lo, aw[L], 0) + sh * __dp4a((int)hi, aw[8 + L], 0);
      }
    }
    const int16_t *bs = act_bsums<AL>(act);
#pragma unroll
    for (int l = 0; l < 4; l++) {
      const uint32_t mw = l < 2 ? u2 : u3;
      Mn[l] = byte_of(mw, (2 * l) & 3) * ((int)bs[4 * l] + (int)bs[4 * l + 1]) +
              byte_of(mw, (2 * l + 1) & 3) * ((int)bs[4 * l + 2] + (int)bs[4 * l + 3]);
    }
  } else {  // Q6_K: S[L] = sum_{h,k} sc * sum_t (q - 32) a, one dp4a of the centered levels
    dw = h2f(ld16(blk + 208));
    dmw = 0.0f;
    // Word i of the block (any even address): two aligned words and a
    // funnel shift; neighbouring words share their aligned loads.
    const uint32_t *wb = (const uint32_t *)((uintptr_t)blk & ~(uintptr_t)3);
    const uint32_t wsh = (uint32_t)((uintptr_t)blk & 3) * 8u;
    auto word = [&](int i) { return __funnelshift_r(wb[i], wb[i + 1], wsh); };
    const uint32_t sw[4] = {word(48), word(49), word(50), word(51)};
#pragma unroll
    for (int L = 0; L < 8; L++) S[L] = 0;
#pragma unroll
    for (int h = 0; h < 2; h++) {
      int aw[32];  // activation words 32h .. 32h+31
      if constexpr (AL) {
#pragma unroll
        for (int v = 0; v < 8; v++) {
          const int4 a4 = *(const int4 *)(aq + 32 * h + 4 * v);
          aw[4 * v] = a4.x;
          aw[4 * v + 1] = a4.y;
          aw[4 * v + 2] = a4.z;
          aw[4 * v + 3] = a4.w;
        }
      } else {
#pragma unroll
        for (int v = 0; v < 32; v++) aw[v] = aq[32 * h + v];
      }
#pragma unroll
      for (int L = 0; L < 8; L++) {
        const uint32_t ql0 = word(16 * h + L), ql1 = word(16 * h + 8 + L);
        const uint32_t qh = word(32 + 8 * h + L);
        const uint32_t v[4] = {(ql0 & 0x0F0F0F0Fu) | ((qh & 0x03030303u) << 4),
                               (ql1 & 0x0F0F0F0Fu) | (((qh >> 2) & 0x03030303u) << 4),
                               ((ql0 >> 4) & 0x0F0F0F0Fu) | (((qh >> 4) & 0x03030303u) << 4),
                               ((ql1 >> 4) & 0x0F0F0F0Fu) | (((qh >> 6) & 0x03030303u) << 4)};
#pragma unroll
        for (int k = 0; k < 4; k++) {
          const int w = 32 * h + 8 * k + L;  // activation word
          const int sidx = 8 * h + 2 * k + (L >= 4 ? 1 : 0);
          const int sc = (int)(int8_t)byte_of(sw[sidx >> 2], sidx & 3);
          S[L] += sc * __dp4a((int)q6_centered(v[k]), aw[w - 32 * h], 0);
        }
      }
    }
#pragma unroll
    for (int l = 0; l < 4; l++) Mn[l] = 0;
  }
}

// One block's float step for all eight lanes (avx2.rs:557-562, 598; 836).
template <int FMT>
RV_DEVFN void lanes_fma(const int (&S)[8], const int (&Mn)[4], float dw, float dmw, float yd,
                        float (&acc)[8], float (&accm)[4]) {
  if constexpr (FMT != RV_Q6_K) {
    const float dmin = __fmul_rn(dmw, yd);
#pragma unroll
    for (int l = 0; l < 4; l++) accm[l] = __fmaf_rn(dmin, __int2float_rn(Mn[l]), accm[l]);
  }
  const float d = __fmul_rn(dw, yd);
#pragma unroll
  for (int L = 0; L < 8; L++) acc[L] = __fmaf_rn(d, __int2float_rn(S[L]), acc[L]);
}

// hsum_ps_8(acc) - hsum_ps_4(accm) (avx2.rs:494-510), or hsum_ps_8 alone.
template <int FMT>
RV_DEVFN float lanes_final(const float (&acc)[8], const float (&accm)[4]) {
  const float a = __fadd_rn(__fadd_rn(__fadd_rn(acc[0], acc[4]), __fadd_rn(acc[2], acc[6])),
                            __fadd_rn(__fadd_rn(acc[1], acc[5]), __fadd_rn(acc[3], acc[7])));
  if constexpr (FMT == RV_Q6_K) return a;
  const float m = __fadd_rn(__fadd_rn(accm[0], accm[2]), __fadd_rn(accm[1], accm[3]));
  return __fsub_rn(a, m);
}

// One row against MT activation rows (token m at acts + m*astride), all
// blocks by this thread: the reference dot per token, exactly.
template <int FMT, int MT>
RV_DEVFN void row_dot_tokens(const uint8_t *wrow, int nb, const uint8_t *acts, size_t astride, int mt,
                             float (&out)[MT]) {
  constexpr int BB = FMT == RV_Q4_K ? 144 : FMT == RV_Q5_K ? 176 : 210;
  float acc[MT][8], accm[MT][4];
#pragma unroll
  for (int m = 0; m < MT; m++) {
#pragma unroll
    for (int L = 0; L < 8; L++) acc[m][L] = 0.0f;
#pragma unroll
    for (int l = 0; l < 4; l++) accm[m][l] = 0.0f;
  }
  for (int b = 0; b < nb; b++) {
#pragma unroll
    for (int m = 0; m < MT; m++) {
      if (m < mt) {
        const uint8_t *act = acts + (size_t)m * astride + (size_t)b * 292;
        int S[8], Mn[4];
        float dw, dmw;
        block_lanes<FMT>(wrow + (size_t)b * BB, act, S, Mn, dw, dmw);
        lanes_fma<FMT>(S, Mn, dw, dmw, *(const float *)act, acc[m], accm[m]);
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MT; m++) out[m] = lanes_final<FMT>(acc[m], accm[m]);
}

// One row, one token, the row's nb = G*NBG blocks split over G consecutive
// lanes of the warp (g = lane % G owns blocks [g*NBG, (g+1)*NBG); a row's G
// lanes never straddle two warps, and the callers keep 32/G rows per warp).  The
// integer lane sums are formed in parallel; the FMA chain then runs through
// the G lanes in block order, handed on with shuffles.  All 32 lanes must
// call; the result is valid on lanes with g == G-1.
template <int FMT, int G, int NBG, bool AL = false>
RV_DEVFN float row_dot_split(const uint8_t *wrow, const uint8_t *act_row, int g) {
  constexpr int BB = FMT == RV_Q4_K ? 144 : FMT == RV_Q5_K ? 176 : 210;
  int S[NBG][8], Mn[NBG][4];
  float dw[NBG], dmw[NBG], yd[NBG];
#pragma unroll
  for (int i = 0; i < NBG; i++) {
    const int b = g * NBG + i;
    const uint8_t *act = act_row + (size_t)b * (AL ? RV_ACT_AL : 292);
    block_lanes<FMT, AL>(wrow + (size_t)b * BB, act, S[i], Mn[i], dw[i], dmw[i]);
    yd[i] = act_scale<AL>(act);
  }
  float acc[8], accm[4];
#pragma unroll
  for (int L = 0; L < 8; L++) acc[L] = 0.0f;
#pragma unroll
  for (int l = 0; l < 4; l++) accm[l] = 0.0f;
  if (g == 0) {
#pragma unroll
    for (int i = 0; i < NBG; i++) lanes_fma<FMT>(S[i], Mn[i], dw[i], dmw[i], yd[i], acc, accm);
  }
  const int src = max((int)(threadIdx.x & 31) - 1, 0);  // lane g-1 of the same row
#pragma unroll
  for (int h = 1; h < G; h++) {
    float pa[8], pm[4];
#pragma unroll
    for (int L = 0; L < 8; L++) pa[L] = __shfl_sync(RV_FULL, acc[L], src);
#pragma unroll
    for (int l = 0; l < 4; l++) pm[l] = __shfl_sync(RV_FULL, accm[l], src);
    if (g == h) {
#pragma unroll
      for (int L = 0; L < 8; L++) acc[L] = pa[L];
#pragma unroll
      for (int l = 0; l < 4; l++) accm[l] = pm[l];
#pragma unroll
      for (int i = 0; i < NBG; i++) lanes_fma<FMT>(S[i], Mn[i], dw[i], dmw[i], yd[i], acc, accm);
    }
  }
  return lanes_final<FMT>(acc, accm);
}
