// rv_tc.cuh -- MoE prefill on the 5th-generation tensor cores (RV_MOE_TENSOR).
//
// The expert contractions run as tcgen05 matrix products whose every input
// is an exactly representable small integer, so the tensor cores return the
// reference's per-super-block integer sums exactly:
//   sumi      = sum_j sc_j * sum_{32} q * a      A = sc*q (Q4_K <= 945, Q5_K <= 1953),
//                                                B = a (the Q8_K levels), both exact in f16
//   sumi_mins = sum_j m_j * bsum32_j             one K=16 product per block:
//                                                A = [m_j, 32 m_j], B = [bsum32_j mod 32, bsum32_j div 32]
//   Q6_K: sc = 32*sh + sl, A_l = sl*(q-32), A_h = sh*(q-32), sumi = D_l + 32*D_h
// (every partial sum below 2^24, so the f32 accumulators hold the integers
// exactly).  The epilogue then applies the reference's scalar per-block float
// step (dot.rs:96-116, 152-184): acc += d_w*d_a*sumi - dmin_w*d_a*sumi_mins,
// in block order, with the same roundings.  Routing, SwiGLU, both Q8_K
// quantizations and the top-k-order combine are the exact path's, so the
// layer output equals the reference's scalar CPU path bit for bit.
//
// Operands are K-major in the canonical layout without swizzle: 8x8 f16 core
// matrices of 128 contiguous bytes.  A is dequantized into shared memory by
// four producer warps from raw super-blocks staged with bulk copies; B lives
// in global memory already in core-matrix order (one 1 KB bulk copy per 8
// rows per stage).  The accumulators of a super-block sit in tensor memory,
// double-buffered so the epilogue of block b overlaps the products of
// block b+1.  Per CTA: warp 0 stages, lane 0 of warp 1 issues tcgen05.mma
// and commits, warps 2-5 dequantize, warps 6-13 run the epilogue.  Every
// wait is bounded.
#pragma once
#include <cuda.h>

#include "rv_moe.cuh"

#define RV_TC_NT 128       // pair columns per tile
#define RV_TC_ROWS 128     // weight rows per CTA (the MMA's M)
#define RV_TC_KS 64        // K elements per shared-memory stage
#define RV_TC_THREADS 640  // 20 warps: 5 per scheduler at 96 registers fills its 16K-register file
#define RV_TC_PROD_WARPS 8
#define RV_TC_EPI_WARPS 8

// ------------------------------------------------------ tcgen05 wrappers
RV_DEVFN void tc_alloc(uint32_t *dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)),
               "r"(ncols)
               : "memory");
}
RV_DEVFN void tc_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
RV_DEVFN void tc_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
RV_DEVFN void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
RV_DEVFN void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16, issued by one thread.
RV_DEVFN void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every MMA this thread issued so far has completed.
RV_DEVFN void tc_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
// 16 consecutive f32 columns of this thread's tensor-memory lane.
RV_DEVFN void tc_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
// 4 consecutive f32 columns of this thread's tensor-memory lane.
RV_DEVFN void tc_ld4(uint32_t taddr, uint32_t (&v)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
               : "r"(taddr));
}
// 8 consecutive f32 columns of this thread's tensor-memory lane.
RV_DEVFN void tc_ld8(uint32_t taddr, uint32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(taddr));
}
RV_DEVFN void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
RV_DEVFN void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Shared-memory matrix descriptor: K-major, no swizzle; leading (K) byte
// offset 128 between the two core matrices one K=16 step reads, `sbo`
// bytes between 8-row groups; descriptor version 1 (sm_100).
RV_DEVFN uint64_t tc_desc(uint32_t saddr, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(128u >> 4) << 16) | ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) |
         (1ull << 46);
}
// Instruction descriptor, kind::f16: A, B f16 (K-major), D f32, M = 128.
RV_DEVFN uint32_t tc_idesc(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(RV_TC_ROWS >> 4) << 24);
}
// Byte offset of 16-byte chunk `chunk` (8 f16 of K) of row `row` in a
// [rows][64] K-major tile in the 128-byte-swizzle canonical layout: 8-row
// atoms of 1024 bytes, row r of an atom at r*128 with its chunks permuted by
// c ^ r (so the tensor core's reads of one K slice across rows hit
// different banks).  Atoms must be 1024-byte aligned.
RV_DEVFN uint32_t tc_sw_off(int row, int chunk) {
  return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4));
}
// Byte offset of 16-byte chunk `chunk` of row `row` in a tile without
// swizzle with `cpr` chunks per row (the K=16 mins operands).
RV_DEVFN uint32_t tc_core_off(int row, int chunk, int cpr = 8) {
  return (uint32_t)(((row >> 3) * cpr + chunk) * 128 + (row & 7) * 16);
}

// ------------------------------------------- integer operands in f16
// Inside every 8-element chunk of K the operands hold elements in the order
// PI = {0, 2, 1, 3, 4, 6, 5, 7} (the same for A and B, so the products are
// unchanged): a 32-bit word of four byte-sized levels then turns into two
// half2 (levels 0,2 and 1,3) with one mask each.  0x6400 | v is the f16
// 1024 + v, and one fused multiply-add (1024 + v)*s - 1024*s gives v*s
// exactly, because that integer is representable (|v*s| <= 2048) and
// 1024*s is too.
RV_DEVFN uint32_t tc_fma2(uint32_t bits, __half2 s, __half2 c) {
  __half2 x = *(__half2 *)&bits;
  x = __hfma2(x, s, c);
  return *(uint32_t *)&x;
}
RV_DEVFN __half2 tc_h2i(int v) { return __float2half2_rn((float)v); }
// Levels at bits [0,6) and [16,22) of x -> half2 of level*s.
RV_DEVFN uint32_t tc_lv2(uint32_t x, uint32_t mask, __half2 s, __half2 c) {
  return tc_fma2((x & mask) | 0x64006400u, s, c);
}

// Half h (sub-block 2j+h: 32 elements, chunks 4h..4h+3) of stage j of a
// Q4_K / Q5_K super-block (16-byte aligned in shared memory) for row r:
// values sc*q.  u0..u3: the block's scales and mins (k4_unpack_words).
// Stage 0 also writes chunk h of the row's K=16 mins operand: m_0..m_7
// (h = 0) or 32*m_0..32*m_7 (h = 1).
template <int FMT>
RV_DEVFN void tc_stage_k45(const uint8_t *blk, int j, int h, uint32_t u0, uint32_t u1, uint32_t u2, uint32_t u3,
                           uint8_t *a, uint8_t *a2, int r) {
  const int sb = 2 * j + h;
  const int sc = byte_of(j < 2 ? u0 : u1, sb & 3);
  const __half2 s2 = tc_h2i(sc), c2 = tc_h2i(-1024 * sc);
  const uint8_t *qs = blk + (FMT == RV_Q4_K ? 16 : 48) + 32 * j;
  const uint4 qa = *(const uint4 *)qs, qb = *(const uint4 *)(qs + 16);
  const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
  uint32_t hw[8];
  if constexpr (FMT == RV_Q5_K) {
    const uint4 ha = *(const uint4 *)(blk + 16), hb = *(const uint4 *)(blk + 32);
    hw[0] = ha.x; hw[1] = ha.y; hw[2] = ha.z; hw[3] = ha.w;
    hw[4] = hb.x; hw[5] = hb.y; hw[6] = hb.z; hw[7] = hb.w;
  }
  const int sh = 4 * h;
#pragma unroll
  for (int cc = 0; cc < 4; cc++) {
    uint32_t o[4];
#pragma unroll
    for (int t = 0; t < 2; t++) {
      const uint32_t w = q[2 * cc + t] >> sh;
      uint32_t x0 = w, x1 = w >> 8;
      if constexpr (FMT == RV_Q5_K) {
        const uint32_t hb5 = hw[2 * cc + t] >> sb;
        x0 = (x0 & 0x000F000Fu) | ((hb5 & 0x00010001u) << 4);
        x1 = (x1 & 0x000F000Fu) | (((hb5 >> 8) & 0x00010001u) << 4);
        o[2 * t] = tc_lv2(x0, 0x001F001Fu, s2, c2);
        o[2 * t + 1] = tc_lv2(x1, 0x001F001Fu, s2, c2);
      } else {
        o[2 * t] = tc_lv2(x0, 0x000F000Fu, s2, c2);
        o[2 * t + 1] = tc_lv2(x1, 0x000F000Fu, s2, c2);
      }
    }
    *(uint4 *)(a + tc_sw_off(r, 4 * h + cc)) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  if (j == 0) {  // the mins operand is in natural order on both sides
    const float f = h ? 32.0f : 1.0f;
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const uint32_t mw = k < 2 ? u2 : u3;
      __half2 t2 = __floats2half2_rn((float)byte_of(mw, (2 * k) & 3) * f, (float)byte_of(mw, (2 * k + 1) & 3) * f);
      o[k] = *(uint32_t *)&t2;
    }
    *(uint4 *)(a2 + tc_core_off(r, h, 2)) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Half h (group g = 2(j&1) + h, 32 elements, scales for elements 0-15 and
// 16-31) of stage j of a Q6_K super-block at any even address (rows of a
// whole-tile copy are 630 bytes apart; words go through ld32u) for row r:
// sl*(q-32) into a and sh*(q-32) into ah, scale = 32*sh + sl.
RV_DEVFN void tc_stage_q6(const uint8_t *blk, int j, int h, uint8_t *a, uint8_t *ah, int r) {
  const int hh = j >> 1, g = 2 * (j & 1) + h;
  const uint8_t *ql = blk + 64 * hh + 32 * (g & 1), *qh = blk + 128 + 32 * hh;
  const int lsh = 4 * (g >> 1), hsh = 2 * g;
#pragma unroll
  for (int half16 = 0; half16 < 2; half16++) {
    const int sc = (int8_t)blk[192 + 8 * hh + 2 * g + half16];
    const __half2 sl = tc_h2i(sc & 31), sh = tc_h2i(sc >> 5);
    const __half2 cl = tc_h2i(-1056 * (sc & 31)), chh = tc_h2i(-1056 * (sc >> 5));
#pragma unroll
    for (int c2 = 0; c2 < 2; c2++) {
      const int cc = 2 * half16 + c2;
      uint32_t oa[4], oh[4];
#pragma unroll
      for (int t = 0; t < 2; t++) {
        const uint32_t lw = ld32u(ql + 8 * cc + 4 * t), hw = ld32u(qh + 8 * cc + 4 * t);
        const uint32_t q6 = ((lw >> lsh) & 0x0F0F0F0Fu) | (((hw >> hsh) & 0x03030303u) << 4);
        oa[2 * t] = tc_lv2(q6, 0x003F003Fu, sl, cl);
        oa[2 * t + 1] = tc_lv2(q6 >> 8, 0x003F003Fu, sl, cl);
        oh[2 * t] = tc_lv2(q6, 0x003F003Fu, sh, chh);
        oh[2 * t + 1] = tc_lv2(q6 >> 8, 0x003F003Fu, sh, chh);
      }
      const uint32_t off = tc_sw_off(r, 4 * h + cc);
      *(uint4 *)(a + off) = make_uint4(oa[0], oa[1], oa[2], oa[3]);
      *(uint4 *)(ah + off) = make_uint4(oh[0], oh[1], oh[2], oh[3]);
    }
  }
}

// -------------------------------------------------------------- tiles
// Work list of the tensor path: (expert, pos0, pos1, padded pos0) with at
// most RV_TC_NT positions each, and per expert the padded first row of its
// positions in the operand matrices (every expert starts on a multiple of 16
// so tiles cover whole 8-row core-matrix groups).  One CTA of 256 threads.
__global__ void __launch_bounds__(256) k_tc_tiles(MoeDims d, MoeBufs B) {
  __shared__ int s_t[256], s_p[256];
  const int e = threadIdx.x;
  const int cnt = e < d.E ? (int)(B.index_start[e + 1] - B.index_start[e]) : 0;
  const int nt = (cnt + RV_TC_NT - 1) / RV_TC_NT, np = (cnt + 15) & ~15;
  s_t[e] = nt;
  s_p[e] = np;
  __syncthreads();
  for (int o = 1; o < 256; o <<= 1) {  // inclusive scans
    const int t = e >= o ? s_t[e - o] : 0, p = e >= o ? s_p[e - o] : 0;
    __syncthreads();
    s_t[e] += t;
    s_p[e] += p;
    __syncthreads();
  }
  const int t0 = s_t[e] - nt, pp0 = s_p[e] - np;
  if (e < d.E) {
    // Experts with two or more position tiles get their weight stages
    // dequantized once (k_tc_predeq) instead of once per tile.
    if (B.tc_a) B.tc_apre[e] = nt >= 2;
    B.tc_pstart[e] = (uint32_t)pp0;
    const int p0 = (int)B.index_start[e];
    for (int k = 0; k < nt; k++)
      if (t0 + k < B.max_tc)
        B.tc_units[t0 + k] = make_int4(e, p0 + k * RV_TC_NT, p0 + min(cnt, (k + 1) * RV_TC_NT), pp0 + k * RV_TC_NT);
  }
  if (e == 255) {
    if (s_t[255] > B.max_tc) rv_dev_fail(RV_ERR_LENGTH_MISMATCH);
    *B.n_tc = min(s_t[255], B.max_tc);
  }
}

// Padded row of CSR position pos (binary search for its expert).
RV_DEVFN uint32_t tc_padded(const MoeDims &d, const MoeBufs &B, uint32_t pos) {
  int lo = 0, hi = d.E;  // index_start[lo] <= pos < index_start[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (B.index_start[mid] <= pos) lo = mid;
    else hi = mid;
  }
  return B.tc_pstart[lo] + (pos - B.index_start[lo]);
}

// Operand B in global memory is stage-major, so that one stage of a tile
// (8-row groups g0.. g0+ng, K elements 64*it.. 64*it+63) is one contiguous
// run of ng KB, already in the 128-byte-swizzle layout: f16 element
// (row pp, k) of a matrix with G 8-row groups sits at (it*G + pp/8)*512 +
// (pp%8)*64 + ((chunk ^ pp%8)*8) + k%8, it = k/64, chunk = (k%64)/8.  The K=16 mins operand of super-block b: ((b*G +
// pp/8)*2 + j/8)*64 + (pp%8)*8 + j%8.
RV_DEVFN size_t tc_bidx(uint32_t pp, int k, int G) {
  const uint32_t rr = pp & 7, c = (uint32_t)(k >> 3) & 7;
  return (((size_t)(k >> 6) * G + (pp >> 3)) << 9) + (rr << 6) + ((c ^ rr) << 3) + (k & 7);
}
RV_DEVFN size_t tc_midx(uint32_t pp, int b, int j, int G) {
  return ((((size_t)b * G + (pp >> 3)) * 2 + (j >> 3)) << 6) + ((pp & 7) << 3) + (j & 7);
}

// One warp: Q8_K block b (of nb) -> the B operands of padded row pp: the 256
// levels as f16 (8 per lane), the K=16 mins operand [bsum32 mod 32,
// bsum32 div 32] and the block scale d.
RV_DEVFN void tc_q8k_operands(const uint8_t *blk, int b, int nb, int G, int lane, __half *q, __half *m, float *dsc,
                              uint32_t pp) {
  const uint32_t w0 = *(const uint32_t *)(blk + 4 + 8 * lane), w1 = *(const uint32_t *)(blk + 8 + 8 * lane);
  uint4 o;  // chunk slots in PI order: elements 0,2 | 1,3 | 4,6 | 5,7
  __half2 h;
  h = __floats2half2_rn((float)(int8_t)w0, (float)(int8_t)(w0 >> 16)); o.x = *(uint32_t *)&h;
  h = __floats2half2_rn((float)(int8_t)(w0 >> 8), (float)(int8_t)(w0 >> 24)); o.y = *(uint32_t *)&h;
  h = __floats2half2_rn((float)(int8_t)w1, (float)(int8_t)(w1 >> 16)); o.z = *(uint32_t *)&h;
  h = __floats2half2_rn((float)(int8_t)(w1 >> 8), (float)(int8_t)(w1 >> 24)); o.w = *(uint32_t *)&h;
  *(uint4 *)(q + tc_bidx(pp, b * 256 + 8 * lane, G)) = o;
  if (lane < 8) {
    const int16_t *bs = (const int16_t *)(blk + 260);
    const int s32 = (int)bs[2 * lane] + (int)bs[2 * lane + 1];
    m[tc_midx(pp, b, lane, G)] = __float2half_rn((float)(s32 & 31));
    m[tc_midx(pp, b, 8 + lane, G)] = __float2half_rn((float)(s32 >> 5));
  }
  if (lane == 0) dsc[(size_t)pp * nb + b] = *(const float *)blk;
}

// Gate/up operand B: the Q8_K row of each position's token.  CTAs of hb
// warps stride over the index's positions.
__global__ void k_tc_gather(MoeDims d, MoeBufs B) {
  const uint32_t total = B.index_start[d.E];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (uint32_t pos = blockIdx.x; pos < total; pos += gridDim.x) {
    const uint32_t tok = B.index[pos] / (uint32_t)d.K;
    const uint32_t pp = tc_padded(d, B, pos);
    for (int b = warp; b < d.hb; b += blockDim.x >> 5)
      tc_q8k_operands(B.acts + (size_t)tok * d.act_stride + (size_t)b * 292, b, d.hb, B.tc_groups, lane, B.xq,
                      B.xm, B.xd, pp);
  }
}

// SwiGLU of each position's gate and up rows (the exact path's
// swiglu_ref), the reference's Q8_K of the result (acts_moe, bit-identical
// to the exact path) and the down operand B.  CTAs of mb warps stride over
// the index's positions.
RV_DEVFN void tc_quant_pos(const MoeDims &d, const MoeBufs &B, uint32_t pos, int warp, int lane) {
  const uint32_t pp = tc_padded(d, B, pos);
  const float *g = B.gu + (size_t)pos * 2 * d.M, *u = g + d.M;
  for (int b = warp; b < d.mb; b += blockDim.x >> 5) {
    float v[8];
    const int k0 = b * 256 + 8 * lane;
#pragma unroll
    for (int k = 0; k < 8; k++) {
      v[k] = swiglu_ref(g[k0 + k], u[k0 + k]);
      B.hbuf[(size_t)pos * d.M + k0 + k] = v[k];
    }
    uint8_t *blk = B.acts_moe + (size_t)pos * d.amoe_stride + (size_t)b * 292;
    q8k_quantize_warp(v, lane, blk);
    __syncwarp();
    tc_q8k_operands(blk, b, d.mb, B.tc_groups, lane, B.hq, B.hm, B.hdsc, pp);
  }
}
__global__ void k_tc_quant(MoeDims d, MoeBufs B) {
  const uint32_t total = B.index_start[d.E];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (uint32_t pos = blockIdx.x; pos < total; pos += gridDim.x) tc_quant_pos(d, B, pos, warp, lane);
}

// ----------------------------------------------------- the GEMM kernel
template <int FMT>
struct TcFmt {
  static constexpr int BB = FMT == RV_Q4_K ? 144 : FMT == RV_Q5_K ? 176 : 210;
  static constexpr bool MINS = FMT != RV_Q6_K;   // second accumulator: sumi_mins
  static constexpr bool SPLIT = FMT == RV_Q6_K;  // second accumulator: the sh part of the scale
};
// Stage K per kernel: 128 (two 64-element sub-stages) where shared memory
// allows, so that each dequantizing thread has two independent 32-level
// units per stage and the per-stage waits, fences and commits are paid once
// per 128 K; 64 for the Q6_K down tile (its 80 KB raw tile and two A
// operands leave no room).
template <int FMT, bool DOWN>
struct TcK {
  static constexpr int SUB = (DOWN && FMT == RV_Q6_K) ? 1 : 2;  // 64-K sub-stages per stage
};
// One A stage: SUB swizzled [128][64] sub-tiles (16 KB each), then as many
// A_h sub-tiles (Q6_K) or the K=16 mins operand A2 (4 KB).
template <int FMT, bool DOWN>
struct TcStage {
  static constexpr int SUB = TcK<FMT, DOWN>::SUB;
  static constexpr size_t a = 0;
  static constexpr size_t ah = (size_t)SUB * RV_TC_ROWS * 128;
  static constexpr size_t a2 = ah;
  static constexpr size_t bytes = ah + (TcFmt<FMT>::SPLIT ? (size_t)SUB * RV_TC_ROWS * 128 : (size_t)RV_TC_ROWS * 32);
};
// Per-kernel shape: A stages, raw weight slots, activation ring bytes.
// Shared layout from a 1 KB aligned base: [SA] A stages | raw slots |
// activation ring | s_da [NT][nb] | s_pair [NT] | barriers | tmem address.
template <int FMT, bool DOWN>
struct TcCfg {
  // A stage's buffer comes back only once its MMAs have completed, so
  // throughput needs several stages in flight; sizes fill the 227 KB of
  // shared memory.
  // (The activation ring holds at least two slots of the largest tile.)
  static constexpr int SA = (!DOWN && FMT == RV_Q4_K) || (DOWN && FMT == RV_Q6_K) ? 3 : 2;
  static constexpr int R = DOWN ? 1 : 2;
  static constexpr int SBMAX = 16;
  static constexpr size_t RING = (DOWN && FMT == RV_Q6_K) ? 40 * 1024 : 72 * 1024;
  static constexpr size_t raw = (size_t)SA * TcStage<FMT, DOWN>::bytes;
  __host__ __device__ static size_t raw_slot(size_t row_bytes) {
    return DOWN ? ((RV_TC_ROWS * row_bytes + 16 + 1023) & ~(size_t)1023)
                : (((size_t)RV_TC_ROWS * TcFmt<FMT>::BB + 1023) & ~(size_t)1023);
  }
  __host__ __device__ static size_t ring(size_t rb) { return raw + R * raw_slot(rb); }
  // The epilogue's per-work-item buffers of activation scales ([nb][NT]
  // floats) and down pair ids ([NT]): nbuf(nb) of them, used in turn.  A
  // warp starting item j has seen all eight warps release the accumulator
  // of super-block F_j - 3 (F_j: item j's first), so no warp still reads
  // the buffers of an item older than the one holding that super-block:
  // nbuf must exceed ceil(3 / nb).
  __host__ __device__ static int da_cols(int nb) { return 2 * nb > 8 ? 2 * nb : 8; }
  __host__ __device__ static int nbuf(int nb) { return da_cols(nb) / nb; }
  __host__ __device__ static size_t da(size_t rb) { return ring(rb) + RING; }
  __host__ __device__ static size_t pair(size_t rb, int nb) { return da(rb) + (size_t)RV_TC_NT * da_cols(nb) * 4; }
  __host__ __device__ static size_t bars(size_t rb, int nb) {
    return pair(rb, nb) + (DOWN ? (size_t)nbuf(nb) * RV_TC_NT * 4 : 0);
  }
  static constexpr int NBARS = 2 * R + 2 * SA + 2 * SBMAX + 4;
  // After the barriers: tensor-memory address, failure flag, padding, and
  // the activation ring's stage offsets and lengths ([SBMAX] each).
  __host__ __device__ static size_t total(size_t rb, int nb) {
    return 1024 + bars(rb, nb) + NBARS * 8 + 16 + 2 * SBMAX * 4;
  }
};

// Warp-uniform wait of the dequantizing / draining warps (backing off
// between probes).
RV_DEVFN bool tc_wait_warp(uint64_t *bar, uint32_t parity) {
  const bool ok = mbar_wait_bounded(bar, parity, 64);
  return __all_sync(RV_FULL, ok);
}
// 4-D tiled TMA load (no multicast) of the box at (x, y, z, w).
RV_DEVFN void tma_load_4d(void *dst, const CUtensorMap *map, int x, int y, int z, int w, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
      "%5}], [%6];" ::"r"(smem_addr(dst)),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_addr(bar))
      : "memory");
}

// Warp roles.  A warp's scheduler is warp % 4 and the tensor-memory lanes it
// may read are 32*(warp % 4)..+31.  Warp 0 stages, warp 1 issues the MMAs,
// warps 4-11 drain (two per lane quadrant), and the dequantizing warps 2, 3
// and 12-17 sit two on each scheduler (measured: the down GEMM at 512
// tokens 0.214 against 0.230 ms with three on schedulers 2 and 3 and none
// beside the MMA warp); warps 18 and 19 idle.  (Registers are granted per
// four warps: 20 warps at 96 registers fill the 64K-register file, and so
// would 18.)
RV_DEVFN int tc_prod_index(int warp) {  // -1: not a producer
  return warp == 2 || warp == 3 ? warp - 2 : warp >= 12 && warp < 18 ? warp - 10 : -1;
}
#define RV_TC_W_EPI0 4   // warps 4-11: epilogue
#define RV_TC_W_EPI1 12

// Bytes of the dequantized stages of one expert's matrix (all row tiles).
template <int FMT, bool DOWN>
__host__ __device__ constexpr size_t tc_predeq_bytes(int rows, int kdim) {
  return (size_t)(rows / RV_TC_ROWS) * (4 / TcStage<FMT, DOWN>::SUB) * (kdim / 256) * TcStage<FMT, DOWN>::bytes;
}

// The weight stages of experts holding two or more position tiles, written
// once to B.tc_a exactly as the GEMM's dequantizing warps would write them
// into shared memory (same functions, same layout); the GEMM then copies
// each stage in with one bulk copy per 32 KB.  grid = (row tiles, stages
// per row tile, experts); thread p: weight row p & 127, half p >> 7, as
// the dequantizing warps.  Q6_K rows (2-byte aligned, read through 32-bit
// word pairs) are first copied into shared memory, so no read leaves the
// slab.
template <int FMT, bool DOWN>
__global__ void __launch_bounds__(256) k_tc_predeq(MoeDims d, MoeBufs B, MoeWeights W) {
  using F = TcFmt<FMT>;
  using SL = TcStage<FMT, DOWN>;
  constexpr int BB = F::BB, SUB = SL::SUB, SPB = 4 / SUB;
  __shared__ __align__(16) uint8_t s_raw[FMT == RV_Q6_K ? RV_TC_ROWS * BB + 16 : 16];
  const int e = blockIdx.z;
  if (!B.tc_apre[e]) return;
  const int rt = blockIdx.x, it = blockIdx.y, NS = gridDim.y;
  const size_t rb = DOWN ? W.down_row_bytes : W.gu_row_bytes;
  int mat = 0, row0;
  if constexpr (DOWN) {
    row0 = rt * RV_TC_ROWS;
  } else {
    const int rtm = d.M / RV_TC_ROWS;
    mat = rt / rtm;
    row0 = (rt % rtm) * RV_TC_ROWS;
  }
  const uint8_t *wsrc = W.base + (size_t)e * W.stride + (DOWN ? W.down_off : mat ? W.up_off : W.gate_off) +
                        (size_t)row0 * rb;
  const int b = it / SPB, js = it % SPB;
  const int p = threadIdx.x, r = p & 127, h = p >> 7;
  uint8_t *st = B.tc_a + (((size_t)e * gridDim.x + rt) * NS + it) * SL::bytes;
  if constexpr (FMT == RV_Q6_K) {
    for (int i = threadIdx.x; i < RV_TC_ROWS * (BB / 2); i += blockDim.x) {
      const int rr = i / (BB / 2), c = i % (BB / 2);
      *(uint16_t *)(s_raw + rr * BB + 2 * c) = ld16(wsrc + (size_t)rr * rb + (size_t)b * BB + 2 * c);
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < SUB; u++) {
      const int j = SUB * js + u;
      tc_stage_q6(s_raw + r * BB, j, h, st + SL::a + (size_t)u * RV_TC_ROWS * 128,
                  st + SL::ah + (size_t)u * RV_TC_ROWS * 128, r);
    }
  } else {
    const uint8_t *blk = wsrc + (size_t)r * rb + (size_t)b * BB;  // 16-byte aligned
    const uint4 hdr = *(const uint4 *)blk;
    uint32_t u0, u1, u2, u3;
    k4_unpack_words(hdr.y, hdr.z, hdr.w, u0, u1, u2, u3);
#pragma unroll
    for (int u = 0; u < SUB; u++) {
      const int j = SUB * js + u;
      tc_stage_k45<FMT>(blk, j, h, u0, u1, u2, u3, st + SL::a + (size_t)u * RV_TC_ROWS * 128, st + SL::a2, r);
    }
  }
}

// Work items of the tensor GEMM: (row tile rt, pair tile u) numbered
// w = u * nrt + rt, so the CTAs running at one time share pair tiles (the
// same activation stages) and experts (the same weight stages) in L2.
struct TcTile {
  int e, rt, p0, n, pp0, nmma, mat, row0;
  bool apre;  // the expert's weight stages come from the cache (k_tc_predeq)
  const uint8_t *wsrc;
};
template <bool DOWN>
RV_DEVFN TcTile tc_tile(const MoeDims &d, const MoeBufs &B, const MoeWeights &W, int w, int nrt, size_t rb) {
  TcTile t;
  const int u = w / nrt;
  t.rt = w - u * nrt;
  const int4 tl = B.tc_units[u];
  t.e = tl.x;
  t.p0 = tl.y;
  t.n = tl.z - tl.y;
  t.pp0 = tl.w;
  t.nmma = (t.n + 15) & ~15;
  t.apre = B.tc_a != nullptr && B.tc_apre[t.e] != 0;
  if constexpr (DOWN) {
    t.mat = 0;
    t.row0 = t.rt * RV_TC_ROWS;
  } else {
    const int rtm = d.M / RV_TC_ROWS;
    t.mat = t.rt / rtm;
    t.row0 = (t.rt % rtm) * RV_TC_ROWS;
  }
  t.wsrc = W.base + (size_t)t.e * W.stride + (DOWN ? W.down_off : t.mat ? W.up_off : W.gate_off) + (size_t)t.row0 * rb;
  return t;
}

// The GEMM as a persistent kernel: one CTA per SM walks the work items
// w = blockIdx.x, blockIdx.x + gridDim.x, ... of 128 weight rows x one pair
// tile of one matrix.  Gate/up (DOWN = false): nrt = 2*M/128 row tiles
// (gate tiles first), output rows of gu [pos][gate M | up M]; the raw
// super-blocks arrive one 128-row x 1-block box per block through `wmap`
// (the layer's [E][gate|up][M][row bytes] slabs).  Down: nrt = H/128, the
// whole contiguous 128-row tile in one bulk copy, output staged by (token,
// slot).  Roles: warp 0 lane 0 stages raw weights and lane 1 activations,
// warp 1 lane 0 issues the MMAs, eight warps fill the A stages (dequantized
// here, or copied from the cache), eight warps drain each super-block's
// accumulators out of tensor memory while the next block multiplies (the
// epilogue), two warps idle.  Every ring (raw weights, A stages, activation
// stages, the two accumulator slots) runs on across work items, so one
// item's staging and products overlap the previous item's epilogue; each
// ring has a single filling party, which waits on every phase in order (a
// parity wait cannot tell phase k from phase k + 2).  The activation ring
// hands out byte ranges, so items of different widths share it.
template <int FMT, bool DOWN>
__global__ void __launch_bounds__(RV_TC_THREADS, 1)
    k_tc_gemm(MoeDims d, MoeBufs B, MoeWeights W, const __grid_constant__ CUtensorMap wmap) {
  using F = TcFmt<FMT>;
  using SL = TcStage<FMT, DOWN>;
  using C = TcCfg<FMT, DOWN>;
  constexpr int BB = F::BB, SA = C::SA, R = C::R, SUB = SL::SUB, SPB = 4 / SUB;  // stages per super-block
  constexpr int SBM = C::SBMAX;
  extern __shared__ __align__(16) uint8_t sm_raw_[];
  uint8_t *sm = (uint8_t *)(((uintptr_t)sm_raw_ + 1023) & ~(uintptr_t)1023);
  constexpr int PK = DOWN ? 2 : 1;
  (void)PK;
  RV_PHASE(PK, 0);
  const int kdim = DOWN ? d.M : d.H, nb = kdim / 256, NS = SPB * nb;
  const int nrt = DOWN ? d.H / RV_TC_ROWS : 2 * d.M / RV_TC_ROWS;
  const int nwork = nrt * *B.n_tc;
  if ((int)blockIdx.x >= nwork) return;
  const size_t rb = DOWN ? W.down_row_bytes : W.gu_row_bytes;
  const uint8_t *bq = (const uint8_t *)(DOWN ? B.hq : B.xq), *bm = (const uint8_t *)(DOWN ? B.hm : B.xm);
  const float *bd = DOWN ? B.hdsc : B.xd;
  const size_t rslot = C::raw_slot(rb);
  uint8_t *raw = sm + C::raw, *ring = sm + C::ring(rb);
  float *s_da = (float *)(sm + C::da(rb));                // [nbuf][nb][NT], one per work item in turn
  uint32_t *s_pair = (uint32_t *)(sm + C::pair(rb, nb));  // [nbuf][NT] (down)
  uint64_t *bars = (uint64_t *)(sm + C::bars(rb, nb));
  uint64_t *raw_full = bars, *raw_empty = bars + R, *a_full = bars + 2 * R, *a_empty = a_full + SA,
           *b_full = a_empty + SA, *b_empty = b_full + SBM, *acc_full = b_empty + SBM, *acc_empty = acc_full + 2;
  uint32_t *s_tmem = (uint32_t *)(bars + C::NBARS);
  volatile int *s_fail = (volatile int *)(s_tmem + 1);
  uint32_t *s_boff = s_tmem + 4, *s_blen = s_boff + SBM;  // activation stage byte ranges in the ring
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < R; i++) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], RV_TC_PROD_WARPS);
    }
    for (int i = 0; i < SA; i++) {
      mbar_init(&a_full[i], RV_TC_PROD_WARPS);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < SBM; i++) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], RV_TC_EPI_WARPS);
    }
    *s_fail = 0;
  }
  __syncwarp();
  if (warp == 0) {
    tc_alloc(s_tmem, 4 * RV_TC_NT);
    tc_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  RV_PHASE(PK, 1);

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------- weight staging
      // Raw weights of the work items whose stages are not in the cache;
      // the A stages themselves are the producer warps' (below).
      bool ok = true;
      int graw = 0, gdraw = 0;  // raw gate/up blocks, raw down tiles so far
      for (int w = blockIdx.x; w < nwork && ok && !*s_fail; w += gridDim.x) {
        const TcTile t = tc_tile<DOWN>(d, B, W, w, nrt, rb);
        if (t.apre) continue;
        if constexpr (DOWN) {
          if (!mbar_wait_bounded(&raw_empty[0], (gdraw & 1) ^ 1, 128)) {
            ok = false;
            break;
          }
          gdraw++;
          const size_t tb = (size_t)RV_TC_ROWS * rb;
          mbar_arrive_expect_tx(&raw_full[0], (uint32_t)tb);
          for (size_t o = 0; o < tb; o += 32768)
            bulk_g2s(raw + o, t.wsrc + o, (uint32_t)(tb - o < 32768 ? tb - o : 32768), &raw_full[0]);
        } else {
          // The tile's rows are contiguous: ask the L2 for all of them now so
          // each super-block's box below comes from L2, not HBM.
          const uint32_t tile_b = (uint32_t)(RV_TC_ROWS * rb);
          for (uint32_t o = 0; o < tile_b; o += 32768)
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(t.wsrc + o),
                         "r"(tile_b - o < 32768u ? tile_b - o : 32768u)
                         : "memory");
          for (int b = 0; b < nb; b++, graw++) {
            const int slot = graw % R;
            if (!mbar_wait_bounded(&raw_empty[slot], ((graw / R) & 1) ^ 1, 128)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&raw_full[slot], (uint32_t)(RV_TC_ROWS * BB));
            tma_load_4d(raw + slot * rslot, &wmap, b * BB, t.row0, t.mat, t.e, &raw_full[slot]);
            RV_TRACE(PK + 2, graw, 6);
          }
        }
        RV_PHASE_ANY(PK, 2);
      }
      if (!ok) *s_fail = 1;
    } else if (lane == 1) {
      // ------------------------------------------ activation staging
      // Stage gb takes barrier pair gb % SBM and a byte range of the ring;
      // ranges are released in order (the MMAs consume stages in order), so
      // the ring is a queue: `used` bytes from the oldest unreleased stage
      // `tail` up to `head`, plus any end gap skipped when a range wrapped.
      bool ok = true;
      int gb = 0, tail = 0;
      uint32_t head = 0, used = 0;
      for (int w = blockIdx.x; w < nwork && ok && !*s_fail; w += gridDim.x) {
        const TcTile t = tc_tile<DOWN>(d, B, W, w, nrt, rb);
        const int ng = t.nmma / 8, g0 = t.pp0 / 8;
        const uint32_t sub_b = (uint32_t)t.nmma * 128;  // one 64-K sub-stage (whole 1 KB atoms)
        for (int it = 0; it < NS; it++, gb++) {
          const bool mins = F::MINS && (it % SPB) == 0;
          const uint32_t sz = (SUB * sub_b + (mins ? (uint32_t)t.nmma * 32 : 0u) + 1023u) & ~1023u;
          uint32_t off = 0;
          for (;;) {
            if (gb - tail < SBM) {
              if (gb == tail) head = used = 0;
              const uint32_t fr = (uint32_t)C::RING - used, gap = (uint32_t)C::RING - head;
              if (sz <= gap && sz <= fr) {
                off = head;
                s_blen[gb % SBM] = sz;
                break;
              }
              if (sz > gap && sz + gap <= fr) {
                off = 0;
                s_blen[gb % SBM] = sz + gap;
                break;
              }
            }
            if (!mbar_wait_bounded(&b_empty[tail % SBM], (tail / SBM) & 1, 128)) {
              ok = false;
              break;
            }
            used -= s_blen[tail % SBM];
            tail++;
          }
          if (!ok) break;
          const int sb = gb % SBM;
          used += s_blen[sb];
          head = off + sz;
          s_boff[sb] = off;
          RV_TRACE(PK + 2, gb, 5);
          uint8_t *dst = ring + off;
          mbar_arrive_expect_tx(&b_full[sb], (uint32_t)(SUB * ng * 1024 + (mins ? ng * 256 : 0)));
          for (int u = 0; u < SUB; u++)
            bulk_g2s(dst + u * sub_b, bq + ((size_t)(SUB * it + u) * B.tc_groups + g0) * 1024, (uint32_t)(ng * 1024),
                     &b_full[sb]);
          if (mins)
            bulk_g2s(dst + SUB * sub_b, bm + ((size_t)(it / SPB) * B.tc_groups + g0) * 256, (uint32_t)(ng * 256),
                     &b_full[sb]);
        }
      }
      if (!ok) *s_fail = 1;
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA issue
    if (lane == 0) {
      // The issue loop is kept short: this warp shares its scheduler with
      // four dequantizing warps.  Descriptor words are formed by adding
      // 16-byte units to precomputed low words.
      // A and B tiles: 128-byte swizzle, SBO 1024 (K advances 32 bytes per
      // K=16 step inside the swizzled row); mins tiles: no swizzle, LBO 128,
      // SBO 256.
      const uint32_t hi_sw = (1024u >> 4) | (1u << 14) | (2u << 29), hi256 = (256u >> 4) | (1u << 14);
      const uint32_t lbo_sw = 1u << 16, lbo_none = (128u >> 4) << 16;
      const uint32_t a_lo0 = smem_addr(sm) >> 4, b_lo0 = smem_addr(ring) >> 4;
      const uint32_t a_step = (uint32_t)(SL::bytes >> 4);
      auto mk = [](uint32_t lo, uint32_t hi) { return ((uint64_t)hi << 32) | lo; };
      int ga = 0, gb = 0, gsb = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < nwork && ok && !*s_fail; w += gridDim.x) {
        const TcTile t = tc_tile<DOWN>(d, B, W, w, nrt, rb);
        const uint32_t idesc = tc_idesc(t.nmma), sub_b = (uint32_t)t.nmma * 128;
        for (int b = 0; b < nb && ok; b++, gsb++) {
          const int slot = gsb & 1;
          if (!mbar_wait_bounded(&acc_empty[slot], ((gsb >> 1) & 1) ^ 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d1 = tmem + (uint32_t)(slot * 2 * RV_TC_NT), d2 = d1 + RV_TC_NT;
          for (int j = 0; j < SPB; j++, ga++, gb++) {
            const int sa = ga % SA, sb = gb % SBM;
            if (!mbar_wait_bounded(&a_full[sa], (ga / SA) & 1)) {
              ok = false;
              break;
            }
            RV_TRACE(PK + 2, ga, 2);
            if (!mbar_wait_bounded(&b_full[sb], (gb / SBM) & 1)) {
              ok = false;
              break;
            }
            RV_TRACE(PK + 2, ga, 3);
            tc_fence_after();
            if (gsb == 0 && j == 0) RV_PHASE_ANY(PK, 3);
            const uint32_t al = a_lo0 + (uint32_t)sa * a_step, bl = b_lo0 + (s_boff[sb] >> 4);
            if (F::MINS && j == 0)
              tc_mma_f16(d2, mk(lbo_none | (al + (uint32_t)(SL::a2 >> 4)), hi256),
                         mk(lbo_none | (bl + (uint32_t)(SUB * sub_b >> 4)), hi256), idesc, 0u);
#pragma unroll
            for (int u = 0; u < SUB; u++) {
              const uint32_t au = al + (uint32_t)(u * RV_TC_ROWS * 128 >> 4), bu = bl + (uint32_t)(u * sub_b >> 4);
#pragma unroll
              for (int kk = 0; kk < 4; kk++) {
                const uint32_t acc = (j | u | kk) != 0;
                tc_mma_f16(d1, mk(lbo_sw | (au + 2 * kk), hi_sw), mk(lbo_sw | (bu + 2 * kk), hi_sw), idesc, acc);
                if (F::SPLIT)
                  tc_mma_f16(d2, mk(lbo_sw | (au + (uint32_t)(SL::ah >> 4) + 2 * kk), hi_sw),
                             mk(lbo_sw | (bu + 2 * kk), hi_sw), idesc, acc);
              }
            }
            RV_TRACE(PK + 2, ga, 9);
            tc_commit(&a_empty[sa]);
            tc_commit(&b_empty[sb]);
            RV_TRACE(PK + 2, ga, 4);
          }
          if (!ok) break;
          tc_commit(&acc_full[slot]);
        }
      }
      RV_PHASE_ANY(PK, 4);
      if (!ok) *s_fail = 1;
    }
    __syncwarp();
  } else if (tc_prod_index(warp) >= 0) {
    // ------------------------------------------------------ producers
    // Every A stage of every work item.  Uncached items: thread p
    // dequantizes weight row p & 127, half p >> 7 of each stage.  Cached
    // items (k_tc_predeq wrote the stages): the first producer warp's lane 0
    // copies each stage in with bulk copies and the other warps arrive.
    const int pi = tc_prod_index(warp), p = 32 * pi + lane, r = p & 127, h = p >> 7;
    bool ok = true, first = true;
    int ga = 0, graw = 0, gdraw = 0;
    for (int w = blockIdx.x; w < nwork && ok && !*s_fail; w += gridDim.x) {
      const TcTile t = tc_tile<DOWN>(d, B, W, w, nrt, rb);
      if (t.apre) {
        const uint8_t *asrc = B.tc_a + ((size_t)t.e * nrt + t.rt) * NS * SL::bytes;
        for (int it = 0; it < NS; it++, ga++) {
          const int sa = ga % SA;
          if (!tc_wait_warp(&a_empty[sa], ((ga / SA) & 1) ^ 1)) {
            ok = false;
            break;
          }
          if (lane == 0) {
            if (pi == 0) {
              mbar_arrive_expect_tx(&a_full[sa], (uint32_t)SL::bytes);
              for (size_t o = 0; o < SL::bytes; o += 32768)
                bulk_g2s(sm + (size_t)sa * SL::bytes + o, asrc + (size_t)it * SL::bytes + o,
                         (uint32_t)(SL::bytes - o < 32768 ? SL::bytes - o : 32768), &a_full[sa]);
            } else {
              mbar_arrive(&a_full[sa]);
            }
          }
          __syncwarp();
          if (p == 0) RV_TRACE(PK + 2, ga, 0);
        }
        continue;
      }
      if (DOWN) {
        ok = tc_wait_warp(&raw_full[0], gdraw & 1);
        if (!ok) break;
      }
      uint32_t u0 = 0, u1 = 0, u2 = 0, u3 = 0;
      for (int it = 0; it < NS; it++, ga++) {
        const int b = it / SPB, js = it % SPB, sa = ga % SA;
        if (!DOWN && js == 0 && !tc_wait_warp(&raw_full[graw % R], (graw / R) & 1)) {
          ok = false;
          break;
        }
        if (p == 0 && js == 0) RV_TRACE(PK + 2, ga, 8);
        const uint8_t *blk = DOWN ? raw + (size_t)r * rb + (size_t)b * BB : raw + (graw % R) * rslot + (size_t)r * BB;
        if (F::MINS && js == 0) {
          const uint4 hdr = *(const uint4 *)blk;
          k4_unpack_words(hdr.y, hdr.z, hdr.w, u0, u1, u2, u3);
        }
        if (!tc_wait_warp(&a_empty[sa], ((ga / SA) & 1) ^ 1)) {
          ok = false;
          break;
        }
        if (first && p == 0) RV_PHASE_ANY(PK, 5);
        first = false;
        if (p == 0) RV_TRACE(PK + 2, ga, 0);
        uint8_t *st = sm + (size_t)sa * SL::bytes;
#pragma unroll
        for (int u = 0; u < SUB; u++) {
          const int j = SUB * js + u;  // 64-element stage of the super-block
          uint8_t *a_sub = st + SL::a + (size_t)u * RV_TC_ROWS * 128;
          if constexpr (FMT == RV_Q6_K) tc_stage_q6(blk, j, h, a_sub, st + SL::ah + (size_t)u * RV_TC_ROWS * 128, r);
          else tc_stage_k45<FMT>(blk, j, h, u0, u1, u2, u3, a_sub, st + SL::a2, r);
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&a_full[sa]);
          if (!DOWN && js == SPB - 1) mbar_arrive(&raw_empty[graw % R]);
        }
        if (!DOWN && js == SPB - 1) graw++;
        if (p == 0) RV_TRACE(PK + 2, ga, 1);
      }
      if (!ok) break;
      if (DOWN) {  // the raw tile may take the next uncached work item's weights
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[0]);
        gdraw++;
      }
    }
    if (p == 0) RV_PHASE_ANY(PK, 6);
    if (!ok) *s_fail = 1;
  } else if (warp >= RV_TC_W_EPI0 && warp < RV_TC_W_EPI1) {
    // ------------------------------------------------------- epilogue
    // Thread (quadrant q, lane) owns weight row 32q + lane (its tensor-
    // memory lane) and the 8-column chunks half, half+2, ..., half+14 of the
    // tile, so small tiles spread over both warps of a quadrant.  Each warp
    // copies the activation scales (stored [nb][NT]) and, down, the pair ids
    // of its own columns into the work item's buffer (C::nbuf of them, in
    // turn); warps of the same half write the same values, and no warp
    // still reads a buffer when it comes round again (TcCfg).  The 64
    // running sums stay in registers, so tensor memory is read four columns
    // at a time.
    const int q = warp & 3, half = (warp - RV_TC_W_EPI0) >> 2, er = 32 * q + lane;
    const int nbuf = C::nbuf(nb);
    bool ok = true, first = true;
    int gsb = 0, bi = 0;
    for (int w = blockIdx.x; w < nwork && ok && !*s_fail; w += gridDim.x, bi = bi + 1 == nbuf ? 0 : bi + 1) {
      const TcTile t = tc_tile<DOWN>(d, B, W, w, nrt, rb);
      float *da = s_da + (size_t)bi * RV_TC_NT * nb;
      uint32_t *pr = s_pair + bi * RV_TC_NT;
      for (int i = lane; i < 8 * 8 * nb; i += 32) {
        const int c = i / (8 * nb), rest = i % (8 * nb), col = 8 * (half + 2 * c) + rest / nb;
        if (col < t.nmma) da[(rest % nb) * RV_TC_NT + col] = bd[(size_t)(t.pp0 + col) * nb + rest % nb];
      }
      if (DOWN)
        for (int i = lane; i < 64; i += 32) {
          const int col = 8 * (half + 2 * (i >> 3)) + (i & 7);
          if (col < t.n) pr[col] = B.index[t.p0 + col];
        }
      __syncwarp();
      const int nch = t.nmma > 8 * half ? (t.nmma - 8 * half + 15) / 16 : 0;  // this warp's chunks
      const uint8_t *hrow = t.wsrc + (size_t)er * rb;  // the drained row's super-block headers (global)
      float acc[8][8];
#pragma unroll
      for (int c = 0; c < 8; c++)
#pragma unroll
        for (int i = 0; i < 8; i++) acc[c][i] = 0.0f;
      uint32_t hdr_next = FMT == RV_Q6_K ? (uint32_t)ld16(hrow + 208) : *(const uint32_t *)hrow;
      for (int eb = 0; eb < nb; eb++, gsb++) {
        const int slot = gsb & 1;
        const uint32_t hdr = hdr_next;
        if (eb + 1 < nb)
          hdr_next = FMT == RV_Q6_K ? (uint32_t)ld16(hrow + (size_t)(eb + 1) * BB + 208)
                                    : *(const uint32_t *)(hrow + (size_t)(eb + 1) * BB);
        const float dw = h2f((uint16_t)(hdr & 0xFFFFu)), dmw = h2f((uint16_t)(hdr >> 16));
        if (!tc_wait_warp(&acc_full[slot], (gsb >> 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (first && warp == RV_TC_W_EPI0 && lane == 0) RV_PHASE_ANY(PK, 7);
        first = false;
        if (warp == RV_TC_W_EPI0 && lane == 0) RV_TRACE(PK + 2, SPB * gsb, 7);
        const uint32_t t1 = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(slot * 2 * RV_TC_NT);
        const float *dab = da + (size_t)eb * RV_TC_NT;
#pragma unroll
        for (int c = 0; c < 8; c++) {
          if (c < nch) {
            const int col = 8 * (half + 2 * c);
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
              uint32_t v1[4], v2[4];
              tc_ld4(t1 + (uint32_t)(col + 4 * hh), v1);
              tc_ld4(t1 + (uint32_t)(RV_TC_NT + col + 4 * hh), v2);
              tc_wait_ld();
#pragma unroll
              for (int k = 0; k < 4; k++) {
                const int i = 4 * hh + k;
                const float dav = dab[col + i];
                float blocksum;
                if constexpr (FMT == RV_Q6_K) {
                  const int sumi =
                      __float2int_rn(__uint_as_float(v1[k])) + 32 * __float2int_rn(__uint_as_float(v2[k]));
                  blocksum = __fmul_rn(__fmul_rn(dw, dav), __int2float_rn(sumi));
                } else {
                  const float dd = __fmul_rn(dw, dav), dm = __fmul_rn(dmw, dav);
                  blocksum = __fsub_rn(__fmul_rn(dd, __uint_as_float(v1[k])), __fmul_rn(dm, __uint_as_float(v2[k])));
                }
                acc[c][i] = __fadd_rn(acc[c][i], blocksum);
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[slot]);
      }
      if (!ok || *s_fail) break;
#pragma unroll
      for (int c = 0; c < 8; c++)
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const int col = 8 * (half + 2 * c) + i;
          if (col < t.n) {
            if constexpr (DOWN) down_out_row(B, pr[col], d.H)[t.row0 + er] = acc[c][i];
            else B.gu[(size_t)(t.p0 + col) * 2 * d.M + (size_t)t.mat * d.M + t.row0 + er] = acc[c][i];
          }
        }
    }
    if (warp == RV_TC_W_EPI0 && lane == 0) RV_PHASE_ANY(PK, 8);
    if (!ok) *s_fail = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tc_dealloc(tmem, 4 * RV_TC_NT);
  }
  // Expert-parallel down rows went to other ranks' memory: one system-scope
  // fence after the barrier orders every thread's stores of this CTA.
  if (DOWN && B.ep_out && threadIdx.x == 32) __threadfence_system();
  RV_PHASE(PK, 9);
}
