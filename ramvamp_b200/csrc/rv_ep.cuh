// rv_ep.cuh -- kernels around the expert-parallel exchange.
//
// Experts are spread over the ranks of a group by expert id modulo the
// group size: rank r holds experts r, r + G, r + 2G, ... as its local
// experts 0, 1, 2, ...  A rank routes its own ("home") tokens, sends the
// Q8_K row of every (token, slot) pair to the rank holding the pair's
// expert, receives the expert output rows back in the order it sent them,
// and reduces them in top-k order, so the layer output does not depend on
// the group size (prefill.rs:2734-2778).
#pragma once
#include "rv_moe.cuh"

// Per-expert counts of an externally supplied expert list (one slot per
// row), for k_index.  Ids out of range are reported and not counted.
__global__ void k_count_ids(MoeDims d, MoeBufs B) {
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= B.T) return;
  const uint32_t e = B.ids[p];
  if (e >= (uint32_t)d.E) {
    rv_dev_fail(RV_ERR_ROUTED_OUT_OF_RANGE);
    return;
  }
  atomicAdd(&B.counts[e], 1);
}

// acc = 0; acc += w_k * out_k in top-k order; residual += acc
// (forward.rs:2744-2753), with expert output row pos_of[pair] (or pair).
__global__ void k_combine_rows(MoeDims d, MoeBufs B, const uint32_t *pos_of) {
  const int t = blockIdx.x;
  const int h = blockIdx.y * blockDim.x + threadIdx.x;
  if (h >= d.H) return;
  float acc = 0.0f;
  for (int k = 0; k < d.K; k++) {
    const size_t pair = (size_t)t * d.K + k;
    const size_t row = pos_of ? pos_of[pair] : pair;
    acc = __fadd_rn(acc, __fmul_rn(B.w[pair], B.staged[row * d.H + h]));
  }
  float *res = B.residual + (size_t)t * d.H + h;
  *res = __fadd_rn(*res, acc);
}

// Dispatch plan of P pairs over `world` ranks (one CTA): send_counts[r] =
// pairs bound for rank r; pairs are laid out rank by rank; pos_of[pair] =
// its row in that layout, order[row] = pair, send_local[row] = the
// expert's local id on its rank.  Rows of one rank are in no fixed order
// (every output row is returned to its pair through pos_of).
__global__ void __launch_bounds__(1024) k_ep_plan(MoeDims d, const uint32_t *ids, unsigned P, unsigned world,
                                                  int32_t *send_counts, uint32_t *pos_of, uint32_t *send_local,
                                                  uint32_t *order) {
  __shared__ unsigned s_cnt[64], s_off[64];
  for (unsigned i = threadIdx.x; i < 64; i += blockDim.x) s_cnt[i] = 0;
  __syncthreads();
  for (unsigned p = threadIdx.x; p < P; p += blockDim.x) {
    uint32_t e = ids[p];
    if (e >= (uint32_t)d.E) {
      rv_dev_fail(RV_ERR_ROUTED_OUT_OF_RANGE);
      e = 0;
    }
    atomicAdd(&s_cnt[e % world], 1u);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned o = 0;
    for (unsigned r = 0; r < world; r++) {
      s_off[r] = o;
      send_counts[r] = (int32_t)s_cnt[r];
      o += s_cnt[r];
    }
  }
  __syncthreads();
  for (unsigned p = threadIdx.x; p < P; p += blockDim.x) {
    uint32_t e = ids[p];
    if (e >= (uint32_t)d.E) e = 0;
    const unsigned pos = atomicAdd(&s_off[e % world], 1u);
    pos_of[p] = pos;
    order[pos] = p;
    send_local[pos] = e / world;
  }
}

// send_acts[row] = the Q8_K row of pair order[row]'s token (act_stride
// bytes, 16-byte aligned).  grid = P CTAs.
__global__ void __launch_bounds__(128) k_ep_pack(MoeDims d, const uint8_t *acts, const uint32_t *order,
                                                 uint8_t *send_acts) {
  const unsigned row = blockIdx.x;
  const uint32_t tok = order[row] / (uint32_t)d.K;
  const uint4 *src = (const uint4 *)(acts + (size_t)tok * d.act_stride);
  uint4 *dst = (uint4 *)(send_acts + (size_t)row * d.act_stride);
  for (size_t i = threadIdx.x; i < d.act_stride / 16; i += blockDim.x) dst[i] = src[i];
}
