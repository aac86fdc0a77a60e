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

// ===================================================== peer-memory exchange
// Every rank owns one exchange window in its own HBM, mapped into each peer
// (CUDA IPC, or peer access inside one process).  For a group of `world`
// ranks and `cap` pairs per rank (max tokens per rank x top-k):
//   flag_disp[world]  source s sets its slot to the layer's epoch once its
//                     rows, metadata and count have landed here
//   flag_comb[world]  expert rank x sets its slot once it has stored the
//                     outputs of every pair this rank sent it
//   count[world]      pairs source s sent for this layer
//   home[world][cap]  per received slot: the pair's index (token*top_k +
//                     slot) at its home rank
//   eid[world][cap]   per received slot: the local id of its expert here
//   acts[world][cap]  per received slot: the token's Q8_K row
//   out[cap][H]       the unweighted expert outputs of this rank's own pairs,
//                     stored here by whichever rank ran each expert
// Flags count layers (the epoch) and never reset, so no step has to clear
// a peer's memory.  Reuse is safe by construction: a rank writes layer l+1
// data into a peer's window only after that peer's combine flag for layer l
// arrived, and the peer sends it after its own expert kernels of layer l,
// the last readers of what it received for layer l.
struct EpState {
  uint32_t epoch;          // layers completed by this rank's dispatch
  uint32_t done;           // CTAs of the current dispatch that finished
  uint32_t send_cnt[64];   // slots reserved per destination (zero between calls)
};

struct EpArgs {
  uint8_t *const *win;     // [world] every rank's window, as this GPU addresses it
  uint8_t *mine;           // this rank's window
  EpState *st;
  uint32_t world, rank, cap;
  uint32_t act_stride;
  int H;
  size_t o_fd, o_fc, o_cnt, o_home, o_eid, o_acts, o_out, bytes;  // window layout
};

// Offsets of the window's parts (identical on every rank of a group).
inline void ep_layout(EpArgs &A) {
  auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
  const size_t W = A.world, C = A.cap;
  size_t o = 0;
  A.o_fd = o; o += up(W * 4);
  A.o_fc = o; o += up(W * 4);
  A.o_cnt = o; o += up(W * 4);
  A.o_home = o; o += up(W * C * 4);
  A.o_eid = o; o += up(W * C * 4);
  A.o_acts = o; o += up(W * C * A.act_stride);
  A.o_out = o; o += up(C * (size_t)A.H * 4);
  A.bytes = o;
}

RV_DEVFN uint32_t *ep_u32(uint8_t *w, size_t off) { return (uint32_t *)(w + off); }

// A wait on a peer's flag that gives up at once when an earlier wait has
// already run out (the device error word is set), so a missing peer costs
// one bounded wait, not one per CTA.
RV_DEVFN bool ep_wait(const uint32_t *flag, uint32_t epoch) {
  if (*(volatile int *)&g_rv_dev_error != 0) return flag_reached(ld_acquire_sys(flag), epoch);
  return flag_wait_bounded(flag, epoch);
}

// Dispatch of this rank's P = T*top_k pairs: one thread per pair reserves a
// slot in its expert's rank (warp-aggregated atomics per destination),
// the rank and local id of global expert e coming from `place[e]` (rank <<
// 16 | local id; an entry out of range is reported and its pair dropped) or,
// without a placement, e mod world and e / world;
// writes the slot's metadata there and the warp copies its pairs' Q8_K rows
// with 16-byte stores over NVLink.  The last CTA to finish publishes the
// counts, clears the reservations and raises this layer's flag on every
// rank.  Also clears the router's per-expert counts (`counts`, E ints).
__global__ void __launch_bounds__(256) k_ep_dispatch(EpArgs A, const uint32_t *place, const uint32_t *ids,
                                                     const uint8_t *acts, int P, int K, int E, int *counts) {
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (blockIdx.x == 0)
    for (int e = threadIdx.x; e < E; e += blockDim.x) counts[e] = 0;
  const int p0 = (blockIdx.x * (blockDim.x >> 5) + warp) * 32;
  const int p = p0 + lane;
  uint32_t e = p < P ? ids[p] : ~0u;
  if (p < P && e >= (uint32_t)E) {
    rv_dev_fail(RV_ERR_ROUTED_OUT_OF_RANGE);
    e = ~0u;
  }
  uint32_t dest = ~0u, local = 0;
  if (e != ~0u) {
    if (place) {
      const uint32_t pl = place[e];
      dest = pl >> 16;
      local = pl & 0xFFFFu;
      if (dest >= A.world || local >= (uint32_t)E / A.world) {
        rv_dev_fail(RV_ERR_ROUTED_OUT_OF_RANGE);
        dest = ~0u;
      }
    } else {
      dest = e % A.world;
      local = e / A.world;
    }
  }
  const unsigned same = __match_any_sync(RV_FULL, dest);
  const int leader = __ffs(same) - 1;
  uint32_t base = 0;
  if (dest != ~0u && lane == leader) base = atomicAdd(&A.st->send_cnt[dest], (uint32_t)__popc(same));
  base = __shfl_sync(RV_FULL, base, leader);
  const uint32_t slot = base + (uint32_t)__popc(same & ((1u << lane) - 1u));
  if (dest != ~0u) {
    if (slot < A.cap) {
      uint8_t *w = A.win[dest];
      const size_t i = (size_t)A.rank * A.cap + slot;
      ep_u32(w, A.o_home)[i] = (uint32_t)p;
      ep_u32(w, A.o_eid)[i] = local;
    } else {
      rv_dev_fail(RV_ERR_LENGTH_MISMATCH);  // cannot happen: P <= cap
    }
  }
  const int n16 = (int)(A.act_stride / 16);
  for (int j = 0; j < 32; j++) {
    const uint32_t dj = __shfl_sync(RV_FULL, dest, j), sj = __shfl_sync(RV_FULL, slot, j);
    if (dj == ~0u || sj >= A.cap) continue;
    const uint4 *src = (const uint4 *)(acts + (size_t)((p0 + j) / K) * A.act_stride);
    uint4 *dst = (uint4 *)(A.win[dj] + A.o_acts + ((size_t)A.rank * A.cap + sj) * A.act_stride);
    for (int i = lane; i < n16; i += 32) dst[i] = src[i];
  }
  __threadfence_system();  // this thread's remote stores before the CTA's count
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t old = atomicAdd(&A.st->done, 1u);
    s_last = old == gridDim.x - 1;
    __threadfence();
  }
  __syncthreads();
  if (!s_last) return;
  const uint32_t epoch = A.st->epoch + 1;
  __syncthreads();
  for (uint32_t r = threadIdx.x; r < A.world; r += blockDim.x) {
    const uint32_t n = atomicExch(&A.st->send_cnt[r], 0u);
    ep_u32(A.win[r], A.o_cnt)[A.rank] = min(n, A.cap);
    __threadfence_system();
    st_release_sys(ep_u32(A.win[r], A.o_fd) + A.rank, epoch);
  }
  if (threadIdx.x == 0) {
    A.st->epoch = epoch;
    A.st->done = 0;
  }
}

// Receive side, one CTA: wait for every source's flag of this layer
// (bounded), then lay the received slots out as the expert stage's dispatch
// list (B.ids[s*cap + i] = local expert, or ~0 for an empty slot; K = 1)
// and build its index.  Metadata out of range is reported and its slot
// dropped, so no later store can leave the home rank's output buffer.
__global__ void __launch_bounds__(1024) k_ep_receive(EpArgs A, MoeDims d, MoeBufs B) {
  __shared__ int s_cnt[256];
  __shared__ uint32_t s_st[257], s_cur[256];
  __shared__ int s_us[257];
  __shared__ uint32_t s_n[64];
  __shared__ int s_ok;
  const uint32_t epoch = A.st->epoch;
  if (threadIdx.x == 0) s_ok = 1;
  for (int e = threadIdx.x; e < 256; e += blockDim.x) s_cnt[e] = 0;
  __syncthreads();
  if (threadIdx.x < A.world) {
    const bool ok = ep_wait(ep_u32(A.mine, A.o_fd) + threadIdx.x, epoch);
    if (!ok) atomicExch(&s_ok, 0);
    s_n[threadIdx.x] = ok ? min(ep_u32(A.mine, A.o_cnt)[threadIdx.x], A.cap) : 0u;
  }
  __syncthreads();
  const uint32_t *eid = ep_u32(A.mine, A.o_eid), *home = ep_u32(A.mine, A.o_home);
  // Only the filled slots: slot (s, i) for i < s_n[s].
  for (uint32_t s = 0; s < A.world; s++)
    for (uint32_t i = threadIdx.x; i < s_n[s]; i += blockDim.x) {
      const uint32_t p = s * A.cap + i;
      uint32_t e = eid[p];
      if (e >= (uint32_t)d.E || home[p] >= A.cap) {
        rv_dev_fail(RV_ERR_ROUTED_OUT_OF_RANGE);
        e = ~0u;
      } else {
        atomicAdd(&s_cnt[e], 1);
      }
      B.ids[p] = e;
    }
  __syncthreads();
  build_index_cta(d, B, s_cnt, s_st, s_cur, s_us, /*sparse=*/true, s_n, (int)A.world, (int)A.cap);
}

// After the expert stage: every output row this rank owed has been stored
// (the stores of the kernels before this one in the stream are complete);
// raise this layer's combine flag on every rank.
__global__ void k_ep_signal(EpArgs A) {
  __threadfence_system();
  const uint32_t epoch = A.st->epoch;
  for (uint32_t r = threadIdx.x; r < A.world; r += blockDim.x)
    st_release_sys(ep_u32(A.win[r], A.o_fc) + A.rank, epoch);
}

// Combine (forward.rs:2744-2753, prefill.rs:2749-2778): once every rank's
// combine flag of this layer is up (bounded wait, thread 0 of each CTA),
// acc = 0; acc += w_k * out[t*K + k] in top-k order; residual += acc.
// grid = (max(T, 1), H/256): with no home tokens the CTA only waits, so
// this rank cannot run ahead into the next layer while peers still read.
__global__ void __launch_bounds__(256) k_ep_combine(EpArgs A, MoeDims d, float *residual, const float *w, int T) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    const uint32_t epoch = A.st->epoch;
    int ok = 1;
    for (uint32_t r = 0; r < A.world; r++)
      ok &= ep_wait(ep_u32(A.mine, A.o_fc) + r, epoch) ? 1 : 0;
    s_ok = ok;
  }
  __syncthreads();
  const int t = blockIdx.x, h = blockIdx.y * blockDim.x + threadIdx.x;
  if (!s_ok || t >= T || h >= d.H) return;
  const float *out = (const float *)(A.mine + A.o_out);
  float acc = 0.0f;
  for (int k = 0; k < d.K; k++) {
    const size_t pair = (size_t)t * d.K + k;
    acc = __fadd_rn(acc, __fmul_rn(w[pair], out[pair * d.H + h]));
  }
  float *res = residual + (size_t)t * d.H + h;
  *res = __fadd_rn(*res, acc);
}
