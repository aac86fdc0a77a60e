/*
 * rv_oracle.h -- CPU restatement of ramvamp's routed-expert FFN path.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product (the ramvamp_b200
 * package, its CUDA library, bench.py's GPU arm) links or calls this code.
 * It exists so tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * --impl reference legs can check the GPU path against, and time, the
 * reference's own CPU algorithm.
 *
 * The reference (y0sif/ramvamp) is Rust; no Rust toolchain exists in this
 * image, so every function here restates the Rust source it names, in C,
 * with the same operation order.  Two arms exist for every k-quant dot:
 *   - OR_IMPL_SCALAR: crates/core/src/kernels/quants/dot.rs (ground truth),
 *   - OR_IMPL_AVX2:   crates/core/src/kernels/quants/avx2.rs (the dispatch
 *                     the reference actually runs on an AVX2+FMA host),
 *   - OR_IMPL_LANES:  a portable C model of the AVX2 arm's float order
 *                     (eight i32 lanes per block, FMA per lane, the fixed
 *                     horizontal-sum tree), which is the order the GPU
 *                     kernels reproduce.  Tested bit-identical to AVX2.
 *
 * Parity pins: the reference's known-answer tests (quantize.rs:140-177,
 * f16.rs:97-160, quants/tests.rs:230-467) are re-expressed in
 * tests/test_oracle_kat.py against this library.
 */
#ifndef RV_ORACLE_H
#define RV_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { OR_Q4_K = 0, OR_Q5_K = 1, OR_Q6_K = 2, OR_Q8_0 = 3, OR_Q8_K = 4 };
enum { OR_IMPL_SCALAR = 0, OR_IMPL_AVX2 = 1, OR_IMPL_LANES = 2 };

/* Error codes: one per KernelError variant (kernels/error.rs:20-110). */
enum {
  OR_OK = 0,
  OR_ERR_INDIVISIBLE_ROW = 1,
  OR_ERR_ROW_BYTES_NOT_BLOCK_MULTIPLE = 2,
  OR_ERR_BLOCK_COUNT_MISMATCH = 3,
  OR_ERR_QUANTIZE_LEN_MISMATCH = 4,
  OR_ERR_LENGTH_MISMATCH = 5,
  OR_ERR_EMPTY = 6,
  OR_ERR_INVALID_HEAD_DIM = 7,
  OR_ERR_UNSUPPORTED_FORMAT = 9,
  OR_ERR_ROUTED_OUT_OF_RANGE = 20
};

/* BlockQ8K (blocks.rs:146-153) in a packed 292-byte C layout. */
typedef struct or_block_q8k {
  float d;
  int8_t qs[256];
  int16_t bsums[16];
} or_block_q8k;

/* BlockQ8_0 (blocks.rs:167-178): d already rounded through f16, 36 bytes. */
typedef struct or_block_q8_0 {
  float d;
  int8_t qs[32];
} or_block_q8_0;

/* One MoE layer: norm, router, and 128 expert blobs laid out like the
 * .rvmp expert file (format/layout.rs:1-13): blob e starts at
 * blobs + e * stride; gate/up/down slabs at the given offsets. */
typedef struct or_moe_layer {
  uint32_t hidden, moe, n_experts, top_k;
  int32_t norm_topk_prob;
  float eps;
  const float *ffn_norm;   /* [hidden] */
  const float *router;     /* [n_experts][hidden] */
  const uint8_t *blobs;    /* n_experts * stride bytes */
  uint64_t stride;
  uint64_t gate_off, up_off, down_off;
  int32_t gate_fmt, up_fmt, down_fmt;
} or_moe_layer;

/* Optional intermediate taps of one MoE pass (any pointer may be NULL).
 * Per token t and top-k slot k (pair p = t*top_k + k). */
typedef struct or_moe_taps {
  float *normed;          /* [T][hidden] */
  or_block_q8k *acts;     /* [T][hidden/256] */
  float *logits;          /* [T][n_experts] */
  float *gate_up;         /* [T*top_k][2][moe] */
  or_block_q8k *acts_moe; /* [T*top_k][moe/256] */
  float *staged;          /* [T*top_k][hidden] */
} or_moe_taps;

const char *or_version(void);
int or_has_avx2(void);

/* f16.rs:17-91 */
float or_f16_to_f32(uint16_t bits);
uint16_t or_f32_to_f16(float x);
/* blocks.rs:127-141 */
void or_get_scale_min_k4(int j, const uint8_t *scales, uint8_t *sc, uint8_t *m);
/* avx2.rs:463-485 */
void or_unpack_scales_mins(const uint8_t *scales, uint8_t *sc8, uint8_t *m8);

size_t or_block_bytes(int fmt);
size_t or_block_weights(int fmt);

/* quantize.rs:68-103 (scalar) / avx2.rs:1070-1130 (AVX2). */
int or_quantize_row_q8_k(const float *x, size_t n, or_block_q8k *out, size_t out_blocks, int impl);

/* dot.rs:96-184 / avx2.rs:554-838 / lane model. */
int or_vec_dot(int fmt, const uint8_t *w, size_t w_len, const or_block_q8k *a, size_t n_blocks,
               int impl, float *out);
/* avx2.rs:162-192, 267-329: one weight row against n_acts activation rows. */
int or_vec_dot_rows(int fmt, const uint8_t *w, size_t w_len, const or_block_q8k *a, size_t n_acts,
                    float *out, int impl);
/* Per-block integer taps: the eight AVX2 lane sums (i32) and, for Q4_K/Q5_K,
 * the four min-lane sums, plus the scalar per-block sumi/sumi_mins. */
int or_block_int_sums(int fmt, const uint8_t *wblock, const or_block_q8k *a, int32_t *lanes8,
                      int32_t *mins4, int32_t *sumi, int32_t *sumi_mins);

/* gemv.rs:296-330 and :444-477: out[i*n_acts+a] = row(r0+i) . act_a. */
int or_gemv(int fmt, const uint8_t *w, size_t w_len, size_t in_dim, size_t out_dim,
            const or_block_q8k *acts, size_t n_acts, size_t r0, size_t r1, float *out,
            size_t out_len, int impl, int threads);

/* quantize.rs:37-54 (scalar) / avx2.rs:1022-1056 (AVX2). */
int or_quantize_row_q8_0(const float *x, size_t n, or_block_q8_0 *out, size_t out_blocks, int impl);
/* dot.rs:190-201 / avx2.rs:942-963 / lane model. */
int or_vec_dot_q8_0(const uint8_t *w, size_t w_len, const or_block_q8_0 *a, size_t n_blocks, int impl,
                    float *out);
/* gemv.rs:544-640: out[i*n_acts+a] = row(r0+i) . act_a. */
int or_gemv_q8_0(const uint8_t *w, size_t w_len, size_t in_dim, size_t out_dim, const or_block_q8_0 *acts,
                 size_t acts_len, size_t n_acts, size_t r0, size_t r1, float *out, size_t out_len, int impl,
                 int threads);
/* test_support.rs:221-234 */
void or_quantize_row_q8_0_test(const float *x, size_t n, uint8_t *out);

/* Attention half of the decode step: rope.rs:30-111, attention.rs:1075-1303,
 * kv/mod.rs:336-373, model/forward.rs:2614-2631. */
int or_rope_neox_heads(float *x, size_t n_heads, size_t head_dim, uint32_t position, float theta);
void or_rope_factors(size_t head_dim, uint32_t position, float theta, float *cos_out, float *sin_out);
int or_attention(const float *q, const uint16_t *k_cache, const uint16_t *v_cache, size_t positions,
                 size_t n_heads, size_t n_kv_heads, size_t head_dim, float scale, float *out);
int or_attn_decode_step(float *q, float *k, const float *v, const float *q_norm, const float *k_norm,
                        uint16_t *k_cache, uint16_t *v_cache, size_t position, size_t n_heads, size_t n_kv_heads,
                        size_t head_dim, float eps, float theta, float *out);

/* test_support.rs:23-39 */
uint64_t or_lcg_next_u64(uint64_t *state);
float or_lcg_next_f32(uint64_t *state);
void or_lcg_fill_f32(uint64_t *state, float *out, size_t n, float scale);

/* test_support.rs:106-219: the reference's weight quantizers. */
void or_quantize_row_q4_k_test(const float *x, size_t n, uint8_t *out);
void or_quantize_row_q5_k_test(const float *x, size_t n, uint8_t *out);
void or_quantize_row_q6_k_test(const float *x, size_t n, uint8_t *out);
/* dequant.rs (Q4_K, Q5_K, Q6_K, Q8_0) */
int or_dequantize_row(int fmt, const uint8_t *bytes, size_t len, float *out);

/* primitives: norm.rs:17-60, softmax.rs:18-40, activation.rs:14-42 */
int or_rmsnorm(const float *x, const float *w, size_t n, float eps, float *out);
int or_softmax(float *x, size_t n);
int or_swiglu_combine(float *gate, const float *up, size_t n);
float or_dot_f32(const float *a, const float *b, size_t n);

/* Router for one row: forward.rs:2669-2705 / prefill.rs:2165-2204. */
int or_route(const float *normed, const float *router, uint32_t hidden, uint32_t n_experts,
             uint32_t top_k, int norm_topk_prob, float *logits, uint32_t *ids, float *weights);

/* Decode MoE block for T tokens, token-major (forward.rs:2654-2754,
 * run_expert_window :2159-2261).  residual [T][hidden] is updated in place. */
int or_moe_decode(const or_moe_layer *L, float *residual, size_t T, uint32_t *topk_ids,
                  float *topk_w, const or_moe_taps *taps, int impl, int threads);
/* Prefill MoE block: router per row, CSR inverse index (prefill.rs:2536-2580),
 * per-expert batched FFN (:2585-2732), top-k-order reduce (:2749-2778). */
int or_moe_prefill(const or_moe_layer *L, float *residual, size_t T, uint32_t *topk_ids,
                   float *topk_w, int impl, int threads);

/* CPU restatement of the GPU library's seeded synthetic generator
 * (rv_synth_normal: SplitMix64 + Irwin-Hall(12)), bit-identical, so the CPU
 * reference arm can build the same expert weights without the GPU. */
void or_synth_normal(uint64_t seed, uint64_t offset, float sigma, float *out, size_t n);
/* Fills n_experts blobs (stride bytes each) the way the GPU library's
 * rv_expert_table_fill_synthetic does: per expert e, 3*moe*hidden values at
 * offset e*3*moe*hidden, quantized by the reference's test quantizers. */
void or_fill_layer_synthetic(uint32_t hidden, uint32_t moe, uint32_t n_experts, uint64_t stride,
                             uint64_t gate_off, uint64_t up_off, uint64_t down_off, int gate_fmt,
                             int up_fmt, int down_fmt, uint64_t seed, float sigma, uint8_t *blobs,
                             int threads);

/* CSR inverse index alone, for dispatch parity tests. index_start has
 * n_experts+1 entries; index holds T*top_k (row<<16 | slot) entries. */
int or_build_index(const uint32_t *topk_ids, size_t T, uint32_t top_k, uint32_t n_experts,
                   uint32_t *index_start, uint32_t *index);

#ifdef __cplusplus
}
#endif
#endif
