/*
 * ramvamp_b200.h -- C ABI of the B200 (sm_100a) routed-expert FFN path.
 *
 * A drop-in replacement for ramvamp's CPU MoE-layer and quantized-matvec
 * entry points.  Every function takes plain pointers and sizes (no
 * CUDA, torch or Rust types), returns an rv_status, and never panics or
 * aborts on bad input: validation happens once per call, before any launch,
 * with the same checks and error precedence as the Rust function it
 * replaces.  A human-readable detail of the most recent failure on the
 * calling thread is available from rv_last_error().
 *
 * Pointers documented as "device" are CUDA device addresses on the device
 * current when the call is made; "host" pointers are ordinary CPU memory.
 * `stream` is a cudaStream_t passed as void* (NULL = the legacy default
 * stream).  Calls that only enqueue work do not synchronize, so they can be
 * captured into a CUDA graph; the *_host variants synchronize on `stream`.
 *
 * Reference citations are paths inside the ramvamp tree
 * (crates/core/src/...).
 */
#ifndef RAMVAMP_B200_H
#define RAMVAMP_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RV_ABI_VERSION 1

#if defined(__GNUC__)
#define RV_API __attribute__((visibility("default")))
#else
#define RV_API
#endif

typedef void *rv_stream;

/* Status codes.  1..9 map one-to-one onto the variants of
 * kernels/error.rs:20-110 (KernelError); the rest are GPU-side conditions
 * the CPU reference cannot hit. */
typedef enum rv_status {
  RV_OK = 0,
  RV_ERR_INDIVISIBLE_ROW = 1,              /* KernelError::IndivisibleRow */
  RV_ERR_ROW_BYTES_NOT_BLOCK_MULTIPLE = 2, /* KernelError::RowBytesNotBlockMultiple */
  RV_ERR_BLOCK_COUNT_MISMATCH = 3,         /* KernelError::BlockCountMismatch */
  RV_ERR_QUANTIZE_LEN_MISMATCH = 4,        /* KernelError::QuantizeLenMismatch */
  RV_ERR_LENGTH_MISMATCH = 5,              /* KernelError::LengthMismatch */
  RV_ERR_EMPTY = 6,                        /* KernelError::Empty */
  RV_ERR_INVALID_HEAD_DIM = 7,             /* KernelError::InvalidHeadDim */
  RV_ERR_UNIMPLEMENTED = 8,                /* KernelError::Unimplemented */
  RV_ERR_UNSUPPORTED_FORMAT = 9,           /* KernelError::UnsupportedFormat */
  RV_ERR_ROUTED_OUT_OF_RANGE = 10,         /* ForwardError::RoutedExpertOutOfRange */
  RV_ERR_LAYER_OUT_OF_RANGE = 11,          /* IoError::LayerOutOfRange */
  RV_ERR_PROTOCOL = 12,                    /* IoError::Io protocol misuse (step state) */
  RV_ERR_INVALID_ARGUMENT = 13,            /* null pointer, misaligned buffer, bad flag */
  RV_ERR_CUDA = 14,                        /* a CUDA runtime call failed */
  RV_ERR_NCCL = 15,                        /* a collective failed */
  RV_ERR_TIMEOUT = 16,                     /* a bounded device-side wait ran out */
  RV_ERR_IO = 17,                          /* IoError::Io: a file could not be opened or read */
  RV_ERR_TOKEN_OUT_OF_RANGE = 18,          /* ModelError::TokenOutOfRange (a row id past the matrix) */
  RV_ERR_POSITION_MISMATCH = 19,           /* ForwardError::PositionMismatch (position != cached length) */
  RV_ERR_CAPACITY_EXCEEDED = 20,           /* KvError::CapacityExceeded (the layer's cache is full) */
  RV_ERR_PEER = 21                         /* an expert-parallel peer's handle does not fit this group,
                                              or its memory could not be mapped */
} rv_status;

/* Quantization formats (kernels/quants/mod.rs:57-70). */
typedef enum rv_quant_format {
  RV_Q4_K = 0, /* 144 B / 256 weights */
  RV_Q5_K = 1, /* 176 B / 256 weights */
  RV_Q6_K = 2, /* 210 B / 256 weights */
  RV_Q8_0 = 3, /*  34 B /  32 weights */
  RV_Q8_K = 4  /* 292 B / 256 weights (activations) */
} rv_quant_format;

/* One Q8_K activation block.  The reference's BlockQ8K
 * (kernels/quants/blocks.rs:146-153) is not repr(C); this is the packed
 * 292-byte C layout every rv_ call uses: d at 0, qs at 4, bsums at 260. */
typedef struct rv_block_q8k {
  float d;
  int8_t qs[256];
  int16_t bsums[16];
} rv_block_q8k;

/* One Q8_0 activation block: the reference's BlockQ8_0
 * (kernels/quants/blocks.rs:167-178), d already rounded through f16, in a
 * 36-byte C layout: d at 0, qs at 4. */
typedef struct rv_block_q8_0 {
  float d;
  int8_t qs[32];
} rv_block_q8_0;

/* ------------------------------------------------------------ library */
/* Version string of the library build. */
RV_API const char *rv_version(void);
/* Name of a status code ("LengthMismatch", ...). */
RV_API const char *rv_status_name(int status);
/* Copies the detail message of the calling thread's most recent failure
 * into buf (NUL-terminated, truncated to len); returns its full length. */
RV_API size_t rv_last_error(char *buf, size_t len);
/* Block geometry: QuantFormat::block_bytes / block_weights
 * (kernels/quants/mod.rs:74-90). 0 for an unknown format. */
RV_API size_t rv_block_bytes(int format);
RV_API size_t rv_block_weights(int format);
/* QuantFormat::row_bytes (kernels/quants/mod.rs:96-105):
 * RV_ERR_INDIVISIBLE_ROW when in_dim is not a block multiple. */
RV_API int rv_row_bytes(int format, size_t in_dim, size_t *out);
/* Reads and clears the device-side error word the kernels of this library
 * set when a bounded wait ran out (RV_ERR_TIMEOUT) or a device check failed.
 * Synchronizes `stream`. */
RV_API int rv_device_status(int device, rv_stream stream);
/* Failure-path probe.  No counterpart in the reference; its analogue there
 * is the injected EBUSY of io/stream.rs:2794-2830, which drives the
 * streamer's typed-error path in tests.  Launches one small kernel that
 * waits, through the same bounded-wait helper the library's kernels use, on
 * something nothing will complete -- what = 0: an mbarrier phase no thread
 * arrives on (the tensor GEMM's and bulk-copy waits); 1: a device flag no
 * peer sets (the expert-parallel exchange's waits) -- and gives up after
 * `cycles` SM cycles (1..2e9).  The kernel returns normally and the timeout
 * lands in the device error word: the next rv_device_status reports
 * RV_ERR_TIMEOUT, and the device stays usable for the calls after it. */
RV_API int rv_debug_wait_probe(int device, uint32_t what, uint64_t cycles, rv_stream stream);

/* ----------------------------------------------------------- kernels */
/* Replaces quants::quantize_row_q8_k (kernels/quants/quantize.rs:68-103,
 * AVX2 arm avx2.rs:1070-1130).  x: device, n floats; out: device,
 * out_blocks blocks.  Byte-identical to the reference on finite input.
 * Any number of rows may be passed as one long row (blocks are
 * independent).  RV_ERR_QUANTIZE_LEN_MISMATCH when n != 256*out_blocks. */
RV_API int rv_quantize_row_q8_k(const float *x, size_t n, rv_block_q8k *out, size_t out_blocks,
                         rv_stream stream);

/* Replaces gemv::gemv_q8_k / Backend::gemv_q8_k (kernels/gemv.rs:347-371,
 * kernels/backend.rs:115-124): out[r] = weight_row_r . acts for r in
 * 0..out_dim.  weight: device, weight_len bytes (any byte alignment);
 * acts: device, acts_len blocks; out: device, out_len floats.  Bit-identical
 * to the reference's AVX2 path. */
RV_API int rv_gemv_q8_k(int format, const uint8_t *weight, size_t weight_len, size_t in_dim,
                 size_t out_dim, const rv_block_q8k *acts, size_t acts_len, float *out,
                 size_t out_len, rv_stream stream);

/* Replaces gemv::gemv_q8_k_rows (kernels/gemv.rs:386-410): the rows
 * [row_start, row_end) only; weight/in_dim/out_dim describe the whole
 * matrix, out holds row_end-row_start floats. */
RV_API int rv_gemv_q8_k_rows(int format, const uint8_t *weight, size_t weight_len, size_t in_dim,
                      size_t out_dim, const rv_block_q8k *acts, size_t acts_len, size_t row_start,
                      size_t row_end, float *out, size_t out_len, rv_stream stream);

/* Replaces gemv::gemv_q8_k_batched (kernels/gemv.rs:444-477):
 * out[i*n_acts + a] = weight_row_(row_start+i) . act_row_a. */
RV_API int rv_gemv_q8_k_batched(int format, const uint8_t *weight, size_t weight_len, size_t in_dim,
                         size_t out_dim, const rv_block_q8k *acts, size_t acts_len, size_t n_acts,
                         size_t row_start, size_t row_end, float *out, size_t out_len,
                         rv_stream stream);

/* Replaces quants::quantize_row_q8_0 (kernels/quants/quantize.rs:37-54):
 * per 32 floats d = amax/127, values times 1/d rounded half away from zero
 * with Rust's saturating cast (NaN -> 0), d stored rounded through f16.
 * x: device, n floats; out: device, out_blocks blocks.  Byte-identical to
 * the scalar arm on every input.  (The AVX2 arm, avx2.rs:1022-1056, agrees
 * with it except on blocks whose amax is below ~3.7e-37, where 1/d
 * overflows and cvtps_epi32 turns every value into -128.)
 * RV_ERR_QUANTIZE_LEN_MISMATCH when n != 32*out_blocks. */
RV_API int rv_quantize_row_q8_0(const float *x, size_t n, rv_block_q8_0 *out, size_t out_blocks,
                         rv_stream stream);

/* Replaces gemv::gemv_q8_0 / Backend::gemv_q8_0 (kernels/gemv.rs:544-565,
 * kernels/backend.rs:89-98): Q8_0 weights (34 B / 32 weights) against Q8_0
 * activations, out[r] = weight_row_r . acts.  weight: device, any 2-byte
 * alignment; acts: device, acts_len blocks; out: device.  Bit-identical to
 * the AVX2 arm (avx2.rs:942-963): eight i32 lanes of four products per
 * block, one FMA per lane per block, then hsum_ps_8's fixed tree. */
RV_API int rv_gemv_q8_0(const uint8_t *weight, size_t weight_len, size_t in_dim, size_t out_dim,
                 const rv_block_q8_0 *acts, size_t acts_len, float *out, size_t out_len,
                 rv_stream stream);

/* Replaces gemv::gemv_q8_0_rows (kernels/gemv.rs:579-601): rows
 * [row_start, row_end) only, out holds row_end-row_start floats. */
RV_API int rv_gemv_q8_0_rows(const uint8_t *weight, size_t weight_len, size_t in_dim, size_t out_dim,
                      const rv_block_q8_0 *acts, size_t acts_len, size_t row_start, size_t row_end,
                      float *out, size_t out_len, rv_stream stream);

/* Replaces gemv::gemv_q8_0_batched (kernels/gemv.rs:616-640):
 * out[i*n_acts + a] = weight_row_(row_start+i) . act_row_a. */
RV_API int rv_gemv_q8_0_batched(const uint8_t *weight, size_t weight_len, size_t in_dim, size_t out_dim,
                         const rv_block_q8_0 *acts, size_t acts_len, size_t n_acts, size_t row_start,
                         size_t row_end, float *out, size_t out_len, rv_stream stream);

/* Replaces quants::dequantize_row_{q4_k,q5_k,q6_k,q8_0}
 * (kernels/quants/dequant.rs:28-147) over chosen rows of a matrix, which is
 * also Weights::embed (model/weights.rs:371-384) for token ids:
 * out[i][0..in_dim) = dequantize(row rows[i]).  weight: device, out_dim
 * rows of row_bytes(in_dim); rows: device, n_rows ids, or NULL for rows
 * 0..n_rows-1; out: device, n_rows*in_dim floats.  Bit-identical (every
 * product and difference rounded as the reference's f32 expressions).
 * A device id >= out_dim cannot be checked before the launch: its row is
 * written as zeros and the device error word is set to
 * RV_ERR_TOKEN_OUT_OF_RANGE, which rv_device_status reports. */
RV_API int rv_dequantize_rows(int format, const uint8_t *weight, size_t weight_len, size_t in_dim,
                       size_t out_dim, const uint32_t *rows, size_t n_rows, float *out, size_t out_len,
                       rv_stream stream);

/* One matrix of a fused row space (gemv::FusedPart, kernels/gemv.rs:655-686).
 * weight and acts are device pointers. */
typedef struct rv_fused_part {
  int32_t format;
  const uint8_t *weight;
  size_t weight_len;
  size_t in_dim;
  size_t out_dim;
  const rv_block_q8k *acts;
  size_t acts_len;
} rv_fused_part;

/* Replaces gemv::gemv_q8_k_fused_rows (kernels/gemv.rs:747-823): rows
 * [row_start,row_end) of the concatenated row spaces of parts (host array).
 * out: device, row_end-row_start floats. */
RV_API int rv_gemv_q8_k_fused_rows(const rv_fused_part *parts, size_t n_parts, size_t row_start,
                            size_t row_end, float *out, size_t out_len, rv_stream stream);

/* Replaces Backend::rmsnorm / primitives::rmsnorm (kernels/primitives/norm.rs:
 * 275-298) for n_rows rows of `n` floats (x, out: device [n_rows][n];
 * weight: device [n]).  f64 mean of squares, bit-identical. */
RV_API int rv_rmsnorm(const float *x, const float *weight, size_t n, size_t n_rows, float eps, float *out,
               rv_stream stream);

/* Replaces Backend::softmax / primitives::softmax (kernels/primitives/softmax.rs:
 * 18-40), in place on n_rows rows of n floats (device).  n <= 1024. */
RV_API int rv_softmax(float *x, size_t n, size_t n_rows, rv_stream stream);

/* Replaces Backend::swiglu_combine / primitives::swiglu_combine
 * (kernels/primitives/activation.rs:30-42): gate[i] <- silu(gate[i]) * up[i]
 * (device).  The SiLU's exponential reproduces glibc expf bit for bit. */
RV_API int rv_swiglu_combine(float *gate, size_t gate_len, const float *up, size_t up_len,
                      rv_stream stream);

/* Integer taps for parity tests (no reference counterpart beyond the
 * integer stages of avx2.rs:554-838): for each of the n_blocks blocks of one
 * weight row against one activation row, the eight i32 lane sums the AVX2
 * dot forms (lanes_out[n_blocks][8]) and, for Q4_K/Q5_K, the four min-lane
 * sums (mins_out[n_blocks][4], zero for Q6_K).  All device pointers. */
RV_API int rv_debug_block_sums(int format, const uint8_t *weight_row, size_t w_len,
                        const rv_block_q8k *acts, size_t n_blocks, int32_t *lanes_out,
                        int32_t *mins_out, rv_stream stream);

/* ------------------------------------------------------- expert table */
/* Geometry of one layer's expert file (format/layout.rs:1-60,
 * io/expert.rs:27-86): blob e occupies [e*stride, (e+1)*stride). */
typedef struct rv_layer_layout {
  uint32_t n_experts;
  uint32_t _pad;
  uint64_t stride;
  uint64_t gate_off, gate_len;
  uint64_t up_off, up_len;
  uint64_t down_off, down_len;
  int32_t gate_format, up_format, down_format;
  uint32_t hidden, moe; /* gate/up are [moe][hidden], down [hidden][moe] */
} rv_layer_layout;

/* Device pointers of one resident expert (io/expert.rs:49-86). */
typedef struct rv_expert_view {
  const uint8_t *blob;
  const uint8_t *gate, *up, *down;
  uint64_t gate_len, up_len, down_len;
  int32_t gate_format, up_format, down_format;
} rv_expert_view;

typedef struct rv_expert_table rv_expert_table;

/* Creates the HBM-resident expert table that stands in for
 * io::ExpertStream (io/stream.rs:1147-1472): every layer's expert file is
 * allocated once on `device` (n_layers layouts, host array). */
RV_API int rv_expert_table_create(int device, const rv_layer_layout *layers, uint32_t n_layers,
                           rv_expert_table **out);
RV_API void rv_expert_table_destroy(rv_expert_table *t);
/* Copies n_experts consecutive blobs starting at expert_first into layer
 * `layer`.  src is host memory unless src_on_device != 0; len must be
 * n_experts*stride.  Synchronizes `stream`. */
RV_API int rv_expert_table_upload(rv_expert_table *t, uint32_t layer, uint32_t expert_first,
                           uint32_t n_experts, const void *src, size_t len, int src_on_device,
                           rv_stream stream);
/* Loads layer `layer` from an install's expert file (the file behind
 * layers[i].file of experts/layout.json, format/layout.rs:1-13): the
 * n_experts*stride bytes from file_offset on, read in chunks and copied to
 * the device as they arrive (the load-time half of io/stream.rs, whose
 * steady-state reads become table hits).  RV_ERR_IO when the file cannot be
 * opened or read, RV_ERR_LENGTH_MISMATCH when it is shorter than the layer.
 * Synchronizes `stream`. */
RV_API int rv_expert_table_load_file(rv_expert_table *t, uint32_t layer, const char *path,
                                     uint64_t file_offset, rv_stream stream);
RV_API int rv_expert_table_layout(const rv_expert_table *t, uint32_t layer, rv_layer_layout *out);
RV_API uint32_t rv_expert_table_n_layers(const rv_expert_table *t);
/* io/stream.rs:1472 (begin_layer): opens a step for `experts` (host array).
 * Every expert is resident, so every request is a hit; a duplicate id is
 * listed once, at its first position, like the reference. */
RV_API int rv_expert_table_begin_layer(rv_expert_table *t, uint32_t layer, const uint32_t *experts,
                                size_t n);
/* io/stream.rs:1551/1558 (hits/misses): (index into the request, slot)
 * pairs of the open step, written to host arrays of capacity cap; the
 * count is returned in *n_out.  The slot of expert e is e.  misses is
 * always empty. */
RV_API int rv_expert_table_hits(const rv_expert_table *t, uint32_t *index_out, uint32_t *slot_out,
                         size_t cap, size_t *n_out);
RV_API int rv_expert_table_misses(const rv_expert_table *t, uint32_t *index_out, uint32_t *slot_out,
                           size_t cap, size_t *n_out);
/* io/stream.rs:1575 (await_misses): nothing is ever in flight; returns
 * RV_OK, or RV_ERR_PROTOCOL without an open step. */
RV_API int rv_expert_table_await_misses(rv_expert_table *t);
/* io/stream.rs:1604 (view): device view of a resident slot. */
RV_API int rv_expert_table_view(const rv_expert_table *t, uint32_t layer, uint32_t slot,
                         rv_expert_view *out);
/* io/stream.rs:2123 (end_layer): closes the open step. */
RV_API int rv_expert_table_end_layer(rv_expert_table *t, uint32_t layer);
/* Access counters (io/stream.rs:297-400 StreamStats subset): requests and
 * hits since creation. */
RV_API int rv_expert_table_stats(const rv_expert_table *t, uint64_t *accesses, uint64_t *hits);

/* ------------------------------------------------------ MoE layer */
/* Layer geometry (model ArchInfo subset, format/manifest.rs:72-105). */
typedef struct rv_moe_config {
  uint32_t hidden;     /* 2048 for Qwen3-30B-A3B */
  uint32_t moe;        /* moe_intermediate, 768 */
  uint32_t n_experts;  /* 128 (GPU path: <= 256) */
  uint32_t top_k;      /* 8 (<= 16) */
  int32_t norm_topk_prob;
  float eps;           /* rms_norm_eps, 1e-6 */
} rv_moe_config;

typedef struct rv_moe rv_moe;

/* Flags of rv_moe_forward. */
#define RV_MOE_EXACT 0u        /* every stage bit-identical to the reference */
#define RV_MOE_TENSOR 1u       /* prefill experts on tcgen05 tensor cores:
                                  integer sub-block sums exact, fp32 outputs
                                  within tolerance */

/* Creates a MoE engine on `device` with scratch for up to max_tokens rows per
 * call.  All device memory the hot path touches is allocated here; forward
 * calls allocate nothing. */
RV_API int rv_moe_create(int device, const rv_moe_config *cfg, size_t max_tokens, rv_moe **out);
RV_API void rv_moe_destroy(rv_moe *m);

/* The MoE block of one layer for n_tokens rows, in place on `residual`:
 * residual += sum_k w_k * expert_k(quantize(rmsnorm(residual))).
 * Replaces the inline MoE blocks of model::forward_token_traced
 * (model/forward.rs:2654-2754) and model::prefill::run_chunk
 * (model/prefill.rs:2136-2263, 2749-2778): same RMSNorm, router, top-k,
 * renormalization, Q8_K activations, expert FFN and fixed top-k-order
 * reduction.  Device pointers: ffn_norm [hidden], router [n_experts][hidden],
 * residual [n_tokens][hidden]; topk_ids/topk_weights [n_tokens][top_k] are
 * optional outputs (NULL to skip).  Experts come from `table`'s `layer`. */
RV_API int rv_moe_forward(rv_moe *m, const rv_expert_table *table, uint32_t layer,
                   const float *ffn_norm, const float *router, float *residual, size_t n_tokens,
                   uint32_t *topk_ids, float *topk_weights, uint32_t flags, rv_stream stream);

/* rv_moe_forward with a HOST residual (and optional host top-k outputs):
 * copies in, runs, copies out and synchronizes `stream`.  This is the call
 * a Rust caller holding `&mut [f32]` makes. */
RV_API int rv_moe_forward_host(rv_moe *m, const rv_expert_table *table, uint32_t layer,
                        const float *ffn_norm, const float *router, float *residual_host,
                        size_t n_tokens, uint32_t *topk_ids_host, float *topk_weights_host,
                        uint32_t flags, rv_stream stream);

/* ---- the MoE block in three parts (expert-parallel serving) ------------
 * The same arithmetic as rv_moe_forward, split where an expert-parallel
 * caller exchanges data between ranks.  The reference runs the block on one
 * host and has no such split; these entries let its run_chunk
 * (model/prefill.rs:2136-2263) run across GPUs with bit-identical results. */

/* Bytes per Q8_K activation row (hidden/256 blocks of 292 bytes, rounded
 * up to 16). */
RV_API size_t rv_moe_act_stride(const rv_moe *m);

/* Routing half (forward.rs:2655-2705, prefill.rs:2165-2204): ffn RMSNorm,
 * Q8_K of the normed rows, router logits, softmax, top-k, renormalization.
 * Writes topk_ids/topk_weights [n_tokens][top_k] and, if acts is not NULL,
 * the Q8_K rows [n_tokens][rv_moe_act_stride] (16-byte aligned).  The
 * residual is only read.  All device pointers. */
RV_API int rv_moe_route(rv_moe *m, const float *ffn_norm, const float *router, const float *residual,
                        size_t n_tokens, uint32_t *topk_ids, float *topk_weights, uint8_t *acts,
                        rv_stream stream);

/* Expert half for n_pairs (expert, Q8_K row) pairs of `layer` of `table`:
 * gate/up, SwiGLU, Q8_K, down (forward.rs:2159-2261).  expert_ids
 * [n_pairs] index the table's experts (0..n_experts-1 of that table);
 * acts [n_pairs][rv_moe_act_stride]; out [n_pairs][hidden] receives the
 * unweighted expert outputs.  n_pairs <= max_tokens * top_k of the engine.
 * flags: RV_MOE_EXACT or RV_MOE_TENSOR. */
RV_API int rv_moe_experts(rv_moe *m, const rv_expert_table *table, uint32_t layer, const uint32_t *expert_ids,
                          const uint8_t *acts, size_t n_pairs, float *out, uint32_t flags, rv_stream stream);

/* Weighted combine (forward.rs:2744-2753, prefill.rs:2749-2778): for each
 * token, acc = 0; acc += w_k * out[row(t, k)] in top-k order; residual +=
 * acc.  row(t, k) = pos_of[t*top_k + k], or t*top_k + k when pos_of is
 * NULL.  expert_out has hidden floats per row. */
RV_API int rv_moe_combine(rv_moe *m, float *residual, const float *topk_weights, const float *expert_out,
                          const uint32_t *pos_of, size_t n_tokens, rv_stream stream);

/* Expert-parallel dispatch plan over `world` ranks (1..64), expert e living
 * on rank e % world as local expert e / world: send_counts[world] (int32)
 * pairs per destination rank; pairs laid out rank by rank, pos_of
 * [n_tokens*top_k] = each pair's row; send_local[row] = the local expert id;
 * send_acts[row] = the pair's token's Q8_K row from acts.  No counterpart
 * in the reference, which has no expert parallelism. */
RV_API int rv_ep_plan(rv_moe *m, const uint32_t *topk_ids, const uint8_t *acts, size_t n_tokens, uint32_t world,
                      int32_t *send_counts, uint32_t *pos_of, uint32_t *send_local, uint8_t *send_acts,
                      rv_stream stream);

/* ---- expert parallelism over the GPUs of one node -----------------------
 * No counterpart in the reference, which runs the MoE block on one host.
 * The 128 experts of a layer are spread over `world` ranks (one process or
 * thread per GPU), n_experts / world per rank, by a placement: rank r's
 * rv_expert_table holds its experts as local experts 0, 1, ...  Without an
 * explicit placement expert e lives on rank e % world as local expert
 * e / world; a placement built from measured expert loads (see
 * rv_ep_check_placement) evens out a skewed router.
 * Each rank routes its own tokens; the exchange runs through GPU memory:
 * every rank owns an exchange window in its HBM that the others map (CUDA
 * IPC across processes, peer access inside one), dispatch stores each
 * pair's Q8_K row into the window of its expert's rank, the down projection
 * there stores the expert output row straight back into the home rank's
 * window over NVLink, and release/acquire flags at system scope, counted
 * per layer, order the steps.  No host synchronization and no collective
 * library call sits on the data path, so a layer's call can be captured
 * into a CUDA graph.  Every pair's output comes from the same kernels on
 * the same bytes as on one GPU and each home rank reduces in top-k order,
 * so the result is bit-identical to rv_moe_forward for every world size
 * (prefill.rs:2734-2778).
 *
 * Set-up (once per rank): rv_ep_create, then rv_ep_handle; the caller
 * gathers the world handles (RV_EP_HANDLE_BYTES each, in rank order) by any
 * out-of-band means (a TCP store, MPI, torch.distributed) and passes them
 * all to rv_ep_connect on every rank.  Each rank must be on its own GPU.
 * Every rank then calls rv_moe_ep_forward for the same layers in the same
 * order (n_tokens may differ, 0 included).  Waits on peers are bounded
 * (~1 s): a peer that does not arrive leaves RV_ERR_TIMEOUT in the device
 * error word (rv_device_status) and the layer's result undefined; the group
 * must then be destroyed and created again on every rank. */
#define RV_EP_HANDLE_BYTES 256
typedef struct rv_ep rv_ep;
/* `m`'s geometry and device; max_tokens = home tokens per call on this rank.
 * The engine runs the experts on up to world * max_tokens received rows, so
 * it must have been created with max_tokens >= world * max_tokens.  The
 * window holds world * max_tokens * top_k received rows plus max_tokens *
 * top_k output rows (77 MB + 34 MB for Qwen3 at 512 tokens per rank). */
RV_API int rv_ep_create(rv_moe *m, uint32_t world, uint32_t rank, size_t max_tokens, rv_ep **out);
RV_API void rv_ep_destroy(rv_ep *ep);
/* Writes this rank's handle (RV_EP_HANDLE_BYTES bytes, host) to out. */
RV_API int rv_ep_handle(const rv_ep *ep, void *out, size_t len);
/* handles: world * RV_EP_HANDLE_BYTES bytes (host), rank order.
 * RV_ERR_PEER if a handle is not one of this group's (wrong world, rank,
 * geometry or capacity, two ranks on one GPU) or cannot be mapped; nothing
 * is mapped then. */
RV_API int rv_ep_connect(rv_ep *ep, const void *handles, size_t len);
/* The MoE block of one layer for this rank's n_tokens home rows, in place on
 * `residual` (device), as rv_moe_forward: ffn_norm [hidden], router
 * [n_experts][hidden] (all experts, device), table = this rank's experts;
 * topk_ids/topk_weights optional [n_tokens][top_k] outputs.  placement:
 * device [n_experts], entry e = rank << 16 | local id of global expert e,
 * the same on every rank for this layer (NULL: e % world, e / world); an
 * entry out of range is reported in the device error word.  flags:
 * RV_MOE_EXACT or RV_MOE_TENSOR.  Enqueues only (no host synchronization).
 * RV_ERR_PROTOCOL before rv_ep_connect. */
RV_API int rv_moe_ep_forward(rv_ep *ep, const rv_expert_table *table, uint32_t layer, const float *ffn_norm,
                             const float *router, float *residual, size_t n_tokens, uint32_t *topk_ids,
                             float *topk_weights, const uint32_t *placement, uint32_t flags, rv_stream stream);
/* Checks a placement (host, len == n_experts) before it is used: every rank
 * holds exactly n_experts / world experts with local ids 0..n_experts/world-1
 * each used once (RV_ERR_ROUTED_OUT_OF_RANGE, RV_ERR_INVALID_ARGUMENT). */
RV_API int rv_ep_check_placement(uint32_t n_experts, uint32_t world, const uint32_t *placement, size_t len);
/* received[r] = pairs rank r sent this rank in the most recent layer (host,
 * len >= world); synchronizes the device. */
RV_API int rv_ep_counts(const rv_ep *ep, uint32_t *received, size_t len);

/* Device addresses of the intermediates the most recent forward left in the
 * engine's scratch, for parity tests.  Layout per field below. */
typedef struct rv_moe_taps {
  const float *normed;          /* [n_tokens][hidden] ffn RMSNorm output */
  const rv_block_q8k *acts;     /* Q8_K of normed, acts_stride bytes per token */
  size_t acts_stride;           /* bytes between tokens' Q8_K rows */
  const float *logits;          /* [n_tokens][n_experts] router logits */
  const float *weights;         /* [n_tokens][top_k] renormalized weights */
  const uint32_t *ids;          /* [n_tokens][top_k] expert ids */
  const uint32_t *index;        /* [index_start[n_experts]] pair ids (t*top_k+k) by expert;
                                   decode (<= 8 tokens) lays out the speculated pairs, and
                                   a position the exact routing did not select holds ~0 */
  const uint32_t *index_start;  /* [n_experts+1] CSR offsets into index */
  const float *swiglu;          /* [positions][moe] SwiGLU output, CSR order */
  const uint8_t *acts_moe;      /* CSR order, acts_moe_stride bytes per position */
  size_t acts_moe_stride;       /* bytes between positions' Q8_K rows */
  const float *staged;          /* [n_tokens][top_k][hidden] expert outputs */
  const float *logit_bounds;    /* decode: [n_tokens][n_experts] (lo, hi) pairs holding
                                   each router logit, from which the speculated experts
                                   are chosen; null when the engine has none */
} rv_moe_taps;
RV_API int rv_moe_get_taps(const rv_moe *m, rv_moe_taps *out);

/* Per-stage timing, the GPU analogue of the reference's PhaseClock
 * (model/prefill.rs:414-520): rv_moe_profile_enable(m, slots) creates
 * `slots` sets of five CUDA events (0 releases them).  Each following
 * rv_moe_forward -- also one being captured into a CUDA graph, which then
 * records into the same set on every replay -- takes the next unused set and
 * records an event before routing, before the gate/up kernel, before the
 * down kernel, before the combine and after it.  rv_moe_profile_rewind makes
 * the next forward take set 0 again.  rv_moe_profile_read synchronizes the
 * used sets and writes four floats per set (routing, gate_up, down, combine
 * milliseconds) to ms_out (host, capacity cap floats); *n_sets gets the
 * number of sets used. */
RV_API int rv_moe_profile_enable(rv_moe *m, size_t slots);
RV_API int rv_moe_profile_rewind(rv_moe *m);
RV_API int rv_moe_profile_read(rv_moe *m, float *ms_out, size_t cap, size_t *n_sets);

/* ------------------------------------------- allocation-free decode */
/* No counterpart in the reference (which never runs on a GPU): the MoE block
 * of rv_moe_forward for callers that cannot call cudaMalloc -- a host whose
 * device memory belongs to another allocator (a serving runtime's pool, a
 * process under a hard memory cap) or code that runs where allocation is not
 * allowed (a real-time decode loop, a stream being captured into a graph).
 * Nothing is allocated: the caller passes the layer's expert blobs
 * (device, layout->n_experts * layout->stride bytes, laid out as in
 * rv_layer_layout) and the other inputs and outputs exactly as for
 * rv_moe_forward (device pointers), and the intermediates live in one
 * file-scope device array of RV_STATIC_SCRATCH_BYTES that every GPU loading
 * the library holds until the process exits.
 * Limits: n_tokens <= RV_STATIC_MAX_TOKENS, hidden <= 2048, moe <= 1024,
 * n_experts <= 128, top_k <= 8; anything larger returns
 * RV_ERR_LENGTH_MISMATCH (or RV_ERR_UNIMPLEMENTED for the geometry) before
 * any work is queued.  The first call on each device looks up the array's
 * device address and uploads the SiLU exception table, so make that first
 * call before any stream capture.  The looked-up address is kept for the
 * life of the process, so the library must not be used across a
 * cudaDeviceReset of that device.  Every call shares the one array and it
 * keeps the previous call's contents (counters are cleared at the start of
 * each call): calls that overlap on the GPU -- on two streams, or from two
 * threads -- race and must be serialized by the caller.  Results are
 * bit-identical to rv_moe_forward. */
#define RV_STATIC_MAX_TOKENS 4
#define RV_STATIC_SCRATCH_BYTES (1u << 20)
RV_API int rv_moe_forward_static(const rv_moe_config *cfg, const rv_layer_layout *layout,
                                 const uint8_t *expert_blobs, const float *ffn_norm,
                                 const float *router, float *residual, size_t n_tokens,
                                 uint32_t *topk_ids, float *topk_weights, rv_stream stream);

/* ------------------------------------------------ synthetic inputs */
/* ---------------------------------------------------------- attention */
/* The attention half of a decode step (model/forward.rs:2614-2631): the
 * KV cache of every layer (f16, the reference's KvCache, kv/mod.rs), the
 * NeoX rotation table and scratch, on one device. */
typedef struct rv_attn_config {
  uint32_t n_layers;
  uint32_t n_heads;       /* query heads (32 for Qwen3-30B-A3B) */
  uint32_t n_kv_heads;    /* key/value heads (4); n_heads % n_kv_heads == 0 */
  uint32_t head_dim;      /* 128; even, a multiple of 8, <= 256 */
  uint32_t max_positions; /* cache capacity per layer */
  float rope_theta;       /* the manifest's rope_theta as f32 (model/forward.rs:2474) */
  float eps;              /* the QK-norm epsilon (the layer norms' eps) */
  uint32_t hidden;        /* model width for rv_attn_block's scratch (0: rv_attn_decode only) */
} rv_attn_config;

typedef struct rv_attn rv_attn;

/* Allocates the caches (2 * n_layers * max_positions * n_kv_heads *
 * head_dim f16) and scratch, and builds the rotation table: for every
 * position p < max_positions and i < head_dim/2, (cos, sin) of
 * p * theta^(-2i/head_dim) formed in f64 with the host libm and rounded to
 * f32, exactly as rope.rs:30-45 computes them per call. */
RV_API int rv_attn_create(int device, const rv_attn_config *cfg, rv_attn **out);
RV_API void rv_attn_destroy(rv_attn *a);
/* KvCache::len / clear (kv/mod.rs). */
RV_API int rv_attn_len(const rv_attn *a, uint32_t layer, uint32_t *len_out);
RV_API int rv_attn_clear(rv_attn *a);
/* Device pointers to one layer's caches, [max_positions][n_kv_heads * head_dim]. */
RV_API int rv_attn_cache(const rv_attn *a, uint32_t layer, const uint16_t **k_out, const uint16_t **v_out);
/* Copies rows 0..positions-1 of one layer's caches to k_out / v_out
 * (device, positions * n_kv_heads * head_dim halves each), on `stream`. */
RV_API int rv_attn_copy_cache(const rv_attn *a, uint32_t layer, uint32_t positions, uint16_t *k_out, uint16_t *v_out,
                       rv_stream stream);

/* One layer of one decode step (forward.rs:2614-2631): per-head
 * QK-RMSNorm of q and k (norm.rs:72-90, weights q_norm / k_norm
 * [head_dim]), NeoX RoPE of both at `position` (rope.rs:80-111), the f16
 * append of k and v (kv/mod.rs:336-373), then decode attention over
 * positions 0..position (attention.rs:1075-1303, scale 1/sqrt(head_dim) in
 * f32).  q [n_heads*head_dim] and k [n_kv_heads*head_dim] are updated in
 * place (normed and rotated), as the reference does; v is read; out
 * [n_heads*head_dim] receives the attention output.  All device pointers.
 * RV_ERR_POSITION_MISMATCH unless position == rv_attn_len(layer);
 * RV_ERR_CAPACITY_EXCEEDED when the layer is full; nothing is written then.
 * Bit-identical to the reference except that its f64 exp (glibc) and
 * CUDA's may differ in the last bit, which changes an f32 probability only
 * when the exact value lies within ~2^-29 ulp of a rounding boundary. */
RV_API int rv_attn_decode(rv_attn *a, uint32_t layer, uint32_t position, float *q, float *k, const float *v,
                   const float *q_norm, const float *k_norm, float *out, rv_stream stream);

/* rv_attn_decode for graph-driven decoding: the position is read from
 * position_dev (device int32) when the kernels run, so one captured CUDA
 * graph serves every step.  The host length bookkeeping is not used
 * (rv_attn_len does not change).  A position outside [0, max_positions)
 * makes every kernel write nothing and sets RV_ERR_CAPACITY_EXCEEDED in
 * the device error word (rv_device_status). */
RV_API int rv_attn_decode_dev(rv_attn *a, uint32_t layer, const int32_t *position_dev, float *q, float *k,
                       const float *v, const float *q_norm, const float *k_norm, float *out, rv_stream stream);
/* The end of a graph-driven decode step, on the device: when next_token
 * is given, ids_out[position] = next_token[0] (if ids_out and position <
 * ids_cap) and token[0] = next_token[0] (if token); then position += 1. */
RV_API int rv_decode_advance(int32_t *position_dev, const uint32_t *next_token, int32_t *token, uint32_t *ids_out,
                      size_t ids_cap, rv_stream stream);

/* Sampler::argmax (generate/mod.rs:321-331): out[0] = the first index of
 * the largest of x[0..n) (device); NaN never wins; 0 when nothing beats
 * -inf.  RV_ERR_EMPTY for n == 0. */
RV_API int rv_argmax(const float *x, size_t n, uint32_t *out, rv_stream stream);
/* primitives::vec_add (kernels/primitives/vec.rs:10-22): a[i] += b[i]. */
RV_API int rv_vec_add(float *a, const float *b, size_t n, rv_stream stream);

/* One layer's weights for rv_attn_block (device pointers, the GGUF-style
 * row-major packed matrices of model/shapes.rs:14-35). */
typedef struct rv_attn_weights {
  const float *attn_norm;      /* [hidden] */
  const uint8_t *attn_q;       /* [n_heads*head_dim][hidden], Q4_K/Q5_K/Q6_K */
  const uint8_t *attn_k;       /* [n_kv_heads*head_dim][hidden], Q8_0 */
  const uint8_t *attn_v;       /* [n_kv_heads*head_dim][hidden], Q4_K/Q5_K/Q6_K */
  const uint8_t *attn_output;  /* [hidden][n_heads*head_dim], Q4_K/Q5_K/Q6_K */
  const float *q_norm;         /* [head_dim] */
  const float *k_norm;         /* [head_dim] */
  int32_t attn_q_format, attn_v_format, attn_output_format;
} rv_attn_weights;

/* The whole attention half of one decode step for one layer
 * (model/forward.rs:2572-2652), residual in place: rmsnorm(residual,
 * attn_norm) -> Q8_K and Q8_0 (one fused kernel) -> the q, k, v projections
 * (one launch) -> QK-norm, RoPE, f16 append, attention -> Q8_K ->
 * attn_output with the residual add in its epilogue.  Needs cfg.hidden.
 * position_dev NULL: `position` is checked as in rv_attn_decode; else the
 * position is read on the device as in rv_attn_decode_dev.  Bit-identical
 * to the reference's sequence (same caveat as rv_attn_decode). */
RV_API int rv_attn_block(rv_attn *a, uint32_t layer, const rv_attn_weights *w, float *residual,
                  const int32_t *position_dev, uint32_t position, rv_stream stream);

/* rmsnorm (norm.rs:38-60) of x [n] with weight w fused with
 * quantize_row_q8_k (q8k_out: n/256 blocks) and, when q80_out is given,
 * quantize_row_q8_0 (n/32 blocks); n a multiple of 256, <= 16384. */
RV_API int rv_rmsnorm_quantize(const float *x, const float *w, size_t n, float eps, rv_block_q8k *q8k_out,
                        rv_block_q8_0 *q80_out, rv_stream stream);

/* Replaces primitives::rope_neox_heads / Backend::rope_neox_heads
 * (kernels/primitives/rope.rs:80-111): x [n_heads*head_dim] (device)
 * rotated in place at `position`.  RV_ERR_INVALID_HEAD_DIM for a zero or odd
 * head_dim; RV_ERR_LENGTH_MISMATCH when x_len != n_heads*head_dim. */
RV_API int rv_rope_neox_heads(float *x, size_t x_len, size_t n_heads, size_t head_dim, uint32_t position,
                       float theta, rv_stream stream);

/* Replaces kernels::attention::decode_attention (attention.rs:426-438,
 * body :1075-1303) over caller caches: q [n_heads*head_dim] f32, k_cache /
 * v_cache [positions][n_kv_heads*head_dim] f16 bits, out [n_heads*head_dim];
 * scratch: 2*n_heads*positions floats.  All device pointers. */
RV_API int rv_attention(const float *q, const uint16_t *k_cache, const uint16_t *v_cache, size_t positions,
                 size_t n_heads, size_t n_kv_heads, size_t head_dim, float scale, float *scratch,
                 size_t scratch_len, float *out, rv_stream stream);

/* Seeded N(0, sigma^2)-like values: element i is the Irwin-Hall sum of
 * twelve 24-bit uniforms drawn from SplitMix64(seed, offset + i), so the
 * same (seed, offset) gives the same floats on every device and host.
 * out: device. */
RV_API int rv_synth_normal(uint64_t seed, uint64_t offset, float sigma, float *out, size_t n,
                    rv_stream stream);
/* The reference's weight quantizers on the GPU
 * (kernels/quants/test_support.rs:106-219), byte-identical to them:
 * n floats (device) -> n/256 blocks of `format` (device). */
RV_API int rv_quantize_weights(int format, const float *x, size_t n, uint8_t *out, rv_stream stream);
/* Fills every expert blob of `layer` with seeded N(0, sigma^2) weights
 * quantized by rv_quantize_weights (gate, up, down at their offsets). */
RV_API int rv_expert_table_fill_synthetic(rv_expert_table *t, uint32_t layer, uint64_t seed, float sigma,
                                   rv_stream stream);
/* The same weights for a shard of the experts: the table's expert i gets the
 * weights of global expert first_expert + i*expert_step (an expert-parallel
 * rank holding experts r, r+G, r+2G, ...). */
RV_API int rv_expert_table_fill_synthetic_strided(rv_expert_table *t, uint32_t layer, uint64_t seed, float sigma,
                                                  uint32_t first_expert, uint32_t expert_step, rv_stream stream);
/* Local expert i of `layer` gets global expert experts[i]'s synthetic
 * weights (host list, n == the layer's n_experts): an expert-parallel
 * rank's experts under any placement. */
RV_API int rv_expert_table_fill_synthetic_list(rv_expert_table *t, uint32_t layer, uint64_t seed, float sigma,
                                               const uint32_t *experts, size_t n, rv_stream stream);

#ifdef __cplusplus
}
#endif
#endif /* RAMVAMP_B200_H */
