// rv_lib.cu -- host side of libramvamp_b200.so: the C ABI declared in
// include/ramvamp_b200.h.  One translation unit (the kernels come in as
// headers) so every device global lives in one module.
#include <algorithm>
#include <cerrno>
#include <cstdio>
#include <cstring>
#include <cstdlib>
#include <mutex>
#include <new>
#include <unistd.h>
#include <vector>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "rv_expf.cuh"
#include "rv_internal.cuh"
#include "rv_kernels.cuh"
#include "rv_moe.cuh"
#include "rv_tc.cuh"
#include "rv_ep.cuh"
#include "rv_attn.cuh"

#include "_gen/expf_exceptions.inc"

#define RV_VERSION_STRING "ramvamp_b200 0.1 (sm_100a)"

// ================================================================ errors
static thread_local char t_err[1024];
static thread_local size_t t_err_len;

void rv_set_error(int status, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  int n = snprintf(t_err, sizeof t_err, "%s: ", rv_status_name(status));
  if (n < 0) n = 0;
  int m = vsnprintf(t_err + n, sizeof t_err - (size_t)n, fmt, ap);
  va_end(ap);
  t_err_len = (size_t)n + (m > 0 ? (size_t)m : 0);
}

extern "C" const char *rv_version(void) { return RV_VERSION_STRING; }

extern "C" const char *rv_status_name(int s) {
  switch (s) {
    case RV_OK: return "Ok";
    case RV_ERR_INDIVISIBLE_ROW: return "IndivisibleRow";
    case RV_ERR_ROW_BYTES_NOT_BLOCK_MULTIPLE: return "RowBytesNotBlockMultiple";
    case RV_ERR_BLOCK_COUNT_MISMATCH: return "BlockCountMismatch";
    case RV_ERR_QUANTIZE_LEN_MISMATCH: return "QuantizeLenMismatch";
    case RV_ERR_LENGTH_MISMATCH: return "LengthMismatch";
    case RV_ERR_EMPTY: return "Empty";
    case RV_ERR_INVALID_HEAD_DIM: return "InvalidHeadDim";
    case RV_ERR_UNIMPLEMENTED: return "Unimplemented";
    case RV_ERR_UNSUPPORTED_FORMAT: return "UnsupportedFormat";
    case RV_ERR_ROUTED_OUT_OF_RANGE: return "RoutedExpertOutOfRange";
    case RV_ERR_LAYER_OUT_OF_RANGE: return "LayerOutOfRange";
    case RV_ERR_PROTOCOL: return "Protocol";
    case RV_ERR_INVALID_ARGUMENT: return "InvalidArgument";
    case RV_ERR_CUDA: return "Cuda";
    case RV_ERR_NCCL: return "Nccl";
    case RV_ERR_TIMEOUT: return "Timeout";
    case RV_ERR_IO: return "Io";
    case RV_ERR_TOKEN_OUT_OF_RANGE: return "TokenOutOfRange";
    case RV_ERR_POSITION_MISMATCH: return "PositionMismatch";
    case RV_ERR_CAPACITY_EXCEEDED: return "CapacityExceeded";
    case RV_ERR_PEER: return "Peer";
  }
  return "Unknown";
}

extern "C" size_t rv_last_error(char *buf, size_t len) {
  if (buf && len) {
    size_t k = t_err_len < len - 1 ? t_err_len : len - 1;
    memcpy(buf, t_err, k);
    buf[k] = 0;
  }
  return t_err_len;
}

extern "C" size_t rv_block_bytes(int f) { return (size_t)rv_fmt_block_bytes(f); }
extern "C" size_t rv_block_weights(int f) {
  return f == RV_Q8_0 ? 32 : (f >= RV_Q4_K && f <= RV_Q8_K ? 256 : 0);
}

extern "C" int rv_row_bytes(int f, size_t in_dim, size_t *out) {
  const size_t bw = rv_block_weights(f);
  if (bw == 0) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "unknown format %d", f);
  if (in_dim % bw != 0)
    RV_FAIL(RV_ERR_INDIVISIBLE_ROW, "format %d row of %zu weights: not a multiple of the %zu-weight block",
            f, in_dim, bw);
  if (out) *out = in_dim / bw * (size_t)rv_fmt_block_bytes(f);
  return RV_OK;
}

// Saturating multiply, as gemv.rs:207-211 validates with saturating_mul.
static size_t sat_mul(size_t a, size_t b) {
  if (a == 0 || b == 0) return 0;
  return a > SIZE_MAX / b ? SIZE_MAX : a * b;
}

// ===================================================== per-device set-up
// The SiLU exception table goes to each device once, before the first
// kernel that uses it; rv_moe_create does it, so forward calls never do.
static std::mutex g_init_mu;
static bool g_dev_ready[64];
static int g_dev_sms[64];  // multiprocessor count, read at set-up

#define RV_ROUTE_SMEM_ONE_PER_SM (120u * 1024u)
// Speculative decode: router rows per exact-chain CTA.  The expert grids
// cover T*K units (usually all there are); CTAs stride over any more.
#define RV_CHAIN_EXPERTS 16

#define RV_SMEM_PER_CTA (227u * 1024u)  // the per-CTA shared-memory limit of sm_100

static int ensure_device(int dev) {
  if (dev < 0 || dev >= 64) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_init_mu);
  if (g_dev_ready[dev]) return RV_OK;
  std::vector<uint2> table(RV_EXPF_TABLE_SIZE, make_uint2(RV_EXPF_EMPTY, 0u));
  int max_probe = 0;
  for (unsigned i = 0; i < kExpfExceptionCount; i++) {
    const uint32_t key = kExpfExceptions[i][0];
    if (key == RV_EXPF_EMPTY) continue;
    uint32_t h = rv_expf_hash(key);
    int p = 0;
    while (table[(h + p) & (RV_EXPF_TABLE_SIZE - 1)].x != RV_EXPF_EMPTY) p++;
    table[(h + p) & (RV_EXPF_TABLE_SIZE - 1)] = make_uint2(key, kExpfExceptions[i][1]);
    if (p > max_probe) max_probe = p;
  }
  int prev = -1;
  RV_CUDA(cudaGetDevice(&prev));
  RV_CUDA(cudaSetDevice(dev));
  cudaError_t e1 = cudaMemcpyToSymbol(g_expf_table, table.data(), table.size() * sizeof(uint2));
  cudaError_t e2 = cudaMemcpyToSymbol(g_expf_max_probe, &max_probe, sizeof(int));
  // Kernels whose shared memory exceeds the 48 KB default.
  const int big = 200 * 1024;
  cudaFuncSetAttribute(k_gemv<RV_Q4_K, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  cudaFuncSetAttribute(k_gemv<RV_Q4_K, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  cudaFuncSetAttribute(k_gemv<RV_Q5_K, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  cudaFuncSetAttribute(k_gemv<RV_Q5_K, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  cudaFuncSetAttribute(k_gemv<RV_Q6_K, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  cudaFuncSetAttribute(k_gemv<RV_Q6_K, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  cudaFuncSetAttribute(k_gemv_lm_head, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  cudaFuncSetAttribute(k_gemv_lm_head, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  cudaFuncSetAttribute(k_gemv_q8_0<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  cudaFuncSetAttribute(k_gemv_multi, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  cudaFuncSetAttribute(k_norm_quant, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  cudaFuncSetAttribute(k_attn_softmax_out<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  cudaFuncSetAttribute(k_attn_softmax_out<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  cudaFuncSetAttribute(k_attn_fused, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  cudaFuncSetAttribute(k_gemv_q8_0<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  g_dev_sms[dev] = 148;
  cudaDeviceGetAttribute(&g_dev_sms[dev], cudaDevAttrMultiProcessorCount, dev);
  cudaFuncSetAttribute(k_rmsnorm, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  cudaFuncSetAttribute(k_prologue, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  cudaFuncSetAttribute(k_route_decode, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  cudaFuncSetAttribute(k_route_spec<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  cudaFuncSetAttribute(k_route_spec<RV_GEO_QWEN3>, cudaFuncAttributeMaxDynamicSharedMemorySize, big);

  cudaFuncSetAttribute(k_router_logits, cudaFuncAttributeMaxDynamicSharedMemorySize, big);
  cudaError_t e3 = cudaGetLastError();
  cudaSetDevice(prev);
  if (e1 != cudaSuccess || e2 != cudaSuccess || e3 != cudaSuccess)
    RV_FAIL(RV_ERR_CUDA, "device %d set-up failed: %s", dev,
            cudaGetErrorString(e1 != cudaSuccess ? e1 : e2 != cudaSuccess ? e2 : e3));
  g_dev_ready[dev] = true;
  return RV_OK;
}

static int ensure_current_device() {
  int dev = 0;
  RV_CUDA(cudaGetDevice(&dev));
  return ensure_device(dev);
}

extern "C" int rv_device_status(int device, rv_stream stream) {
  int prev = -1;
  RV_CUDA(cudaGetDevice(&prev));
  RV_CUDA(cudaSetDevice(device));
  int v = 0, zero = 0;
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_rv_dev_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(g_rv_dev_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  cudaSetDevice(prev);
  if (e != cudaSuccess) RV_FAIL(RV_ERR_CUDA, "rv_device_status: %s", cudaGetErrorString(e));
  if (v != 0) RV_FAIL(v, "a device-side check failed on device %d", device);
  return RV_OK;
}

// One CTA waits, through the library's bounded-wait helpers, on something
// nothing will complete, and gives up after `limit` cycles.
__global__ void k_wait_probe(uint32_t what, long long limit, const uint32_t *flag) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  if (what == 0) {
    mbar_init(&bar, 1);  // one arrival expected; none comes
    mbar_wait_bounded(&bar, 0, 0, limit);
  } else {
    flag_wait_bounded(flag, 1u, limit);  // the flag stays 0
  }
}

extern "C" int rv_debug_wait_probe(int device, uint32_t what, uint64_t cycles, rv_stream stream) {
  if (what > 1) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "wait probe: unknown target %u", what);
  if (cycles == 0 || cycles > (uint64_t)RV_WAIT_CYCLES)
    RV_FAIL(RV_ERR_INVALID_ARGUMENT, "wait probe: %llu cycles (1..%lld)", (unsigned long long)cycles,
            (long long)RV_WAIT_CYCLES);
  int prev = -1;
  RV_CUDA(cudaGetDevice(&prev));
  RV_CUDA(cudaSetDevice(device));
  cudaStream_t s = (cudaStream_t)stream;
  uint32_t *flag = nullptr;
  cudaError_t e = cudaSuccess;
  if (what == 1) {
    // A flag nothing sets: 4 bytes of the library's own zeroed memory.
    e = cudaMallocAsync((void **)&flag, 4, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(flag, 0, 4, s);
  }
  if (e == cudaSuccess) {
    cudaGetLastError();  // clear any earlier error so the check below sees this launch's
    k_wait_probe<<<1, 32, 0, s>>>(what, (long long)cycles, flag);
    e = cudaGetLastError();
  }
  if (flag) {
    const cudaError_t f = cudaFreeAsync(flag, s);
    if (e == cudaSuccess) e = f;
  }
  cudaSetDevice(prev);
  if (e != cudaSuccess) RV_FAIL(RV_ERR_CUDA, "wait probe: %s", cudaGetErrorString(e));
  return RV_OK;
}

// =============================================================== kernels
extern "C" int rv_quantize_row_q8_k(const float *x, size_t n, rv_block_q8k *out, size_t out_blocks,
                                    rv_stream stream) {
  if (n != sat_mul(out_blocks, 256))
    RV_FAIL(RV_ERR_QUANTIZE_LEN_MISMATCH, "Q8_K quantize: %zu input floats do not fill %zu output blocks exactly",
            n, out_blocks);
  if (out_blocks == 0) return RV_OK;
  if (!x || !out || ((uintptr_t)x & 3) || ((uintptr_t)out & 3))
    RV_FAIL(RV_ERR_INVALID_ARGUMENT, "quantize_row_q8_k: null or misaligned pointer");
  const size_t grid = (out_blocks + 7) / 8;
  k_quantize_q8k<<<(unsigned)grid, 256, 0, (cudaStream_t)stream>>>(x, (uint8_t *)out, out_blocks);
  RV_LAUNCH_CHECK();
  return RV_OK;
}

// gemv.rs:212-264 (validate): same checks, same precedence.
static int validate_gemv(const char *what, int format, size_t weight_len, size_t in_dim,
                         size_t out_dim, size_t acts_len, size_t n_acts, size_t r0, size_t r1,
                         size_t out_len, size_t *row_bytes) {
  if (!rv_fmt_is_kquant(format))
    RV_FAIL(RV_ERR_UNSUPPORTED_FORMAT, "%s: unsupported weight format %d", what, format);
  int rc = rv_row_bytes(format, in_dim, row_bytes);
  if (rc) return rc;
  if (sat_mul(*row_bytes, out_dim) != weight_len)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "%s: weight bytes vs rows (%zu vs %zu)", what, weight_len,
            sat_mul(*row_bytes, out_dim));
  if (r0 > r1) RV_FAIL(RV_ERR_LENGTH_MISMATCH, "gemv rows: row range start vs end (%zu vs %zu)", r0, r1);
  if (r1 > out_dim)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "gemv rows: row range end vs out_dim (%zu vs %zu)", r1, out_dim);
  if (out_len != sat_mul(r1 - r0, n_acts))
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "%s: out vs range (%zu vs %zu)", what, out_len, sat_mul(r1 - r0, n_acts));
  const size_t wb = sat_mul(in_dim / 256, n_acts);
  if (wb != acts_len)
    RV_FAIL(RV_ERR_BLOCK_COUNT_MISMATCH,
            "dot length mismatch: weight row has %zu blocks, activations %zu", wb, acts_len);
  return RV_OK;
}

template <int FMT>
static void launch_gemv(const GemvArgs &g, cudaStream_t s) {
  // One activation row and 8 or 16 blocks per row: the warp-per-row tile,
  // R rows per CTA (fewer until the grid covers two waves of SMs).
  const int nbg = g.n_acts == 1 ? gemv_wide_nbg(FMT, g.nb) : 0;
  if (nbg) {
    GemvArgs w = g;
    w.R = 8;
    while (w.R > 1 && (w.nrows + w.R - 1) / w.R < 2 * 148) w.R /= 2;
    const size_t smem = gemv_tile_smem(w.R, w.row_bytes, (size_t)w.nb * 292);
    const unsigned grid = (unsigned)((w.nrows + w.R - 1) / w.R);
    if (nbg == 2) k_gemv_wide<FMT, 2><<<grid, 32 * w.R, smem, s>>>(w);
    else k_gemv_wide<FMT, 4><<<grid, 32 * w.R, smem, s>>>(w);
    return;
  }
  const size_t act_row = (size_t)g.nb * 292;
  const int mt = g.n_acts > 1 ? 8 : 1;
  const size_t smem = 16 + ((g.R * g.row_bytes + 15) & ~(size_t)15) + 16 + mt * act_row + 16;
  const unsigned grid = (unsigned)((g.nrows + g.R - 1) / g.R);
  if (mt == 1) k_gemv<FMT, 1><<<grid, g.R * 8, smem, s>>>(g);
  else k_gemv<FMT, 8><<<grid, g.R * 8, smem, s>>>(g);
}

static int gemv_launch(int format, const uint8_t *weight, size_t row_bytes, size_t in_dim,
                       const rv_block_q8k *acts, size_t n_acts, size_t r0, size_t r1, float *out,
                       cudaStream_t s) {
  if (n_acts == 0 || r1 == r0) return RV_OK;
  if (!weight || !acts || !out || ((uintptr_t)acts & 3))
    RV_FAIL(RV_ERR_INVALID_ARGUMENT, "gemv: null pointer or activations not 4-byte aligned");
  int rc = ensure_current_device();
  if (rc) return rc;
  GemvArgs g{};
  g.w = weight;
  g.row_bytes = row_bytes;
  g.nb = (int)(in_dim / 256);
  g.r0 = r0;
  g.nrows = r1 - r0;
  g.acts = (const uint8_t *)acts;
  g.n_acts = n_acts;
  g.out = out;
  g.R = row_bytes <= 2048 ? 32 : row_bytes <= 4096 ? 16 : 8;
  // Small matrices (the attention projections: 512-4096 rows): fewer rows
  // per CTA until the grid covers two waves of SMs.
  while (g.R > 4 && (g.nrows + g.R - 1) / g.R < 2 * 148) g.R /= 2;
  const size_t act_row = (size_t)g.nb * 292;
  if ((size_t)g.R * row_bytes + 8 * act_row > 180 * 1024)
    RV_FAIL(RV_ERR_UNIMPLEMENTED, "gemv: rows of %zu bytes exceed the staged-tile limit", row_bytes);
  // lm_head shape (Q6_K, 8 blocks per row, one activation row, more tiles
  // than two waves): the streaming kernel.  Its bulk copies need a
  // 16-byte-aligned first row (rows are 1,680 = 105 x 16 bytes).
  int dev = 0;
  RV_CUDA(cudaGetDevice(&dev));
  const int sms = g_dev_sms[dev] > 0 ? g_dev_sms[dev] : 148;
  const size_t lmh_tiles = (g.nrows + RV_LMH_ROWS - 1) / RV_LMH_ROWS;
  if (format == RV_Q6_K && g.nb == 8 && n_acts == 1 && ((uintptr_t)(weight + r0 * row_bytes) & 15) == 0 &&
      lmh_tiles > (size_t)2 * sms) {
    const size_t smem = 64 + (size_t)RV_LMH_STAGES * RV_LMH_ROWS * row_bytes;
    k_gemv_lm_head<<<(unsigned)std::min(lmh_tiles, (size_t)2 * sms), RV_LMH_ROWS * 8, smem, s>>>(g);
    RV_LAUNCH_CHECK();
    return RV_OK;
  }
  switch (format) {
    case RV_Q4_K: launch_gemv<RV_Q4_K>(g, s); break;
    case RV_Q5_K: launch_gemv<RV_Q5_K>(g, s); break;
    default: launch_gemv<RV_Q6_K>(g, s); break;
  }
  RV_LAUNCH_CHECK();
  return RV_OK;
}

extern "C" int rv_gemv_q8_k(int format, const uint8_t *weight, size_t weight_len, size_t in_dim,
                            size_t out_dim, const rv_block_q8k *acts, size_t acts_len, float *out,
                            size_t out_len, rv_stream stream) {
  size_t rb = 0;
  int rc = validate_gemv("gemv_q8_k", format, weight_len, in_dim, out_dim, acts_len, 1, 0, out_dim,
                         out_len, &rb);
  if (rc) return rc;
  return gemv_launch(format, weight, rb, in_dim, acts, 1, 0, out_dim, out, (cudaStream_t)stream);
}

extern "C" int rv_gemv_q8_k_rows(int format, const uint8_t *weight, size_t weight_len, size_t in_dim,
                                 size_t out_dim, const rv_block_q8k *acts, size_t acts_len,
                                 size_t row_start, size_t row_end, float *out, size_t out_len,
                                 rv_stream stream) {
  size_t rb = 0;
  int rc = validate_gemv("gemv_q8_k_rows", format, weight_len, in_dim, out_dim, acts_len, 1,
                         row_start, row_end, out_len, &rb);
  if (rc) return rc;
  return gemv_launch(format, weight, rb, in_dim, acts, 1, row_start, row_end, out, (cudaStream_t)stream);
}

extern "C" int rv_gemv_q8_k_batched(int format, const uint8_t *weight, size_t weight_len,
                                    size_t in_dim, size_t out_dim, const rv_block_q8k *acts,
                                    size_t acts_len, size_t n_acts, size_t row_start,
                                    size_t row_end, float *out, size_t out_len, rv_stream stream) {
  size_t rb = 0;
  int rc = validate_gemv("gemv_q8_k_batched", format, weight_len, in_dim, out_dim, acts_len, n_acts,
                         row_start, row_end, out_len, &rb);
  if (rc) return rc;
  return gemv_launch(format, weight, rb, in_dim, acts, n_acts, row_start, row_end, out,
                     (cudaStream_t)stream);
}

// ------------------------------------------------------------------ Q8_0
extern "C" int rv_quantize_row_q8_0(const float *x, size_t n, rv_block_q8_0 *out, size_t out_blocks,
                                    rv_stream stream) {
  if (n != sat_mul(out_blocks, 32))
    RV_FAIL(RV_ERR_QUANTIZE_LEN_MISMATCH, "Q8_0 quantize: %zu input floats do not fill %zu output blocks exactly",
            n, out_blocks);
  if (out_blocks == 0) return RV_OK;
  if (!x || !out || ((uintptr_t)x & 3) || ((uintptr_t)out & 3))
    RV_FAIL(RV_ERR_INVALID_ARGUMENT, "quantize_row_q8_0: null or misaligned pointer");
  const size_t grid = (out_blocks + 7) / 8;
  k_quantize_q8_0<<<(unsigned)grid, 256, 0, (cudaStream_t)stream>>>(x, (uint8_t *)out, out_blocks);
  RV_LAUNCH_CHECK();
  return RV_OK;
}

// gemv.rs:212-264 (validate) for Format::Q8_0, same checks and precedence.
static int validate_gemv_q8_0(const char *what, size_t weight_len, size_t in_dim, size_t out_dim,
                              size_t acts_len, size_t n_acts, size_t r0, size_t r1, size_t out_len,
                              size_t *row_bytes) {
  int rc = rv_row_bytes(RV_Q8_0, in_dim, row_bytes);
  if (rc) return rc;
  if (sat_mul(*row_bytes, out_dim) != weight_len)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "%s: weight bytes vs rows (%zu vs %zu)", what, weight_len,
            sat_mul(*row_bytes, out_dim));
  if (r0 > r1) RV_FAIL(RV_ERR_LENGTH_MISMATCH, "gemv rows: row range start vs end (%zu vs %zu)", r0, r1);
  if (r1 > out_dim)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "gemv rows: row range end vs out_dim (%zu vs %zu)", r1, out_dim);
  if (out_len != sat_mul(r1 - r0, n_acts))
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "%s: out vs range (%zu vs %zu)", what, out_len, sat_mul(r1 - r0, n_acts));
  const size_t wb = sat_mul(in_dim / 32, n_acts);
  if (wb != acts_len)
    RV_FAIL(RV_ERR_BLOCK_COUNT_MISMATCH, "dot length mismatch: weight row has %zu blocks, activations %zu", wb,
            acts_len);
  return RV_OK;
}

static int gemv_q8_0_launch(const uint8_t *weight, size_t row_bytes, size_t in_dim, const rv_block_q8_0 *acts,
                            size_t n_acts, size_t r0, size_t r1, float *out, cudaStream_t s) {
  if (n_acts == 0 || r1 == r0) return RV_OK;
  if (!weight || !acts || !out || ((uintptr_t)weight & 1) || ((uintptr_t)acts & 3))
    RV_FAIL(RV_ERR_INVALID_ARGUMENT, "gemv_q8_0: null pointer, weight not 2-byte or activations not 4-byte aligned");
  int rc = ensure_current_device();
  if (rc) return rc;
  GemvArgs g{};
  g.w = weight;
  g.row_bytes = row_bytes;
  g.nb = (int)(in_dim / 32);
  g.r0 = r0;
  g.nrows = r1 - r0;
  g.acts = (const uint8_t *)acts;
  g.n_acts = n_acts;
  g.out = out;
  // Rows per CTA: as many as fit, but at least two CTAs per SM while the
  // matrix allows it (the attention matrices have only 512-4096 rows).
  int R = row_bytes <= 2048 ? 32 : row_bytes <= 4096 ? 16 : 8;
  while (R > 4 && (g.nrows + R - 1) / R < 2 * 148) R /= 2;
  g.R = R;
  const size_t act_row = (size_t)g.nb * 36;
  const int mt = n_acts > 1 ? 8 : 1;
  const size_t smem = 16 + ((R * row_bytes + 15) & ~(size_t)15) + 16 + mt * act_row + 16;
  if (smem > 200 * 1024)
    RV_FAIL(RV_ERR_UNIMPLEMENTED, "gemv_q8_0: rows of %zu bytes exceed the staged-tile limit", row_bytes);
  if (mt == 1 && gemv_wide_nbg(RV_Q8_0, g.nb)) {  // one activation row, 64 blocks: the warp-per-row tile
    g.R = 8;
    while (g.R > 1 && (g.nrows + g.R - 1) / g.R < 2 * 148) g.R /= 2;
    k_gemv_q8_0_wide<16><<<(unsigned)((g.nrows + g.R - 1) / g.R), 32 * g.R,
                           gemv_tile_smem(g.R, row_bytes, act_row), s>>>(g);
    RV_LAUNCH_CHECK();
    return RV_OK;
  }
  const unsigned grid = (unsigned)((g.nrows + R - 1) / R);
  if (mt == 1) k_gemv_q8_0<1><<<grid, R * 8, smem, s>>>(g);
  else k_gemv_q8_0<8><<<grid, R * 8, smem, s>>>(g);
  RV_LAUNCH_CHECK();
  return RV_OK;
}

extern "C" int rv_gemv_q8_0(const uint8_t *weight, size_t weight_len, size_t in_dim, size_t out_dim,
                            const rv_block_q8_0 *acts, size_t acts_len, float *out, size_t out_len,
                            rv_stream stream) {
  size_t rb = 0;
  int rc = validate_gemv_q8_0("gemv_q8_0", weight_len, in_dim, out_dim, acts_len, 1, 0, out_dim, out_len, &rb);
  if (rc) return rc;
  return gemv_q8_0_launch(weight, rb, in_dim, acts, 1, 0, out_dim, out, (cudaStream_t)stream);
}

extern "C" int rv_gemv_q8_0_rows(const uint8_t *weight, size_t weight_len, size_t in_dim, size_t out_dim,
                                 const rv_block_q8_0 *acts, size_t acts_len, size_t row_start, size_t row_end,
                                 float *out, size_t out_len, rv_stream stream) {
  size_t rb = 0;
  int rc = validate_gemv_q8_0("gemv_q8_0_rows", weight_len, in_dim, out_dim, acts_len, 1, row_start, row_end,
                              out_len, &rb);
  if (rc) return rc;
  return gemv_q8_0_launch(weight, rb, in_dim, acts, 1, row_start, row_end, out, (cudaStream_t)stream);
}

extern "C" int rv_gemv_q8_0_batched(const uint8_t *weight, size_t weight_len, size_t in_dim, size_t out_dim,
                                    const rv_block_q8_0 *acts, size_t acts_len, size_t n_acts, size_t row_start,
                                    size_t row_end, float *out, size_t out_len, rv_stream stream) {
  size_t rb = 0;
  int rc = validate_gemv_q8_0("gemv_q8_0_batched", weight_len, in_dim, out_dim, acts_len, n_acts, row_start,
                              row_end, out_len, &rb);
  if (rc) return rc;
  return gemv_q8_0_launch(weight, rb, in_dim, acts, n_acts, row_start, row_end, out, (cudaStream_t)stream);
}

// ------------------------------------------------------- dequantization
extern "C" int rv_dequantize_rows(int format, const uint8_t *weight, size_t weight_len, size_t in_dim,
                                  size_t out_dim, const uint32_t *rows, size_t n_rows, float *out, size_t out_len,
                                  rv_stream stream) {
  if (format != RV_Q4_K && format != RV_Q5_K && format != RV_Q6_K && format != RV_Q8_0)
    RV_FAIL(RV_ERR_UNSUPPORTED_FORMAT, "dequantize_rows: unsupported weight format %d", format);
  size_t rb = 0;
  int rc = rv_row_bytes(format, in_dim, &rb);
  if (rc) return rc;
  if (sat_mul(rb, out_dim) != weight_len)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "dequantize_rows: weight bytes vs rows (%zu vs %zu)", weight_len,
            sat_mul(rb, out_dim));
  if (out_len != sat_mul(n_rows, in_dim))
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "dequantize_rows: out vs rows x in_dim (%zu vs %zu)", out_len,
            sat_mul(n_rows, in_dim));
  if (!rows && n_rows > out_dim)
    RV_FAIL(RV_ERR_TOKEN_OUT_OF_RANGE, "dequantize_rows: %zu rows of a %zu-row matrix", n_rows, out_dim);
  if (out_len == 0) return RV_OK;
  if (!weight || !out || ((uintptr_t)out & 3) || ((uintptr_t)rows & 3))
    RV_FAIL(RV_ERR_INVALID_ARGUMENT, "dequantize_rows: null or misaligned pointer");
  rc = ensure_current_device();
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  const unsigned grid = (unsigned)((out_len + 255) / 256);
  switch (format) {
    case RV_Q4_K: k_dequant_rows<RV_Q4_K><<<grid, 256, 0, s>>>(weight, rb, in_dim, out_dim, rows, n_rows, out); break;
    case RV_Q5_K: k_dequant_rows<RV_Q5_K><<<grid, 256, 0, s>>>(weight, rb, in_dim, out_dim, rows, n_rows, out); break;
    case RV_Q6_K: k_dequant_rows<RV_Q6_K><<<grid, 256, 0, s>>>(weight, rb, in_dim, out_dim, rows, n_rows, out); break;
    default: k_dequant_rows<RV_Q8_0><<<grid, 256, 0, s>>>(weight, rb, in_dim, out_dim, rows, n_rows, out); break;
  }
  RV_LAUNCH_CHECK();
  return RV_OK;
}

// gemv.rs:747-823: rows of the concatenated row spaces, part by part.
extern "C" int rv_gemv_q8_k_fused_rows(const rv_fused_part *parts, size_t n_parts, size_t row_start,
                                       size_t row_end, float *out, size_t out_len,
                                       rv_stream stream) {
  if (n_parts && !parts) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "fused_rows: null parts");
  size_t total = 0;
  for (size_t p = 0; p < n_parts; p++) total = total > SIZE_MAX - parts[p].out_dim ? SIZE_MAX : total + parts[p].out_dim;
  if (row_start > row_end)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "gemv rows: row range start vs end (%zu vs %zu)", row_start, row_end);
  if (row_end > total)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "gemv rows: row range end vs out_dim (%zu vs %zu)", row_end, total);
  if (out_len != row_end - row_start)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "gemv_q8_k_fused_rows: out vs range (%zu vs %zu)", out_len,
            row_end - row_start);
  // Validate every touched part first, then launch (fused_row_parts, gemv.rs:713-728).
  struct Job { size_t p, lo, hi, rb, at; };
  std::vector<Job> jobs;
  size_t base = 0, at = 0;
  for (size_t p = 0; p < n_parts; p++) {
    const size_t end = base > SIZE_MAX - parts[p].out_dim ? SIZE_MAX : base + parts[p].out_dim;
    const size_t lo = row_start < base ? base : (row_start > end ? end : row_start);
    const size_t hi = row_end < base ? base : (row_end > end ? end : row_end);
    if (lo < hi) {
      size_t rb = 0;
      int rc = validate_gemv("gemv_q8_k_fused_rows: part weight bytes vs rows / out vs range",
                             parts[p].format, parts[p].weight_len, parts[p].in_dim, parts[p].out_dim,
                             parts[p].acts_len, 1, lo - base, hi - base, hi - lo, &rb);
      if (rc) return rc;
      jobs.push_back({p, lo - base, hi - base, rb, at});
      at += hi - lo;
    }
    base = end;
  }
  for (const Job &j : jobs) {
    int rc = gemv_launch(parts[j.p].format, parts[j.p].weight, j.rb, parts[j.p].in_dim, parts[j.p].acts,
                         1, j.lo, j.hi, out + j.at, (cudaStream_t)stream);
    if (rc) return rc;
  }
  return RV_OK;
}

extern "C" int rv_rmsnorm(const float *x, const float *weight, size_t n, size_t n_rows, float eps,
                          float *out, rv_stream stream) {
  if (n == 0) RV_FAIL(RV_ERR_EMPTY, "rmsnorm: input is empty");
  if (n > 16384) RV_FAIL(RV_ERR_UNIMPLEMENTED, "rmsnorm rows longer than 16384 are not implemented");
  if (n_rows == 0) return RV_OK;
  if (!x || !weight || !out) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "rmsnorm: null pointer");
  int rc = ensure_current_device();
  if (rc) return rc;
  k_rmsnorm<<<(unsigned)n_rows, 256, 34 * sizeof(double) + n * sizeof(float), (cudaStream_t)stream>>>(
      x, weight, n, eps, out);
  RV_LAUNCH_CHECK();
  return RV_OK;
}

extern "C" int rv_softmax(float *x, size_t n, size_t n_rows, rv_stream stream) {
  if (n == 0) RV_FAIL(RV_ERR_EMPTY, "softmax: input is empty");
  if (n > 1024) RV_FAIL(RV_ERR_UNIMPLEMENTED, "softmax rows longer than 1024 are not implemented");
  if (n_rows == 0) return RV_OK;
  if (!x) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "softmax: null pointer");
  const unsigned grid = (unsigned)((n_rows + 3) / 4);
  k_softmax<<<grid, 128, 4 * n * sizeof(double), (cudaStream_t)stream>>>(x, n, n_rows);
  RV_LAUNCH_CHECK();
  return RV_OK;
}

extern "C" int rv_swiglu_combine(float *gate, size_t gate_len, const float *up, size_t up_len,
                                 rv_stream stream) {
  if (gate_len != up_len)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "swiglu_combine: gate vs up (%zu vs %zu)", gate_len, up_len);
  if (gate_len == 0) return RV_OK;
  if (!gate || !up) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "swiglu_combine: null pointer");
  int rc = ensure_current_device();
  if (rc) return rc;
  k_swiglu<<<(unsigned)((gate_len + 255) / 256), 256, 0, (cudaStream_t)stream>>>(gate, up, gate_len);
  RV_LAUNCH_CHECK();
  return RV_OK;
}

extern "C" int rv_debug_block_sums(int format, const uint8_t *w, size_t w_len, const rv_block_q8k *acts,
                                   size_t n_blocks, int32_t *lanes_out, int32_t *mins_out,
                                   rv_stream stream) {
  if (!rv_fmt_is_kquant(format)) RV_FAIL(RV_ERR_UNSUPPORTED_FORMAT, "debug_block_sums: format %d", format);
  const size_t bb = (size_t)rv_fmt_block_bytes(format);
  if (w_len % bb) RV_FAIL(RV_ERR_ROW_BYTES_NOT_BLOCK_MULTIPLE, "row of %zu bytes", w_len);
  if (w_len / bb != n_blocks)
    RV_FAIL(RV_ERR_BLOCK_COUNT_MISMATCH, "weight row has %zu blocks, activations %zu", w_len / bb, n_blocks);
  if (n_blocks == 0) return RV_OK;
  if (!w || !acts || !lanes_out || !mins_out || ((uintptr_t)acts & 3))
    RV_FAIL(RV_ERR_INVALID_ARGUMENT, "debug_block_sums: bad pointer");
  cudaStream_t s = (cudaStream_t)stream;
  const unsigned g = (unsigned)n_blocks;
  const uint8_t *a = (const uint8_t *)acts;
  if (format == RV_Q4_K) k_block_sums<RV_Q4_K><<<g, 32, 256 + 304, s>>>(w, a, (int)n_blocks, lanes_out, mins_out);
  else if (format == RV_Q5_K) k_block_sums<RV_Q5_K><<<g, 32, 256 + 304, s>>>(w, a, (int)n_blocks, lanes_out, mins_out);
  else k_block_sums<RV_Q6_K><<<g, 32, 256 + 304, s>>>(w, a, (int)n_blocks, lanes_out, mins_out);
  RV_LAUNCH_CHECK();
  return RV_OK;
}

// ========================================================== expert table
struct rv_expert_table {
  int device;
  std::vector<rv_layer_layout> layouts;
  std::vector<uint8_t *> base;  // device, one allocation per layer
  bool step_active = false;
  uint32_t step_layer = 0;
  std::vector<uint32_t> hit_index, hit_slot;
  uint64_t accesses = 0, hits = 0;
};

static int check_layout(const rv_layer_layout &L, uint32_t i) {
  const rv_layer_layout *p = &L;
  if (!rv_fmt_is_kquant(p->gate_format) || !rv_fmt_is_kquant(p->up_format) || !rv_fmt_is_kquant(p->down_format))
    RV_FAIL(RV_ERR_UNSUPPORTED_FORMAT, "layer %u: expert slabs must be Q4_K/Q5_K/Q6_K", i);
  size_t rg, ru, rd;
  int rc = rv_row_bytes(p->gate_format, p->hidden, &rg);
  if (!rc) rc = rv_row_bytes(p->up_format, p->hidden, &ru);
  if (!rc) rc = rv_row_bytes(p->down_format, p->moe, &rd);
  if (rc) return rc;
  if (p->gate_len != (uint64_t)rg * p->moe || p->up_len != (uint64_t)ru * p->moe ||
      p->down_len != (uint64_t)rd * p->hidden)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "layer %u: slab lengths do not match [moe][hidden] / [hidden][moe]", i);
  if (p->gate_off + p->gate_len > p->stride || p->up_off + p->up_len > p->stride ||
      p->down_off + p->down_len > p->stride)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "layer %u: a slab runs past the blob stride", i);
  if (p->n_experts == 0) RV_FAIL(RV_ERR_EMPTY, "layer %u: no experts", i);
  return RV_OK;
}

extern "C" int rv_expert_table_create(int device, const rv_layer_layout *layers, uint32_t n_layers,
                                      rv_expert_table **out) {
  if (!out || (n_layers && !layers)) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "expert_table_create: null pointer");
  *out = nullptr;
  for (uint32_t i = 0; i < n_layers; i++) {
    int rc = check_layout(layers[i], i);
    if (rc) return rc;
  }
  int rc = ensure_device(device);
  if (rc) return rc;
  rv_expert_table *t = new (std::nothrow) rv_expert_table();
  if (!t) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "out of host memory");
  t->device = device;
  t->layouts.assign(layers, layers + n_layers);
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  for (uint32_t i = 0; i < n_layers; i++) {
    uint8_t *p = nullptr;
    cudaError_t e = cudaMalloc(&p, (size_t)layers[i].n_experts * layers[i].stride);
    if (e != cudaSuccess) {
      for (uint8_t *q : t->base) cudaFree(q);
      delete t;
      cudaSetDevice(prev);
      RV_FAIL(RV_ERR_CUDA, "expert table layer %u (%zu bytes): %s", i,
              (size_t)layers[i].n_experts * layers[i].stride, cudaGetErrorString(e));
    }
    t->base.push_back(p);
  }
  cudaSetDevice(prev);
  *out = t;
  return RV_OK;
}

extern "C" void rv_expert_table_destroy(rv_expert_table *t) {
  if (!t) return;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(t->device);
  for (uint8_t *p : t->base) cudaFree(p);
  cudaSetDevice(prev);
  cudaGetLastError();  // a void call: leave no error behind for the caller's next check
  delete t;
}

extern "C" uint32_t rv_expert_table_n_layers(const rv_expert_table *t) {
  return t ? (uint32_t)t->layouts.size() : 0;
}

extern "C" int rv_expert_table_layout(const rv_expert_table *t, uint32_t layer, rv_layer_layout *out) {
  if (!t || !out) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "null pointer");
  if (layer >= t->layouts.size()) RV_FAIL(RV_ERR_LAYER_OUT_OF_RANGE, "layer %u of %zu", layer, t->layouts.size());
  *out = t->layouts[layer];
  return RV_OK;
}

extern "C" int rv_expert_table_upload(rv_expert_table *t, uint32_t layer, uint32_t expert_first,
                                      uint32_t n_experts, const void *src, size_t len,
                                      int src_on_device, rv_stream stream) {
  if (!t || (!src && len)) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "null pointer");
  if (layer >= t->layouts.size()) RV_FAIL(RV_ERR_LAYER_OUT_OF_RANGE, "layer %u of %zu", layer, t->layouts.size());
  const rv_layer_layout &L = t->layouts[layer];
  if ((uint64_t)expert_first + n_experts > L.n_experts)
    RV_FAIL(RV_ERR_ROUTED_OUT_OF_RANGE, "experts [%u, %u) of %u", expert_first, expert_first + n_experts, L.n_experts);
  if (len != (size_t)n_experts * L.stride)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "upload: %zu bytes vs %zu expected", len, (size_t)n_experts * L.stride);
  if (len == 0) return RV_OK;
  cudaStream_t s = (cudaStream_t)stream;
  RV_CUDA(cudaMemcpyAsync(t->base[layer] + (size_t)expert_first * L.stride, src, len,
                          src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s));
  RV_CUDA(cudaStreamSynchronize(s));
  return RV_OK;
}

// One layer's expert file (`experts/layer_XX.bin` of an install: n_experts
// blobs of `stride` bytes from file_offset on; format/layout.rs:1-13) into
// the table.  The file is read in 8 MiB chunks into two pinned staging
// buffers, each chunk copied to the device while the next is read.
extern "C" int rv_expert_table_load_file(rv_expert_table *t, uint32_t layer, const char *path,
                                         uint64_t file_offset, rv_stream stream) {
  if (!t || !path) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "load_file: null pointer");
  if (layer >= t->layouts.size()) RV_FAIL(RV_ERR_LAYER_OUT_OF_RANGE, "layer %u of %zu", layer, t->layouts.size());
  const rv_layer_layout &L = t->layouts[layer];
  const uint64_t total = (uint64_t)L.n_experts * L.stride;
  FILE *f = fopen(path, "rb");
  if (!f) RV_FAIL(RV_ERR_IO, "layer %u: cannot open %s: %s", layer, path, strerror(errno));
  struct Closer {
    FILE *f;
    ~Closer() { fclose(f); }
  } closer{f};
  if (fseeko(f, 0, SEEK_END) != 0) RV_FAIL(RV_ERR_IO, "layer %u: cannot seek %s", layer, path);
  const uint64_t size = (uint64_t)ftello(f);
  if (size < file_offset || size - file_offset < total)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "layer %u: %s holds %llu bytes from offset %llu, the layer needs %llu", layer,
            path, (unsigned long long)(size - std::min(size, file_offset)), (unsigned long long)file_offset,
            (unsigned long long)total);
  if (fseeko(f, (off_t)file_offset, SEEK_SET) != 0) RV_FAIL(RV_ERR_IO, "layer %u: cannot seek %s", layer, path);
  int prev = -1;
  RV_CUDA(cudaGetDevice(&prev));
  RV_CUDA(cudaSetDevice(t->device));
  const size_t chunk = 8u << 20;
  void *stage[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  cudaStream_t s = (cudaStream_t)stream;
  int rc = RV_OK;
  cudaError_t e = cudaSuccess;
  for (int i = 0; i < 2 && e == cudaSuccess; i++) {
    e = cudaHostAlloc(&stage[i], chunk, cudaHostAllocDefault);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming);
  }
  if (e != cudaSuccess) {
    rv_set_error(RV_ERR_CUDA, "load_file: staging buffers: %s", cudaGetErrorString(e));
    rc = RV_ERR_CUDA;
  }
  for (uint64_t off = 0, k = 0; rc == RV_OK && off < total; off += chunk, k++) {
    const int b = (int)(k & 1);
    const size_t n = (size_t)std::min<uint64_t>(chunk, total - off);
    if (k >= 2 && (e = cudaEventSynchronize(done[b])) != cudaSuccess) {  // the copy that used this buffer
      rv_set_error(RV_ERR_CUDA, "load_file: %s", cudaGetErrorString(e));
      rc = RV_ERR_CUDA;
      break;
    }
    if (fread(stage[b], 1, n, f) != n) {
      rv_set_error(RV_ERR_IO, "layer %u: short read of %s at byte %llu", layer, path,
                   (unsigned long long)(file_offset + off));
      rc = RV_ERR_IO;
      break;
    }
    if ((e = cudaMemcpyAsync(t->base[layer] + off, stage[b], n, cudaMemcpyHostToDevice, s)) != cudaSuccess ||
        (e = cudaEventRecord(done[b], s)) != cudaSuccess) {
      rv_set_error(RV_ERR_CUDA, "load_file: %s", cudaGetErrorString(e));
      rc = RV_ERR_CUDA;
    }
  }
  const cudaError_t es = cudaStreamSynchronize(s);
  if (rc == RV_OK && es != cudaSuccess) {
    rv_set_error(RV_ERR_CUDA, "load_file: %s", cudaGetErrorString(es));
    rc = RV_ERR_CUDA;
  }
  for (int i = 0; i < 2; i++) {
    if (done[i]) cudaEventDestroy(done[i]);
    if (stage[i]) cudaFreeHost(stage[i]);
  }
  cudaSetDevice(prev);
  return rc;
}

extern "C" int rv_expert_table_begin_layer(rv_expert_table *t, uint32_t layer, const uint32_t *experts,
                                           size_t n) {
  if (!t || (n && !experts)) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "null pointer");
  if (layer >= t->layouts.size()) RV_FAIL(RV_ERR_LAYER_OUT_OF_RANGE, "layer %u of %zu", layer, t->layouts.size());
  if (t->step_active)
    RV_FAIL(RV_ERR_PROTOCOL, "layer %u: begin_layer called with a step already open; end_layer first", layer);
  for (size_t i = 0; i < n; i++)
    if (experts[i] >= t->layouts[layer].n_experts)
      RV_FAIL(RV_ERR_ROUTED_OUT_OF_RANGE, "expert %u of %u", experts[i], t->layouts[layer].n_experts);
  t->hit_index.clear();
  t->hit_slot.clear();
  for (size_t i = 0; i < n; i++) {
    bool dup = false;
    for (size_t j = 0; j < i; j++) dup |= experts[j] == experts[i];
    if (dup) continue;  // a duplicate resolves once, at its first position
    t->hit_index.push_back((uint32_t)i);
    t->hit_slot.push_back(experts[i]);
  }
  t->accesses += t->hit_slot.size();
  t->hits += t->hit_slot.size();
  t->step_active = true;
  t->step_layer = layer;
  return RV_OK;
}

extern "C" int rv_expert_table_hits(const rv_expert_table *t, uint32_t *index_out, uint32_t *slot_out,
                                    size_t cap, size_t *n_out) {
  if (!t || !n_out) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "null pointer");
  const size_t n = t->step_active ? t->hit_slot.size() : 0;
  *n_out = n;
  for (size_t i = 0; i < n && i < cap; i++) {
    if (index_out) index_out[i] = t->hit_index[i];
    if (slot_out) slot_out[i] = t->hit_slot[i];
  }
  return RV_OK;
}

extern "C" int rv_expert_table_misses(const rv_expert_table *t, uint32_t *index_out, uint32_t *slot_out,
                                      size_t cap, size_t *n_out) {
  (void)index_out;
  (void)slot_out;
  (void)cap;
  if (!t || !n_out) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "null pointer");
  *n_out = 0;
  return RV_OK;
}

extern "C" int rv_expert_table_await_misses(rv_expert_table *t) {
  if (!t) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "null pointer");
  return RV_OK;
}

extern "C" int rv_expert_table_view(const rv_expert_table *t, uint32_t layer, uint32_t slot,
                                    rv_expert_view *out) {
  if (!t || !out) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "null pointer");
  if (layer >= t->layouts.size()) RV_FAIL(RV_ERR_LAYER_OUT_OF_RANGE, "layer %u of %zu", layer, t->layouts.size());
  const rv_layer_layout &L = t->layouts[layer];
  if (slot >= L.n_experts) RV_FAIL(RV_ERR_PROTOCOL, "layer %u: slot %u is not in the pool", layer, slot);
  const uint8_t *b = t->base[layer] + (size_t)slot * L.stride;
  out->blob = b;
  out->gate = b + L.gate_off;
  out->up = b + L.up_off;
  out->down = b + L.down_off;
  out->gate_len = L.gate_len;
  out->up_len = L.up_len;
  out->down_len = L.down_len;
  out->gate_format = L.gate_format;
  out->up_format = L.up_format;
  out->down_format = L.down_format;
  return RV_OK;
}

extern "C" int rv_expert_table_end_layer(rv_expert_table *t, uint32_t layer) {
  if (!t) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "null pointer");
  if (!t->step_active) RV_FAIL(RV_ERR_PROTOCOL, "layer %u: end_layer without an open step", layer);
  t->step_active = false;
  t->hit_index.clear();
  t->hit_slot.clear();
  return RV_OK;
}

extern "C" int rv_expert_table_stats(const rv_expert_table *t, uint64_t *accesses, uint64_t *hits) {
  if (!t) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "null pointer");
  if (accesses) *accesses = t->accesses;
  if (hits) *hits = t->hits;
  return RV_OK;
}

// ============================================================ MoE engine
struct rv_moe {
  int device;
  rv_moe_config cfg;
  size_t max_tokens;
  MoeDims d;
  MoeBufs B;  // T and residual/ffn_norm/router set per call
  int max_units;
  void *arena;
  float *dres;  // [max_tokens][H] device residual of rv_moe_forward_host
  int last_T = 0;
  bool spec = true;   // speculative expert dispatch for decode (RV_DECODE_SPEC=0 turns it off)
  std::vector<cudaEvent_t> prof;  // 5 events per set
  size_t prof_next = 0;
};

static void prof_release(rv_moe *m) {
  for (cudaEvent_t e : m->prof) cudaEventDestroy(e);
  m->prof.clear();
  m->prof_next = 0;
}

extern "C" int rv_moe_profile_enable(rv_moe *m, size_t slots) {
  if (!m) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "null engine");
  int prev = -1;
  RV_CUDA(cudaGetDevice(&prev));
  RV_CUDA(cudaSetDevice(m->device));
  prof_release(m);
  for (size_t i = 0; i < 5 * slots; i++) {
    cudaEvent_t e;
    cudaError_t err = cudaEventCreate(&e);
    if (err != cudaSuccess) {
      prof_release(m);
      cudaSetDevice(prev);
      RV_FAIL(RV_ERR_CUDA, "profile events: %s", cudaGetErrorString(err));
    }
    m->prof.push_back(e);
  }
  cudaSetDevice(prev);
  return RV_OK;
}

extern "C" int rv_moe_profile_rewind(rv_moe *m) {
  if (!m) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "null engine");
  m->prof_next = 0;
  return RV_OK;
}

extern "C" int rv_moe_profile_read(rv_moe *m, float *ms_out, size_t cap, size_t *n_sets) {
  if (!m || !n_sets) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "null pointer");
  const size_t used = m->prof_next;
  *n_sets = used;
  for (size_t i = 0; i < used; i++) {
    cudaEvent_t *ev = &m->prof[5 * i];
    RV_CUDA(cudaEventSynchronize(ev[4]));
    for (int k = 0; k < 4; k++) {
      float ms = 0.0f;
      RV_CUDA(cudaEventElapsedTime(&ms, ev[k], ev[k + 1]));
      if (ms_out && 4 * i + k < cap) ms_out[4 * i + k] = ms;
    }
  }
  return RV_OK;
}

static size_t round16(size_t x) { return (x + 15) & ~(size_t)15; }

// Bytes of the tensor path's dequantized-stage cache: room for every expert's
// largest matrix (gate|up, or down in any format), for engines of at least
// 1024 tokens (where experts often hold several 128-position tiles); 0
// otherwise.
static size_t tc_cache_bytes(const MoeDims &d, size_t max_tokens) {
  if (max_tokens < 1024 || d.H % RV_TC_ROWS || d.M % RV_TC_ROWS) return 0;
  const size_t gu = tc_predeq_bytes<RV_Q4_K, false>(2 * d.M, d.H);
  const size_t dn = std::max(tc_predeq_bytes<RV_Q6_K, true>(d.H, d.M), tc_predeq_bytes<RV_Q4_K, true>(d.H, d.M));
  return (size_t)d.E * std::max(gu, dn);
}

extern "C" int rv_moe_create(int device, const rv_moe_config *cfg, size_t max_tokens, rv_moe **out) {
  if (!cfg || !out) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "moe_create: null pointer");
  *out = nullptr;
  if (cfg->hidden == 0 || cfg->hidden % 256)
    RV_FAIL(RV_ERR_INDIVISIBLE_ROW, "hidden %u: not a multiple of the 256-weight block", cfg->hidden);
  if (cfg->moe == 0 || cfg->moe % 256)
    RV_FAIL(RV_ERR_INDIVISIBLE_ROW, "moe_intermediate %u: not a multiple of the 256-weight block", cfg->moe);
  if (cfg->hidden > 4096 || cfg->moe > 4096)
    RV_FAIL(RV_ERR_UNIMPLEMENTED, "hidden/moe above 4096 are not implemented on the GPU path");
  if (cfg->n_experts == 0 || cfg->n_experts > 256)
    RV_FAIL(RV_ERR_UNIMPLEMENTED, "n_experts %u: the GPU path handles 1..256", cfg->n_experts);
  if (cfg->top_k == 0 || cfg->top_k > 16 || cfg->top_k > cfg->n_experts)
    RV_FAIL(RV_ERR_UNIMPLEMENTED, "top_k %u: the GPU path handles 1..min(16, n_experts)", cfg->top_k);
  if (max_tokens == 0 || max_tokens > (1u << 20) / cfg->top_k)
    RV_FAIL(RV_ERR_INVALID_ARGUMENT, "max_tokens %zu out of range", max_tokens);
  int rc = ensure_device(device);
  if (rc) return rc;
  rv_moe *m = new (std::nothrow) rv_moe();
  if (!m) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "out of host memory");
  m->device = device;
  m->cfg = *cfg;
  m->max_tokens = max_tokens;
  MoeDims &d = m->d;
  d.H = (int)cfg->hidden;
  d.M = (int)cfg->moe;
  d.E = (int)cfg->n_experts;
  d.K = (int)cfg->top_k;
  d.hb = d.H / 256;
  d.mb = d.M / 256;
  d.act_stride = round16((size_t)d.hb * 292);
  d.amoe_stride = round16((size_t)d.mb * 292);
  d.eps = cfg->eps;
  d.norm_topk = cfg->norm_topk_prob;
  const size_t T = max_tokens, K = d.K, P = T * K;
  m->max_units = (int)(std::min<size_t>((size_t)d.E, P) + (P + RV_MOE_TOK_CHUNK - 1) / RV_MOE_TOK_CHUNK);
  // Speculative decode lays out up to min(T, 8) * E positions, one unit per expert.
  const size_t PS = std::max(P, std::min<size_t>(T, RV_SPEC_MAX_T) * (size_t)d.E);
  const size_t units_cap = std::max<size_t>((size_t)m->max_units, (size_t)d.E);
  if (const char *v = getenv("RV_DECODE_SPEC")) m->spec = atoi(v) != 0;
  const size_t max_tc = std::min<size_t>((size_t)d.E, P) + P / RV_TC_NT + 1;
  const size_t padded_rows = (P + 16 * (size_t)d.E + 16 + 15) & ~(size_t)15;  // every expert's rows rounded up to 16
  // One arena for every scratch buffer the forward touches.
  struct Part { size_t bytes; void **slot; };
  MoeBufs &B = m->B;
  const Part parts[] = {
      {T * d.H * 4, (void **)&B.normed},
      {T * d.act_stride, (void **)&B.acts},
      {T * d.E * 4, (void **)&B.logits},
      {P * 4, (void **)&B.ids},
      {P * 4, (void **)&B.w},
      {(size_t)d.E * 4, (void **)&B.counts},
      {((size_t)d.E + 1) * 4, (void **)&B.index_start},
      {PS * 4, (void **)&B.index},
      {(size_t)m->max_units * 16, (void **)&B.units},
      {16, (void **)&B.n_units},
      {PS * d.M * 4, (void **)&B.hbuf},
      {PS * d.amoe_stride, (void **)&B.acts_moe},
      {P * d.H * 4, (void **)&B.staged},
      {units_cap * d.mb * 4, (void **)&B.tile_cnt},
      {16, (void **)&B.route_cnt},
      {((size_t)d.H / 4 + 1) * 4, (void **)&B.down_cnt},  // one per down row tile (>= 4 rows)
      {std::min<size_t>(T, RV_SPEC_MAX_T) * (size_t)d.E * 8, (void **)&B.spec},
      {T * d.H * 4, (void **)&m->dres},
      {padded_rows * d.H * 2, (void **)&B.xq},
      {padded_rows * d.hb * 32, (void **)&B.xm},
      {padded_rows * d.hb * 4, (void **)&B.xd},
      {padded_rows * d.M * 2, (void **)&B.hq},
      {padded_rows * d.mb * 32, (void **)&B.hm},
      {padded_rows * d.mb * 4, (void **)&B.hdsc},
      {P * d.M * 8, (void **)&B.gu},
      {max_tc * 16, (void **)&B.tc_units},
      {16, (void **)&B.n_tc},
      {(size_t)d.E * 4, (void **)&B.tc_pstart},
      // Dequantized weight stages (tensor path, experts with two or more
      // position tiles): only engines large enough for that to happen often.
      {tc_cache_bytes(d, max_tokens), (void **)&B.tc_a},
      {(size_t)d.E * 4, (void **)&B.tc_apre},
  };
  size_t total = 0;
  for (const Part &p : parts) total += (p.bytes + 255) & ~(size_t)255;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  cudaError_t e = cudaMalloc(&m->arena, total);
  if (e == cudaSuccess) e = cudaMemset(m->arena, 0, total);
  cudaSetDevice(prev);
  if (e != cudaSuccess) {
    delete m;
    RV_FAIL(RV_ERR_CUDA, "moe_create: %zu bytes of scratch: %s", total, cudaGetErrorString(e));
  }
  size_t off = 0;
  for (const Part &p : parts) {
    *p.slot = (uint8_t *)m->arena + off;
    off += (p.bytes + 255) & ~(size_t)255;
  }
  if (tc_cache_bytes(d, max_tokens) == 0) B.tc_a = nullptr;
  B.max_units = m->max_units;
  B.max_tc = (int)max_tc;
  B.tc_groups = (int)(padded_rows / 8);
  *out = m;
  return RV_OK;
}

extern "C" void rv_moe_destroy(rv_moe *m) {
  if (!m) return;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(m->device);
  prof_release(m);
  cudaFree(m->arena);
  cudaSetDevice(prev);
  cudaGetLastError();  // a void call: leave no error behind for the caller's next check
  delete m;
}

// Launch with programmatic stream serialization (the kernel may start
// while the previous kernel of the stream runs; it calls pdl_wait()).
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// The decode kernels come in a Qwen3-geometry instantiation (hidden 2048,
// moe 768, 128 experts, top-8) with the dimensions as constants.
static bool geo_qwen3(const MoeDims &d) { return d.H == 2048 && d.M == 768 && d.E == 128 && d.K == 8; }

// The exact router chains of speculative decode: RV_CHAIN_EXPERTS router
// rows per CTA (fewer when the rows and T residual rows would not fit), one
// cluster of all the CTAs when there are at most 8 of them.  Each CTA takes
// a whole SM's shared memory, so no other kernel's CTA shares an SM with a
// serial chain.
static void (*route_chain_kernel(bool cluster, bool q3))(MoeDims, MoeBufs, int, MoeWeights) {
  if (cluster) return q3 ? k_route_chain<true, RV_GEO_QWEN3> : k_route_chain<true, 0>;
  return q3 ? k_route_chain<false, RV_GEO_QWEN3> : k_route_chain<false, 0>;
}

static int launch_route_chain(const MoeDims &d, const MoeBufs &B, int T, const MoeWeights &W, cudaStream_t s) {
  const size_t xrow = (size_t)(d.H + 4) * 4;
  const size_t fixed = 16 + (size_t)T * xrow + (size_t)d.H * 4;
  int ch = 0, grid = 0;
  bool cluster = false;
  void (*kern)(MoeDims, MoeBufs, int, MoeWeights) = nullptr;
  size_t room = 0;
  for (int v = 0; v < 2 && !kern; v++) {  // the cluster variant first
    const bool q3 = geo_qwen3(d);
    void (*k)(MoeDims, MoeBufs, int, MoeWeights) = route_chain_kernel(v == 0, q3);
    cudaFuncAttributes fa;
    RV_CUDA(cudaFuncGetAttributes(&fa, k));
    room = (size_t)RV_SMEM_PER_CTA - fa.sharedSizeBytes;
    if (room < fixed + xrow) continue;
    ch = (int)std::min<size_t>(RV_CHAIN_EXPERTS, (room - fixed) / xrow);
    grid = (d.E + ch - 1) / ch;
    if (v == 0 && grid > 8) continue;
    kern = k;
    cluster = v == 0;
  }
  if (!kern) RV_FAIL(RV_ERR_UNIMPLEMENTED, "router chains: %d tokens of hidden %d do not fit in shared memory", T, d.H);
  const size_t smem = room;
  RV_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(RV_CHAIN_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = (unsigned)grid;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = cluster ? 2 : 1;
  RV_CUDA(cudaLaunchKernelEx(&cfg, kern, d, B, ch, W));
  return RV_OK;
}

// Split mode (G lanes per row, one token at a time) serves decode; token
// mode (a thread per row, up to 8 tokens in flight) serves larger batches.
// units: the grid's first dimension (the unit capacity, or for the
// speculative kernels the units expected; they stride over the rest).

template <int FMT, int G, int NBG, int R, bool SPEC, int GEO>
static void launch_gate_up_t(const MoeDims &d, const MoeBufs &B, const MoeWeights &W, int units, cudaStream_t s) {
  const size_t st = FMT == RV_Q6_K ? W.gu_row_bytes : W.gu_row_bytes + 16;
  const size_t smem = 16 + round16(2 * (size_t)R * st) + 16 + (size_t)B.ms * d.act_stride + 2 * R * RV_MOE_MT * 4;
  dim3 grid((unsigned)units, (unsigned)(d.M / R));
  cudaFuncSetAttribute(k_gate_up<FMT, G, NBG, R, SPEC, GEO>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  launch_pdl(k_gate_up<FMT, G, NBG, R, SPEC, GEO>, grid, dim3(2 * R * G), smem, s, d, B, W);
}
template <int FMT>
static void launch_gate_up(const MoeDims &d, const MoeBufs &B, const MoeWeights &W, int T, int spec_units,
                           cudaStream_t s) {
  const bool q3 = geo_qwen3(d);
  if (spec_units) {
    if (q3) launch_gate_up_t<FMT, 4, 2, 8, true, RV_GEO_QWEN3>(d, B, W, spec_units, s);
    else if (d.hb == 8) launch_gate_up_t<FMT, 4, 2, 8, true, 0>(d, B, W, spec_units, s);
    else launch_gate_up_t<FMT, 1, 1, 32, true, 0>(d, B, W, spec_units, s);
  } else if (T <= RV_SMALL_T && d.hb == 8) {
    if (q3) launch_gate_up_t<FMT, 4, 2, 8, false, RV_GEO_QWEN3>(d, B, W, B.max_units, s);
    else launch_gate_up_t<FMT, 4, 2, 8, false, 0>(d, B, W, B.max_units, s);
  } else {
    launch_gate_up_t<FMT, 1, 1, 32, false, 0>(d, B, W, B.max_units, s);
  }
}
template <int FMT, int G, int NBG, int ROWS, bool COMBINE, bool SPEC, int GEO>
static cudaError_t launch_down_t(const MoeDims &d, const MoeBufs &B, const MoeWeights &W, int units,
                                 cudaStream_t s) {
  const size_t st = FMT == RV_Q6_K ? W.down_row_bytes : W.down_row_bytes + 16;
  const size_t smem = 16 + round16((size_t)ROWS * st) + 16 + (size_t)B.ms * d.amoe_stride + 16 +
                      (G > 1 ? (size_t)B.ms * d.mb * RV_ACT_AL : 0);
  dim3 grid((unsigned)units, (unsigned)((d.H + ROWS - 1) / ROWS));
  cudaFuncSetAttribute(k_down<FMT, G, NBG, ROWS, COMBINE, SPEC, GEO>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       (int)smem);
  return launch_pdl(k_down<FMT, G, NBG, ROWS, COMBINE, SPEC, GEO>, grid, dim3(32), smem, s, d, B, W);
}
// Returns true when the down kernel also performed the combine (only when
// fuse_combine allows it; always for the speculative kernels).
template <int FMT>
static bool launch_down(const MoeDims &d, const MoeBufs &B, const MoeWeights &W, int T, bool fuse_combine,
                        int spec_units, cudaStream_t s) {
  const bool q3 = geo_qwen3(d);
  if (spec_units) {
    if (q3) launch_down_t<FMT, 3, 1, 8, true, true, RV_GEO_QWEN3>(d, B, W, spec_units, s);
    else if (d.mb == 3) launch_down_t<FMT, 3, 1, 8, true, true, 0>(d, B, W, spec_units, s);
    else launch_down_t<FMT, 1, 1, 32, true, true, 0>(d, B, W, spec_units, s);
    return true;
  }
  if (T <= RV_SMALL_T && d.mb == 3) {
    if (fuse_combine) {
      if (q3) launch_down_t<FMT, 3, 1, 8, true, false, RV_GEO_QWEN3>(d, B, W, B.max_units, s);
      else launch_down_t<FMT, 3, 1, 8, true, false, 0>(d, B, W, B.max_units, s);
      return true;
    }
    launch_down_t<FMT, 3, 1, 8, false, false, 0>(d, B, W, B.max_units, s);
    return false;
  }
  launch_down_t<FMT, 1, 1, 32, false, false, 0>(d, B, W, B.max_units, s);
  return false;
}

// ---------------------------------------------------- tensor-core prefill
static PFN_cuTensorMapEncodeTiled_v12000 g_tmap_encode;

// The driver's tensor-map encoder, looked up once through the runtime.
static int tmap_encoder(PFN_cuTensorMapEncodeTiled_v12000 *out) {
  std::lock_guard<std::mutex> lk(g_init_mu);
  if (!g_tmap_encode) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
      RV_FAIL(RV_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable (%s)", cudaGetErrorString(e));
    g_tmap_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
  }
  *out = g_tmap_encode;
  return RV_OK;
}

// Tensor map over a layer's gate and up slabs as one [E][2][M][row bytes]
// byte array (strides: row bytes, up_off - gate_off, expert stride); box =
// one super-block column of 128 rows.
static int gate_up_map(const MoeWeights &W, const rv_layer_layout &L, CUtensorMap *map) {
  if (L.up_off <= L.gate_off) RV_FAIL(RV_ERR_UNIMPLEMENTED, "the tensor path needs the up slab after the gate slab");
  PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
  int rc = tmap_encoder(&enc);
  if (rc) return rc;
  const cuuint64_t dims[4] = {W.gu_row_bytes, L.moe, 2, L.n_experts};
  const cuuint64_t strides[3] = {W.gu_row_bytes, L.up_off - L.gate_off, L.stride};
  const cuuint32_t box[4] = {(cuuint32_t)rv_fmt_block_bytes(L.gate_format), RV_TC_ROWS, 1, 1};
  const cuuint32_t es[4] = {1, 1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, (void *)(W.base + L.gate_off), dims, strides, box, es,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) RV_FAIL(RV_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return RV_OK;
}

template <int FMT, bool DOWN>
static int launch_tc_gemm(const MoeDims &d, const MoeBufs &B, const MoeWeights &W, const CUtensorMap &map,
                          cudaStream_t s) {
  const size_t rb = DOWN ? W.down_row_bytes : W.gu_row_bytes;
  const size_t smem = TcCfg<FMT, DOWN>::total(rb, (DOWN ? d.M : d.H) / 256);
  RV_CUDA(cudaFuncSetAttribute(k_tc_gemm<FMT, DOWN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const size_t nrt = DOWN ? (size_t)(d.H / RV_TC_ROWS) : (size_t)(2 * d.M / RV_TC_ROWS);
  // Persistent: one CTA per SM walks the (row tile, pair tile) work items;
  // the count of pair tiles is the device's (k_tc_tiles), the capacity
  // bounds the grid.
  int dev = 0;
  RV_CUDA(cudaGetDevice(&dev));
  const size_t sms = g_dev_sms[dev] > 0 ? (size_t)g_dev_sms[dev] : 148;
  const unsigned grid = (unsigned)std::min(sms, nrt * (size_t)B.max_tc);
  k_tc_gemm<FMT, DOWN><<<grid, RV_TC_THREADS, smem, s>>>(d, B, W, map);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    cudaFuncAttributes fa = {};
    cudaFuncGetAttributes(&fa, k_tc_gemm<FMT, DOWN>);
    RV_FAIL(RV_ERR_CUDA, "k_tc_gemm launch failed: %s (%d registers, at most %d threads, %zu bytes of shared memory)",
            cudaGetErrorString(e), fa.numRegs, fa.maxThreadsPerBlock, smem);
  }
  return RV_OK;
}

// Checks the tensor path's layout requirements: gate/up Q4_K or Q5_K, and
// every super-block row start and whole down tile 16-byte aligned for the
// bulk copies.
static int tc_check(const rv_layer_layout &L, const MoeWeights &W, uint32_t layer) {
  if (L.gate_format != RV_Q4_K && L.gate_format != RV_Q5_K)
    RV_FAIL(RV_ERR_UNIMPLEMENTED, "layer %u: the tensor path takes Q4_K or Q5_K gate/up (format %d)", layer,
            L.gate_format);
  if (!rv_fmt_is_kquant(L.down_format))
    RV_FAIL(RV_ERR_UNSUPPORTED_FORMAT, "layer %u: down format %d", layer, L.down_format);
  if (((uintptr_t)W.base | W.stride | W.gate_off | W.up_off | W.down_off | W.gu_row_bytes) & 15)
    RV_FAIL(RV_ERR_UNIMPLEMENTED, "layer %u: the tensor path needs 16-byte aligned expert slabs", layer);
  return RV_OK;
}

// Event record for the per-stage profile (an external node inside a stream
// capture, so that every replay of the graph records it).
static int prof_record(cudaEvent_t *ev, int i, unsigned flags, cudaStream_t s) {
  if (ev) RV_CUDA(cudaEventRecordWithFlags(ev[i], s, flags));
  return RV_OK;
}

static MoeWeights layer_weights(const rv_expert_table *table, uint32_t layer) {
  const rv_layer_layout &L = table->layouts[layer];
  MoeWeights W;
  W.base = table->base[layer];
  W.stride = L.stride;
  W.gate_off = L.gate_off;
  W.up_off = L.up_off;
  W.down_off = L.down_off;
  rv_row_bytes(L.gate_format, L.hidden, &W.gu_row_bytes);
  rv_row_bytes(L.down_format, L.moe, &W.down_row_bytes);
  return W;
}

// The expert half for T rows of d.K slots whose dispatch index (B.index,
// B.units, B.index_start) is built: gate/up, SwiGLU, Q8_K, down into
// B.staged [pair][H].  Profile events 1-3 are recorded when ev is set.
// *combined: the down kernel also performed the combine (only with
// fuse_combine).
static int expert_stage(const MoeDims &d, const MoeBufs &B, const MoeWeights &W, const rv_layer_layout &L,
                        uint32_t layer, int T, uint32_t flags, bool fuse_combine, int spec_units, cudaEvent_t *ev,
                        unsigned evflags, cudaStream_t s, bool *combined) {
  *combined = false;
  int rc;
  if (flags & RV_MOE_TENSOR) {
    rc = tc_check(L, W, layer);
    if (rc) return rc;
    const unsigned P = (unsigned)(T * d.K);
    k_tc_tiles<<<1, 256, 0, s>>>(d, B);
    // Position-striding grids: P is the capacity, the index holds how many.
    const unsigned pg = std::min(P, 4096u);
    k_tc_gather<<<pg, 32 * d.hb, 0, s>>>(d, B);
    RV_LAUNCH_CHECK();
    if ((rc = prof_record(ev, 1, evflags, s))) return rc;
    CUtensorMap gmap;
    if ((rc = gate_up_map(W, L, &gmap))) return rc;
    if (B.tc_a) {
      const int spb = 4 / (L.gate_format == RV_Q4_K ? TcStage<RV_Q4_K, false>::SUB : TcStage<RV_Q5_K, false>::SUB);
      const dim3 g((unsigned)(2 * d.M / RV_TC_ROWS), (unsigned)(spb * d.hb), (unsigned)d.E);
      if (L.gate_format == RV_Q4_K) k_tc_predeq<RV_Q4_K, false><<<g, 256, 0, s>>>(d, B, W);
      else k_tc_predeq<RV_Q5_K, false><<<g, 256, 0, s>>>(d, B, W);
      RV_LAUNCH_CHECK();
    }
    rc = L.gate_format == RV_Q4_K ? launch_tc_gemm<RV_Q4_K, false>(d, B, W, gmap, s)
                                  : launch_tc_gemm<RV_Q5_K, false>(d, B, W, gmap, s);
    if (rc) return rc;
    k_tc_quant<<<pg, 32 * d.mb, 0, s>>>(d, B);
    RV_LAUNCH_CHECK();
    if (B.tc_a) {  // after the gate/up GEMM: the cache now takes the down stages
      const unsigned gx = (unsigned)(d.H / RV_TC_ROWS);
      switch (L.down_format) {
        case RV_Q4_K:
          k_tc_predeq<RV_Q4_K, true><<<dim3(gx, 4 / TcStage<RV_Q4_K, true>::SUB * d.mb, d.E), 256, 0, s>>>(d, B, W);
          break;
        case RV_Q5_K:
          k_tc_predeq<RV_Q5_K, true><<<dim3(gx, 4 / TcStage<RV_Q5_K, true>::SUB * d.mb, d.E), 256, 0, s>>>(d, B, W);
          break;
        default:
          k_tc_predeq<RV_Q6_K, true><<<dim3(gx, 4 / TcStage<RV_Q6_K, true>::SUB * d.mb, d.E), 256, 0, s>>>(d, B, W);
          break;
      }
      RV_LAUNCH_CHECK();
    }
    if ((rc = prof_record(ev, 2, evflags, s))) return rc;
    switch (L.down_format) {
      case RV_Q4_K: rc = launch_tc_gemm<RV_Q4_K, true>(d, B, W, gmap, s); break;
      case RV_Q5_K: rc = launch_tc_gemm<RV_Q5_K, true>(d, B, W, gmap, s); break;
      default: rc = launch_tc_gemm<RV_Q6_K, true>(d, B, W, gmap, s); break;
    }
    if (rc) return rc;
    return prof_record(ev, 3, evflags, s);
  }
  if ((rc = prof_record(ev, 1, evflags, s))) return rc;
  switch (L.gate_format) {
    case RV_Q4_K: launch_gate_up<RV_Q4_K>(d, B, W, T, spec_units, s); break;
    case RV_Q5_K: launch_gate_up<RV_Q5_K>(d, B, W, T, spec_units, s); break;
    default: launch_gate_up<RV_Q6_K>(d, B, W, T, spec_units, s); break;
  }
  if ((rc = prof_record(ev, 2, evflags, s))) return rc;
  switch (L.down_format) {
    case RV_Q4_K: *combined = launch_down<RV_Q4_K>(d, B, W, T, fuse_combine, spec_units, s); break;
    case RV_Q5_K: *combined = launch_down<RV_Q5_K>(d, B, W, T, fuse_combine, spec_units, s); break;
    default: *combined = launch_down<RV_Q6_K>(d, B, W, T, fuse_combine, spec_units, s); break;
  }
  RV_LAUNCH_CHECK();
  return prof_record(ev, 3, evflags, s);
}

// Routing for T rows through the large-batch kernels: RMSNorm + Q8_K,
// serial router chains, softmax/top-k/renormalization (counts into
// B.counts).
static int route_stage(const MoeDims &d, const MoeBufs &B, int T, cudaStream_t s) {
  k_prologue<<<T, 256, 34 * sizeof(double) + (size_t)d.H * 4, s>>>(d, B);
  k_router_logits<<<dim3((unsigned)((T + 31) / 32), (unsigned)((d.E + RV_REXP - 1) / RV_REXP)), 128,
                    router_logits_smem(), s>>>(d, B);
  k_route<<<(unsigned)((T + 3) / 4), 128, 0, s>>>(d, B);
  RV_LAUNCH_CHECK();
  return RV_OK;
}

static int check_engine_layer(const rv_moe *m, const rv_expert_table *table, uint32_t layer, bool local) {
  if (layer >= table->layouts.size())
    RV_FAIL(RV_ERR_LAYER_OUT_OF_RANGE, "layer %u of %zu", layer, table->layouts.size());
  const rv_layer_layout &L = table->layouts[layer];
  const MoeDims &d = m->d;
  if (L.hidden != (uint32_t)d.H || L.moe != (uint32_t)d.M || (!local && L.n_experts != (uint32_t)d.E))
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "layer %u geometry (%u, %u, %u) vs engine (%d, %d, %d)", layer, L.hidden,
            L.moe, L.n_experts, d.H, d.M, d.E);
  if (L.n_experts > 256) RV_FAIL(RV_ERR_UNIMPLEMENTED, "layer %u: more than 256 experts", layer);
  if (L.gate_format != L.up_format)
    RV_FAIL(RV_ERR_UNIMPLEMENTED, "layer %u: gate and up in different formats", layer);
  return RV_OK;
}

extern "C" int rv_moe_forward(rv_moe *m, const rv_expert_table *table, uint32_t layer,
                              const float *ffn_norm, const float *router, float *residual,
                              size_t n_tokens, uint32_t *topk_ids, float *topk_weights,
                              uint32_t flags, rv_stream stream) {
  if (!m || !table) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "moe_forward: null engine or table");
  int rc = check_engine_layer(m, table, layer, false);
  if (rc) return rc;
  const rv_layer_layout &L = table->layouts[layer];
  const MoeDims &d = m->d;
  if (flags & ~RV_MOE_TENSOR) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "unknown flags 0x%x", flags);
  if (n_tokens > m->max_tokens)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "moe_forward: %zu tokens vs engine capacity %zu", n_tokens, m->max_tokens);
  if (n_tokens == 0) return RV_OK;
  if (!ffn_norm || !router || !residual) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "moe_forward: null pointer");
  if (((uintptr_t)router & 15) || (d.H & 3))
    RV_FAIL(RV_ERR_INVALID_ARGUMENT, "moe_forward: router must be 16-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  MoeBufs B = m->B;
  B.ffn_norm = ffn_norm;
  B.router = router;
  B.residual = residual;
  B.T = (int)n_tokens;
  const MoeWeights W = layer_weights(table, layer);
  const int T = (int)n_tokens;
  cudaEvent_t *ev = nullptr;
  unsigned evflags = 0;
  if (m->prof_next < m->prof.size() / 5) {
    ev = &m->prof[5 * m->prof_next++];
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    RV_CUDA(cudaStreamIsCapturing(s, &cs));
    if (cs == cudaStreamCaptureStatusActive) evflags = cudaEventRecordExternal;
  }
  if ((rc = prof_record(ev, 0, evflags, s))) return rc;
  B.ms = T < RV_MOE_MT ? T : RV_MOE_MT;
  int spec_units = 0;
  if (!(flags & RV_MOE_TENSOR) && T <= RV_SMALL_T && m->spec) {
    // decode, speculative: norm, Q8_K and logit bounds; then the exact
    // router chains beside gate/up on the speculated experts; then down
    // and combine on the exact routing.
    const size_t xrow = (size_t)(d.H + 4) * 4;
    // Shared memory padded past half an SM's: one routing CTA per SM.
    const size_t rs_need = 16 + (size_t)(RV_SPEC_EPC + 1) * d.H * 4 + T * xrow;
    // The expert CTAs, then one CTA per four Q8_K blocks of the normed rows.
    RV_CUDA(launch_pdl(geo_qwen3(d) ? k_route_spec<RV_GEO_QWEN3> : k_route_spec<0>,
                       dim3((unsigned)((d.E + RV_SPEC_EPC - 1) / RV_SPEC_EPC + (T * d.hb + 3) / 4)), dim3(128),
                       std::max(rs_need, (size_t)RV_ROUTE_SMEM_ONE_PER_SM), s, d, B));
    if ((rc = launch_route_chain(d, B, T, W, s))) return rc;
    spec_units = std::min(d.E, T * d.K);
  } else if (!(flags & RV_MOE_TENSOR) && T <= RV_SMALL_T) {
    // decode: routing, norm, Q8_K and dispatch in one launch
    // Shared memory padded past half an SM's so that no two routing CTAs
    // (each running one serial router chain) share an SM.
    const size_t need = 16 + (size_t)2 * d.H * 4 + (size_t)T * (d.H + 4) * 4 + 4 * (size_t)T * sizeof(double) + 16;
    const size_t smem = need < RV_ROUTE_SMEM_ONE_PER_SM ? RV_ROUTE_SMEM_ONE_PER_SM : need;
    RV_CUDA(launch_pdl(k_route_decode, dim3((unsigned)d.E), dim3(128), smem, s, d, B));
  } else {
    if ((rc = route_stage(d, B, T, s))) return rc;
    k_index<<<1, 1024, 0, s>>>(d, B);
  }
  bool combined = false;
  if ((rc = expert_stage(d, B, W, L, layer, T, flags, true, spec_units, ev, evflags, s, &combined))) return rc;
  if (!combined) k_combine<<<dim3((unsigned)T, (unsigned)((d.H + 255) / 256)), 256, 0, s>>>(d, B);
  if ((rc = prof_record(ev, 4, evflags, s))) return rc;
  RV_LAUNCH_CHECK();
  if (topk_ids) RV_CUDA(cudaMemcpyAsync(topk_ids, B.ids, n_tokens * d.K * 4, cudaMemcpyDeviceToDevice, s));
  if (topk_weights) RV_CUDA(cudaMemcpyAsync(topk_weights, B.w, n_tokens * d.K * 4, cudaMemcpyDeviceToDevice, s));
  m->last_T = T;
  return RV_OK;
}

extern "C" size_t rv_moe_act_stride(const rv_moe *m) { return m ? m->d.act_stride : 0; }

extern "C" int rv_moe_route(rv_moe *m, const float *ffn_norm, const float *router, const float *residual,
                            size_t n_tokens, uint32_t *topk_ids, float *topk_weights, uint8_t *acts,
                            rv_stream stream) {
  if (!m) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "moe_route: null engine");
  if (n_tokens > m->max_tokens)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "moe_route: %zu tokens vs engine capacity %zu", n_tokens, m->max_tokens);
  if (n_tokens == 0) return RV_OK;
  if (!ffn_norm || !router || !residual || !topk_ids || !topk_weights)
    RV_FAIL(RV_ERR_INVALID_ARGUMENT, "moe_route: null pointer");
  if ((uintptr_t)router & 15) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "moe_route: router must be 16-byte aligned");
  if (acts && ((uintptr_t)acts & 15)) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "moe_route: acts must be 16-byte aligned");
  const MoeDims &d = m->d;
  cudaStream_t s = (cudaStream_t)stream;
  MoeBufs B = m->B;
  B.ffn_norm = ffn_norm;
  B.router = router;
  B.residual = (float *)residual;  // read only by the prologue
  B.T = (int)n_tokens;
  if (acts) B.acts = acts;
  int rc = route_stage(d, B, (int)n_tokens, s);
  if (rc) return rc;
  RV_CUDA(cudaMemsetAsync(B.counts, 0, (size_t)d.E * 4, s));
  RV_CUDA(cudaMemcpyAsync(topk_ids, B.ids, n_tokens * d.K * 4, cudaMemcpyDeviceToDevice, s));
  RV_CUDA(cudaMemcpyAsync(topk_weights, B.w, n_tokens * d.K * 4, cudaMemcpyDeviceToDevice, s));
  m->last_T = (int)n_tokens;
  return RV_OK;
}

extern "C" int rv_moe_experts(rv_moe *m, const rv_expert_table *table, uint32_t layer, const uint32_t *expert_ids,
                              const uint8_t *acts, size_t n_pairs, float *out, uint32_t flags, rv_stream stream) {
  if (!m || !table) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "moe_experts: null engine or table");
  int rc = check_engine_layer(m, table, layer, true);
  if (rc) return rc;
  if (flags & ~RV_MOE_TENSOR) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "unknown flags 0x%x", flags);
  const size_t cap = m->max_tokens * (size_t)m->d.K;
  if (n_pairs > cap) RV_FAIL(RV_ERR_LENGTH_MISMATCH, "moe_experts: %zu pairs vs engine capacity %zu", n_pairs, cap);
  if (n_pairs == 0) return RV_OK;
  if (!expert_ids || !acts || !out) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "moe_experts: null pointer");
  if ((uintptr_t)acts & 15) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "moe_experts: acts must be 16-byte aligned");
  const rv_layer_layout &L = table->layouts[layer];
  MoeDims d = m->d;  // one slot per row, the table's local experts
  d.K = 1;
  d.E = (int)L.n_experts;
  cudaStream_t s = (cudaStream_t)stream;
  MoeBufs B = m->B;
  B.T = (int)n_pairs;
  B.ms = B.T < RV_MOE_MT ? B.T : RV_MOE_MT;
  B.acts = (uint8_t *)acts;  // read only
  B.staged = out;
  RV_CUDA(cudaMemcpyAsync(B.ids, expert_ids, n_pairs * 4, cudaMemcpyDeviceToDevice, s));
  k_count_ids<<<(unsigned)((n_pairs + 255) / 256), 256, 0, s>>>(d, B);
  k_index<<<1, 1024, 0, s>>>(d, B);
  RV_LAUNCH_CHECK();
  bool combined = false;
  return expert_stage(d, B, layer_weights(table, layer), L, layer, (int)n_pairs, flags, false, 0, nullptr, 0, s,
                      &combined);
}

extern "C" int rv_moe_combine(rv_moe *m, float *residual, const float *topk_weights, const float *expert_out,
                              const uint32_t *pos_of, size_t n_tokens, rv_stream stream) {
  if (!m) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "moe_combine: null engine");
  if (n_tokens == 0) return RV_OK;
  if (!residual || !topk_weights || !expert_out) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "moe_combine: null pointer");
  const MoeDims &d = m->d;
  MoeBufs B = m->B;
  B.residual = residual;
  B.w = (float *)topk_weights;
  B.staged = (float *)expert_out;
  B.T = (int)n_tokens;
  k_combine_rows<<<dim3((unsigned)n_tokens, (unsigned)((d.H + 255) / 256)), 256, 0, (cudaStream_t)stream>>>(
      d, B, pos_of);
  RV_LAUNCH_CHECK();
  return RV_OK;
}

extern "C" int rv_ep_plan(rv_moe *m, const uint32_t *topk_ids, const uint8_t *acts, size_t n_tokens, uint32_t world,
                          int32_t *send_counts, uint32_t *pos_of, uint32_t *send_local, uint8_t *send_acts,
                          rv_stream stream) {
  if (!m) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "ep_plan: null engine");
  if (world == 0 || world > 64) RV_FAIL(RV_ERR_UNIMPLEMENTED, "ep_plan: world size %u (1..64)", world);
  if (n_tokens > m->max_tokens)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "ep_plan: %zu tokens vs engine capacity %zu", n_tokens, m->max_tokens);
  if (!topk_ids || !acts || !send_counts || !pos_of || !send_local || !send_acts)
    RV_FAIL(RV_ERR_INVALID_ARGUMENT, "ep_plan: null pointer");
  if (((uintptr_t)acts | (uintptr_t)send_acts) & 15)
    RV_FAIL(RV_ERR_INVALID_ARGUMENT, "ep_plan: activation rows must be 16-byte aligned");
  const MoeDims &d = m->d;
  cudaStream_t s = (cudaStream_t)stream;
  const unsigned P = (unsigned)(n_tokens * d.K);
  k_ep_plan<<<1, 1024, 0, s>>>(d, topk_ids, P, world, send_counts, pos_of, send_local, m->B.index);
  if (P) k_ep_pack<<<P, 128, 0, s>>>(d, acts, m->B.index, send_acts);
  RV_LAUNCH_CHECK();
  return RV_OK;
}

// ============================================== expert-parallel exchange
// One rv_ep per rank: its exchange window (see rv_ep.cuh), the peers'
// windows as this GPU addresses them, and the state of the step protocol.
#define RV_EP_MAGIC "RVEPWIN1"
struct EpHandle {  // what rv_ep_handle exports (RV_EP_HANDLE_BYTES)
  char magic[8];
  uint32_t world, rank, cap, act_stride, hidden, n_experts;
  int64_t pid;
  uint64_t win_bytes, win_ptr;
  char bus_id[32];
  cudaIpcMemHandle_t ipc;
};
static_assert(sizeof(EpHandle) <= RV_EP_HANDLE_BYTES, "handle layout");

struct rv_ep {
  rv_moe *m = nullptr;
  int device = 0;              // the engine's device (kept here: destroy does not touch the engine)
  uint32_t world = 0, rank = 0;
  size_t max_tokens = 0;
  uint8_t *window = nullptr;   // this rank's window (cudaMalloc, exported)
  EpState *state = nullptr;    // device
  uint8_t **d_win = nullptr;   // device [world]: every rank's window
  float **d_out = nullptr;     // device [world]: every rank's output rows (window + o_out)
  uint32_t *slot_ids = nullptr;  // device [world*cap]: the received slots' local experts
  std::vector<void *> opened;  // peer windows mapped through IPC (closed on destroy)
  bool connected = false;
  char bus_id[32] = {0};
  EpArgs A{};
};

extern "C" void rv_ep_destroy(rv_ep *ep) {
  if (!ep) return;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(ep->device);
  cudaStreamSynchronize(nullptr);
  for (void *p : ep->opened) cudaIpcCloseMemHandle(p);
  cudaFree(ep->window);
  cudaFree(ep->state);
  cudaFree(ep->d_win);
  cudaFree(ep->d_out);
  cudaFree(ep->slot_ids);
  if (prev >= 0) cudaSetDevice(prev);
  cudaGetLastError();  // a void call: leave no error behind for the caller's next check
  delete ep;
}

extern "C" int rv_ep_create(rv_moe *m, uint32_t world, uint32_t rank, size_t max_tokens, rv_ep **out) {
  if (!m || !out) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "ep_create: null pointer");
  *out = nullptr;
  if (world == 0 || world > 64) RV_FAIL(RV_ERR_UNIMPLEMENTED, "ep_create: world size %u (1..64)", world);
  if (rank >= world) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "ep_create: rank %u of %u", rank, world);
  if ((uint32_t)m->d.E % world)
    RV_FAIL(RV_ERR_UNIMPLEMENTED, "ep_create: %d experts do not split evenly over %u ranks", m->d.E, world);
  if (max_tokens == 0 || max_tokens > m->max_tokens)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "ep_create: %zu tokens per rank vs engine capacity %zu", max_tokens,
            m->max_tokens);
  if ((size_t)world * max_tokens > m->max_tokens)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH,
            "ep_create: the engine runs the experts on up to world x max_tokens = %zu rows; it holds %zu",
            (size_t)world * max_tokens, m->max_tokens);
  rv_ep *ep = new (std::nothrow) rv_ep();
  if (!ep) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "out of host memory");
  ep->m = m;
  ep->device = m->device;
  ep->world = world;
  ep->rank = rank;
  ep->max_tokens = max_tokens;
  EpArgs &A = ep->A;
  A.world = world;
  A.rank = rank;
  A.cap = (uint32_t)(max_tokens * (size_t)m->d.K);
  A.act_stride = (uint32_t)m->d.act_stride;
  A.H = m->d.H;
  ep_layout(A);
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(m->device);
  cudaError_t e = cudaMalloc((void **)&ep->window, A.bytes);
  if (e == cudaSuccess) e = cudaMemset(ep->window, 0, A.bytes);
  if (e == cudaSuccess) e = cudaMalloc((void **)&ep->state, sizeof(EpState));
  if (e == cudaSuccess) e = cudaMemset(ep->state, 0, sizeof(EpState));
  if (e == cudaSuccess) e = cudaMalloc((void **)&ep->d_win, world * sizeof(uint8_t *));
  if (e == cudaSuccess) e = cudaMalloc((void **)&ep->d_out, world * sizeof(float *));
  if (e == cudaSuccess) e = cudaMalloc((void **)&ep->slot_ids, (size_t)world * A.cap * 4);
  if (e == cudaSuccess) e = cudaDeviceGetPCIBusId(ep->bus_id, (int)sizeof ep->bus_id, m->device);
  cudaSetDevice(prev);
  if (e != cudaSuccess) {
    rv_ep_destroy(ep);
    RV_FAIL(RV_ERR_CUDA, "ep_create: %zu-byte exchange window: %s", A.bytes, cudaGetErrorString(e));
  }
  A.mine = ep->window;
  A.st = ep->state;
  A.win = ep->d_win;
  *out = ep;
  return RV_OK;
}

extern "C" int rv_ep_handle(const rv_ep *ep, void *out, size_t len) {
  if (!ep || !out) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "ep_handle: null pointer");
  if (len < RV_EP_HANDLE_BYTES) RV_FAIL(RV_ERR_LENGTH_MISMATCH, "ep_handle: %zu bytes (needs %d)", len,
                                        RV_EP_HANDLE_BYTES);
  EpHandle h;
  memset(&h, 0, sizeof h);
  memcpy(h.magic, RV_EP_MAGIC, 8);
  h.world = ep->world;
  h.rank = ep->rank;
  h.cap = ep->A.cap;
  h.act_stride = ep->A.act_stride;
  h.hidden = (uint32_t)ep->m->d.H;
  h.n_experts = (uint32_t)ep->m->d.E;
  h.pid = (int64_t)getpid();
  h.win_bytes = ep->A.bytes;
  h.win_ptr = (uint64_t)(uintptr_t)ep->window;
  memcpy(h.bus_id, ep->bus_id, sizeof h.bus_id);
  int prev = -1;
  RV_CUDA(cudaGetDevice(&prev));
  RV_CUDA(cudaSetDevice(ep->m->device));
  const cudaError_t e = cudaIpcGetMemHandle(&h.ipc, ep->window);
  cudaSetDevice(prev);
  if (e != cudaSuccess) RV_FAIL(RV_ERR_CUDA, "ep_handle: cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  memset(out, 0, RV_EP_HANDLE_BYTES);
  memcpy(out, &h, sizeof h);
  return RV_OK;
}

extern "C" int rv_ep_connect(rv_ep *ep, const void *handles, size_t len) {
  if (!ep || !handles) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "ep_connect: null pointer");
  if (ep->connected) RV_FAIL(RV_ERR_PROTOCOL, "ep_connect: already connected");
  if (len != (size_t)ep->world * RV_EP_HANDLE_BYTES)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "ep_connect: %zu bytes for %u handles of %d", len, ep->world,
            RV_EP_HANDLE_BYTES);
  // Check every handle before mapping anything.
  std::vector<EpHandle> hs(ep->world);
  for (uint32_t r = 0; r < ep->world; r++) {
    EpHandle &h = hs[r];
    memcpy(&h, (const uint8_t *)handles + (size_t)r * RV_EP_HANDLE_BYTES, sizeof h);
    if (memcmp(h.magic, RV_EP_MAGIC, 8) != 0) RV_FAIL(RV_ERR_PEER, "ep_connect: handle %u is not an exchange handle", r);
    if (h.world != ep->world || h.rank != r)
      RV_FAIL(RV_ERR_PEER, "ep_connect: handle %u is rank %u of %u; this group is %u ranks", r, h.rank, h.world,
              ep->world);
    if (h.cap != ep->A.cap || h.act_stride != ep->A.act_stride || h.hidden != (uint32_t)ep->m->d.H ||
        h.n_experts != (uint32_t)ep->m->d.E || h.win_bytes != ep->A.bytes)
      RV_FAIL(RV_ERR_PEER, "ep_connect: rank %u was created with another geometry or capacity", r);
    h.bus_id[sizeof h.bus_id - 1] = 0;
    if (r != ep->rank && strcmp(h.bus_id, ep->bus_id) == 0)
      RV_FAIL(RV_ERR_PEER, "ep_connect: ranks %u and %u are on the same GPU (%s); each rank needs its own", r,
              ep->rank, ep->bus_id);
  }
  if (hs[ep->rank].win_ptr != (uint64_t)(uintptr_t)ep->window || hs[ep->rank].pid != (int64_t)getpid())
    RV_FAIL(RV_ERR_PEER, "ep_connect: handle %u is not this rank's own", ep->rank);
  int prev = -1;
  RV_CUDA(cudaGetDevice(&prev));
  RV_CUDA(cudaSetDevice(ep->m->device));
  std::vector<uint8_t *> win(ep->world, nullptr);
  int status = RV_OK;
  for (uint32_t r = 0; r < ep->world && status == RV_OK; r++) {
    const EpHandle &h = hs[r];
    if (r == ep->rank) {
      win[r] = ep->window;
    } else if (h.pid == (int64_t)getpid()) {
      // Another device of this process: direct peer access.
      int pdev = -1, can = 0;
      cudaError_t e = cudaDeviceGetByPCIBusId(&pdev, h.bus_id);
      if (e == cudaSuccess) e = cudaDeviceCanAccessPeer(&can, ep->m->device, pdev);
      if (e == cudaSuccess && !can) {
        rv_set_error(RV_ERR_PEER, "ep_connect: device %d cannot access rank %u's device %d", ep->m->device, r, pdev);
        status = RV_ERR_PEER;
        break;
      }
      if (e == cudaSuccess) {
        e = cudaDeviceEnablePeerAccess(pdev, 0);
        if (e == cudaErrorPeerAccessAlreadyEnabled) {
          cudaGetLastError();
          e = cudaSuccess;
        }
      }
      if (e != cudaSuccess) {
        rv_set_error(RV_ERR_PEER, "ep_connect: peer access to rank %u: %s", r, cudaGetErrorString(e));
        status = RV_ERR_PEER;
        break;
      }
      win[r] = (uint8_t *)(uintptr_t)h.win_ptr;
    } else {
      void *p = nullptr;
      const cudaError_t e = cudaIpcOpenMemHandle(&p, h.ipc, cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess) {
        rv_set_error(RV_ERR_PEER, "ep_connect: mapping rank %u's window: %s", r, cudaGetErrorString(e));
        status = RV_ERR_PEER;
        break;
      }
      ep->opened.push_back(p);
      win[r] = (uint8_t *)p;
    }
  }
  if (status == RV_OK) {
    std::vector<float *> outs(ep->world);
    for (uint32_t r = 0; r < ep->world; r++) outs[r] = (float *)(win[r] + ep->A.o_out);
    cudaError_t e = cudaMemcpy(ep->d_win, win.data(), ep->world * sizeof(uint8_t *), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(ep->d_out, outs.data(), ep->world * sizeof(float *), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      rv_set_error(RV_ERR_CUDA, "ep_connect: %s", cudaGetErrorString(e));
      status = RV_ERR_CUDA;
    }
  }
  if (status != RV_OK) {
    for (void *p : ep->opened) cudaIpcCloseMemHandle(p);
    ep->opened.clear();
  } else {
    ep->connected = true;
  }
  cudaSetDevice(prev);
  return status;
}

extern "C" int rv_moe_ep_forward(rv_ep *ep, const rv_expert_table *table, uint32_t layer, const float *ffn_norm,
                                 const float *router, float *residual, size_t n_tokens, uint32_t *topk_ids,
                                 float *topk_weights, const uint32_t *placement, uint32_t flags, rv_stream stream) {
  if (!ep || !table) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "moe_ep_forward: null exchange or table");
  if (!ep->connected) RV_FAIL(RV_ERR_PROTOCOL, "moe_ep_forward: rv_ep_connect has not completed");
  rv_moe *m = ep->m;
  int rc = check_engine_layer(m, table, layer, true);
  if (rc) return rc;
  const rv_layer_layout &L = table->layouts[layer];
  if (L.n_experts * ep->world != (uint32_t)m->d.E)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "moe_ep_forward: layer %u holds %u experts; rank %u of %u needs %d", layer,
            L.n_experts, ep->rank, ep->world, m->d.E / (int)ep->world);
  if (flags & ~RV_MOE_TENSOR) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "unknown flags 0x%x", flags);
  if (n_tokens > ep->max_tokens)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "moe_ep_forward: %zu tokens vs capacity %zu", n_tokens, ep->max_tokens);
  if (n_tokens && (!ffn_norm || !router || !residual)) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "moe_ep_forward: null pointer");
  if ((uintptr_t)router & 15) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "moe_ep_forward: router must be 16-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  const MoeDims &d = m->d;
  const int T = (int)n_tokens;
  MoeBufs B = m->B;
  B.ffn_norm = ffn_norm;
  B.router = router;
  B.residual = residual;
  B.T = T;
  // 1. route the home tokens (forward.rs:2655-2705, prefill.rs:2165-2204)
  if (T > 0 && (rc = route_stage(d, B, T, s))) return rc;
  // 2. dispatch: rows and metadata into the experts' ranks, then the flags
  const int P = T * d.K;
  const unsigned dgrid = (unsigned)std::max(1, (P + 255) / 256);
  k_ep_dispatch<<<dgrid, 256, 0, s>>>(ep->A, placement, B.ids, B.acts, P, d.K, d.E, B.counts);
  RV_LAUNCH_CHECK();
  if (topk_ids) RV_CUDA(cudaMemcpyAsync(topk_ids, B.ids, (size_t)P * 4, cudaMemcpyDeviceToDevice, s));
  if (topk_weights) RV_CUDA(cudaMemcpyAsync(topk_weights, B.w, (size_t)P * 4, cudaMemcpyDeviceToDevice, s));
  // 3. receive: wait for every source, lay out this rank's dispatch list
  MoeDims dx = d;  // the expert stage: one slot per received row, local experts
  dx.K = 1;
  dx.E = (int)L.n_experts;
  MoeBufs X = m->B;
  X.T = (int)(ep->world * ep->A.cap);
  X.ms = X.T < RV_MOE_MT ? X.T : RV_MOE_MT;
  X.ids = ep->slot_ids;
  X.acts = ep->window + ep->A.o_acts;
  X.ep_out = ep->d_out;
  X.ep_home = (const uint32_t *)(ep->window + ep->A.o_home);
  X.ep_cap = ep->A.cap;
  k_ep_receive<<<1, 1024, 0, s>>>(ep->A, dx, X);
  RV_LAUNCH_CHECK();
  // 4. the experts; the down projection stores each row into its home rank
  bool combined = false;
  if ((rc = expert_stage(dx, X, layer_weights(table, layer), L, layer, X.T, flags, false, 0, nullptr, 0, s,
                         &combined)))
    return rc;
  // 5. tell every rank its rows are in, 6. combine once every rank has
  k_ep_signal<<<1, 64, 0, s>>>(ep->A);
  k_ep_combine<<<dim3((unsigned)std::max(T, 1), (unsigned)((d.H + 255) / 256)), 256, 0, s>>>(ep->A, d, residual,
                                                                                            B.w, T);
  RV_LAUNCH_CHECK();
  return RV_OK;
}

extern "C" int rv_ep_check_placement(uint32_t n_experts, uint32_t world, const uint32_t *placement, size_t len) {
  if (!placement) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "ep_check_placement: null placement");
  if (world == 0 || world > 64 || n_experts % world)
    RV_FAIL(RV_ERR_UNIMPLEMENTED, "ep_check_placement: %u experts over %u ranks", n_experts, world);
  if (len != n_experts) RV_FAIL(RV_ERR_LENGTH_MISMATCH, "ep_check_placement: %zu entries for %u experts", len, n_experts);
  const uint32_t per = n_experts / world;
  std::vector<uint8_t> seen((size_t)n_experts, 0);
  for (uint32_t e = 0; e < n_experts; e++) {
    const uint32_t r = placement[e] >> 16, l = placement[e] & 0xFFFFu;
    if (r >= world || l >= per)
      RV_FAIL(RV_ERR_ROUTED_OUT_OF_RANGE, "ep_check_placement: expert %u -> rank %u local %u (of %u x %u)", e, r, l,
              world, per);
    if (seen[(size_t)r * per + l]++)
      RV_FAIL(RV_ERR_INVALID_ARGUMENT, "ep_check_placement: rank %u local %u holds two experts", r, l);
  }
  return RV_OK;
}

extern "C" int rv_ep_counts(const rv_ep *ep, uint32_t *received, size_t len) {
  if (!ep || !received) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "ep_counts: null pointer");
  if (len < ep->world) RV_FAIL(RV_ERR_LENGTH_MISMATCH, "ep_counts: %zu entries for %u ranks", len, ep->world);
  int prev = -1;
  RV_CUDA(cudaGetDevice(&prev));
  RV_CUDA(cudaSetDevice(ep->m->device));
  const cudaError_t e = cudaMemcpy(received, ep->window + ep->A.o_cnt, ep->world * 4, cudaMemcpyDeviceToHost);
  cudaSetDevice(prev);
  if (e != cudaSuccess) RV_FAIL(RV_ERR_CUDA, "ep_counts: %s", cudaGetErrorString(e));
  return RV_OK;
}

extern "C" int rv_moe_forward_host(rv_moe *m, const rv_expert_table *table, uint32_t layer,
                                   const float *ffn_norm, const float *router, float *residual_host,
                                   size_t n_tokens, uint32_t *topk_ids_host, float *topk_weights_host,
                                   uint32_t flags, rv_stream stream) {
  if (!m) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "moe_forward_host: null engine");
  if (n_tokens > m->max_tokens)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "moe_forward: %zu tokens vs engine capacity %zu", n_tokens, m->max_tokens);
  if (n_tokens == 0) return RV_OK;
  if (!residual_host) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "moe_forward_host: null residual");
  cudaStream_t s = (cudaStream_t)stream;
  const MoeDims &d = m->d;
  float *dres = m->dres;
  const size_t rbytes = n_tokens * (size_t)d.H * 4;
  RV_CUDA(cudaMemcpyAsync(dres, residual_host, rbytes, cudaMemcpyHostToDevice, s));
  int rc = rv_moe_forward(m, table, layer, ffn_norm, router, dres, n_tokens, nullptr, nullptr, flags, stream);
  if (rc) return rc;
  RV_CUDA(cudaMemcpyAsync(residual_host, dres, rbytes, cudaMemcpyDeviceToHost, s));
  if (topk_ids_host) RV_CUDA(cudaMemcpyAsync(topk_ids_host, m->B.ids, n_tokens * d.K * 4, cudaMemcpyDeviceToHost, s));
  if (topk_weights_host) RV_CUDA(cudaMemcpyAsync(topk_weights_host, m->B.w, n_tokens * d.K * 4, cudaMemcpyDeviceToHost, s));
  RV_CUDA(cudaStreamSynchronize(s));
  return RV_OK;
}

extern "C" int rv_moe_get_taps(const rv_moe *m, rv_moe_taps *o) {
  if (!m || !o) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "null pointer");
  o->normed = m->B.normed;
  o->acts = (const rv_block_q8k *)m->B.acts;
  o->acts_stride = m->d.act_stride;
  o->logits = m->B.logits;
  o->weights = m->B.w;
  o->ids = m->B.ids;
  o->index = m->B.index;
  o->index_start = m->B.index_start;
  o->swiglu = m->B.hbuf;
  o->acts_moe = m->B.acts_moe;
  o->acts_moe_stride = m->d.amoe_stride;
  o->staged = m->B.staged;
  o->logit_bounds = (const float *)m->B.spec;
  return RV_OK;
}

// ==================================================== synthetic inputs
// ============================================================ attention
// rope.rs:30-45: inv_freq = theta^(-2i/dim) and the angle in f64 (host
// libm pow), cos and sin of the angle (host libm), rounded to f32.
static void rope_inv_freq(size_t hd, float theta, std::vector<double> &inv) {
  const double base = (double)theta, dim = (double)hd;
  inv.resize(hd / 2);
  for (size_t i = 0; i < hd / 2; i++) inv[i] = pow(base, -2.0 * (double)i / dim);
}
static void rope_row(const std::vector<double> &inv, uint32_t position, float2 *out) {
  const double pos = (double)position;
  for (size_t i = 0; i < inv.size(); i++) {
    const double ang = pos * inv[i];
    out[i] = make_float2((float)cos(ang), (float)sin(ang));
  }
}

struct rv_attn {
  int device = 0;
  rv_attn_config cfg{};
  uint16_t *k_cache = nullptr, *v_cache = nullptr;
  float2 *rot = nullptr;
  float *scratch = nullptr;
  std::vector<uint32_t> lens;
  float scale = 0.0f;
  size_t plane = 0;  // halves per layer and cache
  // rv_attn_block scratch (cfg.hidden > 0)
  uint8_t *acts_k = nullptr, *acts_0 = nullptr, *acts_attn = nullptr;
  float *q = nullptr, *k = nullptr, *v = nullptr, *attn_out = nullptr;
};

extern "C" void rv_attn_destroy(rv_attn *a) {
  if (!a) return;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(a->device);
  cudaFree(a->k_cache);
  cudaFree(a->v_cache);
  cudaFree(a->rot);
  cudaFree(a->scratch);
  cudaFree(a->acts_k);
  cudaFree(a->acts_0);
  cudaFree(a->acts_attn);
  cudaFree(a->q);
  cudaFree(a->k);
  cudaFree(a->v);
  cudaFree(a->attn_out);
  if (prev >= 0) cudaSetDevice(prev);
  cudaGetLastError();  // a void call: leave no error behind for the caller's next check
  delete a;
}

extern "C" int rv_attn_create(int device, const rv_attn_config *cfg, rv_attn **out) {
  if (!cfg || !out) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "rv_attn_create: null argument");
  *out = nullptr;
  const rv_attn_config c = *cfg;
  if (c.head_dim == 0 || c.head_dim % 2) RV_FAIL(RV_ERR_INVALID_HEAD_DIM, "head_dim %u", c.head_dim);
  if (c.head_dim % 8 || c.head_dim > 256)
    RV_FAIL(RV_ERR_UNIMPLEMENTED, "head_dim %u: the kernels take multiples of 8 up to 256", c.head_dim);
  if (c.n_layers == 0 || c.n_heads == 0 || c.n_kv_heads == 0 || c.max_positions == 0)
    RV_FAIL(RV_ERR_EMPTY, "rv_attn_create: zero layers, heads or positions");
  if (c.n_heads % c.n_kv_heads)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "n_heads %u is not a multiple of n_kv_heads %u", c.n_heads, c.n_kv_heads);
  if (c.max_positions > (1u << 20)) RV_FAIL(RV_ERR_UNIMPLEMENTED, "max_positions %u > 2^20", c.max_positions);
  if (c.hidden % 256 || c.hidden > 16384)
    RV_FAIL(RV_ERR_INDIVISIBLE_ROW, "hidden %u: a multiple of 256 up to 16384 (0 for no block scratch)", c.hidden);
  if (c.hidden && ((c.n_heads * c.head_dim) % 256))
    RV_FAIL(RV_ERR_INDIVISIBLE_ROW, "n_heads * head_dim %u is not a multiple of 256", c.n_heads * c.head_dim);
  int rc = ensure_device(device);
  if (rc) return rc;
  int prev = -1;
  RV_CUDA(cudaGetDevice(&prev));
  RV_CUDA(cudaSetDevice(device));
  rv_attn *a = new rv_attn;
  a->device = device;
  a->cfg = c;
  a->lens.assign(c.n_layers, 0);
  a->scale = 1.0f / sqrtf((float)c.head_dim);  // model/forward.rs:2475
  a->plane = (size_t)c.max_positions * c.n_kv_heads * c.head_dim;
  const size_t half = c.head_dim / 2;
  cudaError_t e = cudaMalloc(&a->k_cache, 2 * a->plane * c.n_layers);
  if (e == cudaSuccess) e = cudaMalloc(&a->v_cache, 2 * a->plane * c.n_layers);
  if (e == cudaSuccess) e = cudaMalloc(&a->rot, sizeof(float2) * half * c.max_positions);
  if (e == cudaSuccess) e = cudaMalloc(&a->scratch, sizeof(float) * 2 * (size_t)c.n_heads * c.max_positions);
  if (e == cudaSuccess && c.hidden) {
    const size_t qd = (size_t)c.n_heads * c.head_dim, kvd = (size_t)c.n_kv_heads * c.head_dim;
    e = cudaMalloc(&a->acts_k, c.hidden / 256 * 292);
    if (e == cudaSuccess) e = cudaMalloc(&a->acts_0, c.hidden / 32 * 36);
    if (e == cudaSuccess) e = cudaMalloc(&a->acts_attn, qd / 256 * 292);
    if (e == cudaSuccess) e = cudaMalloc(&a->q, qd * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&a->k, kvd * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&a->v, kvd * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&a->attn_out, qd * sizeof(float));
  }
  if (e == cudaSuccess) {
    std::vector<double> inv;
    rope_inv_freq(c.head_dim, c.rope_theta, inv);
    std::vector<float2> table(half * c.max_positions);
    for (uint32_t p = 0; p < c.max_positions; p++) rope_row(inv, p, table.data() + (size_t)p * half);
    e = cudaMemcpy(a->rot, table.data(), sizeof(float2) * table.size(), cudaMemcpyHostToDevice);
  }
  cudaSetDevice(prev);
  if (e != cudaSuccess) {
    rv_attn_destroy(a);
    RV_FAIL(RV_ERR_CUDA, "rv_attn_create: %s", cudaGetErrorString(e));
  }
  *out = a;
  return RV_OK;
}

extern "C" int rv_attn_len(const rv_attn *a, uint32_t layer, uint32_t *len_out) {
  if (!a || !len_out) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "rv_attn_len: null argument");
  if (layer >= a->cfg.n_layers) RV_FAIL(RV_ERR_LAYER_OUT_OF_RANGE, "layer %u of %u", layer, a->cfg.n_layers);
  *len_out = a->lens[layer];
  return RV_OK;
}

extern "C" int rv_attn_clear(rv_attn *a) {
  if (!a) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "rv_attn_clear: null engine");
  std::fill(a->lens.begin(), a->lens.end(), 0u);
  return RV_OK;
}

extern "C" int rv_attn_cache(const rv_attn *a, uint32_t layer, const uint16_t **k_out, const uint16_t **v_out) {
  if (!a) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "rv_attn_cache: null engine");
  if (layer >= a->cfg.n_layers) RV_FAIL(RV_ERR_LAYER_OUT_OF_RANGE, "layer %u of %u", layer, a->cfg.n_layers);
  if (k_out) *k_out = a->k_cache + (size_t)layer * a->plane;
  if (v_out) *v_out = a->v_cache + (size_t)layer * a->plane;
  return RV_OK;
}

extern "C" int rv_attn_copy_cache(const rv_attn *a, uint32_t layer, uint32_t positions, uint16_t *k_out,
                                  uint16_t *v_out, rv_stream stream) {
  if (!a) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "rv_attn_copy_cache: null engine");
  if (layer >= a->cfg.n_layers) RV_FAIL(RV_ERR_LAYER_OUT_OF_RANGE, "layer %u of %u", layer, a->cfg.n_layers);
  if (positions > a->cfg.max_positions)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "%u positions of a %u-position cache", positions, a->cfg.max_positions);
  const size_t bytes = 2 * (size_t)positions * a->cfg.n_kv_heads * a->cfg.head_dim;
  if (bytes == 0) return RV_OK;
  cudaStream_t s = (cudaStream_t)stream;
  if (k_out) RV_CUDA(cudaMemcpyAsync(k_out, a->k_cache + (size_t)layer * a->plane, bytes, cudaMemcpyDeviceToDevice, s));
  if (v_out) RV_CUDA(cudaMemcpyAsync(v_out, a->v_cache + (size_t)layer * a->plane, bytes, cudaMemcpyDeviceToDevice, s));
  return RV_OK;
}

// Scores and softmax-out over positions 0..args.position, shared by
// rv_attn_decode and rv_attention.
// The Q8_K of the attention output is formed inside the softmax-out kernel
// when two heads of 128 (one Q8_K block) share a CTA and a kv head.
static bool attn_fold_q8k(const AttnArgs &args) {
  return args.q8k_out && args.hd == 128 && (args.n_heads / args.n_kv) % 2 == 0;
}

static int attn_launch_core(const AttnArgs &args, cudaStream_t s, bool fused_prep = false) {
  // Host mode: one 128-position tile per CTA row.  Device mode (the
  // position known only when the kernels run): up to 16 tile rows that
  // stride over the positions.
  const int positions = args.pos_dev ? args.max_positions : args.position + 1;
  const int tiles = (positions + 127) / 128;
  dim3 grid((unsigned)args.n_heads, (unsigned)(args.pos_dev ? std::min(tiles, 16) : tiles));
  // The attention block's whole attention in one launch per head pair
  // (k_attn_fused) up to RV_ATTN_FUSED_MAX positions (the position of a
  // host-driven call; the cache's capacity when the position is read on the
  // device).  Its scores run on n_heads / 2 CTAs: measured on the Qwen3
  // geometry, 2.61 against 2.79 ms per decode step at positions 64-127,
  // 3.42 against 3.30 ms at 512-575.
  if (fused_prep && attn_fold_q8k(args) && positions <= RV_ATTN_FUSED_MAX) {
    k_attn_fused<<<(unsigned)args.n_heads / 2, 256, attn_fused_smem(positions), s>>>(args);
    RV_LAUNCH_CHECK();
    return RV_OK;
  }
  if (fused_prep)
    k_attn_scores_prep<<<grid, 128, 34 * sizeof(double) + 2 * args.hd * sizeof(float), s>>>(args);
  else
    k_attn_scores<<<grid, 128, args.hd * sizeof(float), s>>>(args);
  if (attn_fold_q8k(args))
    k_attn_softmax_out<2><<<(unsigned)args.n_heads / 2, 256, attn_out_smem(args.hd, 2), s>>>(args);
  else
    k_attn_softmax_out<1><<<(unsigned)args.n_heads, args.hd > 128 ? args.hd : 128, attn_out_smem(args.hd), s>>>(args);
  RV_LAUNCH_CHECK();
  return RV_OK;
}

extern "C" int rv_attn_decode(rv_attn *a, uint32_t layer, uint32_t position, float *q, float *k, const float *v,
                              const float *q_norm, const float *k_norm, float *out, rv_stream stream) {
  if (!a) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "rv_attn_decode: null engine");
  const rv_attn_config &c = a->cfg;
  if (layer >= c.n_layers) RV_FAIL(RV_ERR_LAYER_OUT_OF_RANGE, "layer %u of %u", layer, c.n_layers);
  if (position != a->lens[layer])
    RV_FAIL(RV_ERR_POSITION_MISMATCH, "position %u, layer %u holds %u", position, layer, a->lens[layer]);
  if (position >= c.max_positions)
    RV_FAIL(RV_ERR_CAPACITY_EXCEEDED, "layer %u is full (%u positions)", layer, c.max_positions);
  if (!q || !k || !v || !q_norm || !k_norm || !out)
    RV_FAIL(RV_ERR_INVALID_ARGUMENT, "rv_attn_decode: null pointer");
  int prev = -1;
  RV_CUDA(cudaGetDevice(&prev));
  if (prev != a->device) RV_CUDA(cudaSetDevice(a->device));
  AttnArgs args{};
  args.q = q;
  args.k = k;
  args.v = v;
  args.q_norm = q_norm;
  args.k_norm = k_norm;
  args.k_cache = a->k_cache + (size_t)layer * a->plane;
  args.v_cache = a->v_cache + (size_t)layer * a->plane;
  args.rot = a->rot;
  args.scores = a->scratch;
  args.probs = a->scratch + (size_t)c.n_heads * c.max_positions;
  args.out = out;
  args.n_heads = (int)c.n_heads;
  args.n_kv = (int)c.n_kv_heads;
  args.hd = (int)c.head_dim;
  args.position = (int)position;
  args.pos_dev = nullptr;
  args.max_positions = (int)c.max_positions;
  args.eps = c.eps;
  args.scale = a->scale;
  cudaStream_t s = (cudaStream_t)stream;
  k_attn_prep<<<c.n_heads + c.n_kv_heads, c.head_dim, 34 * sizeof(double) + c.head_dim * sizeof(float), s>>>(args);
  int rc = attn_launch_core(args, s);
  if (prev != a->device) cudaSetDevice(prev);
  if (rc) return rc;
  a->lens[layer] = position + 1;
  return RV_OK;
}

// One GEMV job of the multi-job launch: whole matrix, one activation row.
static GemvArgs gemv_job(const uint8_t *w, size_t row_bytes, int nb, size_t rows, const uint8_t *acts, float *out,
                         int R) {
  GemvArgs g{};
  g.w = w;
  g.row_bytes = row_bytes;
  g.nb = nb;
  g.r0 = 0;
  g.nrows = rows;
  g.acts = acts;
  g.n_acts = 1;
  g.out = out;
  g.R = R;
  g.accumulate = 0;
  return g;
}

extern "C" int rv_rmsnorm_quantize(const float *x, const float *w, size_t n, float eps, rv_block_q8k *q8k_out,
                                   rv_block_q8_0 *q80_out, rv_stream stream) {
  if (n == 0) RV_FAIL(RV_ERR_EMPTY, "rmsnorm_quantize: empty row");
  if (n % 256 || n > 16384) RV_FAIL(RV_ERR_QUANTIZE_LEN_MISMATCH, "rmsnorm_quantize: n %zu (multiples of 256 <= 16384)", n);
  if (!x || !w || !q8k_out || ((uintptr_t)q8k_out & 3) || ((uintptr_t)q80_out & 3))
    RV_FAIL(RV_ERR_INVALID_ARGUMENT, "rmsnorm_quantize: null or misaligned pointer");
  int rc = ensure_current_device();
  if (rc) return rc;
  const size_t smem = 34 * sizeof(double) + (n + 256) * sizeof(float);
  k_norm_quant<<<(unsigned)(n / 256), 256, smem, (cudaStream_t)stream>>>(x, w, (int)n, eps, (uint8_t *)q8k_out,
                                                                         (uint8_t *)q80_out);
  RV_LAUNCH_CHECK();
  return RV_OK;
}

extern "C" int rv_attn_block(rv_attn *a, uint32_t layer, const rv_attn_weights *w, float *residual,
                             const int32_t *position_dev, uint32_t position, rv_stream stream) {
  if (!a || !w || !residual) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "rv_attn_block: null argument");
  const rv_attn_config &c = a->cfg;
  if (!c.hidden) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "rv_attn_block: the engine was created with hidden = 0");
  if (layer >= c.n_layers) RV_FAIL(RV_ERR_LAYER_OUT_OF_RANGE, "layer %u of %u", layer, c.n_layers);
  if (!w->attn_norm || !w->attn_q || !w->attn_k || !w->attn_v || !w->attn_output || !w->q_norm || !w->k_norm)
    RV_FAIL(RV_ERR_INVALID_ARGUMENT, "rv_attn_block: null weight");
  for (int f : {w->attn_q_format, w->attn_v_format, w->attn_output_format})
    if (!rv_fmt_is_kquant(f)) RV_FAIL(RV_ERR_UNSUPPORTED_FORMAT, "rv_attn_block: weight format %d", f);
  if (!position_dev) {
    if (position != a->lens[layer])
      RV_FAIL(RV_ERR_POSITION_MISMATCH, "position %u, layer %u holds %u", position, layer, a->lens[layer]);
    if (position >= c.max_positions)
      RV_FAIL(RV_ERR_CAPACITY_EXCEEDED, "layer %u is full (%u positions)", layer, c.max_positions);
  } else if ((uintptr_t)position_dev & 3) {
    RV_FAIL(RV_ERR_INVALID_ARGUMENT, "rv_attn_block: misaligned position pointer");
  }
  int prev = -1;
  RV_CUDA(cudaGetDevice(&prev));
  if (prev != a->device) RV_CUDA(cudaSetDevice(a->device));
  cudaStream_t s = (cudaStream_t)stream;
  const size_t H = c.hidden, qd = (size_t)c.n_heads * c.head_dim, kvd = (size_t)c.n_kv_heads * c.head_dim;
  // 1. attn_norm -> Q8_K and Q8_0 of the normed row
  k_norm_quant<<<(unsigned)(H / 256), 256, 34 * sizeof(double) + (H + 256) * sizeof(float), s>>>(
      residual, w->attn_norm, (int)H, c.eps, a->acts_k, a->acts_0);
  // 2. q, k, v projections in one launch of 256-thread CTAs: 8 rows per CTA
  // for the warp-per-row tiles (gemv_wide_nbg), 32 for the others.
  const int TPB = 256;
  auto rows_per_cta = [&](int fmt, int nb) { return gemv_wide_nbg(fmt, nb) ? TPB / 32 : TPB / 8; };
  GemvMulti m{};
  const size_t rb_q = H / 256 * rv_fmt_block_bytes(w->attn_q_format);
  const size_t rb_v = H / 256 * rv_fmt_block_bytes(w->attn_v_format);
  const size_t rb_k = H / 32 * 34;
  const int nb_k = (int)(H / 256), nb_0 = (int)(H / 32);
  m.job[0] = gemv_job(w->attn_q, rb_q, nb_k, qd, a->acts_k, a->q, rows_per_cta(w->attn_q_format, nb_k));
  m.fmt[0] = w->attn_q_format;
  m.job[1] = gemv_job(w->attn_k, rb_k, nb_0, kvd, a->acts_0, a->k, rows_per_cta(RV_Q8_0, nb_0));
  m.fmt[1] = RV_Q8_0;
  m.job[2] = gemv_job(w->attn_v, rb_v, nb_k, kvd, a->acts_k, a->v, rows_per_cta(w->attn_v_format, nb_k));
  m.fmt[2] = w->attn_v_format;
  m.n = 3;
  m.cta0[0] = 0;
  size_t smem = 0;
  for (int j = 0; j < 3; j++) {
    const GemvArgs &g = m.job[j];
    m.cta0[j + 1] = m.cta0[j] + (unsigned)((g.nrows + g.R - 1) / g.R);
    const size_t act_row = m.fmt[j] == RV_Q8_0 ? (size_t)g.nb * 36 : (size_t)g.nb * 292;
    smem = std::max(smem, gemv_tile_smem(g.R, g.row_bytes, act_row));
  }
  k_gemv_multi<<<m.cta0[3], TPB, smem, s>>>(m);
  // 3. QK-norm, RoPE, append, attention
  AttnArgs args{};
  args.q = a->q;
  args.k = a->k;
  args.v = a->v;
  args.q_norm = w->q_norm;
  args.k_norm = w->k_norm;
  args.k_cache = a->k_cache + (size_t)layer * a->plane;
  args.v_cache = a->v_cache + (size_t)layer * a->plane;
  args.rot = a->rot;
  args.scores = a->scratch;
  args.probs = a->scratch + (size_t)c.n_heads * c.max_positions;
  args.out = a->attn_out;
  args.q8k_out = a->acts_attn;  // the block quantizes the output in the softmax-out kernel where it can
  args.n_heads = (int)c.n_heads;
  args.n_kv = (int)c.n_kv_heads;
  args.hd = (int)c.head_dim;
  args.position = (int)position;
  args.pos_dev = position_dev;
  args.max_positions = (int)c.max_positions;
  args.eps = c.eps;
  args.scale = a->scale;
  int rc = attn_launch_core(args, s, /*fused_prep=*/true);
  if (rc) {
    if (prev != a->device) cudaSetDevice(prev);
    return rc;
  }
  // 4. Q8_K of the attention output, 5. attn_output + residual add
  if (!attn_fold_q8k(args))
    k_quantize_q8k<<<(unsigned)((qd / 256 + 7) / 8), 256, 0, s>>>(a->attn_out, a->acts_attn, qd / 256);
  GemvArgs g = gemv_job(w->attn_output, qd / 256 * rv_fmt_block_bytes(w->attn_output_format), (int)(qd / 256), H,
                        a->acts_attn, residual, 4);
  g.accumulate = 1;
  switch (w->attn_output_format) {
    case RV_Q4_K: launch_gemv<RV_Q4_K>(g, s); break;
    case RV_Q5_K: launch_gemv<RV_Q5_K>(g, s); break;
    default: launch_gemv<RV_Q6_K>(g, s); break;
  }
  RV_LAUNCH_CHECK();
  if (prev != a->device) cudaSetDevice(prev);
  if (!position_dev) a->lens[layer] = position + 1;
  return RV_OK;
}

extern "C" int rv_rope_neox_heads(float *x, size_t x_len, size_t n_heads, size_t head_dim, uint32_t position,
                                  float theta, rv_stream stream) {
  if (head_dim == 0 || head_dim % 2) RV_FAIL(RV_ERR_INVALID_HEAD_DIM, "rope_neox_heads: head_dim %zu", head_dim);
  if (x_len != sat_mul(n_heads, head_dim))
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "rope_neox_heads: x vs n_heads * head_dim (%zu vs %zu)", x_len,
            sat_mul(n_heads, head_dim));
  if (head_dim / 2 > RV_ROPE_MAX_HALF) RV_FAIL(RV_ERR_UNIMPLEMENTED, "rope_neox_heads: head_dim %zu > 512", head_dim);
  if (x_len == 0) return RV_OK;
  if (!x || ((uintptr_t)x & 3)) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "rope_neox_heads: null or misaligned x");
  int rc = ensure_current_device();
  if (rc) return rc;
  std::vector<double> inv;
  rope_inv_freq(head_dim, theta, inv);
  RopeFactors f;
  rope_row(inv, position, f.cs);
  const size_t pairs = n_heads * (head_dim / 2);
  k_rope_heads<<<(unsigned)((pairs + 255) / 256), 256, 0, (cudaStream_t)stream>>>(x, (int)n_heads, (int)head_dim, f);
  RV_LAUNCH_CHECK();
  return RV_OK;
}

extern "C" int rv_attention(const float *q, const uint16_t *k_cache, const uint16_t *v_cache, size_t positions,
                            size_t n_heads, size_t n_kv_heads, size_t head_dim, float scale, float *scratch,
                            size_t scratch_len, float *out, rv_stream stream) {
  if (positions == 0 || n_heads == 0 || n_kv_heads == 0) RV_FAIL(RV_ERR_EMPTY, "attention: nothing to attend");
  if (head_dim == 0 || head_dim % 2) RV_FAIL(RV_ERR_INVALID_HEAD_DIM, "attention: head_dim %zu", head_dim);
  if (head_dim % 8 || head_dim > 256)
    RV_FAIL(RV_ERR_UNIMPLEMENTED, "attention: head_dim %zu (multiples of 8 up to 256)", head_dim);
  if (n_heads % n_kv_heads)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "attention: %zu query heads over %zu kv heads", n_heads, n_kv_heads);
  if (positions > (1u << 20)) RV_FAIL(RV_ERR_UNIMPLEMENTED, "attention: %zu positions > 2^20", positions);
  if (scratch_len < sat_mul(2 * n_heads, positions))
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "attention: scratch of %zu floats, needs %zu", scratch_len,
            sat_mul(2 * n_heads, positions));
  if (!q || !k_cache || !v_cache || !scratch || !out || ((uintptr_t)k_cache & 15) || ((uintptr_t)v_cache & 15))
    RV_FAIL(RV_ERR_INVALID_ARGUMENT, "attention: null pointer or caches not 16-byte aligned");
  int rc = ensure_current_device();
  if (rc) return rc;
  AttnArgs args{};
  args.q8k_out = nullptr;
  args.q = const_cast<float *>(q);
  args.k_cache = const_cast<uint16_t *>(k_cache);
  args.v_cache = const_cast<uint16_t *>(v_cache);
  args.scores = scratch;
  args.probs = scratch + n_heads * positions;
  args.out = out;
  args.n_heads = (int)n_heads;
  args.n_kv = (int)n_kv_heads;
  args.hd = (int)head_dim;
  args.position = (int)positions - 1;
  args.pos_dev = nullptr;
  args.max_positions = (int)positions;
  args.scale = scale;
  return attn_launch_core(args, (cudaStream_t)stream);
}

extern "C" int rv_attn_decode_dev(rv_attn *a, uint32_t layer, const int32_t *position_dev, float *q, float *k,
                                  const float *v, const float *q_norm, const float *k_norm, float *out,
                                  rv_stream stream) {
  if (!a) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "rv_attn_decode_dev: null engine");
  const rv_attn_config &c = a->cfg;
  if (layer >= c.n_layers) RV_FAIL(RV_ERR_LAYER_OUT_OF_RANGE, "layer %u of %u", layer, c.n_layers);
  if (!position_dev || !q || !k || !v || !q_norm || !k_norm || !out || ((uintptr_t)position_dev & 3))
    RV_FAIL(RV_ERR_INVALID_ARGUMENT, "rv_attn_decode_dev: null or misaligned pointer");
  int prev = -1;
  RV_CUDA(cudaGetDevice(&prev));
  if (prev != a->device) RV_CUDA(cudaSetDevice(a->device));
  AttnArgs args{};
  args.q = q;
  args.k = k;
  args.v = v;
  args.q_norm = q_norm;
  args.k_norm = k_norm;
  args.k_cache = a->k_cache + (size_t)layer * a->plane;
  args.v_cache = a->v_cache + (size_t)layer * a->plane;
  args.rot = a->rot;
  args.scores = a->scratch;
  args.probs = a->scratch + (size_t)c.n_heads * c.max_positions;
  args.out = out;
  args.n_heads = (int)c.n_heads;
  args.n_kv = (int)c.n_kv_heads;
  args.hd = (int)c.head_dim;
  args.position = 0;
  args.pos_dev = position_dev;
  args.max_positions = (int)c.max_positions;
  args.eps = c.eps;
  args.scale = a->scale;
  cudaStream_t s = (cudaStream_t)stream;
  k_attn_prep<<<c.n_heads + c.n_kv_heads, c.head_dim, 34 * sizeof(double) + c.head_dim * sizeof(float), s>>>(args);
  int rc = attn_launch_core(args, s);
  if (prev != a->device) cudaSetDevice(prev);
  return rc;
}

extern "C" int rv_decode_advance(int32_t *position_dev, const uint32_t *next_token, int32_t *token,
                                 uint32_t *ids_out, size_t ids_cap, rv_stream stream) {
  if (!position_dev || ((uintptr_t)position_dev & 3)) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "rv_decode_advance: bad pointer");
  k_decode_advance<<<1, 1, 0, (cudaStream_t)stream>>>(position_dev, next_token, token, ids_out,
                                                      (int)std::min(ids_cap, (size_t)INT32_MAX));
  RV_LAUNCH_CHECK();
  return RV_OK;
}

extern "C" int rv_argmax(const float *x, size_t n, uint32_t *out, rv_stream stream) {
  if (n == 0) RV_FAIL(RV_ERR_EMPTY, "argmax: no logits");
  if (!x || !out || ((uintptr_t)x & 3) || ((uintptr_t)out & 3)) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "argmax: bad pointer");
  k_argmax<<<1, 1024, 0, (cudaStream_t)stream>>>(x, n, out);
  RV_LAUNCH_CHECK();
  return RV_OK;
}

extern "C" int rv_vec_add(float *a, const float *b, size_t n, rv_stream stream) {
  if (n == 0) return RV_OK;
  if (!a || !b) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "vec_add: null pointer");
  k_vec_add<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(a, b, n);
  RV_LAUNCH_CHECK();
  return RV_OK;
}

extern "C" int rv_synth_normal(uint64_t seed, uint64_t offset, float sigma, float *out, size_t n,
                               rv_stream stream) {
  if (n == 0) return RV_OK;
  if (!out) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "synth_normal: null pointer");
  k_synth_normal<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(seed, offset, sigma, out, n);
  RV_LAUNCH_CHECK();
  return RV_OK;
}

extern "C" int rv_quantize_weights(int format, const float *x, size_t n, uint8_t *out, rv_stream stream) {
  if (!rv_fmt_is_kquant(format)) RV_FAIL(RV_ERR_UNSUPPORTED_FORMAT, "quantize_weights: format %d", format);
  if (n % 256) RV_FAIL(RV_ERR_INDIVISIBLE_ROW, "quantize_weights: %zu weights", n);
  if (n == 0) return RV_OK;
  if (!x || !out) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "quantize_weights: null pointer");
  const size_t nb = n / 256;
  const unsigned grid = (unsigned)((nb + 127) / 128);
  cudaStream_t s = (cudaStream_t)stream;
  if (format == RV_Q4_K) k_quantize_weights<RV_Q4_K><<<grid, 128, 0, s>>>(x, out, nb);
  else if (format == RV_Q5_K) k_quantize_weights<RV_Q5_K><<<grid, 128, 0, s>>>(x, out, nb);
  else k_quantize_weights<RV_Q6_K><<<grid, 128, 0, s>>>(x, out, nb);
  RV_LAUNCH_CHECK();
  return RV_OK;
}

extern "C" int rv_expert_table_fill_synthetic(rv_expert_table *t, uint32_t layer, uint64_t seed, float sigma,
                                              rv_stream stream) {
  return rv_expert_table_fill_synthetic_strided(t, layer, seed, sigma, 0, 1, stream);
}

// Local expert ex of the layer gets global expert ge(ex)'s weights.
template <typename GE>
static int fill_synthetic(rv_expert_table *t, uint32_t layer, uint64_t seed, float sigma, GE ge_of, rv_stream stream);

extern "C" int rv_expert_table_fill_synthetic_strided(rv_expert_table *t, uint32_t layer, uint64_t seed, float sigma,
                                                      uint32_t first_expert, uint32_t expert_step, rv_stream stream) {
  if (!t) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "null table");
  if (expert_step == 0) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "fill_synthetic: expert_step 0");
  return fill_synthetic(t, layer, seed, sigma,
                        [&](uint32_t ex) { return (uint64_t)first_expert + (uint64_t)ex * expert_step; }, stream);
}

extern "C" int rv_expert_table_fill_synthetic_list(rv_expert_table *t, uint32_t layer, uint64_t seed, float sigma,
                                                   const uint32_t *experts, size_t n, rv_stream stream) {
  if (!t || !experts) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "fill_synthetic_list: null pointer");
  if (layer >= t->layouts.size()) RV_FAIL(RV_ERR_LAYER_OUT_OF_RANGE, "layer %u of %zu", layer, t->layouts.size());
  if (n != t->layouts[layer].n_experts)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "fill_synthetic_list: %zu experts for a layer of %u", n,
            t->layouts[layer].n_experts);
  return fill_synthetic(t, layer, seed, sigma, [&](uint32_t ex) { return (uint64_t)experts[ex]; }, stream);
}

template <typename GE>
static int fill_synthetic(rv_expert_table *t, uint32_t layer, uint64_t seed, float sigma, GE ge_of, rv_stream stream) {
  if (layer >= t->layouts.size()) RV_FAIL(RV_ERR_LAYER_OUT_OF_RANGE, "layer %u of %zu", layer, t->layouts.size());
  const rv_layer_layout &L = t->layouts[layer];
  const size_t mh = (size_t)L.moe * L.hidden;
  int prev = -1;
  RV_CUDA(cudaGetDevice(&prev));
  RV_CUDA(cudaSetDevice(t->device));
  float *tmp = nullptr;
  cudaError_t e = cudaMalloc(&tmp, 3 * mh * sizeof(float));
  if (e != cudaSuccess) {
    cudaSetDevice(prev);
    RV_FAIL(RV_ERR_CUDA, "fill_synthetic scratch: %s", cudaGetErrorString(e));
  }
  int rc = RV_OK;
  cudaStream_t s = (cudaStream_t)stream;
  for (uint32_t ex = 0; ex < L.n_experts && rc == RV_OK; ex++) {
    uint8_t *blob = t->base[layer] + (size_t)ex * L.stride;
    const uint64_t ge = ge_of(ex);  // global expert id
    rc = rv_synth_normal(seed, ge * 3 * mh, sigma, tmp, 3 * mh, stream);
    if (!rc) rc = rv_quantize_weights(L.gate_format, tmp, mh, blob + L.gate_off, stream);
    if (!rc) rc = rv_quantize_weights(L.up_format, tmp + mh, mh, blob + L.up_off, stream);
    if (!rc) rc = rv_quantize_weights(L.down_format, tmp + 2 * mh, mh, blob + L.down_off, stream);
  }
  e = cudaStreamSynchronize(s);
  cudaFree(tmp);
  cudaSetDevice(prev);
  if (rc) return rc;
  if (e != cudaSuccess) RV_FAIL(RV_ERR_CUDA, "fill_synthetic: %s", cudaGetErrorString(e));
  return RV_OK;
}

#ifdef RV_PHASE_CLOCK
// Copies the phase clocks of kernel k (0 route, 1 gate_up, 2 down) to out
// ([RV_PHASE_CTAS][RV_PHASES] int64) and clears them.
extern "C" __attribute__((visibility("default"))) int rv_debug_phase_clock(int k, long long *out) {
  if (k < 0 || k >= RV_PHASE_KERNELS || !out) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "phase clock slot %d", k);
  RV_CUDA(cudaDeviceSynchronize());
  RV_CUDA(cudaMemcpyFromSymbol(out, g_rv_phase, sizeof(long long) * RV_PHASE_CTAS * RV_PHASES,
                               sizeof(long long) * RV_PHASE_CTAS * RV_PHASES * k));
  static long long zero[RV_PHASE_CTAS * RV_PHASES];
  RV_CUDA(cudaMemcpyToSymbol(g_rv_phase, zero, sizeof zero, sizeof(long long) * RV_PHASE_CTAS * RV_PHASES * k));
  return RV_OK;
}
#endif

// ================================================ allocation-free decode
// The MoE block for callers that cannot allocate device memory: every
// intermediate lives in this file-scope array.  Host code reaches it only
// through the address cudaGetSymbolAddress returns for the current device.
static __device__ __align__(256) uint8_t g_rv_static_scratch[RV_STATIC_SCRATCH_BYTES];
static std::mutex g_static_mu;
static void *g_static_ptr[64];

extern "C" int rv_moe_forward_static(const rv_moe_config *cfg, const rv_layer_layout *L,
                                     const uint8_t *expert_blobs, const float *ffn_norm,
                                     const float *router, float *residual, size_t n_tokens,
                                     uint32_t *topk_ids, float *topk_weights, rv_stream stream) {
  if (!cfg || !L) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "moe_forward_static: null config or layout");
  if (cfg->hidden == 0 || cfg->hidden % 256 || cfg->moe == 0 || cfg->moe % 256)
    RV_FAIL(RV_ERR_INDIVISIBLE_ROW, "hidden %u / moe %u: not multiples of 256", cfg->hidden, cfg->moe);
  if (cfg->hidden > 2048 || cfg->moe > 1024 || cfg->n_experts == 0 || cfg->n_experts > 128 ||
      cfg->top_k == 0 || cfg->top_k > 8 || cfg->top_k > cfg->n_experts)
    RV_FAIL(RV_ERR_UNIMPLEMENTED,
            "moe_forward_static handles hidden <= 2048, moe <= 1024, n_experts <= 128, top_k <= 8");
  if (n_tokens > RV_STATIC_MAX_TOKENS)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "moe_forward_static: %zu tokens exceed the static limit of %d",
            n_tokens, RV_STATIC_MAX_TOKENS);
  int rc = check_layout(*L, 0);
  if (rc) return rc;
  if (L->hidden != cfg->hidden || L->moe != cfg->moe || L->n_experts != cfg->n_experts)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "layout geometry (%u, %u, %u) vs config (%u, %u, %u)", L->hidden, L->moe,
            L->n_experts, cfg->hidden, cfg->moe, cfg->n_experts);
  if (L->gate_format != L->up_format) RV_FAIL(RV_ERR_UNIMPLEMENTED, "gate and up in different formats");
  if (n_tokens == 0) return RV_OK;
  if (!expert_blobs || !ffn_norm || !router || !residual)
    RV_FAIL(RV_ERR_INVALID_ARGUMENT, "moe_forward_static: null pointer");
  if ((uintptr_t)router & 15) RV_FAIL(RV_ERR_INVALID_ARGUMENT, "moe_forward_static: router must be 16-byte aligned");
  int dev = 0;
  RV_CUDA(cudaGetDevice(&dev));
  rc = ensure_device(dev);
  if (rc) return rc;
  uint8_t *base = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_static_mu);
    if (!g_static_ptr[dev]) {
      void *ptr = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&ptr, g_rv_static_scratch);
      if (e != cudaSuccess || !ptr)
        RV_FAIL(RV_ERR_CUDA, "moe_forward_static: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      g_static_ptr[dev] = ptr;
    }
    base = (uint8_t *)g_static_ptr[dev];
  }
  // The same geometry and scratch carving as rv_moe_create, for
  // RV_STATIC_MAX_TOKENS rows; counters first so one memset clears them.
  // Value-initialized: every buffer this path does not carve stays null.
  rv_moe m{};
  m.device = dev;
  m.cfg = *cfg;
  m.max_tokens = RV_STATIC_MAX_TOKENS;
  MoeDims &d = m.d;
  d.H = (int)cfg->hidden;
  d.M = (int)cfg->moe;
  d.E = (int)cfg->n_experts;
  d.K = (int)cfg->top_k;
  d.hb = d.H / 256;
  d.mb = d.M / 256;
  d.act_stride = round16((size_t)d.hb * 292);
  d.amoe_stride = round16((size_t)d.mb * 292);
  d.eps = cfg->eps;
  d.norm_topk = cfg->norm_topk_prob;
  const size_t T = RV_STATIC_MAX_TOKENS, K = d.K, P = T * K;
  m.max_units = (int)(std::min<size_t>((size_t)d.E, P) + (P + RV_MOE_TOK_CHUNK - 1) / RV_MOE_TOK_CHUNK);
  MoeBufs &B = m.B;
  struct Part { size_t bytes; void **slot; };
  const Part parts[] = {
      {(size_t)d.E * 4, (void **)&B.counts},
      {(size_t)m.max_units * d.mb * 4, (void **)&B.tile_cnt},
      {16, (void **)&B.route_cnt},
      {((size_t)d.H / 4 + 1) * 4, (void **)&B.down_cnt},  // as rv_moe_create: one per down row tile
      {16, (void **)&B.n_units},
      {T * d.H * 4, (void **)&B.normed},
      {T * d.act_stride, (void **)&B.acts},
      {T * d.E * 4, (void **)&B.logits},
      {P * 4, (void **)&B.ids},
      {P * 4, (void **)&B.w},
      {((size_t)d.E + 1) * 4, (void **)&B.index_start},
      {P * 4, (void **)&B.index},
      {(size_t)m.max_units * 16, (void **)&B.units},
      {P * d.M * 4, (void **)&B.hbuf},
      {P * d.amoe_stride, (void **)&B.acts_moe},
      {P * d.H * 4, (void **)&B.staged},
  };
  size_t off = 0, counters = 0;
  for (size_t i = 0; i < sizeof parts / sizeof parts[0]; i++) {
    *parts[i].slot = base + off;
    off += (parts[i].bytes + 255) & ~(size_t)255;
    if (i == 4) counters = off;
  }
  if (off > RV_STATIC_SCRATCH_BYTES)
    RV_FAIL(RV_ERR_LENGTH_MISMATCH, "moe_forward_static: needs %zu scratch bytes, has %u", off,
            (unsigned)RV_STATIC_SCRATCH_BYTES);
  B.max_units = m.max_units;
  cudaStream_t s = (cudaStream_t)stream;
  RV_CUDA(cudaMemsetAsync(base, 0, counters, s));
  B.ffn_norm = ffn_norm;
  B.router = router;
  B.residual = residual;
  B.T = (int)n_tokens;
  B.ms = B.T < RV_MOE_MT ? B.T : RV_MOE_MT;
  MoeWeights W;
  W.base = expert_blobs;
  W.stride = L->stride;
  W.gate_off = L->gate_off;
  W.up_off = L->up_off;
  W.down_off = L->down_off;
  rv_row_bytes(L->gate_format, L->hidden, &W.gu_row_bytes);
  rv_row_bytes(L->down_format, L->moe, &W.down_row_bytes);
  const int Tn = (int)n_tokens;
  // Shared memory padded past half an SM's, as in rv_moe_forward: no two
  // routing CTAs (each running one serial router chain) share an SM.
  const size_t need = 16 + (size_t)2 * d.H * 4 + (size_t)Tn * (d.H + 4) * 4 + 4 * (size_t)Tn * sizeof(double) + 16;
  const size_t smem = need < RV_ROUTE_SMEM_ONE_PER_SM ? RV_ROUTE_SMEM_ONE_PER_SM : need;
  RV_CUDA(launch_pdl(k_route_decode, dim3((unsigned)d.E), dim3(128), smem, s, d, B));
  switch (L->gate_format) {
    case RV_Q4_K: launch_gate_up<RV_Q4_K>(d, B, W, Tn, 0, s); break;
    case RV_Q5_K: launch_gate_up<RV_Q5_K>(d, B, W, Tn, 0, s); break;
    default: launch_gate_up<RV_Q6_K>(d, B, W, Tn, 0, s); break;
  }
  bool combined;
  switch (L->down_format) {
    case RV_Q4_K: combined = launch_down<RV_Q4_K>(d, B, W, Tn, true, 0, s); break;
    case RV_Q5_K: combined = launch_down<RV_Q5_K>(d, B, W, Tn, true, 0, s); break;
    default: combined = launch_down<RV_Q6_K>(d, B, W, Tn, true, 0, s); break;
  }
  if (!combined) k_combine<<<dim3((unsigned)Tn, (unsigned)((d.H + 255) / 256)), 256, 0, s>>>(d, B);
  RV_LAUNCH_CHECK();
  if (topk_ids) RV_CUDA(cudaMemcpyAsync(topk_ids, B.ids, n_tokens * d.K * 4, cudaMemcpyDeviceToDevice, s));
  if (topk_weights) RV_CUDA(cudaMemcpyAsync(topk_weights, B.w, n_tokens * d.K * 4, cudaMemcpyDeviceToDevice, s));
  return RV_OK;
}
