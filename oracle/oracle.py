"""ctypes front end of the CPU oracle (oracle/rv_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference legs.  The product (ramvamp_b200) never
imports it.  Every function restates the ramvamp Rust source cited in
rv_oracle.c; numpy arrays carry the data.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "librv_oracle.so")

Q4_K, Q5_K, Q6_K, Q8_0, Q8_K = 0, 1, 2, 3, 4
SCALAR, AVX2, LANES = 0, 1, 2
BLOCK_BYTES = {Q4_K: 144, Q5_K: 176, Q6_K: 210, Q8_0: 34, Q8_K: 292}

# BlockQ8K (blocks.rs:146-153) as a packed 292-byte record.
Q8K_DTYPE = np.dtype([("d", "<f4"), ("qs", "i1", (256,)), ("bsums", "<i2", (16,))])
assert Q8K_DTYPE.itemsize == 292
# BlockQ8_0 (blocks.rs:167-178): d (already f16-rounded) + 32 i8, 36 bytes.
Q8_0_DTYPE = np.dtype([("d", "<f4"), ("qs", "i1", (32,))])
assert Q8_0_DTYPE.itemsize == 36

ERRORS = {
    0: "Ok",
    1: "IndivisibleRow",
    2: "RowBytesNotBlockMultiple",
    3: "BlockCountMismatch",
    4: "QuantizeLenMismatch",
    5: "LengthMismatch",
    6: "Empty",
    7: "InvalidHeadDim",
    9: "UnsupportedFormat",
    20: "RoutedExpertOutOfRange",
}


class OracleError(RuntimeError):
    def __init__(self, code: int, what: str):
        super().__init__(f"{what}: {ERRORS.get(code, code)}")
        self.code = code
        self.kind = ERRORS.get(code, str(code))


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (system gcc, no fast-math)."""
    src = os.path.join(HERE, "rv_oracle.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-C", HERE, "-s"], check=True)
    return LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = ctypes.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


P = ctypes.c_void_p
SZ = ctypes.c_size_t
I32 = ctypes.c_int


class MoeLayer(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_uint32), ("moe", ctypes.c_uint32),
        ("n_experts", ctypes.c_uint32), ("top_k", ctypes.c_uint32),
        ("norm_topk_prob", ctypes.c_int32), ("eps", ctypes.c_float),
        ("ffn_norm", P), ("router", P), ("blobs", P), ("stride", ctypes.c_uint64),
        ("gate_off", ctypes.c_uint64), ("up_off", ctypes.c_uint64), ("down_off", ctypes.c_uint64),
        ("gate_fmt", ctypes.c_int32), ("up_fmt", ctypes.c_int32), ("down_fmt", ctypes.c_int32),
    ]


class MoeTaps(ctypes.Structure):
    _fields_ = [("normed", P), ("acts", P), ("logits", P), ("gate_up", P), ("acts_moe", P),
                ("staged", P)]


def _declare(L):
    L.or_f16_to_f32.argtypes = [ctypes.c_uint16]; L.or_f16_to_f32.restype = ctypes.c_float
    L.or_f32_to_f16.argtypes = [ctypes.c_float]; L.or_f32_to_f16.restype = ctypes.c_uint16
    L.or_has_avx2.restype = I32
    L.or_quantize_row_q8_k.argtypes = [P, SZ, P, SZ, I32]
    L.or_vec_dot.argtypes = [I32, P, SZ, P, SZ, I32, P]
    L.or_vec_dot_rows.argtypes = [I32, P, SZ, P, SZ, P, I32]
    L.or_block_int_sums.argtypes = [I32, P, P, P, P, P, P]
    L.or_gemv.argtypes = [I32, P, SZ, SZ, SZ, P, SZ, SZ, SZ, P, SZ, I32, I32]
    L.or_lcg_next_u64.argtypes = [P]; L.or_lcg_next_u64.restype = ctypes.c_uint64
    L.or_lcg_fill_f32.argtypes = [P, P, SZ, ctypes.c_float]
    L.or_rope_neox_heads.argtypes = [P, SZ, SZ, ctypes.c_uint32, ctypes.c_float]
    L.or_rope_factors.argtypes = [SZ, ctypes.c_uint32, ctypes.c_float, P, P]
    L.or_attention.argtypes = [P, P, P, SZ, SZ, SZ, SZ, ctypes.c_float, P]
    L.or_attn_decode_step.argtypes = [P, P, P, P, P, P, P, SZ, SZ, SZ, SZ, ctypes.c_float, ctypes.c_float, P]
    L.or_quantize_row_q8_0.argtypes = [P, SZ, P, SZ, I32]
    L.or_vec_dot_q8_0.argtypes = [P, SZ, P, SZ, I32, P]
    L.or_gemv_q8_0.argtypes = [P, SZ, SZ, SZ, P, SZ, SZ, SZ, SZ, P, SZ, I32, I32]
    for f in ("or_quantize_row_q4_k_test", "or_quantize_row_q5_k_test", "or_quantize_row_q6_k_test",
              "or_quantize_row_q8_0_test"):
        getattr(L, f).argtypes = [P, SZ, P]
    L.or_dequantize_row.argtypes = [I32, P, SZ, P]
    L.or_rmsnorm.argtypes = [P, P, SZ, ctypes.c_float, P]
    L.or_softmax.argtypes = [P, SZ]
    L.or_swiglu_combine.argtypes = [P, P, SZ]
    L.or_route.argtypes = [P, P, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, I32, P, P, P]
    L.or_moe_decode.argtypes = [ctypes.POINTER(MoeLayer), P, SZ, P, P, ctypes.POINTER(MoeTaps), I32, I32]
    L.or_moe_prefill.argtypes = [ctypes.POINTER(MoeLayer), P, SZ, P, P, I32, I32]
    L.or_build_index.argtypes = [P, SZ, ctypes.c_uint32, ctypes.c_uint32, P, P]
    L.or_synth_normal.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float, P, SZ]
    L.or_fill_layer_synthetic.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                          ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64,
                                          ctypes.c_uint64, I32, I32, I32, ctypes.c_uint64,
                                          ctypes.c_float, P, I32]


def _p(a):
    return None if a is None else a.ctypes.data_as(P)


def _check(code, what):
    if code != 0:
        raise OracleError(code, what)


def has_avx2() -> bool:
    return bool(lib().or_has_avx2())


def default_impl() -> int:
    """The arm the reference's dispatch would pick on this host (avx2.rs:65)."""
    return AVX2 if has_avx2() else SCALAR


# ----------------------------------------------------------------- f16
def f16_to_f32(bits: int) -> float:
    return lib().or_f16_to_f32(bits)


def f32_to_f16(x: float) -> int:
    return lib().or_f32_to_f16(ctypes.c_float(x))


# -------------------------------------------------------------- Q8_K
def quantize_row_q8_k(x, impl: int | None = None, out_blocks: int | None = None) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    nb = x.size // 256 if out_blocks is None else out_blocks
    out = np.zeros(max(nb, 0), dtype=Q8K_DTYPE)
    _check(lib().or_quantize_row_q8_k(_p(x), x.size, _p(out), nb,
                                      default_impl() if impl is None else impl), "quantize_row_q8_k")
    return out


# -------------------------------------------------------------- dots
def vec_dot(fmt: int, w, acts, impl: int | None = None) -> float:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    acts = np.ascontiguousarray(acts, dtype=Q8K_DTYPE)
    out = np.zeros(1, dtype=np.float32)
    _check(lib().or_vec_dot(fmt, _p(w), w.size, _p(acts), acts.size,
                            default_impl() if impl is None else impl, _p(out)), "vec_dot")
    return float(out[0])


def vec_dot_rows(fmt: int, w, acts, n_acts: int, impl: int | None = None) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    acts = np.ascontiguousarray(acts, dtype=Q8K_DTYPE)
    out = np.zeros(n_acts, dtype=np.float32)
    _check(lib().or_vec_dot_rows(fmt, _p(w), w.size, _p(acts), n_acts, _p(out),
                                 default_impl() if impl is None else impl), "vec_dot_rows")
    return out


def block_int_sums(fmt: int, wblock, act_block):
    """Eight AVX2 lane sums, four min-lane sums, scalar sumi, sumi_mins."""
    wblock = np.ascontiguousarray(wblock, dtype=np.uint8)
    act_block = np.ascontiguousarray(act_block, dtype=Q8K_DTYPE)
    lanes = np.zeros(8, np.int32); mins = np.zeros(4, np.int32)
    s = np.zeros(1, np.int32); sm = np.zeros(1, np.int32)
    _check(lib().or_block_int_sums(fmt, _p(wblock), _p(act_block), _p(lanes), _p(mins), _p(s), _p(sm)),
           "block_int_sums")
    return lanes, mins, int(s[0]), int(sm[0])


def gemv(fmt: int, w, in_dim: int, out_dim: int, acts, n_acts: int = 1, rows=None,
         impl: int | None = None, threads: int = 1) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    acts = np.ascontiguousarray(acts, dtype=Q8K_DTYPE)
    r0, r1 = (0, out_dim) if rows is None else rows
    out = np.zeros(max(r1 - r0, 0) * n_acts, dtype=np.float32)
    _check(lib().or_gemv(fmt, _p(w), w.size, in_dim, out_dim, _p(acts), n_acts, r0, r1, _p(out),
                         out.size, default_impl() if impl is None else impl, threads), "gemv")
    return out


# -------------------------------------------------------------- Q8_0
def quantize_row_q8_0(x, impl: int | None = None, out_blocks: int | None = None) -> np.ndarray:
    """quantize.rs:37-54 (scalar) / avx2.rs:1022-1056 (AVX2)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    nb = x.size // 32 if out_blocks is None else out_blocks
    out = np.zeros(max(nb, 0), dtype=Q8_0_DTYPE)
    _check(lib().or_quantize_row_q8_0(_p(x), x.size, _p(out), nb,
                                      default_impl() if impl is None else impl), "quantize_row_q8_0")
    return out


def vec_dot_q8_0(w, acts, impl: int | None = None) -> float:
    """dot.rs:190-201 / avx2.rs:942-963 / the lane model."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    acts = np.ascontiguousarray(acts, dtype=Q8_0_DTYPE)
    out = np.zeros(1, dtype=np.float32)
    _check(lib().or_vec_dot_q8_0(_p(w), w.size, _p(acts), acts.size,
                                 default_impl() if impl is None else impl, _p(out)), "vec_dot_q8_0")
    return float(out[0])


def gemv_q8_0(w, in_dim: int, out_dim: int, acts, n_acts: int = 1, rows=None,
              impl: int | None = None, threads: int = 1) -> np.ndarray:
    """gemv.rs:544-640 (gemv_q8_0 / _rows / _batched)."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    acts = np.ascontiguousarray(acts, dtype=Q8_0_DTYPE)
    r0, r1 = (0, out_dim) if rows is None else rows
    out = np.zeros(max(r1 - r0, 0) * n_acts, dtype=np.float32)
    _check(lib().or_gemv_q8_0(_p(w), w.size, in_dim, out_dim, _p(acts), acts.size, n_acts, r0, r1, _p(out),
                              out.size, default_impl() if impl is None else impl, threads), "gemv_q8_0")
    return out


# --------------------------------------------------------- attention
def rope_neox_heads(x, n_heads: int, head_dim: int, position: int, theta: float) -> np.ndarray:
    """rope.rs:80-111 (returns a rotated copy)."""
    x = np.array(x, dtype=np.float32, copy=True)
    _check(lib().or_rope_neox_heads(_p(x), n_heads, head_dim, position, ctypes.c_float(theta)), "rope_neox_heads")
    return x


def rope_factors(head_dim: int, position: int, theta: float):
    """The f32 (cos, sin) pairs rope.rs:30-45 forms at one position."""
    c = np.zeros(head_dim // 2, np.float32)
    s = np.zeros(head_dim // 2, np.float32)
    lib().or_rope_factors(head_dim, position, ctypes.c_float(theta), _p(c), _p(s))
    return c, s


def attention(q, k_cache, v_cache, positions: int, n_heads: int, n_kv_heads: int, head_dim: int,
              scale: float) -> np.ndarray:
    """attention.rs:1075-1303 (scalar arm); caches are f16 bits [pos][kv_dim]."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k_cache = np.ascontiguousarray(k_cache, dtype=np.uint16)
    v_cache = np.ascontiguousarray(v_cache, dtype=np.uint16)
    out = np.zeros(n_heads * head_dim, np.float32)
    _check(lib().or_attention(_p(q), _p(k_cache), _p(v_cache), positions, n_heads, n_kv_heads, head_dim,
                              ctypes.c_float(scale), _p(out)), "attention")
    return out


def attn_decode_step(q, k, v, q_norm, k_norm, k_cache, v_cache, position: int, n_heads: int, n_kv_heads: int,
                     head_dim: int, eps: float, theta: float):
    """model/forward.rs:2614-2631: QK-norm, RoPE, f16 append (into the given
    cache arrays, in place), attention.  Returns (out, q_rotated, k_rotated)."""
    q = np.array(q, dtype=np.float32, copy=True)
    k = np.array(k, dtype=np.float32, copy=True)
    v = np.ascontiguousarray(v, dtype=np.float32)
    qn = np.ascontiguousarray(q_norm, dtype=np.float32)
    kn = np.ascontiguousarray(k_norm, dtype=np.float32)
    assert k_cache.dtype == np.uint16 and v_cache.dtype == np.uint16
    assert k_cache.flags.c_contiguous and v_cache.flags.c_contiguous
    out = np.zeros(n_heads * head_dim, np.float32)
    _check(lib().or_attn_decode_step(_p(q), _p(k), _p(v), _p(qn), _p(kn), _p(k_cache), _p(v_cache), position,
                                     n_heads, n_kv_heads, head_dim, ctypes.c_float(eps), ctypes.c_float(theta),
                                     _p(out)), "attn_decode_step")
    return out, q, k


# -------------------------------------------------------------- Lcg
class Lcg:
    """test_support.rs:23-39."""

    def __init__(self, seed: int):
        self.state = np.array([seed & 0xFFFFFFFFFFFFFFFF], dtype=np.uint64)

    def next_u64(self) -> int:
        return int(lib().or_lcg_next_u64(_p(self.state)))

    def fill(self, n: int, scale: float = 1.0) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        lib().or_lcg_fill_f32(_p(self.state), _p(out), n, ctypes.c_float(scale))
        return out


# ------------------------------------------------- weight quantizers
def quantize_weights(fmt: int, x) -> np.ndarray:
    """The reference's weight quantizers (test_support.rs:106-234)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    bw = 32 if fmt == Q8_0 else 256
    assert x.size % bw == 0
    out = np.zeros(x.size // bw * BLOCK_BYTES[fmt], dtype=np.uint8)
    fn = {Q4_K: "or_quantize_row_q4_k_test", Q5_K: "or_quantize_row_q5_k_test",
          Q6_K: "or_quantize_row_q6_k_test", Q8_0: "or_quantize_row_q8_0_test"}[fmt]
    getattr(lib(), fn)(_p(x), x.size, _p(out))
    return out


def dequantize_row(fmt: int, b) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint8)
    out = np.zeros(b.size // BLOCK_BYTES[fmt] * (32 if fmt == Q8_0 else 256), dtype=np.float32)
    _check(lib().or_dequantize_row(fmt, _p(b), b.size, _p(out)), "dequantize_row")
    return out


# -------------------------------------------------------- primitives
def rmsnorm(x, w, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32); w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.empty_like(x)
    _check(lib().or_rmsnorm(_p(x), _p(w), x.size, ctypes.c_float(eps), _p(out)), "rmsnorm")
    return out


def softmax(x) -> np.ndarray:
    x = np.array(x, dtype=np.float32)
    _check(lib().or_softmax(_p(x), x.size), "softmax")
    return x


def swiglu_combine(gate, up) -> np.ndarray:
    g = np.array(gate, dtype=np.float32); u = np.ascontiguousarray(up, dtype=np.float32)
    lib().or_swiglu_combine(_p(g), _p(u), g.size)
    return g


def route(normed, router, top_k: int, norm_topk_prob: bool = True):
    normed = np.ascontiguousarray(normed, dtype=np.float32)
    router = np.ascontiguousarray(router, dtype=np.float32)
    E, H = router.shape
    logits = np.zeros(E, np.float32); ids = np.zeros(top_k, np.uint32); w = np.zeros(top_k, np.float32)
    _check(lib().or_route(_p(normed), _p(router), H, E, top_k, int(norm_topk_prob), _p(logits),
                          _p(ids), _p(w)), "route")
    return logits, ids, w


# ----------------------------------------------------------- MoE layer
def make_layer(hidden, moe, n_experts, top_k, eps, ffn_norm, router, blobs, stride, gate_off,
               up_off, down_off, gate_fmt, up_fmt, down_fmt, norm_topk_prob=True):
    keep = (ffn_norm, router, blobs)
    L = MoeLayer(hidden, moe, n_experts, top_k, int(norm_topk_prob), eps,
                 ffn_norm.ctypes.data, router.ctypes.data, blobs.ctypes.data, stride,
                 gate_off, up_off, down_off, gate_fmt, up_fmt, down_fmt)
    L._keep = keep  # arrays must outlive the struct
    return L


def moe_decode(L: MoeLayer, residual, impl: int | None = None, threads: int = 1, taps: bool = False):
    """forward.rs:2654-2754, token by token. Returns (residual', ids, w, taps)."""
    res = np.array(residual, dtype=np.float32, copy=True)
    T = res.shape[0] if res.ndim == 2 else 1
    K = L.top_k
    ids = np.zeros((T, K), np.uint32); w = np.zeros((T, K), np.float32)
    tp = None
    t = None
    if taps:
        H, M, E = L.hidden, L.moe, L.n_experts
        t = dict(normed=np.zeros((T, H), np.float32), acts=np.zeros(T * H // 256, Q8K_DTYPE),
                 logits=np.zeros((T, E), np.float32), gate_up=np.zeros((T * K, 2, M), np.float32),
                 acts_moe=np.zeros(T * K * M // 256, Q8K_DTYPE),
                 staged=np.zeros((T * K, H), np.float32))
        tp = MoeTaps(*(t[k].ctypes.data for k in ("normed", "acts", "logits", "gate_up", "acts_moe", "staged")))
    _check(lib().or_moe_decode(ctypes.byref(L), _p(res), T, _p(ids), _p(w),
                               ctypes.byref(tp) if tp is not None else None,
                               default_impl() if impl is None else impl, threads), "moe_decode")
    return res, ids, w, t


def moe_prefill(L: MoeLayer, residual, impl: int | None = None, threads: int = 1):
    res = np.array(residual, dtype=np.float32, copy=True)
    T = res.shape[0]
    K = L.top_k
    ids = np.zeros((T, K), np.uint32); w = np.zeros((T, K), np.float32)
    _check(lib().or_moe_prefill(ctypes.byref(L), _p(res), T, _p(ids), _p(w),
                                default_impl() if impl is None else impl, threads), "moe_prefill")
    return res, ids, w


def build_index(topk_ids, n_experts: int):
    ids = np.ascontiguousarray(topk_ids, dtype=np.uint32)
    T, K = ids.shape
    start = np.zeros(n_experts + 1, np.uint32); index = np.zeros(T * K, np.uint32)
    _check(lib().or_build_index(_p(ids), T, K, n_experts, _p(start), _p(index)), "build_index")
    return start, index


# ------------------------------------------------------- synthetic data
def synth_normal(seed: int, offset: int, sigma: float, n: int) -> np.ndarray:
    """Bit-identical CPU restatement of the GPU library's rv_synth_normal."""
    out = np.empty(n, np.float32)
    lib().or_synth_normal(seed, offset, ctypes.c_float(sigma), _p(out), n)
    return out


def fill_layer_synthetic(layout, seed: int, sigma: float = 0.02, threads: int = 1) -> np.ndarray:
    """All expert blobs of one layer, as rv_expert_table_fill_synthetic makes them."""
    blobs = np.zeros(layout.n_experts * layout.stride, np.uint8)
    lib().or_fill_layer_synthetic(layout.hidden, layout.moe, layout.n_experts, layout.stride,
                                  layout.gate_off, layout.up_off, layout.down_off,
                                  layout.gate_format, layout.up_format, layout.down_format,
                                  seed, ctypes.c_float(sigma), _p(blobs), threads)
    return blobs
