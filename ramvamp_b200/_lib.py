"""ctypes binding of libramvamp_b200.so (the C ABI in include/ramvamp_b200.h).

The shared library is built in-tree by ``ramvamp_b200.build.build()``.  There
is no fallback: if the library is missing or fails to load, importing this
module raises, so nothing can silently run on the CPU instead.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libramvamp_b200.so")

P = ctypes.c_void_p
SZ = ctypes.c_size_t
I32 = ctypes.c_int
U32 = ctypes.c_uint32
U64 = ctypes.c_uint64
F32 = ctypes.c_float

STATUS_NAMES = {
    0: "Ok", 1: "IndivisibleRow", 2: "RowBytesNotBlockMultiple", 3: "BlockCountMismatch",
    4: "QuantizeLenMismatch", 5: "LengthMismatch", 6: "Empty", 7: "InvalidHeadDim",
    8: "Unimplemented", 9: "UnsupportedFormat", 10: "RoutedExpertOutOfRange",
    11: "LayerOutOfRange", 12: "Protocol", 13: "InvalidArgument", 14: "Cuda", 15: "Nccl",
    16: "Timeout",
    17: "Io",
    18: "TokenOutOfRange",
    19: "PositionMismatch",
    20: "CapacityExceeded",
    21: "Peer",
}


class RvError(RuntimeError):
    """A non-zero rv_status.  ``kind`` is the reference's KernelError variant
    name for codes 1..9 (kernels/error.rs:20-110)."""

    def __init__(self, code: int, detail: str):
        self.code = code
        self.kind = STATUS_NAMES.get(code, str(code))
        super().__init__(detail or self.kind)


class LayerLayout(ctypes.Structure):
    _fields_ = [
        ("n_experts", U32), ("_pad", U32), ("stride", U64),
        ("gate_off", U64), ("gate_len", U64), ("up_off", U64), ("up_len", U64),
        ("down_off", U64), ("down_len", U64),
        ("gate_format", ctypes.c_int32), ("up_format", ctypes.c_int32), ("down_format", ctypes.c_int32),
        ("hidden", U32), ("moe", U32),
    ]


class ExpertView(ctypes.Structure):
    _fields_ = [
        ("blob", P), ("gate", P), ("up", P), ("down", P),
        ("gate_len", U64), ("up_len", U64), ("down_len", U64),
        ("gate_format", ctypes.c_int32), ("up_format", ctypes.c_int32), ("down_format", ctypes.c_int32),
    ]


class FusedPartC(ctypes.Structure):
    _fields_ = [("format", ctypes.c_int32), ("weight", P), ("weight_len", SZ), ("in_dim", SZ),
                ("out_dim", SZ), ("acts", P), ("acts_len", SZ)]


class MoeConfig(ctypes.Structure):
    _fields_ = [("hidden", U32), ("moe", U32), ("n_experts", U32), ("top_k", U32),
                ("norm_topk_prob", ctypes.c_int32), ("eps", F32)]


class AttnConfig(ctypes.Structure):
    _fields_ = [("n_layers", U32), ("n_heads", U32), ("n_kv_heads", U32), ("head_dim", U32),
                ("max_positions", U32), ("rope_theta", F32), ("eps", F32), ("hidden", U32)]


class AttnWeights(ctypes.Structure):
    _fields_ = [("attn_norm", P), ("attn_q", P), ("attn_k", P), ("attn_v", P), ("attn_output", P),
                ("q_norm", P), ("k_norm", P), ("attn_q_format", ctypes.c_int32), ("attn_v_format", ctypes.c_int32),
                ("attn_output_format", ctypes.c_int32)]


class MoeTaps(ctypes.Structure):
    _fields_ = [("normed", P), ("acts", P), ("acts_stride", SZ), ("logits", P), ("weights", P),
                ("ids", P), ("index", P), ("index_start", P), ("swiglu", P), ("acts_moe", P),
                ("acts_moe_stride", SZ), ("staged", P), ("logit_bounds", P)]


# name -> (restype, argtypes); every symbol the header declares.
SIGNATURES = {
    "rv_version": (ctypes.c_char_p, []),
    "rv_status_name": (ctypes.c_char_p, [I32]),
    "rv_last_error": (SZ, [ctypes.c_char_p, SZ]),
    "rv_block_bytes": (SZ, [I32]),
    "rv_block_weights": (SZ, [I32]),
    "rv_row_bytes": (I32, [I32, SZ, ctypes.POINTER(SZ)]),
    "rv_device_status": (I32, [I32, P]),
    "rv_debug_wait_probe": (I32, [I32, U32, U64, P]),
    "rv_quantize_row_q8_k": (I32, [P, SZ, P, SZ, P]),
    "rv_gemv_q8_k": (I32, [I32, P, SZ, SZ, SZ, P, SZ, P, SZ, P]),
    "rv_gemv_q8_k_rows": (I32, [I32, P, SZ, SZ, SZ, P, SZ, SZ, SZ, P, SZ, P]),
    "rv_gemv_q8_k_batched": (I32, [I32, P, SZ, SZ, SZ, P, SZ, SZ, SZ, SZ, P, SZ, P]),
    "rv_quantize_row_q8_0": (I32, [P, SZ, P, SZ, P]),
    "rv_gemv_q8_0": (I32, [P, SZ, SZ, SZ, P, SZ, P, SZ, P]),
    "rv_gemv_q8_0_rows": (I32, [P, SZ, SZ, SZ, P, SZ, SZ, SZ, P, SZ, P]),
    "rv_gemv_q8_0_batched": (I32, [P, SZ, SZ, SZ, P, SZ, SZ, SZ, SZ, P, SZ, P]),
    "rv_dequantize_rows": (I32, [I32, P, SZ, SZ, SZ, P, SZ, P, SZ, P]),
    "rv_attn_create": (I32, [I32, ctypes.POINTER(AttnConfig), ctypes.POINTER(P)]),
    "rv_attn_destroy": (None, [P]),
    "rv_attn_len": (I32, [P, U32, ctypes.POINTER(U32)]),
    "rv_attn_clear": (I32, [P]),
    "rv_attn_cache": (I32, [P, U32, ctypes.POINTER(P), ctypes.POINTER(P)]),
    "rv_attn_copy_cache": (I32, [P, U32, U32, P, P, P]),
    "rv_attn_decode": (I32, [P, U32, U32, P, P, P, P, P, P, P]),
    "rv_rope_neox_heads": (I32, [P, SZ, SZ, SZ, U32, F32, P]),
    "rv_attn_decode_dev": (I32, [P, U32, P, P, P, P, P, P, P, P]),
    "rv_decode_advance": (I32, [P, P, P, P, SZ, P]),
    "rv_attn_block": (I32, [P, U32, ctypes.POINTER(AttnWeights), P, P, U32, P]),
    "rv_rmsnorm_quantize": (I32, [P, P, SZ, F32, P, P, P]),
    "rv_argmax": (I32, [P, SZ, P, P]),
    "rv_vec_add": (I32, [P, P, SZ, P]),
    "rv_attention": (I32, [P, P, P, SZ, SZ, SZ, SZ, F32, P, SZ, P, P]),
    "rv_gemv_q8_k_fused_rows": (I32, [ctypes.POINTER(FusedPartC), SZ, SZ, SZ, P, SZ, P]),
    "rv_rmsnorm": (I32, [P, P, SZ, SZ, F32, P, P]),
    "rv_softmax": (I32, [P, SZ, SZ, P]),
    "rv_swiglu_combine": (I32, [P, SZ, P, SZ, P]),
    "rv_debug_block_sums": (I32, [I32, P, SZ, P, SZ, P, P, P]),
    "rv_expert_table_create": (I32, [I32, ctypes.POINTER(LayerLayout), U32, ctypes.POINTER(P)]),
    "rv_expert_table_destroy": (None, [P]),
    "rv_expert_table_upload": (I32, [P, U32, U32, U32, P, SZ, I32, P]),
    "rv_expert_table_load_file": (I32, [P, U32, ctypes.c_char_p, U64, P]),
    "rv_expert_table_layout": (I32, [P, U32, ctypes.POINTER(LayerLayout)]),
    "rv_expert_table_n_layers": (U32, [P]),
    "rv_expert_table_begin_layer": (I32, [P, U32, P, SZ]),
    "rv_expert_table_hits": (I32, [P, P, P, SZ, ctypes.POINTER(SZ)]),
    "rv_expert_table_misses": (I32, [P, P, P, SZ, ctypes.POINTER(SZ)]),
    "rv_expert_table_await_misses": (I32, [P]),
    "rv_expert_table_view": (I32, [P, U32, U32, ctypes.POINTER(ExpertView)]),
    "rv_expert_table_end_layer": (I32, [P, U32]),
    "rv_expert_table_stats": (I32, [P, ctypes.POINTER(U64), ctypes.POINTER(U64)]),
    "rv_moe_create": (I32, [I32, ctypes.POINTER(MoeConfig), SZ, ctypes.POINTER(P)]),
    "rv_moe_destroy": (None, [P]),
    "rv_moe_forward": (I32, [P, P, U32, P, P, P, SZ, P, P, U32, P]),
    "rv_moe_forward_host": (I32, [P, P, U32, P, P, P, SZ, P, P, U32, P]),
    "rv_moe_get_taps": (I32, [P, ctypes.POINTER(MoeTaps)]),
    "rv_moe_act_stride": (SZ, [P]),
    "rv_moe_route": (I32, [P, P, P, P, SZ, P, P, P, P]),
    "rv_moe_experts": (I32, [P, P, U32, P, P, SZ, P, U32, P]),
    "rv_moe_combine": (I32, [P, P, P, P, P, SZ, P]),
    "rv_ep_plan": (I32, [P, P, P, SZ, U32, P, P, P, P, P]),
    "rv_ep_create": (I32, [P, U32, U32, SZ, ctypes.POINTER(P)]),
    "rv_ep_destroy": (None, [P]),
    "rv_ep_handle": (I32, [P, P, SZ]),
    "rv_ep_connect": (I32, [P, P, SZ]),
    "rv_moe_ep_forward": (I32, [P, P, U32, P, P, P, SZ, P, P, P, U32, P]),
    "rv_ep_check_placement": (I32, [U32, U32, P, SZ]),
    "rv_ep_counts": (I32, [P, P, SZ]),
    "rv_moe_profile_enable": (I32, [P, SZ]),
    "rv_moe_profile_rewind": (I32, [P]),
    "rv_moe_profile_read": (I32, [P, P, SZ, ctypes.POINTER(SZ)]),
    "rv_moe_forward_static": (I32, [ctypes.POINTER(MoeConfig), ctypes.POINTER(LayerLayout), P, P, P, P, SZ, P, P, P]),
    "rv_synth_normal": (I32, [U64, U64, F32, P, SZ, P]),
    "rv_quantize_weights": (I32, [I32, P, SZ, P, P]),
    "rv_expert_table_fill_synthetic": (I32, [P, U32, U64, F32, P]),
    "rv_expert_table_fill_synthetic_strided": (I32, [P, U32, U64, F32, U32, U32, P]),
    "rv_expert_table_fill_synthetic_list": (I32, [P, U32, U64, F32, P, SZ, P]),
}

_lib = None


def load() -> ctypes.CDLL:
    """Load the in-tree library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run ramvamp_b200.build.build() first")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    load().rv_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(code: int) -> None:
    if code != 0:
        raise RvError(code, last_error())
