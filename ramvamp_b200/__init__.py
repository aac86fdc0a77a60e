"""ramvamp_b200: the routed-expert FFN of ramvamp on B200 (sm_100a).

Host-side mirror of ramvamp's kernel and MoE entry points, backed by the C
ABI of libramvamp_b200.so (include/ramvamp_b200.h).  Device memory is
carried in torch CUDA tensors; every call enqueues on the current torch
stream.  Names and error kinds follow the reference:

- ``quantize_row_q8_k``                    kernels/quants/quantize.rs:68
- ``gemv_q8_k`` / ``_rows`` / ``_batched``   kernels/gemv.rs:347, 386, 444
- ``FusedPart`` / ``gemv_q8_k_fused_rows``   kernels/gemv.rs:655, 747
- ``quantize_row_q8_0``                    kernels/quants/quantize.rs:37
- ``gemv_q8_0`` / ``_rows`` / ``_batched``   kernels/gemv.rs:544, 579, 616
- ``dequantize_rows`` / ``embed``          kernels/quants/dequant.rs:28-147,
                                             model/weights.rs:371-384
- ``rope_neox_heads``, ``attention``       kernels/primitives/rope.rs:80,
                                             kernels/attention.rs:426
- ``AttnEngine`` (KV cache + decode step)  kv/mod.rs, model/forward.rs:2614-2631
- ``CudaBackend`` (the ``Backend`` trait)    kernels/backend.rs:23-59
- ``ExpertTable`` (``ExpertStream`` API)      io/stream.rs:1472-2160
- ``rvmp.load_expert_table`` (install files) format/layout.rs, io/expert.rs
- ``MoeEngine.forward`` (the MoE block)      model/forward.rs:2654-2754,
                                             model/prefill.rs:2136-2263
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from enum import IntEnum
from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import RvError as KernelError
from ._lib import check as _check

__all__ = [
    "QuantFormat", "KernelError", "Q8K_BYTES", "quantize_row_q8_k", "gemv_q8_k", "gemv_q8_k_rows",
    "gemv_q8_k_batched", "FusedPart", "gemv_q8_k_fused_rows", "rmsnorm", "softmax",
    "swiglu_combine", "debug_block_sums", "CudaBackend", "ExpertTable", "MoeEngine", "MoeConfig",
    "LayerLayout", "qwen3_layer_layout", "QWEN3_Q6K_DOWN_LAYERS", "synth_normal",
    "quantize_weights", "EXACT", "TENSOR", "lib", "Q8_0_BYTES", "quantize_row_q8_0", "gemv_q8_0",
    "gemv_q8_0_rows", "gemv_q8_0_batched", "dequantize_rows", "embed", "device_status",
    "rope_neox_heads", "attention", "AttnEngine", "attn_weights", "rmsnorm_quantize", "ExpertParallel",
    "EP_HANDLE_BYTES", "wait_probe",
]

Q8K_BYTES = 292
Q8_0_BYTES = 36  # rv_block_q8_0: f32 d + 32 i8
EXACT = 0
TENSOR = 1

lib = _lib.load  # the loaded CDLL (raises if the library was not built)


class QuantFormat(IntEnum):
    """kernels/quants/mod.rs:57-106."""

    Q4_K = 0
    Q5_K = 1
    Q6_K = 2
    Q8_0 = 3
    Q8_K = 4

    def block_weights(self) -> int:
        return 32 if self is QuantFormat.Q8_0 else 256

    def block_bytes(self) -> int:
        return {0: 144, 1: 176, 2: 210, 3: 34, 4: 292}[int(self)]

    def row_bytes(self, in_dim: int) -> int:
        out = ctypes.c_size_t()
        _check(lib().rv_row_bytes(int(self), in_dim, ctypes.byref(out)))
        return out.value


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _p(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _nbytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


def _blocks(acts: torch.Tensor) -> int:
    n = _nbytes(acts)
    if n % Q8K_BYTES:
        raise ValueError("Q8_K activations must be a whole number of 292-byte blocks")
    return n // Q8K_BYTES


def _blocks_q8_0(acts: torch.Tensor) -> int:
    n = _nbytes(acts)
    if n % Q8_0_BYTES:
        raise ValueError("Q8_0 activations must be a whole number of 36-byte blocks")
    return n // Q8_0_BYTES


# ---------------------------------------------------------------- kernels
def quantize_row_q8_k(x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Q8_K of ``x`` (device f32) into ``out`` (device uint8, 292 B/block)."""
    n = x.numel()
    if out is None:
        out = torch.empty((n // 256) * Q8K_BYTES, dtype=torch.uint8, device=x.device)
    _check(lib().rv_quantize_row_q8_k(_p(x), n, _p(out), _blocks(out), _stream()))
    return out


def gemv_q8_k(format, weight, in_dim, out_dim, acts, out):
    _check(lib().rv_gemv_q8_k(int(format), _p(weight), _nbytes(weight), in_dim, out_dim, _p(acts),
                              _blocks(acts), _p(out), out.numel(), _stream()))
    return out


def gemv_q8_k_rows(format, weight, in_dim, out_dim, acts, rows: range, out):
    _check(lib().rv_gemv_q8_k_rows(int(format), _p(weight), _nbytes(weight), in_dim, out_dim,
                                   _p(acts), _blocks(acts), rows.start, rows.stop, _p(out),
                                   out.numel(), _stream()))
    return out


def gemv_q8_k_batched(format, weight, in_dim, out_dim, acts, n_acts, rows: range, out):
    _check(lib().rv_gemv_q8_k_batched(int(format), _p(weight), _nbytes(weight), in_dim, out_dim,
                                      _p(acts), _blocks(acts), n_acts, rows.start, rows.stop,
                                      _p(out), out.numel(), _stream()))
    return out


def quantize_row_q8_0(x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Q8_0 of ``x`` (device f32) into ``out`` (device uint8, 36 B/block):
    quantize.rs:37-54."""
    n = x.numel()
    if out is None:
        out = torch.empty((n // 32) * Q8_0_BYTES, dtype=torch.uint8, device=x.device)
    _check(lib().rv_quantize_row_q8_0(_p(x), n, _p(out), _blocks_q8_0(out), _stream()))
    return out


def gemv_q8_0(weight, in_dim, out_dim, acts, out):
    """gemv.rs:544-565: Q8_0 weights against Q8_0 activations."""
    _check(lib().rv_gemv_q8_0(_p(weight), _nbytes(weight), in_dim, out_dim, _p(acts), _blocks_q8_0(acts),
                              _p(out), out.numel(), _stream()))
    return out


def gemv_q8_0_rows(weight, in_dim, out_dim, acts, rows: range, out):
    """gemv.rs:579-601."""
    _check(lib().rv_gemv_q8_0_rows(_p(weight), _nbytes(weight), in_dim, out_dim, _p(acts), _blocks_q8_0(acts),
                                   rows.start, rows.stop, _p(out), out.numel(), _stream()))
    return out


def gemv_q8_0_batched(weight, in_dim, out_dim, acts, n_acts, rows: range, out):
    """gemv.rs:616-640: out[i * n_acts + a] = row(rows.start + i) . act_a."""
    _check(lib().rv_gemv_q8_0_batched(_p(weight), _nbytes(weight), in_dim, out_dim, _p(acts),
                                      _blocks_q8_0(acts), n_acts, rows.start, rows.stop, _p(out), out.numel(),
                                      _stream()))
    return out


def dequantize_rows(format, weight, in_dim, out_dim, rows: Optional[torch.Tensor] = None,
                    n_rows: Optional[int] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """dequant.rs:28-147 over chosen rows: out[i] = dequantize(row rows[i])
    (rows: device int32/uint32 ids, or None for rows 0..n_rows-1)."""
    if rows is not None:
        if rows.dtype not in (torch.int32, torch.uint32):
            raise ValueError("row ids must be 32-bit")
        n_rows = rows.numel()
    elif n_rows is None:
        n_rows = out_dim
    if out is None:
        out = torch.empty(n_rows * in_dim, dtype=torch.float32, device=weight.device)
    _check(lib().rv_dequantize_rows(int(format), _p(weight), _nbytes(weight), in_dim, out_dim, _p(rows), n_rows,
                                    _p(out), out.numel(), _stream()))
    return out


def embed(embedding, hidden, vocab, tokens: torch.Tensor, format=None, out=None) -> torch.Tensor:
    """Weights::embed (model/weights.rs:371-384) for a batch of token ids on
    the device: one dequantized embedding row (``hidden`` floats) per token.
    An id >= vocab zeroes its row and is reported by ``device_status`` as
    TokenOutOfRange."""
    fmt = QuantFormat.Q4_K if format is None else format
    return dequantize_rows(fmt, embedding, hidden, vocab, rows=tokens, out=out)


def rope_neox_heads(x: torch.Tensor, n_heads: int, head_dim: int, position: int, theta_base: float):
    """rope.rs:80-111, in place on a device tensor."""
    _check(lib().rv_rope_neox_heads(_p(x), x.numel(), n_heads, head_dim, position, theta_base, _stream()))
    return x


def attention(q, k_cache, v_cache, positions: int, n_heads: int, n_kv_heads: int, head_dim: int, scale: float,
              out: Optional[torch.Tensor] = None, scratch: Optional[torch.Tensor] = None) -> torch.Tensor:
    """kernels/attention.rs:426-438 over device caches (f16 bits as int16 /
    uint16 / float16 tensors, [positions][n_kv_heads * head_dim])."""
    if out is None:
        out = torch.empty(n_heads * head_dim, dtype=torch.float32, device=q.device)
    if scratch is None:
        scratch = torch.empty(2 * n_heads * positions, dtype=torch.float32, device=q.device)
    _check(lib().rv_attention(_p(q), _p(k_cache), _p(v_cache), positions, n_heads, n_kv_heads, head_dim, scale,
                              _p(scratch), scratch.numel(), _p(out), _stream()))
    return out


@dataclass
class FusedPart:
    """kernels/gemv.rs:655-686."""

    format: int
    weight: torch.Tensor
    in_dim: int
    out_dim: int
    acts: torch.Tensor


def gemv_q8_k_fused_rows(parts: Sequence[FusedPart], rows: range, out: torch.Tensor):
    arr = (_lib.FusedPartC * max(len(parts), 1))()
    for i, p in enumerate(parts):
        arr[i] = _lib.FusedPartC(int(p.format), _p(p.weight), _nbytes(p.weight), p.in_dim,
                                 p.out_dim, _p(p.acts), _blocks(p.acts))
    _check(lib().rv_gemv_q8_k_fused_rows(arr, len(parts), rows.start, rows.stop, _p(out),
                                         out.numel(), _stream()))
    return out


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor):
    n = weight.numel()
    rows = x.numel() // n if n else 0
    if x.numel() != out.numel() or (n and x.numel() % n):
        raise KernelError(5, "rmsnorm: x vs out / weight length mismatch")
    _check(lib().rv_rmsnorm(_p(x), _p(weight), n, rows, eps, _p(out), _stream()))
    return out


def softmax(x: torch.Tensor):
    n = x.shape[-1] if x.dim() else 0
    rows = x.numel() // n if n else 0
    _check(lib().rv_softmax(_p(x), n, rows, _stream()))
    return x


def swiglu_combine(gate: torch.Tensor, up: torch.Tensor):
    _check(lib().rv_swiglu_combine(_p(gate), gate.numel(), _p(up), up.numel(), _stream()))
    return gate


def debug_block_sums(format, weight_row, acts):
    """Per-block AVX2 lane sums [n_blocks][8] and min lanes [n_blocks][4]."""
    nb = _blocks(acts)
    lanes = torch.zeros(nb * 8, dtype=torch.int32, device=acts.device)
    mins = torch.zeros(nb * 4, dtype=torch.int32, device=acts.device)
    _check(lib().rv_debug_block_sums(int(format), _p(weight_row), _nbytes(weight_row), _p(acts), nb,
                                     _p(lanes), _p(mins), _stream()))
    return lanes.view(nb, 8), mins.view(nb, 4)


def synth_normal(seed: int, offset: int, sigma: float, n: int, device="cuda") -> torch.Tensor:
    out = torch.empty(n, dtype=torch.float32, device=device)
    _check(lib().rv_synth_normal(seed, offset, sigma, _p(out), n, _stream()))
    return out


def quantize_weights(format, x: torch.Tensor) -> torch.Tensor:
    """The reference's weight quantizers (test_support.rs:106-219) on the GPU."""
    fmt = QuantFormat(format)
    out = torch.empty(x.numel() // 256 * fmt.block_bytes(), dtype=torch.uint8, device=x.device)
    _check(lib().rv_quantize_weights(int(fmt), _p(x), x.numel(), _p(out), _stream()))
    return out


class CudaBackend:
    """The ``Backend`` trait (kernels/backend.rs:23-59) on the GPU."""

    def gemv_q8_k(self, format, weight, in_dim, out_dim, acts, out):
        return gemv_q8_k(format, weight, in_dim, out_dim, acts, out)

    def gemv_q8_0(self, weight, in_dim, out_dim, acts, out):
        return gemv_q8_0(weight, in_dim, out_dim, acts, out)

    def rmsnorm(self, x, weight, eps, out):
        return rmsnorm(x, weight, eps, out)

    def rope_neox_heads(self, x, n_heads, head_dim, position, theta_base):
        return rope_neox_heads(x, n_heads, head_dim, position, theta_base)

    def softmax(self, x):
        return softmax(x)

    def swiglu_combine(self, gate, up):
        return swiglu_combine(gate, up)


# ------------------------------------------------------------ expert table
LayerLayout = _lib.LayerLayout

# Layers whose expert down projection is Q6_K in Qwen3-30B-A3B Q4_K_M
# (model/shapes.rs:30-35); the rest are Q4_K.
QWEN3_Q6K_DOWN_LAYERS = frozenset(list(range(0, 6)) + [8, 11, 14, 17, 20, 23, 26, 29, 32, 35, 38]
                                  + list(range(41, 48)))


def qwen3_layer_layout(layer: int = 0, hidden=2048, moe=768, n_experts=128, down_format=None,
                       align=4096) -> LayerLayout:
    """Blob geometry of one .rvmp expert file (format/layout.rs:1-60):
    gate, up, down slabs, each starting on an `align` boundary."""
    if down_format is None:
        down_format = QuantFormat.Q6_K if layer in QWEN3_Q6K_DOWN_LAYERS else QuantFormat.Q4_K
    g_len = moe * QuantFormat.Q4_K.row_bytes(hidden)
    d_len = hidden * QuantFormat(down_format).row_bytes(moe)
    up_off = -(-g_len // align) * align
    down_off = up_off + (-(-g_len // align) * align)
    stride = -(-(down_off + d_len) // align) * align
    return LayerLayout(n_experts, 0, stride, 0, g_len, up_off, g_len, down_off, d_len,
                       int(QuantFormat.Q4_K), int(QuantFormat.Q4_K), int(down_format), hidden, moe)


@dataclass
class ExpertSlabs:
    """io/expert.rs:27-86: device addresses and formats of one expert."""

    blob: int
    gate: int
    up: int
    down: int
    gate_len: int
    up_len: int
    down_len: int
    gate_format: QuantFormat
    up_format: QuantFormat
    down_format: QuantFormat


class ExpertTable:
    """HBM-resident expert table behind the ``ExpertStream`` step API
    (io/stream.rs:1472-2160).  Every expert of every layer is resident, so a
    step's request is all hits and ``await_misses`` never blocks."""

    def __init__(self, layouts: Sequence[LayerLayout], device: int = 0):
        arr = (LayerLayout * len(layouts))(*layouts)
        h = ctypes.c_void_p()
        _check(lib().rv_expert_table_create(device, arr, len(layouts), ctypes.byref(h)))
        self.handle = h
        self.device = device
        self.layouts = list(layouts)

    def close(self):
        if getattr(self, "handle", None):
            lib().rv_expert_table_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def n_layers(self) -> int:
        return lib().rv_expert_table_n_layers(self.handle)

    def upload(self, layer: int, expert_first: int, blobs) -> None:
        """Copy whole blobs (bytes-like host buffer or device uint8 tensor)."""
        if isinstance(blobs, torch.Tensor):
            on_dev = blobs.is_cuda
            blobs = blobs.contiguous()
            n = _nbytes(blobs) // self.layouts[layer].stride
            _check(lib().rv_expert_table_upload(self.handle, layer, expert_first, n, _p(blobs),
                                                _nbytes(blobs), int(on_dev), _stream()))
        else:
            mv = memoryview(blobs).cast("B")
            buf = (ctypes.c_char * len(mv)).from_buffer_copy(mv)
            n = len(mv) // self.layouts[layer].stride
            _check(lib().rv_expert_table_upload(self.handle, layer, expert_first, n, buf, len(mv), 0,
                                                _stream()))

    def load_file(self, layer: int, path: str, offset: int = 0) -> None:
        """Layer `layer`'s expert file (n_experts * stride bytes from
        `offset`), read and copied to the device by the native loader."""
        _check(lib().rv_expert_table_load_file(self.handle, layer, os.fsencode(path), offset, _stream()))

    def fill_synthetic(self, layer: int, seed: int, sigma: float = 0.02, first_expert: int = 0,
                       expert_step: int = 1) -> None:
        """Seeded N(0, sigma^2) weights quantized by the reference's
        quantizers; expert i of this table gets global expert
        first_expert + i*expert_step's weights (an expert-parallel shard)."""
        _check(lib().rv_expert_table_fill_synthetic_strided(self.handle, layer, seed, sigma, first_expert,
                                                            expert_step, _stream()))

    def fill_synthetic_list(self, layer: int, seed: int, sigma: float, experts: Sequence[int]) -> None:
        """Local expert i gets global expert experts[i]'s synthetic weights."""
        arr = (ctypes.c_uint32 * max(len(experts), 1))(*experts)
        _check(lib().rv_expert_table_fill_synthetic_list(self.handle, layer, seed, sigma, arr, len(experts),
                                                         _stream()))

    def begin_layer(self, layer: int, experts: Sequence[int]) -> None:
        arr = (ctypes.c_uint32 * max(len(experts), 1))(*experts)
        _check(lib().rv_expert_table_begin_layer(self.handle, layer, arr, len(experts)))

    def _pairs(self, fn):
        n = ctypes.c_size_t()
        _check(fn(self.handle, None, None, 0, ctypes.byref(n)))
        idx = (ctypes.c_uint32 * max(n.value, 1))()
        slot = (ctypes.c_uint32 * max(n.value, 1))()
        _check(fn(self.handle, idx, slot, n.value, ctypes.byref(n)))
        return [(idx[i], slot[i]) for i in range(n.value)]

    def hits(self):
        return self._pairs(lib().rv_expert_table_hits)

    def misses(self):
        return self._pairs(lib().rv_expert_table_misses)

    def await_misses(self) -> None:
        _check(lib().rv_expert_table_await_misses(self.handle))

    def view(self, layer: int, slot: int) -> ExpertSlabs:
        v = _lib.ExpertView()
        _check(lib().rv_expert_table_view(self.handle, layer, slot, ctypes.byref(v)))
        return ExpertSlabs(v.blob, v.gate, v.up, v.down, v.gate_len, v.up_len, v.down_len,
                           QuantFormat(v.gate_format), QuantFormat(v.up_format), QuantFormat(v.down_format))

    def end_layer(self, layer: int) -> None:
        _check(lib().rv_expert_table_end_layer(self.handle, layer))

    def stats(self):
        a, h = ctypes.c_uint64(), ctypes.c_uint64()
        _check(lib().rv_expert_table_stats(self.handle, ctypes.byref(a), ctypes.byref(h)))
        return {"accesses": a.value, "hits": h.value}

    def blob_tensor(self, layer: int, expert: int) -> torch.Tensor:
        """A uint8 device tensor aliasing one blob (for tests: copy it out)."""
        v = self.view(layer, expert)
        L = self.layouts[layer]
        return _alias_u8(v.blob, L.stride, self.device)


class _DevBuf:
    """A raw device range exposed through __cuda_array_interface__."""

    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


def alias(ptr: int, n: int, dtype=torch.uint8, device: int = 0) -> torch.Tensor:
    """A torch tensor aliasing n elements of `dtype` at a device address."""
    typestr = {torch.uint8: "|u1", torch.float32: "<f4", torch.int32: "<i4", torch.int16: "<i2"}[dtype]
    return torch.as_tensor(_DevBuf(ptr, n, typestr), device=f"cuda:{device}")


def _alias_u8(ptr: int, n: int, device: int) -> torch.Tensor:
    return alias(ptr, n, torch.uint8, device).clone()


# ------------------------------------------------------------- MoE engine
MoeConfig = _lib.MoeConfig


class MoeEngine:
    """The MoE block of one layer on the GPU: RMSNorm, router, top-k,
    Q8_K, expert FFN and the fixed-order combine, for up to max_tokens rows
    per call.  Scratch is allocated here; forward allocates nothing."""

    def __init__(self, hidden=2048, moe=768, n_experts=128, top_k=8, norm_topk_prob=True,
                 eps=1e-6, max_tokens=1, device: int = 0):
        self.cfg = MoeConfig(hidden, moe, n_experts, top_k, int(norm_topk_prob), eps)
        h = ctypes.c_void_p()
        _check(lib().rv_moe_create(device, ctypes.byref(self.cfg), max_tokens, ctypes.byref(h)))
        self.handle = h
        self.max_tokens = max_tokens
        self.device = device

    def close(self):
        if getattr(self, "handle", None):
            lib().rv_moe_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, table: ExpertTable, layer: int, ffn_norm: torch.Tensor, router: torch.Tensor,
                residual: torch.Tensor, topk_ids: Optional[torch.Tensor] = None,
                topk_weights: Optional[torch.Tensor] = None, flags: int = EXACT) -> torch.Tensor:
        """In place: residual += MoE(residual).  Device tensors."""
        T = residual.numel() // self.cfg.hidden
        _check(lib().rv_moe_forward(self.handle, table.handle, layer, _p(ffn_norm), _p(router),
                                    _p(residual), T, _p(topk_ids), _p(topk_weights), flags, _stream()))
        return residual

    def forward_host(self, table: ExpertTable, layer: int, ffn_norm, router, residual_host,
                     topk_ids_host=None, topk_weights_host=None, flags: int = EXACT):
        """Host-buffer variant (numpy / pinned CPU tensors); synchronizes."""
        def hp(a):
            if a is None:
                return None
            if isinstance(a, torch.Tensor):
                return a.data_ptr()
            return a.ctypes.data
        T = (residual_host.numel() if isinstance(residual_host, torch.Tensor) else residual_host.size) // self.cfg.hidden
        _check(lib().rv_moe_forward_host(self.handle, table.handle, layer, _p(ffn_norm), _p(router),
                                         hp(residual_host), T, hp(topk_ids_host), hp(topk_weights_host),
                                         flags, _stream()))
        return residual_host

    def profile_enable(self, slots: int) -> None:
        _check(lib().rv_moe_profile_enable(self.handle, slots))

    def profile_rewind(self) -> None:
        _check(lib().rv_moe_profile_rewind(self.handle))

    def profile_read(self):
        """[n_sets][4] ms: routing, gate_up, down, combine per recorded forward."""
        import numpy as np
        n = ctypes.c_size_t()
        _check(lib().rv_moe_profile_read(self.handle, None, 0, ctypes.byref(n)))
        out = np.zeros(max(n.value, 1) * 4, dtype=np.float32)
        _check(lib().rv_moe_profile_read(self.handle, out.ctypes.data, out.size, ctypes.byref(n)))
        return out[: n.value * 4].reshape(n.value, 4)

    # -- the block in three parts (expert-parallel serving) -------------
    @property
    def act_stride(self) -> int:
        return int(lib().rv_moe_act_stride(self.handle))

    def route(self, ffn_norm: torch.Tensor, router: torch.Tensor, residual: torch.Tensor):
        """Routing half: (topk_ids int32 [T, K], topk_weights f32 [T, K],
        acts uint8 [T, act_stride] Q8_K rows).  residual is only read."""
        T, K = residual.numel() // self.cfg.hidden, self.cfg.top_k
        dev = residual.device
        ids = torch.empty(T, K, dtype=torch.int32, device=dev)
        w = torch.empty(T, K, dtype=torch.float32, device=dev)
        acts = torch.empty(T, self.act_stride, dtype=torch.uint8, device=dev)
        _check(lib().rv_moe_route(self.handle, _p(ffn_norm), _p(router), _p(residual), T, _p(ids), _p(w),
                                  _p(acts), _stream()))
        return ids, w, acts

    def experts(self, table: ExpertTable, layer: int, expert_ids: torch.Tensor, acts: torch.Tensor,
                flags: int = EXACT) -> torch.Tensor:
        """Expert half for (expert id in `table`, Q8_K row) pairs: f32 [n, hidden]."""
        n = expert_ids.numel()
        out = torch.empty(n, self.cfg.hidden, dtype=torch.float32, device=acts.device)
        _check(lib().rv_moe_experts(self.handle, table.handle, layer, _p(expert_ids), _p(acts), n, _p(out), flags,
                                    _stream()))
        return out

    def combine(self, residual: torch.Tensor, topk_weights: torch.Tensor, expert_out: torch.Tensor,
                pos_of: Optional[torch.Tensor] = None) -> torch.Tensor:
        """In place: residual += sum_k w_k * expert_out[row(t, k)] in top-k order."""
        T = residual.numel() // self.cfg.hidden
        _check(lib().rv_moe_combine(self.handle, _p(residual), _p(topk_weights), _p(expert_out), _p(pos_of), T,
                                    _stream()))
        return residual

    def ep_plan(self, topk_ids: torch.Tensor, acts: torch.Tensor, world: int):
        """Dispatch plan over `world` ranks (expert e on rank e % world):
        (send_counts int32 [world], pos_of int32 [T*K], send_local int32
        [T*K], send_acts uint8 [T*K, act_stride])."""
        T, K = topk_ids.shape[0], self.cfg.top_k
        dev = acts.device
        counts = torch.empty(world, dtype=torch.int32, device=dev)
        pos_of = torch.empty(T * K, dtype=torch.int32, device=dev)
        send_local = torch.empty(T * K, dtype=torch.int32, device=dev)
        send_acts = torch.empty(T * K, self.act_stride, dtype=torch.uint8, device=dev)
        _check(lib().rv_ep_plan(self.handle, _p(topk_ids), _p(acts), T, world, _p(counts), _p(pos_of),
                                _p(send_local), _p(send_acts), _stream()))
        return counts, pos_of, send_local, send_acts

    def taps(self) -> _lib.MoeTaps:
        t = _lib.MoeTaps()
        _check(lib().rv_moe_get_taps(self.handle, ctypes.byref(t)))
        return t


EP_HANDLE_BYTES = 256  # RV_EP_HANDLE_BYTES


class ExpertParallel:
    """One rank of an expert-parallel group (rv_ep_*): experts spread over
    `world` GPUs by id modulo world, tokens dispatched and expert outputs
    returned through GPU memory with no host synchronization.  Usage, on
    every rank: ``ep = ExpertParallel(engine, world, rank, max_tokens)``;
    gather every rank's ``ep.handle()`` in rank order (any out-of-band
    channel; ``ramvamp_b200.ep.connect_group`` uses torch.distributed);
    ``ep.connect(handles)``; then ``ep.forward(...)`` per layer on every
    rank.  The engine must hold world * max_tokens rows."""

    def __init__(self, engine: "MoeEngine", world: int, rank: int, max_tokens: int):
        h = ctypes.c_void_p()
        _check(lib().rv_ep_create(engine.handle, world, rank, max_tokens, ctypes.byref(h)))
        self.handle, self.engine = h, engine
        self.world, self.rank, self.max_tokens = world, rank, max_tokens

    def handle_bytes(self) -> bytes:
        buf = ctypes.create_string_buffer(EP_HANDLE_BYTES)
        _check(lib().rv_ep_handle(self.handle, buf, EP_HANDLE_BYTES))
        return buf.raw

    def connect(self, handles: Sequence[bytes]) -> None:
        blob = b"".join(handles)
        buf = ctypes.create_string_buffer(blob, len(blob))
        _check(lib().rv_ep_connect(self.handle, buf, len(blob)))

    def forward(self, table: ExpertTable, layer: int, ffn_norm: torch.Tensor, router: torch.Tensor,
                residual: torch.Tensor, topk_ids: Optional[torch.Tensor] = None,
                topk_weights: Optional[torch.Tensor] = None, flags: int = EXACT,
                placement: Optional[torch.Tensor] = None) -> torch.Tensor:
        """In place on this rank's home rows: residual += MoE(residual).
        placement: device int32 [n_experts] of rank << 16 | local id (the
        same on every rank), from ``ramvamp_b200.ep.placement_tensor``;
        None: expert e on rank e % world."""
        T = residual.numel() // self.engine.cfg.hidden
        _check(lib().rv_moe_ep_forward(self.handle, table.handle, layer, _p(ffn_norm), _p(router),
                                       _p(residual), T, _p(topk_ids), _p(topk_weights), _p(placement), flags,
                                       _stream()))
        return residual

    def received(self) -> list:
        """Pairs each rank sent this rank in the most recent layer."""
        arr = (ctypes.c_uint32 * self.world)()
        _check(lib().rv_ep_counts(self.handle, arr, self.world))
        return list(arr)

    def close(self):
        if getattr(self, "handle", None):
            lib().rv_ep_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class AttnEngine:
    """The attention half of a decode step on one device: the f16 KV cache
    of every layer (kv/mod.rs ``KvCache``), the NeoX rotation table and
    scratch.  ``decode`` is model/forward.rs:2614-2631 for one layer."""

    def __init__(self, n_layers=48, n_heads=32, n_kv_heads=4, head_dim=128, max_positions=4096,
                 rope_theta=1e7, eps=1e-6, device: int = 0, hidden: int = 0):
        self.cfg = _lib.AttnConfig(n_layers, n_heads, n_kv_heads, head_dim, max_positions, rope_theta, eps,
                                   hidden)
        h = ctypes.c_void_p()
        _check(lib().rv_attn_create(device, ctypes.byref(self.cfg), ctypes.byref(h)))
        self.handle = h
        self.device = device

    def close(self):
        if getattr(self, "handle", None):
            lib().rv_attn_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def len(self, layer: int) -> int:
        n = ctypes.c_uint32()
        _check(lib().rv_attn_len(self.handle, layer, ctypes.byref(n)))
        return n.value

    def clear(self):
        _check(lib().rv_attn_clear(self.handle))

    def cache(self, layer: int):
        """(k, v) device addresses of one layer's caches."""
        k, v = ctypes.c_void_p(), ctypes.c_void_p()
        _check(lib().rv_attn_cache(self.handle, layer, ctypes.byref(k), ctypes.byref(v)))
        return k.value, v.value

    def cache_tensors(self, layer: int, positions: Optional[int] = None):
        """Copies (k, v) of one layer's first `positions` rows, f16 bits as
        int16 device tensors [positions][n_kv_heads * head_dim]."""
        n = self.len(layer) if positions is None else positions
        kv_dim = self.cfg.n_kv_heads * self.cfg.head_dim
        k = torch.empty((n, kv_dim), dtype=torch.int16, device=f"cuda:{self.device}")
        v = torch.empty_like(k)
        _check(lib().rv_attn_copy_cache(self.handle, layer, n, _p(k), _p(v), _stream()))
        return k, v

    def block(self, layer: int, weights, residual: torch.Tensor, position: Optional[int] = None,
              position_dev: Optional[torch.Tensor] = None) -> torch.Tensor:
        """model/forward.rs:2572-2652 for one layer, residual in place.
        `weights` is an rv_attn_weights (``attn_weights(...)``); the
        position is a host int (checked) or an int32 device tensor."""
        _check(lib().rv_attn_block(self.handle, layer, ctypes.byref(weights), _p(residual), _p(position_dev),
                                   0 if position is None else position, _stream()))
        return residual

    def decode(self, layer: int, position: int, q, k, v, q_norm, k_norm, out=None) -> torch.Tensor:
        """QK-norm + RoPE of q and k (in place), f16 append of k and v at
        `position`, attention over positions 0..position into `out`."""
        if out is None:
            out = torch.empty_like(q)
        _check(lib().rv_attn_decode(self.handle, layer, position, _p(q), _p(k), _p(v), _p(q_norm), _p(k_norm),
                                    _p(out), _stream()))
        return out


def attn_weights(attn_norm, attn_q, attn_k, attn_v, attn_output, q_norm, k_norm, attn_q_format=QuantFormat.Q4_K,
                 attn_v_format=QuantFormat.Q6_K, attn_output_format=QuantFormat.Q5_K):
    """An rv_attn_weights for AttnEngine.block (device tensors; the caller
    keeps them alive)."""
    return _lib.AttnWeights(_p(attn_norm), _p(attn_q), _p(attn_k), _p(attn_v), _p(attn_output), _p(q_norm),
                            _p(k_norm), int(attn_q_format), int(attn_v_format), int(attn_output_format))


def rmsnorm_quantize(x: torch.Tensor, w: torch.Tensor, eps: float, q8k_out: torch.Tensor,
                     q80_out: Optional[torch.Tensor] = None):
    """rmsnorm fused with quantize_row_q8_k (and quantize_row_q8_0)."""
    _check(lib().rv_rmsnorm_quantize(_p(x), _p(w), x.numel(), eps, _p(q8k_out), _p(q80_out), _stream()))
    return q8k_out


def device_status(device: int = 0) -> None:
    """Raise if a device-side bounded wait or check failed since the last call."""
    _check(lib().rv_device_status(device, _stream()))


WAIT_MBARRIER, WAIT_FLAG = 0, 1


def wait_probe(what: int, cycles: int, device: int = 0) -> None:
    """rv_debug_wait_probe: one kernel whose bounded wait on `what`
    (WAIT_MBARRIER or WAIT_FLAG) runs out after `cycles` SM cycles; the
    next device_status raises Timeout."""
    _check(lib().rv_debug_wait_probe(device, what, cycles, _stream()))

from . import rvmp  # noqa: E402  (install reader; imports this module lazily)
