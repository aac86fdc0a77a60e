"""Expert-blob geometry and greedy sampling, restated without the product.

TEST INFRASTRUCTURE ONLY: the reference arm of bench.py and the oracle's
whole-model twin use these so that they never load libramvamp_b200.so.  A
CPU test checks that the product's own ``qwen3_layer_layout`` gives the same
numbers.

- ``layer_layout`` follows format/layout.rs:1-13 (each layer's expert file is
  n_experts fixed-stride blobs with the gate, up and down slabs at 4 KiB
  aligned offsets; stride a 4 KiB multiple) and the slab order of the
  repacker (crates/repack/src/plan.rs:323-349: gate at 0, up after it, down
  after up).
- ``Q6K_DOWN_LAYERS`` is the down-projection format split of the audited
  Qwen3-30B-A3B Q4_K_M file (model/shapes.rs:30-35).
- ``top1`` is Sampler::argmax (generate/mod.rs:321-331).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

Q4_K, Q5_K, Q6_K, Q8_0 = 0, 1, 2, 3
BLOCK_BYTES = {Q4_K: 144, Q5_K: 176, Q6_K: 210, Q8_0: 34}
BLOCK_WEIGHTS = {Q4_K: 256, Q5_K: 256, Q6_K: 256, Q8_0: 32}
EXPERT_BLOB_ALIGN = 4096  # format/mod.rs:73

Q6K_DOWN_LAYERS = frozenset(list(range(0, 6)) + [8, 11, 14, 17, 20, 23, 26, 29, 32, 35, 38] + list(range(41, 48)))


def row_bytes(fmt: int, in_dim: int) -> int:
    """QuantFormat::row_bytes (kernels/quants/mod.rs:96-105)."""
    w = BLOCK_WEIGHTS[fmt]
    if in_dim % w:
        raise ValueError(f"in_dim {in_dim} is not a multiple of {w}")
    return in_dim // w * BLOCK_BYTES[fmt]


@dataclass(frozen=True)
class Layout:
    """One layer's blob geometry (the fields of rv_layer_layout)."""

    n_experts: int
    stride: int
    gate_off: int
    gate_len: int
    up_off: int
    up_len: int
    down_off: int
    down_len: int
    gate_format: int
    up_format: int
    down_format: int
    hidden: int
    moe: int


def layer_layout(layer: int = 0, hidden: int = 2048, moe: int = 768, n_experts: int = 128, down_format=None,
                 align: int = EXPERT_BLOB_ALIGN) -> Layout:
    if down_format is None:
        down_format = Q6_K if layer in Q6K_DOWN_LAYERS else Q4_K
    g_len = moe * row_bytes(Q4_K, hidden)
    d_len = hidden * row_bytes(int(down_format), moe)
    up_off = -(-g_len // align) * align
    down_off = up_off + (-(-g_len // align) * align)
    stride = -(-(down_off + d_len) // align) * align
    return Layout(n_experts, stride, 0, g_len, up_off, g_len, down_off, d_len, Q4_K, Q4_K, int(down_format), hidden,
                  moe)


def top1(logits) -> int:
    """The first index of the largest value; NaN never wins; 0 when nothing
    beats -inf."""
    x = np.asarray(logits, np.float32)
    valid = x > -np.inf  # False for NaN
    if not valid.any():
        return 0
    return int(np.flatnonzero(valid & (x == x[valid].max()))[0])


@dataclass(frozen=True)
class ModelShape:
    """Qwen3-30B-A3B's shapes (model/shapes.rs:14-35 and the manifest's arch
    block) for the reference arm's whole-model twin; the fields of the
    product's ModelConfig."""

    n_layers: int = 48
    hidden: int = 2048
    n_heads: int = 32
    n_kv_heads: int = 4
    head_dim: int = 128
    moe: int = 768
    n_experts: int = 128
    top_k: int = 8
    vocab: int = 151936
    rope_theta: float = 1e6
    eps: float = 1e-6
    norm_topk_prob: bool = True

    @property
    def q_dim(self):
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self):
        return self.n_kv_heads * self.head_dim

    def q6k_layer(self, layer: int) -> bool:
        """attn_v and ffn_down are Q6_K on the pinned layer set of the
        48-layer model, Q4_K elsewhere (alternating on smaller test models)."""
        return layer in Q6K_DOWN_LAYERS if self.n_layers == 48 else layer % 2 == 0
