"""Whole-model Qwen3-30B-A3B decode on the GPU: the per-token step of
model/forward.rs:2548-2780 (embedding, 48 x (attention half + MoE block),
final norm, lm_head) and the greedy loop of generate/mod.rs (argmax, first
index wins ties), plus the KL / top-1 comparison the reference's
scripts/kl_vs_reference.py applies to two logit streams.

The step runs entirely on the device: the input token id, the position and
the sampled id live in device memory, so one CUDA graph captured once serves
every step (``Decoder.capture``), with no host work between tokens while
generating.  Every kernel on the step is this package's own; weights are
synthetic (seeded values through the reference's quantizers) or come from an
install.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np
import torch

from . import (AttnEngine, ExpertTable, MoeEngine, QuantFormat, QWEN3_Q6K_DOWN_LAYERS, _check, _p, _stream,
               attn_weights, dequantize_rows, gemv_q8_k, lib, qwen3_layer_layout, quantize_row_q8_0,
               quantize_weights, rmsnorm_quantize, synth_normal)

Q = QuantFormat


@dataclass
class ModelConfig:
    """model/shapes.rs:14-35 and the manifest's arch block; defaults are
    Qwen3-30B-A3B."""

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
        48-layer model (model/shapes.rs:30-35), Q4_K elsewhere."""
        return layer in QWEN3_Q6K_DOWN_LAYERS if self.n_layers == 48 else layer % 2 == 0


@dataclass
class LayerWeights:
    attn_norm: torch.Tensor
    attn_q: torch.Tensor       # Q4_K [q_dim][hidden]
    attn_k: torch.Tensor       # Q8_0 [kv_dim][hidden]
    attn_v: torch.Tensor       # Q6_K or Q4_K [kv_dim][hidden]
    attn_v_format: int
    attn_output: torch.Tensor  # Q5_K [hidden][q_dim]
    attn_q_norm: torch.Tensor
    attn_k_norm: torch.Tensor
    ffn_norm: torch.Tensor
    router: torch.Tensor       # f32 [n_experts][hidden]


def _q8_0_weights(x: torch.Tensor) -> torch.Tensor:
    """Packed Q8_0 weight rows (34 B / 32 weights): the activation quantizer
    with d stored as f16, which is test_support.rs:221-234's recipe."""
    blocks = quantize_row_q8_0(x).view(-1, 36)
    d16 = blocks[:, :4].contiguous().view(torch.float32).half().view(torch.uint8)
    return torch.cat([d16, blocks[:, 4:]], dim=1).contiguous().view(-1)


@dataclass
class Qwen3Weights:
    cfg: ModelConfig
    token_embd: torch.Tensor   # Q4_K [vocab][hidden]
    output_norm: torch.Tensor
    lm_head: torch.Tensor      # Q6_K [vocab][hidden]
    layers: List[LayerWeights]
    experts: ExpertTable

    @classmethod
    def synthetic(cls, cfg: ModelConfig, seed: int = 1, device: int = 0, expert_sigma: float = 0.02):
        """Seeded random-init weights (config 1): every matrix N(0, 0.02)
        through the reference's quantizers (embedding N(0, 1)), norms
        1 + N(0, 0.05), router N(0, 0.02) f32."""
        dev = f"cuda:{device}"
        offset = [0]

        def normal(n, sigma):
            x = synth_normal(seed, offset[0], sigma, n, device=dev)
            offset[0] += n
            return x

        def norm_w(n):
            return 1.0 + normal(n, 0.05)

        H = cfg.hidden
        layers = []
        for l in range(cfg.n_layers):
            v_fmt = Q.Q6_K if cfg.q6k_layer(l) else Q.Q4_K
            layers.append(LayerWeights(
                attn_norm=norm_w(H),
                attn_q=quantize_weights(Q.Q4_K, normal(cfg.q_dim * H, 0.02)),
                attn_k=_q8_0_weights(normal(cfg.kv_dim * H, 0.02)),
                attn_v=quantize_weights(v_fmt, normal(cfg.kv_dim * H, 0.02)),
                attn_v_format=int(v_fmt),
                attn_output=quantize_weights(Q.Q5_K, normal(H * cfg.q_dim, 0.02)),
                attn_q_norm=norm_w(cfg.head_dim),
                attn_k_norm=norm_w(cfg.head_dim),
                ffn_norm=norm_w(H),
                router=normal(cfg.n_experts * H, 0.02),
            ))
        layouts = [qwen3_layer_layout(l, hidden=H, moe=cfg.moe, n_experts=cfg.n_experts,
                                      down_format=Q.Q6_K if cfg.q6k_layer(l) else Q.Q4_K)
                   for l in range(cfg.n_layers)]
        table = ExpertTable(layouts, device=device)
        for l in range(cfg.n_layers):
            table.fill_synthetic(l, seed * 1000 + l, expert_sigma)
        token_embd = quantize_weights(Q.Q4_K, normal(cfg.vocab * H, 1.0))
        output_norm = norm_w(H)
        lm_head = quantize_weights(Q.Q6_K, normal(cfg.vocab * H, 0.02))
        torch.cuda.synchronize(device)
        return cls(cfg, token_embd, output_norm, lm_head, layers, table)


class Decoder:
    """Batch-1 decoding over Qwen3Weights.  ``step`` runs one token of
    forward_token_traced (model/forward.rs:2548-2780) plus the greedy
    argmax; all state (token, position, caches) is on the device."""

    def __init__(self, weights: Qwen3Weights, max_positions: int = 1024, device: int = 0):
        cfg = weights.cfg
        self.w, self.cfg, self.device = weights, cfg, device
        self.max_positions = max_positions
        self.attn = AttnEngine(cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, max_positions,
                               cfg.rope_theta, cfg.eps, device, hidden=cfg.hidden)
        self.attn_w = [attn_weights(l.attn_norm, l.attn_q, l.attn_k, l.attn_v, l.attn_output, l.attn_q_norm,
                                    l.attn_k_norm, Q.Q4_K, l.attn_v_format, Q.Q5_K) for l in weights.layers]
        self.moe = MoeEngine(cfg.hidden, cfg.moe, cfg.n_experts, cfg.top_k, cfg.norm_topk_prob, cfg.eps,
                             max_tokens=1, device=device)
        d = f"cuda:{device}"
        f32 = lambda n: torch.zeros(n, dtype=torch.float32, device=d)
        H = cfg.hidden
        self.residual = f32(H)
        self.acts_k = torch.zeros(H // 256 * 292, dtype=torch.uint8, device=d)
        self.logits = f32(cfg.vocab)
        self.token = torch.zeros(1, dtype=torch.int32, device=d)
        self.next_token = torch.zeros(1, dtype=torch.int32, device=d)
        self.position = torch.zeros(1, dtype=torch.int32, device=d)
        self.ids = torch.zeros(max_positions, dtype=torch.int32, device=d)
        self.graph: Optional[torch.cuda.CUDAGraph] = None

    def reset(self):
        """KvCache::clear and position 0."""
        self.attn.clear()
        self.position.zero_()
        self.ids.zero_()

    def _launch_step(self):
        cfg, w, s = self.cfg, self.w, _stream()
        H = cfg.hidden
        dequantize_rows(Q.Q4_K, w.token_embd, H, cfg.vocab, rows=self.token, out=self.residual)
        for l, lw in enumerate(w.layers):
            # attention half (forward.rs:2572-2652), residual in place
            self.attn.block(l, self.attn_w[l], self.residual, position_dev=self.position)
            # MoE block (forward.rs:2654-2754), residual in place
            self.moe.forward(w.experts, l, lw.ffn_norm, lw.router, self.residual)
        rmsnorm_quantize(self.residual, w.output_norm, cfg.eps, self.acts_k)
        gemv_q8_k(Q.Q6_K, w.lm_head, H, cfg.vocab, self.acts_k, self.logits)
        _check(lib().rv_argmax(_p(self.logits), cfg.vocab, _p(self.next_token), s))
        _check(lib().rv_decode_advance(_p(self.position), _p(self.next_token), _p(self.token), _p(self.ids),
                                       self.ids.numel(), s))

    def capture(self):
        """Capture one step as a CUDA graph (replayed by ``step``)."""
        torch.cuda.synchronize(self.device)
        side = torch.cuda.Stream(self.device)
        saved = (self.token.clone(), self.position.clone(), self.ids.clone())
        with torch.cuda.stream(side):
            self._launch_step()  # warm-up outside capture (lazy set-up)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            self._launch_step()
        torch.cuda.synchronize(self.device)
        self.token.copy_(saved[0])
        self.position.copy_(saved[1])
        self.ids.copy_(saved[2])
        self.attn.clear()
        self.graph = g
        return g

    def step(self):
        """One token: reads self.token / self.position, writes self.logits,
        self.next_token (= self.token for the next step), self.ids[pos]."""
        if self.graph is not None:
            self.graph.replay()
        else:
            self._launch_step()

    def generate(self, prompt: Sequence[int], n_new: int, on_logits=None) -> List[int]:
        """Greedy continuation of `prompt` by n_new tokens (generate/mod.rs:
        the prompt is fed one token per step, then each argmax becomes the
        next input).  on_logits(step_index, logits) sees every step's logits
        (prompt steps included)."""
        if len(prompt) + n_new > self.max_positions:
            raise ValueError("prompt + new tokens exceed max_positions")
        self.reset()
        prompt_t = torch.tensor(list(prompt), dtype=torch.int32, device=self.token.device)
        self.token.copy_(prompt_t[:1])
        for i in range(len(prompt) + n_new - 1):
            self.step()
            if on_logits is not None:
                on_logits(i, self.logits)
            if i + 1 < len(prompt):
                self.token.copy_(prompt_t[i + 1:i + 2])
        torch.cuda.synchronize(self.device)
        ids = self.ids[:len(prompt) + n_new - 1].cpu().numpy()
        return [int(x) for x in ids[len(prompt) - 1:]]


def kl_divergence(ref_logits, logits) -> float:
    """Full-vocab KL(p_ref || p) in f64 from two logit vectors (the
    comparison of scripts/kl_vs_reference.py)."""
    a = np.asarray(ref_logits, np.float64)
    b = np.asarray(logits, np.float64)
    la = a - a.max() - math.log(np.exp(a - a.max()).sum())
    lb = b - b.max() - math.log(np.exp(b - b.max()).sum())
    return float(np.sum(np.exp(la) * (la - lb)))


def top1(logits) -> int:
    """Sampler::argmax (generate/mod.rs:321-331): the first index of the
    largest value; NaN never wins; 0 when nothing beats -inf."""
    x = np.asarray(logits, np.float32)
    valid = x > -np.inf  # False for NaN
    if not valid.any():
        return 0
    return int(np.flatnonzero(valid & (x == x[valid].max()))[0])


def _main(argv=None):
    """python -m ramvamp_b200.model [--layers N] [--profile-step K]: build
    the synthetic Qwen3 model, run K eager steps, then one more inside the
    NVTX range "step" (for a profiler restricted to that range)."""
    import argparse

    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--profile-step", type=int, default=8)
    a = ap.parse_args(argv)
    w = Qwen3Weights.synthetic(ModelConfig(n_layers=a.layers), seed=1)
    dec = Decoder(w, max_positions=a.profile_step + 8)
    dec.reset()
    dec.token.fill_(5)
    for _ in range(a.profile_step):
        dec.step()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("step")
    dec.step()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    print("next token", int(dec.next_token.item()))


if __name__ == "__main__":
    _main()
