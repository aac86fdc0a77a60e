"""CPU restatement of one whole decode step of the reference
(model/forward.rs:2548-2780) and of its greedy loop (generate/mod.rs).

TEST INFRASTRUCTURE ONLY: imported by tests/ to check the GPU decoder.  The
arithmetic is the oracle library's (oracle/rv_oracle.c); this module only
sequences it the way forward_token_traced does: embedding row, then per
layer attn_norm -> Q8_K / Q8_0 -> attn_q / attn_k / attn_v GEMVs -> QK-norm,
RoPE, f16 append, attention -> Q8_K -> attn_output GEMV -> residual add ->
the MoE block; final norm -> Q8_K -> lm_head.  Every dot uses the lane model
of the AVX2 arm (bit-identical to it, and portable).
"""
from __future__ import annotations

import numpy as np

from . import oracle as O


def synthetic_host(cfg, seed: int, layers, threads: int = 8):
    """CPU twin of ramvamp_b200.model.Qwen3Weights.synthetic for the listed
    layers: the same seeded values (or_synth_normal, bit-identical to the GPU
    generator) at the same offsets, through the oracle's restatement of the
    reference's quantizers.  Returns (weights dict, MoE layers) for RefModel."""
    from .layout import layer_layout

    H, off = cfg.hidden, [0]

    def normal(n, sigma, keep=True):
        x = O.synth_normal(seed, off[0], sigma, n) if keep else None
        off[0] += n
        return x

    def norm_w(n, keep=True):
        x = normal(n, 0.05, keep)
        return None if x is None else (np.float32(1.0) + x).astype(np.float32)

    def q(fmt, x):
        return O.quantize_weights(fmt, x)

    out_layers, moe = [], []
    for l in range(cfg.n_layers):
        keep = l in layers
        v_fmt = O.Q6_K if cfg.q6k_layer(l) else O.Q4_K
        d = dict(attn_norm=norm_w(H, keep))
        x = normal(cfg.q_dim * H, 0.02, keep); d["attn_q"] = q(O.Q4_K, x) if keep else None
        x = normal(cfg.kv_dim * H, 0.02, keep); d["attn_k"] = q(O.Q8_0, x) if keep else None
        x = normal(cfg.kv_dim * H, 0.02, keep); d["attn_v"] = q(v_fmt, x) if keep else None
        d["attn_v_format"] = v_fmt
        x = normal(H * cfg.q_dim, 0.02, keep); d["attn_output"] = q(O.Q5_K, x) if keep else None
        d["attn_q_norm"] = norm_w(cfg.head_dim, keep)
        d["attn_k_norm"] = norm_w(cfg.head_dim, keep)
        ffn_norm = norm_w(H, keep)
        router = normal(cfg.n_experts * H, 0.02, keep)
        if keep:
            lay = layer_layout(l, hidden=H, moe=cfg.moe, n_experts=cfg.n_experts,
                               down_format=O.Q6_K if cfg.q6k_layer(l) else O.Q4_K)
            blobs = O.fill_layer_synthetic(lay, seed * 1000 + l, 0.02, threads)
            moe.append(O.make_layer(H, cfg.moe, cfg.n_experts, cfg.top_k, cfg.eps, ffn_norm, router, blobs,
                                    lay.stride, lay.gate_off, lay.up_off, lay.down_off, lay.gate_format,
                                    lay.up_format, lay.down_format))
            out_layers.append(d)
    weights = dict(layers=out_layers)
    weights["token_embd"] = q(O.Q4_K, normal(cfg.vocab * H, 1.0))
    weights["output_norm"] = norm_w(H)
    weights["lm_head"] = q(O.Q6_K, normal(cfg.vocab * H, 0.02))
    return weights, moe


class RefModel:
    def __init__(self, cfg, weights: dict, moe_layers, max_positions: int, threads: int = 8, impl=None):
        """weights: host numpy copies -- token_embd, output_norm, lm_head and
        a list `layers` of dicts (attn_norm, attn_q, attn_k, attn_v,
        attn_v_format, attn_output, attn_q_norm, attn_k_norm); moe_layers:
        one oracle MoeLayer per layer (ffn_norm, router, expert blobs).
        impl: the dot arm (default the lane model, bit-identical to AVX2)."""
        self.cfg, self.w, self.moe_layers, self.threads = cfg, weights, moe_layers, threads
        self.impl = O.LANES if impl is None else impl
        kv = max_positions * cfg.kv_dim
        self.caches = [(np.zeros(kv, np.uint16), np.zeros(kv, np.uint16)) for _ in range(cfg.n_layers)]

    def step(self, token: int, position: int) -> np.ndarray:
        cfg, w, T = self.cfg, self.w, self.threads
        H, L = cfg.hidden, self.impl
        rb = H // 256 * 144
        x = O.dequantize_row(O.Q4_K, w["token_embd"][token * rb:(token + 1) * rb])
        for l, lw in enumerate(w["layers"]):
            normed = O.rmsnorm(x, lw["attn_norm"], cfg.eps)
            a8k = O.quantize_row_q8_k(normed)
            a80 = O.quantize_row_q8_0(normed, O.SCALAR)
            q = O.gemv(O.Q4_K, lw["attn_q"], H, cfg.q_dim, a8k, impl=L, threads=T)
            k = O.gemv_q8_0(lw["attn_k"], H, cfg.kv_dim, a80, impl=L, threads=T)
            v = O.gemv(lw["attn_v_format"], lw["attn_v"], H, cfg.kv_dim, a8k, impl=L, threads=T)
            kc, vc = self.caches[l]
            out, _, _ = O.attn_decode_step(q, k, v, lw["attn_q_norm"], lw["attn_k_norm"], kc, vc, position,
                                           cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.eps, cfg.rope_theta)
            o = O.gemv(O.Q5_K, lw["attn_output"], cfg.q_dim, H, O.quantize_row_q8_k(out), impl=L, threads=T)
            x = (x + o).astype(np.float32)  # vec_add
            x, _, _, _ = O.moe_decode(self.moe_layers[l], x[None, :], impl=L, threads=T)
            x = x.reshape(-1)
        normed = O.rmsnorm(x, w["output_norm"], cfg.eps)
        return O.gemv(O.Q6_K, w["lm_head"], H, cfg.vocab, O.quantize_row_q8_k(normed), impl=L, threads=T)

    def generate(self, prompt, n_new: int, on_logits=None):
        """Greedy continuation: the prompt one token per step, then each
        argmax (first index wins ties) as the next input."""
        from .layout import top1

        tok, out = prompt[0], []
        for i in range(len(prompt) + n_new - 1):
            logits = self.step(tok, i)
            if on_logits is not None:
                on_logits(i, logits)
            nxt = top1(logits)
            if i + 1 < len(prompt):
                tok = prompt[i + 1]
            else:
                out.append(nxt)
                tok = nxt
        return out
