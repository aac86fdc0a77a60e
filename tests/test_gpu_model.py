"""Whole-model greedy decode (config 1's acceptance: identical top-1 tokens
and full-vocab KL <= 1e-4 against the reference) on the GPU decoder against
the CPU restatement of the reference's step, on small and on Qwen3-geometry
models with synthetic weights.  Logits are compared bit for bit."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rv():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import ramvamp_b200

    return ramvamp_b200


def _ref_model(rv, orc, w, max_positions, threads=8):
    from oracle.model_ref import RefModel

    cfg = w.cfg
    host = lambda t: t.cpu().numpy()
    weights = dict(token_embd=host(w.token_embd), output_norm=host(w.output_norm), lm_head=host(w.lm_head),
                   layers=[dict(attn_norm=host(l.attn_norm), attn_q=host(l.attn_q), attn_k=host(l.attn_k),
                                attn_v=host(l.attn_v), attn_v_format=l.attn_v_format,
                                attn_output=host(l.attn_output), attn_q_norm=host(l.attn_q_norm),
                                attn_k_norm=host(l.attn_k_norm)) for l in w.layers])
    moe = []
    for li, l in enumerate(w.layers):
        lay = w.experts.layouts[li]
        blobs = orc.fill_layer_synthetic(lay, 1 * 1000 + li, 0.02, threads=threads)
        moe.append(orc.make_layer(cfg.hidden, cfg.moe, cfg.n_experts, cfg.top_k, cfg.eps, host(l.ffn_norm),
                                  host(l.router), blobs, lay.stride, lay.gate_off, lay.up_off, lay.down_off,
                                  lay.gate_format, lay.up_format, lay.down_format))
    return RefModel(cfg, weights, moe, max_positions, threads)


def _compare(rv, orc, cfg, prompt, n_new, graph):
    from ramvamp_b200.model import Decoder, Qwen3Weights, kl_divergence, top1

    w = Qwen3Weights.synthetic(cfg, seed=1)
    dec = Decoder(w, max_positions=64)
    if graph:
        dec.capture()
    got = []
    toks = dec.generate(prompt, n_new, on_logits=lambda i, t: got.append(t.cpu().numpy().copy()))
    ref = _ref_model(rv, orc, w, 64)
    want = []
    ref_toks = ref.generate(prompt, n_new, on_logits=lambda i, x: want.append(x.copy()))
    assert toks == ref_toks
    for i, (g, r) in enumerate(zip(got, want)):
        assert top1(g) == top1(r), i
        assert kl_divergence(r, g) <= 1e-4, i
        assert g.tobytes() == r.tobytes(), i
    rv.device_status(0)
    return toks


@pytest.mark.parametrize("graph", [False, True])
def test_greedy_decode_small_model(rv, orc, graph):
    from ramvamp_b200.model import ModelConfig

    cfg = ModelConfig(n_layers=3, hidden=256, n_heads=4, n_kv_heads=2, head_dim=128, moe=512, n_experts=8,
                      top_k=2, vocab=1000)
    prompt = [int(x) for x in np.random.default_rng(7).integers(0, cfg.vocab, 10)]
    _compare(rv, orc, cfg, prompt, 6, graph)


def test_greedy_decode_qwen3_geometry(rv, orc):
    """Qwen3-30B-A3B shapes (hidden 2048, 32/4 heads, 128 experts, top-8,
    vocab 151,936) with two layers, through the captured graph."""
    from ramvamp_b200.model import ModelConfig

    cfg = ModelConfig(n_layers=2)
    prompt = [int(x) for x in np.random.default_rng(8).integers(0, cfg.vocab, 4)]
    _compare(rv, orc, cfg, prompt, 3, graph=True)


def test_graph_replay_equals_eager(rv):
    """The captured step and the eager step give the same ids."""
    from ramvamp_b200.model import Decoder, ModelConfig, Qwen3Weights

    cfg = ModelConfig(n_layers=2, hidden=256, n_heads=4, n_kv_heads=2, head_dim=128, moe=512, n_experts=8,
                      top_k=2, vocab=1000)
    w = Qwen3Weights.synthetic(cfg, seed=3)
    prompt = [5, 17, 900, 3]
    a = Decoder(w, max_positions=32).generate(prompt, 10)
    d = Decoder(w, max_positions=32)
    d.capture()
    assert d.generate(prompt, 10) == a


def test_host_weight_twin_matches_gpu_weights(rv, orc):
    """oracle.model_ref.synthetic_host (the reference arm's weights) makes the
    same bytes as Qwen3Weights.synthetic on the GPU."""
    from oracle.model_ref import synthetic_host
    from ramvamp_b200.model import ModelConfig, Qwen3Weights

    cfg = ModelConfig(n_layers=3, hidden=256, n_heads=4, n_kv_heads=2, head_dim=128, moe=512, n_experts=8,
                      top_k=2, vocab=1000)
    w = Qwen3Weights.synthetic(cfg, seed=4)
    hw, moe = synthetic_host(cfg, 4, [1, 2])
    for key in ("token_embd", "output_norm", "lm_head"):
        assert getattr(w, key).cpu().numpy().tobytes() == hw[key].tobytes(), key
    for hl, l in zip(hw["layers"], (1, 2)):
        gl = w.layers[l]
        for key in ("attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "attn_q_norm", "attn_k_norm"):
            assert getattr(gl, key).cpu().numpy().tobytes() == hl[key].tobytes(), (l, key)
