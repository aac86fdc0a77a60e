"""GPU parity of the MoE block (rv_moe_forward) against the CPU oracle.

Geometry is Qwen3-30B-A3B's (hidden 2048, moe 768, 128 experts, top-8) with
weights drawn and quantized on the GPU, copied to the host for the oracle.
Every intermediate and the final residual are compared bit for bit.
"""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

H, M, E, K = 2048, 768, 128, 8
THREADS = max(1, min(32, os.cpu_count() or 1))


@pytest.fixture(scope="module")
def rv():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import ramvamp_b200

    return ramvamp_b200


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


class Layer:
    def __init__(self, rv, orc, table, li, router, ffn_norm, router_np, norm_np):
        self.li = li
        L = table.layouts[li]
        v = table.view(li, 0)
        self.blobs = host(rv.alias(v.blob, E * L.stride, torch.uint8))
        self.router, self.ffn_norm = router, ffn_norm
        self.oracle = orc.make_layer(H, M, E, K, 1e-6, norm_np, router_np, self.blobs, L.stride,
                                     L.gate_off, L.up_off, L.down_off, L.gate_format, L.up_format,
                                     L.down_format)


@pytest.fixture(scope="module")
def world(rv, orc):
    layouts = [rv.qwen3_layer_layout(0), rv.qwen3_layer_layout(6)]  # Q6_K down, Q4_K down
    table = rv.ExpertTable(layouts, device=0)
    table.fill_synthetic(0, seed=1234, sigma=0.02)
    table.fill_synthetic(1, seed=4321, sigma=0.02)
    router = rv.synth_normal(99, 0, 0.02, E * H).view(E, H).contiguous()
    ffn_norm = torch.ones(H, dtype=torch.float32, device="cuda")
    router_np, norm_np = host(router), host(ffn_norm)
    layers = [Layer(rv, orc, table, i, router, ffn_norm, router_np, norm_np) for i in range(2)]
    eng = rv.MoeEngine(H, M, E, K, True, 1e-6, max_tokens=512, device=0)
    return table, layers, eng


def inputs(rv, T, seed):
    return rv.synth_normal(seed, 0, 1.0, T * H).view(T, H).contiguous()


def run_gpu(rv, world, li, x):
    table, layers, eng = world
    res = x.clone()
    T = x.shape[0]
    ids = torch.empty(T * K, dtype=torch.int32, device="cuda")
    w = torch.empty(T * K, dtype=torch.float32, device="cuda")
    eng.forward(table, li, layers[li].ffn_norm, layers[li].router, res, ids, w)
    return host(res), host(ids).view(np.uint32).reshape(T, K), host(w).reshape(T, K)


def taps(rv, eng, T):
    t = eng.taps()
    a = lambda p, n, dt=torch.float32: host(rv.alias(p, n, dt))
    n = int(a(t.index_start, E + 1, torch.int32)[E])  # positions: T*K, or the speculated pairs
    return dict(
        normed=a(t.normed, T * H).reshape(T, H),
        acts=a(t.acts, T * t.acts_stride, torch.uint8).reshape(T, t.acts_stride),
        logits=a(t.logits, T * E).reshape(T, E),
        index=a(t.index, n, torch.int32).view(np.uint32),
        swiglu=a(t.swiglu, n * M).reshape(n, M),
        acts_moe=a(t.acts_moe, n * t.acts_moe_stride, torch.uint8).reshape(n, t.acts_moe_stride),
        staged=a(t.staged, T * K * H).reshape(T * K, H),
    )


UNSELECTED = 0xFFFFFFFF  # a speculated position the exact routing did not select


@pytest.mark.parametrize("li", [0, 1])
def test_decode_token_bit_identical_with_every_intermediate(rv, orc, world, li):
    """forward.rs:2654-2754 for one token: normed, Q8_K, logits, top-8,
    weights, SwiGLU, intermediate Q8_K, expert outputs and residual."""
    table, layers, eng = world
    for seed in (1, 2, 3):
        x = inputs(rv, 1, seed)
        res, ids, w = run_gpu(rv, world, li, x)
        g = taps(rv, eng, 1)
        want, wids, ww, t = orc.moe_decode(layers[li].oracle, host(x), threads=THREADS, taps=True)
        assert bits(g["normed"]).tobytes() == bits(t["normed"]).tobytes()
        assert g["acts"][0, :8 * 292].tobytes() == t["acts"].view(np.uint8).tobytes()
        assert bits(g["logits"]).tobytes() == bits(t["logits"]).tobytes()
        assert (ids == wids).all()
        assert bits(w).tobytes() == bits(ww).tobytes()
        gate, up = t["gate_up"][:, 0, :], t["gate_up"][:, 1, :]
        sw = np.stack([orc.swiglu_combine(gate[p], up[p]) for p in range(K)])
        amoe = t["acts_moe"].view(np.uint8).reshape(K, 3 * 292)
        seen = []
        for pos, pair in enumerate(g["index"]):
            if pair == UNSELECTED:
                continue
            seen.append(pair)
            assert bits(g["swiglu"][pos]).tobytes() == bits(sw[pair]).tobytes()
            assert g["acts_moe"][pos, :3 * 292].tobytes() == amoe[pair].tobytes()
        assert sorted(seen) == list(range(K))
        assert bits(g["staged"]).tobytes() == bits(t["staged"]).tobytes()
        assert bits(res).tobytes() == bits(want).tobytes()


def test_batched_decode_tokens_match_token_major(rv, orc, world):
    """Five tokens in one call equal five single-token decodes (bitwise)."""
    table, layers, eng = world
    x = inputs(rv, 5, 17)
    res, ids, w = run_gpu(rv, world, 0, x)
    want, wids, ww, _ = orc.moe_decode(layers[0].oracle, host(x), threads=THREADS)
    assert (ids == wids).all() and bits(w).tobytes() == bits(ww).tobytes()
    assert bits(res).tobytes() == bits(want).tobytes()


@pytest.mark.parametrize("T,li", [(64, 0), (64, 1), (512, 0)])
def test_prefill_bit_identical(rv, orc, world, T, li):
    """run_chunk (prefill.rs:2136-2263): router per row, CSR dispatch,
    per-expert batched FFN, top-k-order reduce."""
    table, layers, eng = world
    x = inputs(rv, T, 100 + T + li)
    res, ids, w = run_gpu(rv, world, li, x)
    want, wids, ww = orc.moe_prefill(layers[li].oracle, host(x), threads=THREADS)
    assert (ids == wids).all()
    assert bits(w).tobytes() == bits(ww).tobytes()
    diff = np.nonzero(bits(res) != bits(want))
    assert diff[0].size == 0, (diff[0][:5], diff[1][:5])
    # The CSR index is a permutation of the T*K pairs (prefill.rs:3698).
    g = taps(rv, eng, T)
    assert sorted(g["index"].tolist()) == list(range(T * K))


def test_forward_host_equals_forward(rv, world):
    table, layers, eng = world
    x = inputs(rv, 7, 55)
    res, ids, w = run_gpu(rv, world, 0, x)
    xh = host(x).copy()
    ih = np.zeros((7, K), np.uint32)
    wh = np.zeros((7, K), np.float32)
    eng.forward_host(table, 0, layers[0].ffn_norm, layers[0].router, xh, ih, wh)
    assert bits(xh).tobytes() == bits(res).tobytes()
    assert (ih == ids).all() and bits(wh).tobytes() == bits(w).tobytes()


def test_router_tie_goes_to_lowest_expert(rv, orc, world):
    """forward.rs:2688-2699: equal probabilities, first index wins."""
    table, layers, eng = world
    x = inputs(rv, 2, 77)
    router = layers[0].router.clone()
    router[5] = 0.01 * x[0]  # aligned with token 0: experts 5 and 9 lead, tied
    router[9] = router[5]
    res = x.clone()
    ids = torch.empty(2 * K, dtype=torch.int32, device="cuda")
    w = torch.empty(2 * K, dtype=torch.float32, device="cuda")
    eng.forward(table, 0, layers[0].ffn_norm, router, res, ids, w)
    got = host(ids).reshape(2, K)
    assert list(got[0][:2]) == [5, 9]
    L = orc.make_layer(H, M, E, K, 1e-6, host(layers[0].ffn_norm), host(router), layers[0].blobs,
                       table.layouts[0].stride, table.layouts[0].gate_off, table.layouts[0].up_off,
                       table.layouts[0].down_off, 0, 0, 2)
    want, wids, ww, _ = orc.moe_decode(L, host(x), threads=THREADS)
    assert (got.view(np.uint32) == wids).all()
    assert bits(host(res)).tobytes() == bits(want).tobytes()


def oracle_with_router(orc, table, layers, router):
    return orc.make_layer(H, M, E, K, 1e-6, host(layers[0].ffn_norm), host(router), layers[0].blobs,
                          table.layouts[0].stride, table.layouts[0].gate_off, table.layouts[0].up_off,
                          table.layouts[0].down_off, 0, 0, 2)


def test_decode_logit_bounds_hold_and_cover_top_k(rv, world):
    """Speculative decode dispatch: every router logit lies in its (lo, hi)
    interval, and the experts with hi + 2^-18 >= the K-th largest lo hold
    the exact top-k -- usually exactly k of them."""
    table, layers, eng = world
    sizes = []
    for li in (0, 1):
        for seed in range(20, 32):
            T = 1 + seed % 4
            x = inputs(rv, T, seed)
            _, ids, _ = run_gpu(rv, world, li, x)
            t = eng.taps()
            lg = host(rv.alias(t.logits, T * E, torch.float32)).reshape(T, E)
            b = host(rv.alias(t.logit_bounds, T * E * 2, torch.float32)).reshape(T, E, 2)
            assert (b[..., 0] <= lg).all() and (lg <= b[..., 1]).all()
            assert (b[..., 1] - b[..., 0] < 1e-2).all()
            for tt in range(T):
                thr = np.sort(b[tt, :, 0])[::-1][K - 1]
                spec = np.nonzero(b[tt, :, 1].astype(np.float64) + 2.0 ** -18 >= thr)[0]
                assert set(ids[tt].tolist()) <= set(spec.tolist())
                sizes.append(len(spec))
    assert np.mean(sizes) < K + 0.5, sizes


def test_decode_speculation_with_a_tie_at_the_cut(rv, orc, world):
    """Two experts tied for the K-th place are both speculated; the exact
    routing keeps the lower index (forward.rs:2688-2699) and the result is
    the oracle's, bit for bit."""
    table, layers, eng = world
    x = inputs(rv, 1, 91)
    run_gpu(rv, world, 0, x)
    order = np.argsort(-taps(rv, eng, 1)["logits"][0], kind="stable")
    kth, nxt = int(order[K - 1]), int(order[K])
    router = layers[0].router.clone()
    router[nxt] = router[kth]
    res = x.clone()
    ids = torch.empty(K, dtype=torch.int32, device="cuda")
    w = torch.empty(K, dtype=torch.float32, device="cuda")
    eng.forward(table, 0, layers[0].ffn_norm, router, res, ids, w)
    g = taps(rv, eng, 1)
    assert len(g["index"]) > K and (g["index"] == UNSELECTED).sum() == len(g["index"]) - K
    want, wids, ww, _ = orc.moe_decode(oracle_with_router(orc, table, layers, router), host(x), threads=THREADS)
    assert (host(ids).view(np.uint32) == wids[0]).all() and min(kth, nxt) in wids[0]
    assert bits(host(w)).tobytes() == bits(ww[0]).tobytes()
    assert bits(host(res)).tobytes() == bits(want).tobytes()


@pytest.mark.parametrize("T", [1, 2])
def test_decode_speculation_of_every_expert(rv, orc, world, T):
    """Identical router rows tie every logit: all experts are speculated
    (more units than the expert grids hold, so their CTAs stride), and the
    exact routing picks experts 0..K-1."""
    table, layers, eng = world
    x = inputs(rv, T, 93)
    router = (0.01 * x[0]).expand(E, H).contiguous()
    res = x.clone()
    ids = torch.empty(T * K, dtype=torch.int32, device="cuda")
    w = torch.empty(T * K, dtype=torch.float32, device="cuda")
    eng.forward(table, 0, layers[0].ffn_norm, router, res, ids, w)
    g = taps(rv, eng, T)
    assert len(g["index"]) == T * E
    want, wids, ww, _ = orc.moe_decode(oracle_with_router(orc, table, layers, router), host(x), threads=THREADS)
    got = host(ids).view(np.uint32).reshape(T, K)
    assert (got == wids).all() and (got == np.arange(K)).all()
    assert bits(host(w)).tobytes() == bits(ww.reshape(-1)).tobytes()
    assert bits(host(res)).tobytes() == bits(want).tobytes()
    rv.device_status(0)


@pytest.mark.parametrize("env,val", [("RV_DECODE_SPEC", "0")])
def test_decode_pipelines_are_identical(rv, world, monkeypatch, env, val):
    """RV_DECODE_SPEC=0 (routing first, then the experts) gives the same
    bits as the default speculative pipeline."""
    table, layers, eng = world
    monkeypatch.setenv(env, val)
    other = rv.MoeEngine(H, M, E, K, True, 1e-6, max_tokens=8, device=0)
    for li, T, seed in ((0, 1, 41), (1, 1, 42), (0, 1, 45), (0, 5, 43), (1, 8, 44)):
        x = inputs(rv, T, seed)
        a = x.clone()
        b = x.clone()
        eng.forward(table, li, layers[li].ffn_norm, layers[li].router, a)
        other.forward(table, li, layers[li].ffn_norm, layers[li].router, b)
        assert bits(host(a)).tobytes() == bits(host(b)).tobytes()
    rv.device_status(0)


def test_forward_errors(rv, world):
    table, layers, eng = world
    x = torch.zeros(513, H, device="cuda")
    with pytest.raises(rv.KernelError) as e:
        eng.forward(table, 0, layers[0].ffn_norm, layers[0].router, x)
    assert e.value.kind == "LengthMismatch"
    with pytest.raises(rv.KernelError) as e:
        eng.forward(table, 5, layers[0].ffn_norm, layers[0].router, x[:1])
    assert e.value.kind == "LayerOutOfRange"
    with pytest.raises(rv.KernelError) as e:
        eng.forward(table, 0, layers[0].ffn_norm, layers[0].router, x[:1], flags=7)
    assert e.value.kind == "InvalidArgument"
    rv.device_status(0)  # no device-side failure recorded by any test above


def test_expert_table_step_protocol(rv, world):
    """io/stream.rs:1472-2160 step API on the resident table."""
    table, layers, eng = world
    table.begin_layer(0, [5, 9, 5, 127])
    assert table.hits() == [(0, 5), (1, 9), (3, 127)]  # duplicate listed once
    assert table.misses() == []
    table.await_misses()
    v = table.view(0, 9)
    L = table.layouts[0]
    assert v.up - v.gate == L.up_off and v.down - v.gate == L.down_off
    assert (v.gate_format, v.down_format) == (rv.QuantFormat.Q4_K, rv.QuantFormat.Q6_K)
    with pytest.raises(rv.KernelError) as e:
        table.begin_layer(1, [0])
    assert e.value.kind == "Protocol"
    table.end_layer(0)
    with pytest.raises(rv.KernelError) as e:
        table.end_layer(0)
    assert e.value.kind == "Protocol"
    with pytest.raises(rv.KernelError) as e:
        table.begin_layer(0, [128])
    assert e.value.kind == "RoutedExpertOutOfRange"
    s = table.stats()
    assert s["accesses"] == s["hits"] >= 3
