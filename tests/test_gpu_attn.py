"""GPU parity of the attention half of the decode step (NeoX RoPE, decode
attention, QK-norm + f16 KV append through the engine) against the CPU
oracle, bit for bit, through the C ABI."""
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

THETA = 1e7


@pytest.fixture(scope="module")
def rv():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import ramvamp_b200

    return ramvamp_b200


def dev(a):
    return torch.from_numpy(np.array(a, copy=True)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def _f16(x):
    return np.asarray(x, np.float32).astype(np.float16).view(np.uint16)


@pytest.mark.parametrize("head_dim", [4, 128, 256])
def test_rope_bit_identical(rv, orc, head_dim):
    """rope.rs:80-111 on the GPU, the reference's test positions and more."""
    rng = np.random.default_rng(head_dim)
    n_heads = 32 if head_dim == 128 else 3
    for position in (0, 1, 2, 3, 17, 511, 4096, 100_000, 2**31 + 5):
        x = rng.uniform(-5, 5, n_heads * head_dim).astype(np.float32)
        got = host(rv.rope_neox_heads(dev(x), n_heads, head_dim, position, THETA))
        assert got.tobytes() == orc.rope_neox_heads(x, n_heads, head_dim, position, THETA).tobytes(), position
    x = dev(rng.uniform(-1, 1, n_heads * head_dim).astype(np.float32))
    want = orc.rope_neox_heads(host(x), n_heads, head_dim, 9, 1e6)
    rv.CudaBackend().rope_neox_heads(x, n_heads, head_dim, 9, 1e6)
    assert host(x).tobytes() == want.tobytes()


@pytest.mark.parametrize("positions", [1, 2, 7, 128, 129, 576, 1000, 4097])
def test_attention_bit_identical(rv, orc, positions):
    """attention.rs:1075-1303 (scalar arm, which its AVX2 arm equals) over
    random f16 caches at Qwen3 geometry (32 query heads, 4 kv heads, 128)."""
    n_q, n_kv, hd = 32, 4, 128
    rng = np.random.default_rng(positions)
    k = _f16(rng.standard_normal(positions * n_kv * hd))
    v = _f16(rng.standard_normal(positions * n_kv * hd))
    q = (rng.standard_normal(n_q * hd) * 0.5).astype(np.float32)
    scale = float(np.float32(1) / np.sqrt(np.float32(hd)))
    want = orc.attention(q, k, v, positions, n_q, n_kv, hd, scale)
    got = host(rv.attention(dev(q), dev(k), dev(v), positions, n_q, n_kv, hd, scale))
    assert got.tobytes() == want.tobytes()


def test_attention_peaked_and_tied_scores(rv, orc):
    """Scores that underflow the exponential for most positions, exact ties,
    and a group of one (attention.rs:2425)."""
    n, hd, P = 4, 8, 300
    rng = np.random.default_rng(11)
    k = np.zeros((P, n * hd), np.float32)
    k[::3, :] = rng.standard_normal((len(range(0, P, 3)), n * hd)) * 30
    k[5] = k[7]  # a tie
    kb, vb = _f16(k).reshape(-1), _f16(rng.standard_normal((P, n * hd))).reshape(-1)
    q = rng.standard_normal(n * hd).astype(np.float32)
    for scale in (1.0, 0.35355339):
        want = orc.attention(q, kb, vb, P, n, n, hd, scale)
        got = host(rv.attention(dev(q), dev(kb), dev(vb), P, n, n, hd, scale))
        assert got.tobytes() == want.tobytes()


def test_decode_steps_bit_identical(rv, orc):
    """forward.rs:2614-2631 step by step on two layers: the normed, rotated
    q and k, the cache rows, and the attention output against the oracle for
    every position 0..299."""
    n_layers, n_q, n_kv, hd, P = 2, 32, 4, 128, 300
    eng = rv.AttnEngine(n_layers, n_q, n_kv, hd, max_positions=P, rope_theta=THETA, eps=1e-6)
    rng = np.random.default_rng(5)
    qn = [rng.uniform(0.5, 1.5, hd).astype(np.float32) for _ in range(n_layers)]
    kn = [rng.uniform(0.5, 1.5, hd).astype(np.float32) for _ in range(n_layers)]
    caches = [(np.zeros(P * n_kv * hd, np.uint16), np.zeros(P * n_kv * hd, np.uint16)) for _ in range(n_layers)]
    qn_d, kn_d = [dev(x) for x in qn], [dev(x) for x in kn]
    for pos in range(P):
        for layer in range(n_layers):
            q = (rng.standard_normal(n_q * hd) * 2).astype(np.float32)
            k = (rng.standard_normal(n_kv * hd) * 2).astype(np.float32)
            v = rng.standard_normal(n_kv * hd).astype(np.float32)
            qd, kd, vd = dev(q), dev(k), dev(v)
            out = eng.decode(layer, pos, qd, kd, vd, qn_d[layer], kn_d[layer])
            want, qr, kr = orc.attn_decode_step(q, k, v, qn[layer], kn[layer], caches[layer][0], caches[layer][1],
                                                pos, n_q, n_kv, hd, 1e-6, THETA)
            if pos % 23 == 0 or pos == P - 1:
                assert host(qd).tobytes() == qr.tobytes(), (pos, layer)
                assert host(kd).tobytes() == kr.tobytes(), (pos, layer)
                assert host(out).tobytes() == want.tobytes(), (pos, layer)
    for layer in range(n_layers):
        kc, vc = eng.cache_tensors(layer)
        assert host(kc).view(np.uint16).reshape(-1).tobytes() == caches[layer][0].tobytes()
        assert host(vc).view(np.uint16).reshape(-1).tobytes() == caches[layer][1].tobytes()
        assert eng.len(layer) == P


def test_engine_errors_and_clear(rv):
    """PositionMismatch, CapacityExceeded, LayerOutOfRange; clear() restarts."""
    eng = rv.AttnEngine(1, 4, 2, 8, max_positions=2)
    z = lambda n: torch.zeros(n, dtype=torch.float32, device="cuda")
    q, k, v, w = z(32), z(16), z(16), torch.ones(8, device="cuda")
    with pytest.raises(rv.KernelError) as e:
        eng.decode(0, 1, q, k, v, w, w)
    assert e.value.kind == "PositionMismatch"
    with pytest.raises(rv.KernelError) as e:
        eng.decode(1, 0, q, k, v, w, w)
    assert e.value.kind == "LayerOutOfRange"
    eng.decode(0, 0, q, k, v, w, w)
    eng.decode(0, 1, q, k, v, w, w)
    with pytest.raises(rv.KernelError) as e:
        eng.decode(0, 2, q, k, v, w, w)
    assert e.value.kind == "CapacityExceeded"
    eng.clear()
    assert eng.len(0) == 0
    eng.decode(0, 0, q, k, v, w, w)
    torch.cuda.synchronize()
    rv.device_status(0)


def test_rmsnorm_quantize_bytes(rv, orc):
    """rmsnorm (norm.rs:38-60) then quantize_row_q8_k and quantize_row_q8_0,
    fused: the same bytes as the separate reference steps."""
    rng = np.random.default_rng(21)
    for n in (256, 2048, 4096):
        x = (rng.standard_normal(n) * 3).astype(np.float32)
        w = rng.uniform(0.5, 1.5, n).astype(np.float32)
        q8k = torch.zeros(n // 256 * 292, dtype=torch.uint8, device="cuda")
        q80 = torch.zeros(n // 32 * 36, dtype=torch.uint8, device="cuda")
        rv.rmsnorm_quantize(dev(x), dev(w), 1e-6, q8k, q80)
        normed = orc.rmsnorm(x, w, 1e-6)
        assert host(q8k).tobytes() == orc.quantize_row_q8_k(normed).tobytes()
        assert host(q80).tobytes() == orc.quantize_row_q8_0(normed, orc.SCALAR).tobytes()


@pytest.mark.parametrize("device_position,P,cap", [(False, 40, 40), (True, 40, 40), (True, 150, 150),
                                                   (True, 150, 300), (False, 300, 300)])
def test_attn_block_matches_reference(rv, orc, device_position, P, cap):
    """rv_attn_block (forward.rs:2572-2652 for one layer, residual in place)
    against the reference's step sequence on the oracle, over P positions
    of a cache of `cap` (the values staged in 64-position chunks).  Up to
    256 positions the block runs attention as one fused launch (host mode:
    by position; device mode: by capacity), beyond that as two: cap 300
    covers the two-launch form in both modes."""
    H, n_q, n_kv, hd = 2048, 32, 4, 128
    rng = np.random.default_rng(31)
    eng = rv.AttnEngine(1, n_q, n_kv, hd, max_positions=cap, rope_theta=1e6, eps=1e-6, hidden=H)
    qd, kvd = n_q * hd, n_kv * hd
    x_norm = rng.uniform(0.8, 1.2, H).astype(np.float32)
    wq = orc.quantize_weights(orc.Q4_K, (rng.standard_normal(qd * H) * 0.02).astype(np.float32))
    wk = orc.quantize_weights(orc.Q8_0, (rng.standard_normal(kvd * H) * 0.02).astype(np.float32))
    wv = orc.quantize_weights(orc.Q6_K, (rng.standard_normal(kvd * H) * 0.02).astype(np.float32))
    wo = orc.quantize_weights(orc.Q5_K, (rng.standard_normal(H * qd) * 0.02).astype(np.float32))
    qn, kn = rng.uniform(0.8, 1.2, hd).astype(np.float32), rng.uniform(0.8, 1.2, hd).astype(np.float32)
    d = [dev(a) for a in (x_norm, wq, wk, wv, wo, qn, kn)]
    aw = rv.attn_weights(*d, attn_q_format=rv.QuantFormat.Q4_K, attn_v_format=rv.QuantFormat.Q6_K,
                         attn_output_format=rv.QuantFormat.Q5_K)
    kc, vc = np.zeros(cap * kvd, np.uint16), np.zeros(cap * kvd, np.uint16)
    pos_d = torch.zeros(1, dtype=torch.int32, device="cuda")
    for pos in range(P):
        x = rng.standard_normal(H).astype(np.float32)
        res = dev(x)
        if device_position:
            pos_d.fill_(pos)
            eng.block(0, aw, res, position_dev=pos_d)
        else:
            eng.block(0, aw, res, position=pos)
        normed = orc.rmsnorm(x, x_norm, 1e-6)
        a8k, a80 = orc.quantize_row_q8_k(normed), orc.quantize_row_q8_0(normed, orc.SCALAR)
        q = orc.gemv(orc.Q4_K, wq, H, qd, a8k, impl=orc.LANES)
        k = orc.gemv_q8_0(wk, H, kvd, a80, impl=orc.LANES)
        v = orc.gemv(orc.Q6_K, wv, H, kvd, a8k, impl=orc.LANES)
        out, _, _ = orc.attn_decode_step(q, k, v, qn, kn, kc, vc, pos, n_q, n_kv, hd, 1e-6, 1e6)
        o = orc.gemv(orc.Q5_K, wo, qd, H, orc.quantize_row_q8_k(out), impl=orc.LANES)
        want = (x + o).astype(np.float32)
        assert host(res).tobytes() == want.tobytes(), pos
    assert eng.len(0) == (0 if device_position else P)
    rv.device_status(0)


def test_argmax_edge_cases(rv):
    """Sampler::argmax: first index wins ties, NaN never wins, all -inf or
    NaN gives 0; unaligned starts and lengths not a multiple of 4."""
    from ramvamp_b200.model import top1

    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    rng = np.random.default_rng(41)
    cases = [rng.standard_normal(151936).astype(np.float32)]
    t = rng.standard_normal(10007).astype(np.float32)
    t[[17, 5000, 9999]] = 50.0
    cases.append(t)
    cases.append(np.full(33, -np.inf, np.float32))
    cases.append(np.full(33, np.nan, np.float32))
    t = rng.standard_normal(1000).astype(np.float32)
    t[::3] = np.nan
    t[500] = np.inf
    t[900] = np.inf
    cases.append(t)
    cases.append(np.array([-np.inf, -1.0], np.float32))
    for x in cases:
        for shift in (0, 1, 2, 3):
            buf = dev(np.concatenate([np.zeros(shift, np.float32), x]))
            rc = rv.lib().rv_argmax(buf.data_ptr() + 4 * shift, x.size, out.data_ptr(), rv._stream())
            assert rc == 0
            assert int(host(out)[0]) == top1(x), (x.size, shift)
