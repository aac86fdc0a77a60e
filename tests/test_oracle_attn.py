"""Pin the oracle's attention half of the decode step (NeoX RoPE, decode
attention, the f16 KV append) against the reference's own tests, and check
the C-ABI's attention validation.  CPU only."""
import math

import numpy as np
import pytest

THETA = 1e7  # rope.rs tests: the v0 pin


def _rope_f64(x, position, theta):
    """rope.rs:113-130 (rope_ref): the formula in f64."""
    x = np.asarray(x, np.float64)
    half = x.size // 2
    out = x.copy()
    for i in range(half):
        ang = position * theta ** (-2.0 * i / x.size)
        c, s = math.cos(ang), math.sin(ang)
        out[i] = x[i] * c - x[i + half] * s
        out[i + half] = x[i] * s + x[i + half] * c
    return out


def test_rope_position_zero_is_identity(orc):
    """rope.rs:133-142."""
    rng = np.random.default_rng(0)
    for dim in (4, 128):
        x = rng.uniform(-5, 5, dim).astype(np.float32)
        assert orc.rope_neox_heads(x, 1, dim, 0, THETA).tobytes() == x.tobytes()


def test_rope_known_angles_head_dim_4(orc):
    """rope.rs:144-176 (hand-computed f64 values, 1e-6 relative)."""
    cases = [(1, [-1.9841106485555495, 1.9987349889570154, 2.4623779024123156, 4.000632255521494]),
             (3, [-1.413352520780047, 1.9962043673770753, -2.828857481741469, 4.001895566311631])]
    for position, want in cases:
        got = orc.rope_neox_heads(np.array([1, 2, 3, 4], np.float32), 1, 4, position, THETA)
        assert np.all(np.abs(got - np.array(want)) <= 1e-6 * np.abs(want) + 1e-30)


def test_rope_matches_f64_reference_head_dim_128(orc):
    """rope.rs:178-194 (1e-6 relative with a 1e-6 absolute floor)."""
    rng = np.random.default_rng(0xD1)
    for position in (1, 2, 17, 4096, 100_000):
        x = rng.uniform(-3, 3, 128).astype(np.float32)
        want = _rope_f64(x, position, THETA)
        got = orc.rope_neox_heads(x, 1, 128, position, THETA).astype(np.float64)
        assert np.all(np.abs(got - want) <= 1e-6 * np.abs(want) + 1e-6)


def test_rope_preserves_pair_magnitude_and_heads_are_independent(orc):
    """rope.rs:196-224."""
    rng = np.random.default_rng(0xF00D)
    x = rng.uniform(-8, 8, 128).astype(np.float32)
    y = orc.rope_neox_heads(x, 1, 128, 90_210, THETA).astype(np.float64)
    before = np.hypot(x[:64].astype(np.float64), x[64:].astype(np.float64))
    after = np.hypot(y[:64], y[64:])
    assert np.all(np.abs(after - before) <= 1e-5 * before)
    heads = rng.uniform(-2, 2, 3 * 128).astype(np.float32)
    multi = orc.rope_neox_heads(heads, 3, 128, 77, THETA)
    for h in range(3):
        one = orc.rope_neox_heads(heads[128 * h:128 * h + 128], 1, 128, 77, THETA)
        assert multi[128 * h:128 * h + 128].tobytes() == one.tobytes()


def test_rope_invalid_head_dim(orc):
    """rope.rs:226-241."""
    for hd in (0, 3):
        with pytest.raises(orc.OracleError) as e:
            orc.rope_neox_heads(np.zeros(max(hd, 1), np.float32), 1, hd, 1, THETA)
        assert e.value.kind == "InvalidHeadDim"


def _f16(x):
    return np.asarray(x, np.float32).astype(np.float16).view(np.uint16)


def test_attention_single_position_returns_v_row(orc):
    """attention.rs:1523-1555: one cached position makes the weight exactly
    1, so each head's output is its kv head's f16-rounded V row, bit-exact."""
    n_kv, n_q, hd = 4, 32, 128
    rng = np.random.default_rng(0x5EED)
    k = _f16(rng.uniform(-1, 1, n_kv * hd))
    v_f = rng.uniform(-1, 1, n_kv * hd).astype(np.float32)
    v = _f16(v_f)
    q = rng.uniform(-1, 1, n_q * hd).astype(np.float32)
    out = orc.attention(q, k, v, 1, n_q, n_kv, hd, 1.0 / math.sqrt(hd))
    for h in range(n_q):
        col = (h // 8) * hd
        want = v[col:col + hd].view(np.float16).astype(np.float32)
        assert out[h * hd:(h + 1) * hd].tobytes() == want.tobytes()


def test_attention_doubling_scale_squares_the_odds_ratio(orc):
    """attention.rs:1894-1927."""
    k = _f16([0, 0, 0, 0, 1, 0, 0, 0])
    v = _f16([0, 0, 0, 0, 1, 1, 1, 1])
    q = np.array([1, 0, 0, 0], np.float32)
    p = lambda s: float(orc.attention(q, k, v, 2, 1, 1, 4, s)[0])
    s = np.float32(0.7)
    p1, p2 = p(s), p(2 * s)
    sig = lambda x: 1 / (1 + math.exp(-x))
    assert abs(p1 - sig(float(s))) <= 1e-5 * sig(float(s))
    assert abs(p2 - sig(2 * float(s))) <= 1e-5 * sig(2 * float(s))
    odds = lambda x: x / (1 - x)
    assert abs(odds(p2) - odds(p1) ** 2) <= 1e-4 * odds(p1) ** 2
    assert p2 > p1


def test_attention_group_of_one_maps_heads(orc):
    """attention.rs:2425-2470: with as many query as kv heads, head h reads kv
    head h (kv head j wins at position j and carries marker 10j + t)."""
    n, hd = 4, 8
    k = np.zeros((n, n * hd), np.float32)
    v = np.zeros((n, n * hd), np.float32)
    for j in range(n):
        k[j, j * hd] = 4.0
        for t in range(n):
            v[t, j * hd:(j + 1) * hd] = 10 * j + t
    q = np.zeros(n * hd, np.float32)
    for h in range(n):
        q[h * hd] = 4.0
    out = orc.attention(q, _f16(k).reshape(-1), _f16(v).reshape(-1), n, n, n, hd, 1.0)
    for h in range(n):
        weights = np.exp([16.0 if t == h else 0.0 for t in range(n)])
        assert abs(out[h * hd] - np.dot(weights / weights.sum(), [10 * h + t for t in range(n)])) < 1e-3


def test_decode_step_appends_f16_and_attends(orc):
    """forward.rs:2614-2631: after a step, cache row `position` holds the f16
    of the normed, rotated k and of v, and the output equals attention over
    the cache."""
    n_q, n_kv, hd, P = 4, 2, 16, 6
    rng = np.random.default_rng(3)
    kc = np.zeros(P * n_kv * hd, np.uint16)
    vc = np.zeros_like(kc)
    qn = rng.uniform(0.5, 1.5, hd).astype(np.float32)
    kn = rng.uniform(0.5, 1.5, hd).astype(np.float32)
    for pos in range(P):
        q = rng.standard_normal(n_q * hd).astype(np.float32)
        k = rng.standard_normal(n_kv * hd).astype(np.float32)
        v = rng.standard_normal(n_kv * hd).astype(np.float32)
        out, qr, kr = orc.attn_decode_step(q, k, v, qn, kn, kc, vc, pos, n_q, n_kv, hd, 1e-6, THETA)
        row = slice(pos * n_kv * hd, (pos + 1) * n_kv * hd)
        assert kc[row].tobytes() == np.array([orc.f32_to_f16(float(x)) for x in kr], np.uint16).tobytes()
        assert vc[row].tobytes() == _f16(v).tobytes()
        want = orc.attention(qr, kc, vc, pos + 1, n_q, n_kv, hd, np.float32(1) / np.sqrt(np.float32(hd)))
        assert out.tobytes() == want.tobytes()


# ------------------------------------------------------ C-ABI validation
@pytest.fixture(scope="module")
def rv():
    import ramvamp_b200

    return ramvamp_b200


def test_c_abi_attention_validation(rv):
    """Geometry is checked before any CUDA call, with the reference's error
    kinds (PrimitiveError::InvalidHeadDim / LengthMismatch, ...)."""
    import ctypes

    lib = rv.lib()
    name = lambda c: lib.rv_status_name(c).decode()
    h = ctypes.c_void_p()
    for cfg, kind in [((2, 32, 4, 0, 16, 1e7, 1e-6), "InvalidHeadDim"), ((2, 32, 4, 7, 16, 1e7, 1e-6), "InvalidHeadDim"),
                      ((2, 32, 5, 128, 16, 1e7, 1e-6), "LengthMismatch"), ((0, 32, 4, 128, 16, 1e7, 1e-6), "Empty"),
                      ((2, 32, 4, 136 * 2, 16, 1e7, 1e-6), "Unimplemented")]:
        c = rv._lib.AttnConfig(*cfg)
        assert name(lib.rv_attn_create(0, ctypes.byref(c), ctypes.byref(h))) == kind
    assert name(lib.rv_rope_neox_heads(None, 8, 2, 3, 1, 1e7, None)) == "InvalidHeadDim"
    assert name(lib.rv_rope_neox_heads(None, 7, 2, 4, 1, 1e7, None)) == "LengthMismatch"
    assert lib.rv_rope_neox_heads(None, 0, 0, 4, 1, 1e7, None) == 0
    a = lambda *args: name(lib.rv_attention(None, None, None, *args, None, None))
    assert a(0, 32, 4, 128, 0.1, None, 0) == "Empty"
    assert a(5, 32, 5, 128, 0.1, None, 1000) == "LengthMismatch"
    assert a(5, 32, 4, 128, 0.1, None, 319) == "LengthMismatch"
    assert a(5, 32, 4, 128, 0.1, None, 320) == "InvalidArgument"
