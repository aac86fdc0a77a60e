"""Pin the CPU oracle against the reference's own known-answer tests.

Each test re-expresses a ramvamp Rust test (file:line in its docstring) on
the C restatement in oracle/.  These run on CPU only.
"""
import math
import struct

import numpy as np
import pytest

F16_SUB_ULP = 2.0 ** -24


def f32(x):
    return struct.unpack("<f", struct.pack("<f", x))[0]


# ------------------------------------------------------------------ f16
def test_f16_to_f32_known_vectors(orc):
    """kernels/quants/f16.rs:97-112."""
    c = orc.f16_to_f32
    assert c(0x0000) == 0.0
    assert c(0x8000) == 0.0 and math.copysign(1, c(0x8000)) < 0
    assert c(0x3C00) == 1.0
    assert c(0xC100) == -2.5
    assert c(0x7BFF) == 65504.0
    assert c(0x0001) == F16_SUB_ULP
    assert c(0x03FF) == 1023.0 * F16_SUB_ULP
    assert c(0x8001) == -F16_SUB_ULP
    assert c(0x7C00) == math.inf and c(0xFC00) == -math.inf
    assert math.isnan(c(0x7E00)) and math.isnan(c(0xFE01))
    assert c(0x3555) == f32(0.333_251_95)


def test_f32_to_f16_known_vectors(orc):
    """kernels/quants/f16.rs:114-133."""
    c = orc.f32_to_f16
    assert c(0.0) == 0x0000
    assert c(-0.0) == 0x8000
    assert c(1.0) == 0x3C00
    assert c(-2.5) == 0xC100
    assert c(65504.0) == 0x7BFF
    assert c(65520.0) == 0x7C00
    assert c(1e9) == 0x7C00
    assert c(math.inf) == 0x7C00 and c(-math.inf) == 0xFC00
    assert c(F16_SUB_ULP) == 0x0001
    assert c(0.5 * F16_SUB_ULP) == 0x0000
    assert c(0.75 * F16_SUB_ULP) == 0x0001
    assert c(1e-10) == 0x0000 and c(-1e-10) == 0x8000
    assert math.isnan(orc.f16_to_f32(c(math.nan)))
    nan_payload = struct.unpack("<f", struct.pack("<I", 0x7F80_0001))[0]
    assert math.isnan(orc.f16_to_f32(c(nan_payload)))


def test_f16_round_trip_all_finite(orc):
    """kernels/quants/f16.rs:135-150 (exhaustive)."""
    for bits in range(0x10000):
        if (bits >> 10) & 0x1F == 0x1F:
            continue
        assert orc.f32_to_f16(orc.f16_to_f32(bits)) == bits


def test_f32_to_f16_nearest_even(orc):
    """kernels/quants/f16.rs:152-160."""
    assert orc.f32_to_f16(1.000_488_3) == 0x3C00
    assert orc.f32_to_f16(1.000_488_4) == 0x3C01
    assert orc.f32_to_f16(1.001_464_8) == 0x3C02


# ----------------------------------------------------------------- Q8_K
@pytest.mark.parametrize("impl", [0, 1])
def test_q8_k_anchors_extreme_to_minus_127(orc, impl):
    """kernels/quants/quantize.rs:140-152."""
    x = np.zeros(256, np.float32)
    x[10] = -3.0
    x[20] = 1.5
    b = orc.quantize_row_q8_k(x, impl)[0]
    assert b["qs"][10] == -127
    assert b["qs"][20] == 64
    assert b["d"] == np.float32(1.0) / (np.float32(-127.0) / np.float32(-3.0))


@pytest.mark.parametrize("impl", [0, 1])
def test_q8_k_positive_extreme_maps_to_minus_127(orc, impl):
    """kernels/quants/quantize.rs:154-165."""
    x = np.zeros(256, np.float32)
    x[0] = 4.0
    x[1] = -2.0
    b = orc.quantize_row_q8_k(x, impl)[0]
    assert b["qs"][0] == -127
    assert b["qs"][1] == 64
    assert b["d"] == np.float32(1.0) / (np.float32(-127.0) / np.float32(4.0))


@pytest.mark.parametrize("impl", [0, 1])
def test_q8_k_zero_row_zeroes_everything(orc, impl):
    """kernels/quants/quantize.rs:167-177."""
    b = orc.quantize_row_q8_k(np.zeros(256, np.float32), impl)[0]
    assert b["d"] == 0.0 and not b["qs"].any() and not b["bsums"].any()


def test_quantize_len_mismatch_errors(orc):
    """kernels/quants/quantize.rs:179-200."""
    with pytest.raises(orc.OracleError) as e:
        orc.quantize_row_q8_k(np.zeros(100, np.float32), out_blocks=1)
    assert e.value.kind == "QuantizeLenMismatch"


def test_q8_k_bsums_match_recomputed_group_sums(orc):
    """kernels/quants/tests.rs:349-364."""
    x = orc.Lcg(9).fill(768, 5.0)
    for b in orc.quantize_row_q8_k(x):
        assert b["d"] != 0.0
        for g in range(16):
            assert int(b["bsums"][g]) == int(b["qs"][16 * g:16 * g + 16].astype(np.int32).sum())


def _tie_rows():
    """Random, tie-heavy, flat and zero rows, as avx2.rs:1568-1642 uses."""
    rng = np.random.default_rng(7)
    rows = [rng.standard_normal(1024).astype(np.float32) * 3]
    t = np.zeros(1024, np.float32)
    t[::7] = 1.0
    t[3::11] = -1.0  # equal |v|: first index must win the signed extreme
    rows.append(t)
    rows.append(np.full(1024, 0.25, np.float32))
    rows.append(np.zeros(1024, np.float32))
    r = rng.integers(-127, 128, 1024).astype(np.float32) / 2.0  # exact .5 ties after scaling
    rows.append(r)
    return rows


def test_q8_k_avx2_byte_identical_to_scalar(orc):
    """kernels/quants/avx2.rs:1568-1642."""
    if not orc.has_avx2():
        pytest.skip("host lacks AVX2")
    for x in _tie_rows():
        a = orc.quantize_row_q8_k(x, orc.SCALAR)
        b = orc.quantize_row_q8_k(x, orc.AVX2)
        assert a.tobytes() == b.tobytes()


# ---------------------------------------------------------------- dots
def _dequant_q8k(blocks):
    return np.concatenate([b["d"] * b["qs"].astype(np.float32) for b in blocks])


def _assert_dot_close(dot, w, a, rel=1e-5):
    """quants/tests.rs:27-46."""
    p = w.astype(np.float64) * a.astype(np.float64)
    r, mag = p.sum(), np.abs(p).sum()
    assert abs(float(dot) - r) <= rel * max(mag, 1e-20), (dot, r, mag)


@pytest.mark.parametrize("fmt", [0, 1, 2])
@pytest.mark.parametrize("n", [2048, 768])
def test_scalar_dot_matches_f64_ground_truth(orc, fmt, n):
    """quants/tests.rs:162-226."""
    rng = orc.Lcg(1000 + n + fmt)
    w = orc.quantize_weights(fmt, rng.fill(n, 2.0))
    acts = orc.quantize_row_q8_k(rng.fill(n, 3.0))
    d = orc.vec_dot(fmt, w, acts, orc.SCALAR)
    _assert_dot_close(d, orc.dequantize_row(fmt, w), _dequant_q8k(acts))


ALL_MIN_SCALES = bytes([0, 0, 0, 0, 0xFF, 0xFF, 0xFF, 0xFF, 0xF0, 0xF0, 0xF0, 0xF0])


def _q4k(orc, d, dmin, scales, qs):
    h = struct.pack("<HH", orc.f32_to_f16(d), orc.f32_to_f16(dmin))
    return np.frombuffer(h + bytes(scales) + bytes([qs]) * 128, np.uint8)


def _q5k(orc, d, dmin, scales, qh, qs):
    h = struct.pack("<HH", orc.f32_to_f16(d), orc.f32_to_f16(dmin))
    return np.frombuffer(h + bytes(scales) + bytes([qh]) * 32 + bytes([qs]) * 128, np.uint8)


def _q6k(orc, ql, qh, scale, d):
    return np.frombuffer(bytes([ql]) * 128 + bytes([qh]) * 64 + bytes([scale & 0xFF]) * 16
                         + struct.pack("<H", orc.f32_to_f16(d)), np.uint8)


def adversarial_blocks(orc):
    """quants/tests.rs:251-321 (q4_K, q5_K, q6_K cases)."""
    return {
        0: [_q4k(orc, 1.0, 0.5, [0xFF] * 12, 0xFF), _q4k(orc, 4.0, 2.0, [0] * 12, 0x5A),
            _q4k(orc, 0.0, 0.0, [0x3F] * 12, 0xFF), _q4k(orc, 1.0, 0.5, ALL_MIN_SCALES, 0x00)],
        1: [_q5k(orc, 1.0, 0.5, [0xFF] * 12, 0xFF, 0xFF), _q5k(orc, 1.0, 0.5, [0xFF] * 12, 0x00, 0xFF),
            _q5k(orc, 4.0, 2.0, [0] * 12, 0xAA, 0x5A), _q5k(orc, 1.0, 0.5, ALL_MIN_SCALES, 0xAA, 0x00)],
        2: [_q6k(orc, 0xFF, 0xFF, -128, 1.0), _q6k(orc, 0xFF, 0xFF, 127, 0.25),
            _q6k(orc, 0x00, 0x00, 127, 1.0), _q6k(orc, 0x5A, 0xA5, 0, 4.0)],
    }


@pytest.mark.parametrize("fmt,seed", [(0, 0xD4), (1, 0xD5), (2, 0xD6)])
def test_adversarial_blocks(orc, fmt, seed):
    """quants/tests.rs:251-321, every arm."""
    acts = orc.quantize_row_q8_k(orc.Lcg(seed).fill(256, 2.0))
    a = _dequant_q8k(acts)
    for blk in adversarial_blocks(orc)[fmt]:
        for impl in (orc.SCALAR, orc.AVX2, orc.LANES):
            _assert_dot_close(orc.vec_dot(fmt, blk, acts, impl), orc.dequantize_row(fmt, blk), a)
    if fmt == 0:
        zero = np.zeros(1, orc.Q8K_DTYPE)
        assert orc.vec_dot(0, adversarial_blocks(orc)[0][1], zero, orc.SCALAR) == 0.0


@pytest.mark.parametrize("fmt", [0, 1, 2])
@pytest.mark.parametrize("n", [2048, 768, 4096])
def test_avx2_matches_scalar_within_tolerance(orc, fmt, n):
    """avx2.rs:1147-1266: AVX2 vs scalar within 1e-6 * sum |w a|."""
    if not orc.has_avx2():
        pytest.skip("host lacks AVX2")
    rng = orc.Lcg(77 + n * 3 + fmt)
    w = orc.quantize_weights(fmt, rng.fill(n, 1.5))
    acts = orc.quantize_row_q8_k(rng.fill(n, 2.0))
    s = orc.vec_dot(fmt, w, acts, orc.SCALAR)
    v = orc.vec_dot(fmt, w, acts, orc.AVX2)
    p = orc.dequantize_row(fmt, w).astype(np.float64) * _dequant_q8k(acts).astype(np.float64)
    assert abs(s - v) <= 1e-6 * np.abs(p).sum()


@pytest.mark.parametrize("fmt", [0, 1, 2])
def test_lane_model_bit_identical_to_avx2(orc, fmt):
    """The portable lane model (the GPU's float order) equals the AVX2 arm."""
    if not orc.has_avx2():
        pytest.skip("host lacks AVX2")
    rng = orc.Lcg(4242 + fmt)
    for n in (256, 768, 2048, 4096):
        for _ in range(8):
            w = orc.quantize_weights(fmt, rng.fill(n, 1.0))
            acts = orc.quantize_row_q8_k(rng.fill(n, 4.0))
            a = orc.vec_dot(fmt, w, acts, orc.AVX2)
            b = orc.vec_dot(fmt, w, acts, orc.LANES)
            assert np.float32(a).tobytes() == np.float32(b).tobytes()
    acts = orc.quantize_row_q8_k(orc.Lcg(0xD6).fill(256, 2.0))
    for blk in adversarial_blocks(orc)[fmt]:
        assert (np.float32(orc.vec_dot(fmt, blk, acts, orc.AVX2)).tobytes()
                == np.float32(orc.vec_dot(fmt, blk, acts, orc.LANES)).tobytes())


@pytest.mark.parametrize("fmt", [0, 2])
def test_four_row_tiles_bit_identical_to_single_row(orc, fmt):
    """avx2.rs:1269-1404."""
    rng = orc.Lcg(31 + fmt)
    n = 2048 if fmt == 0 else 768
    w = orc.quantize_weights(fmt, rng.fill(n, 1.0))
    for n_acts in (1, 3, 4, 5, 9):
        acts = orc.quantize_row_q8_k(rng.fill(n * n_acts, 2.0))
        tile = orc.vec_dot_rows(fmt, w, acts, n_acts)
        nb = n // 256
        for a in range(n_acts):
            one = orc.vec_dot(fmt, w, acts[a * nb:(a + 1) * nb])
            assert np.float32(one).tobytes() == tile[a].tobytes()


def test_scale_unpack_matches_get_scale_min_k4(orc):
    """avx2.rs:1733: the mask-trick unpack equals get_scale_min_k4."""
    import ctypes
    rng = np.random.default_rng(5)
    L = orc.lib()
    L.or_get_scale_min_k4.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    L.or_unpack_scales_mins.argtypes = [ctypes.c_void_p] * 3
    for _ in range(200):
        s = rng.integers(0, 256, 12).astype(np.uint8)
        sc8 = np.zeros(8, np.uint8); m8 = np.zeros(8, np.uint8)
        L.or_unpack_scales_mins(s.ctypes.data, sc8.ctypes.data, m8.ctypes.data)
        for j in range(8):
            a = np.zeros(1, np.uint8); b = np.zeros(1, np.uint8)
            L.or_get_scale_min_k4(j, s.ctypes.data, a.ctypes.data, b.ctypes.data)
            assert (a[0], b[0]) == (sc8[j], m8[j])


def test_dots_reject_bad_lengths(orc):
    """quants/tests.rs:368-441 (k-quant part)."""
    acts2 = np.zeros(2, orc.Q8K_DTYPE)
    with pytest.raises(orc.OracleError) as e:
        orc.vec_dot(0, np.zeros(144, np.uint8), acts2)
    assert e.value.kind == "BlockCountMismatch"
    with pytest.raises(orc.OracleError) as e:
        orc.vec_dot(1, np.zeros(175, np.uint8), acts2)
    assert e.value.kind == "RowBytesNotBlockMultiple"
    with pytest.raises(orc.OracleError) as e:
        orc.vec_dot(2, np.zeros(630, np.uint8), acts2)
    assert e.value.kind == "BlockCountMismatch"


# ------------------------------------------------------------- primitives
def test_softmax_single_element_is_one(orc):
    """primitives/softmax.rs:102-107."""
    assert orc.softmax([-1234.5])[0] == 1.0


def test_softmax_all_equal(orc):
    """primitives/softmax.rs:90-100."""
    for n in (1, 3, 1000):
        got = orc.softmax(np.full(n, 42.5, np.float32))
        assert np.allclose(got, 1.0 / n, rtol=1e-6, atol=0)


def test_swiglu_matches_f64_formula(orc):
    """primitives/activation.rs:78-89."""
    rng = np.random.default_rng(0x5716)
    g = rng.uniform(-12, 12, 768).astype(np.float32)
    u = rng.uniform(-3, 3, 768).astype(np.float32)
    got = orc.swiglu_combine(g, u)
    want = g.astype(np.float64) / (1 + np.exp(-g.astype(np.float64))) * u
    assert np.allclose(got, want, rtol=1e-6, atol=1e-30)


def test_router_topk_lowest_index_wins_ties(orc):
    """forward.rs:2688-2699: strict '>' scan, first index wins a tie."""
    router = np.zeros((8, 256), np.float32)
    router[5, 0] = 1.0
    router[2, 0] = 1.0  # same logit as expert 5
    x = np.zeros(256, np.float32)
    x[0] = 3.0
    _, ids, w = orc.route(x, router, 3)
    assert list(ids[:2]) == [2, 5]
    assert ids[2] == 0
    assert abs(float(w.sum()) - 1.0) < 1e-6


def test_row_bytes(orc):
    """quants/tests.rs:444-467."""
    assert orc.BLOCK_BYTES[0] * 2048 // 256 == 1152
    assert orc.BLOCK_BYTES[1] * 768 // 256 == 528
    assert orc.BLOCK_BYTES[2] * 768 // 256 == 630
