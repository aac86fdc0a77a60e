"""Pin the oracle's Q8_0 family (attn_k's quantizer, dot and GEMV) and the
row dequantizers against the reference's own tests, and check the C-ABI's
Q8_0 / dequantization validation.  CPU only."""
import struct

import numpy as np
import pytest

from test_oracle_kat import _assert_dot_close

DIMS = (2048, 768, 4096)  # avx2.rs:1147


def _dequant_q8_0_act(acts):
    """quants/tests.rs:20-25."""
    return np.concatenate([b["d"] * b["qs"].astype(np.float32) for b in acts])


def quantizer_inputs(orc, n, seed):
    """avx2.rs:1568-1601: random, zero, flat, tie-heavy, signed-extreme and
    duplicate-extreme rows."""
    rng = orc.Lcg(seed)
    cases = [rng.fill(n, 8.0), np.zeros(n, np.float32), np.full(n, -3.75, np.float32),
             np.full(n, 12.5, np.float32)]
    tie = np.array([[2.0, -1.0, 0.5, -0.5][i % 4] for i in range(n)], np.float32)
    cases.append(tie)
    neg = np.full(n, 0.5, np.float32); neg[0] = -4.0
    pos = np.full(n, -0.5, np.float32); pos[1] = 4.0
    dup = np.full(n, 0.25, np.float32); dup[3] = -6.0; dup[7] = 6.0
    return cases + [neg, pos, dup]


# --------------------------------------------------------------- quantizer
@pytest.mark.parametrize("impl", [0, 1])
def test_q8_0_scales_and_signs(orc, impl):
    """quantize.rs:109-124."""
    if impl == 1 and not orc.has_avx2():
        pytest.skip("host lacks AVX2")
    x = np.zeros(32, np.float32)
    x[0], x[1], x[31] = 2.0, -1.0, 0.5
    b = orc.quantize_row_q8_0(x, impl)[0]
    assert b["d"] == orc.f16_to_f32(orc.f32_to_f16(float(np.float32(2.0) / np.float32(127.0))))
    assert (b["qs"][0], b["qs"][1], b["qs"][31], b["qs"][2]) == (127, -64, 32, 0)


@pytest.mark.parametrize("impl", [0, 1])
def test_q8_0_zero_row(orc, impl):
    """quantize.rs:126-138."""
    if impl == 1 and not orc.has_avx2():
        pytest.skip("host lacks AVX2")
    out = orc.quantize_row_q8_0(np.zeros(64, np.float32), impl)
    assert (out["d"] == 0).all() and (out["qs"] == 0).all()


def test_q8_0_len_mismatch(orc):
    with pytest.raises(orc.OracleError) as e:
        orc.quantize_row_q8_0(np.zeros(33, np.float32), out_blocks=1)
    assert e.value.kind == "QuantizeLenMismatch"


def test_q8_0_avx2_byte_identical_to_scalar(orc):
    """avx2.rs:1604-1620."""
    if not orc.has_avx2():
        pytest.skip("host lacks AVX2")
    for n in DIMS:
        for x in quantizer_inputs(orc, n, 0xC0 ^ n):
            assert orc.quantize_row_q8_0(x, orc.SCALAR).tobytes() == orc.quantize_row_q8_0(x, orc.AVX2).tobytes()


def test_q8_0_arms_differ_when_the_inverse_scale_overflows(orc):
    """Outside the reference's own test inputs: with amax < 127/FLT_MAX the
    inverse scale 1/d is +inf.  The scalar arm (quantize.rs:37-54) then
    saturates (inf -> 127, -inf -> -128, 0*inf = NaN -> 0); the AVX2 arm's
    cvtps_epi32 (avx2.rs:1022-1056) maps all three to -128.  The GPU follows
    the scalar arm."""
    x = np.zeros(32, np.float32)
    x[0], x[1] = 1e-37, -5e-38
    s = orc.quantize_row_q8_0(x, orc.SCALAR)[0]
    assert list(s["qs"][:3]) == [127, -128, 0]
    if orc.has_avx2():
        a = orc.quantize_row_q8_0(x, orc.AVX2)[0]
        assert (a["qs"] == -128).all() and a["d"] == s["d"]


def test_round_trip_q8_0(orc):
    """quants/tests.rs:116-133."""
    x = orc.Lcg(45).fill(128, 8.0)
    b = orc.quantize_weights(orc.Q8_0, x)
    w = orc.dequantize_row(orc.Q8_0, b)
    for bi in range(4):
        d = orc.f16_to_f32(int(b[34 * bi]) | (int(b[34 * bi + 1]) << 8))
        assert np.all(np.abs(w[32 * bi:32 * bi + 32] - x[32 * bi:32 * bi + 32]) <= d + 1e-6)


# ------------------------------------------------------------------ dots
@pytest.mark.parametrize("n", [2048, 768])
def test_dot_ground_truth_q8_0(orc, n):
    """quants/tests.rs:211-226 (same seeds, same Lcg draws)."""
    rng = orc.Lcg(0x80 ^ n)
    xw, xa = rng.fill(n, 4.0), rng.fill(n, 3.0)
    wb = orc.quantize_weights(orc.Q8_0, xw)
    acts = orc.quantize_row_q8_0(xa, orc.SCALAR)
    for impl in (orc.SCALAR, orc.AVX2, orc.LANES):
        _assert_dot_close(orc.vec_dot_q8_0(wb, acts, impl), orc.dequantize_row(orc.Q8_0, wb),
                          _dequant_q8_0_act(acts))


def _adversarial(orc):
    wb = np.frombuffer(struct.pack("<H", 0x7BFF) + bytes([0x80]) * 32, np.uint8)  # d = 65504, q = -128
    acts = np.zeros(1, orc.Q8_0_DTYPE)
    acts["d"] = 65504.0
    acts["qs"] = 127
    return wb, acts


def test_adversarial_q8_0(orc):
    """quants/tests.rs:324-344 and avx2.rs:1537-1562, every arm."""
    wb, acts = _adversarial(orc)
    for impl in (orc.SCALAR, orc.AVX2, orc.LANES):
        _assert_dot_close(orc.vec_dot_q8_0(wb, acts, impl), orc.dequantize_row(orc.Q8_0, wb),
                          _dequant_q8_0_act(acts))
        assert orc.vec_dot_q8_0(wb, np.zeros(1, orc.Q8_0_DTYPE), impl) == 0.0


def test_q8_0_dot_rejects_bad_lengths(orc):
    """quants/tests.rs:430-440."""
    acts8 = np.zeros(8, orc.Q8_0_DTYPE)
    with pytest.raises(orc.OracleError) as e:
        orc.vec_dot_q8_0(np.zeros(35, np.uint8), acts8)
    assert e.value.kind == "RowBytesNotBlockMultiple"
    assert orc.vec_dot_q8_0(np.zeros(272, np.uint8), acts8) == 0.0


@pytest.mark.parametrize("n", DIMS)
def test_q8_0_avx2_matches_scalar_within_tolerance(orc, n):
    """avx2.rs:1243-1262: within 1e-6 * sum |w a|."""
    if not orc.has_avx2():
        pytest.skip("host lacks AVX2")
    rng = orc.Lcg(0xB8 ^ n)
    wb = orc.quantize_weights(orc.Q8_0, rng.fill(n, 4.0))
    acts = orc.quantize_row_q8_0(rng.fill(n, 3.0), orc.SCALAR)
    s, v = orc.vec_dot_q8_0(wb, acts, orc.SCALAR), orc.vec_dot_q8_0(wb, acts, orc.AVX2)
    p = orc.dequantize_row(orc.Q8_0, wb).astype(np.float64) * _dequant_q8_0_act(acts).astype(np.float64)
    assert abs(s - v) <= 1e-6 * np.abs(p).sum()


def test_q8_0_lane_model_bit_identical_to_avx2(orc):
    """The portable lane model (the GPU's float order) equals the AVX2 arm."""
    if not orc.has_avx2():
        pytest.skip("host lacks AVX2")
    rng = orc.Lcg(0x51)
    for n in (32, 96, 768, 2048, 4096):
        for _ in range(8):
            wb = orc.quantize_weights(orc.Q8_0, rng.fill(n, 1.0))
            acts = orc.quantize_row_q8_0(rng.fill(n, 4.0))
            a, b = orc.vec_dot_q8_0(wb, acts, orc.AVX2), orc.vec_dot_q8_0(wb, acts, orc.LANES)
            assert np.float32(a).tobytes() == np.float32(b).tobytes()
    wb, acts = _adversarial(orc)
    assert (np.float32(orc.vec_dot_q8_0(wb, acts, orc.AVX2)).tobytes()
            == np.float32(orc.vec_dot_q8_0(wb, acts, orc.LANES)).tobytes())


# ------------------------------------------------------------------ GEMV
def _q8_0_batch(orc, in_dim, n_acts, seed):
    """gemv.rs:887-921 (q8_0_acts per act_seed)."""
    out = []
    for a in range(n_acts):
        s = (seed ^ (((a + 1) * 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF))
        out.append(orc.quantize_row_q8_0(orc.Lcg(s).fill(in_dim, 3.0)))
    return np.concatenate(out)


def test_gemv_q8_0_matches_per_row_dots(orc):
    """gemv.rs:1352-1371."""
    in_dim, out_dim = 2048, 64
    w = orc.quantize_weights(orc.Q8_0, orc.Lcg(0x80).fill(in_dim * out_dim, 1.0))
    acts = orc.quantize_row_q8_0(orc.Lcg(0xAC7).fill(in_dim, 3.0))
    out = orc.gemv_q8_0(w, in_dim, out_dim, acts)
    rb = in_dim // 32 * 34
    for r in range(out_dim):
        assert out[r].tobytes() == np.float32(orc.vec_dot_q8_0(w[r * rb:(r + 1) * rb], acts)).tobytes()


def test_gemv_q8_0_partitions_and_batches_bit_identical(orc):
    """gemv.rs:1394-1406 (row partitions) and :1500-1522 (batched columns)."""
    in_dim, out_dim = 2048, 512  # attn_k
    w = orc.quantize_weights(orc.Q8_0, orc.Lcg(0x8A).fill(in_dim * out_dim, 1.0))
    acts = orc.quantize_row_q8_0(orc.Lcg(0xAC7).fill(in_dim, 3.0))
    whole = orc.gemv_q8_0(w, in_dim, out_dim, acts, threads=4)
    parts = np.concatenate([orc.gemv_q8_0(w, in_dim, out_dim, acts, rows=(a, b))
                            for a, b in ((0, 1), (1, 100), (100, 100), (100, 511), (511, 512))])
    assert parts.tobytes() == whole.tobytes()
    for n_acts in (1, 2, 5, 9):
        batch = _q8_0_batch(orc, in_dim, n_acts, 0xBA70)
        got = orc.gemv_q8_0(w, in_dim, out_dim, batch, n_acts=n_acts, rows=(3, 67)).reshape(64, n_acts)
        nb = in_dim // 32
        for a in range(n_acts):
            one = orc.gemv_q8_0(w, in_dim, out_dim, batch[a * nb:(a + 1) * nb], rows=(3, 67))
            assert got[:, a].tobytes() == one.tobytes()
        if n_acts > 1:
            assert not np.array_equal(got[:, 0], got[:, 1])


def test_gemv_q8_0_validation(orc):
    """gemv.rs:212-264 precedence on the oracle."""
    a = np.zeros(64, orc.Q8_0_DTYPE)
    for args, kind in [((np.zeros(0, np.uint8), 33, 1, a[:1]), "IndivisibleRow"),
                       ((np.zeros(2175, np.uint8), 2048, 1, a), "LengthMismatch"),
                       ((np.zeros(2176, np.uint8), 2048, 1, a[:63]), "BlockCountMismatch")]:
        with pytest.raises(orc.OracleError) as e:
            orc.gemv_q8_0(*args)
        assert e.value.kind == kind


# -------------------------------------------------------- dequantization
def test_dequantize_q8_0_is_d_times_q(orc):
    """dequant.rs:134-147."""
    blk = np.frombuffer(struct.pack("<H", orc.f32_to_f16(0.375)) + bytes(range(0x70, 0x90)), np.uint8)
    w = orc.dequantize_row(orc.Q8_0, blk)
    q = np.arange(0x70, 0x90).astype(np.uint8).view(np.int8).astype(np.float32)
    assert w.tobytes() == (np.float32(0.375) * q).tobytes()


# ------------------------------------------------------ C-ABI validation
@pytest.fixture(scope="module")
def rv():
    import ramvamp_b200

    return ramvamp_b200


def test_c_abi_q8_0_validation(rv):
    """The library's Q8_0 entries check geometry before any CUDA call, with
    gemv.rs:212-264's precedence."""
    lib = rv.lib()
    name = lambda c: lib.rv_status_name(c).decode()
    g = lambda wlen, ind, outd, alen, n, r0, r1, olen: name(lib.rv_gemv_q8_0_batched(
        None, wlen, ind, outd, None, alen, n, r0, r1, None, olen, None))
    assert g(0, 33, 1, 1, 1, 0, 1, 1) == "IndivisibleRow"
    assert g(2175, 2048, 1, 64, 1, 0, 1, 1) == "LengthMismatch"
    assert g(2176, 2048, 1, 64, 1, 1, 0, 0) == "LengthMismatch"
    assert g(2176, 2048, 1, 64, 1, 0, 2, 2) == "LengthMismatch"
    assert g(2176, 2048, 1, 64, 1, 0, 1, 2) == "LengthMismatch"
    assert g(2176, 2048, 1, 63, 1, 0, 1, 1) == "BlockCountMismatch"
    assert g(2176, 2048, 1, 64, 1, 0, 1, 1) == "InvalidArgument"  # null pointers, still before CUDA
    assert g(2176, 2048, 1, 0, 0, 0, 1, 0) == "Ok"  # no activations: a no-op
    assert name(lib.rv_gemv_q8_0(None, 34, 32, 1, None, 2, None, 1, None)) == "BlockCountMismatch"
    assert name(lib.rv_gemv_q8_0_rows(None, 34, 32, 1, None, 1, 0, 1, None, 2, None)) == "LengthMismatch"
    assert name(lib.rv_quantize_row_q8_0(None, 33, None, 1, None)) == "QuantizeLenMismatch"
    assert lib.rv_quantize_row_q8_0(None, 0, None, 0, None) == 0


def test_c_abi_dequantize_validation(rv):
    lib = rv.lib()
    name = lambda c: lib.rv_status_name(c).decode()
    d = lambda fmt, wlen, ind, outd, rows, n, olen: name(lib.rv_dequantize_rows(
        fmt, None, wlen, ind, outd, rows, n, None, olen, None))
    assert d(4, 292, 256, 1, None, 1, 256) == "UnsupportedFormat"  # Q8_K is an activation format
    assert d(0, 144, 100, 1, None, 1, 100) == "IndivisibleRow"
    assert d(0, 143, 256, 1, None, 1, 256) == "LengthMismatch"
    assert d(0, 144, 256, 1, None, 1, 255) == "LengthMismatch"
    assert d(0, 144, 256, 1, None, 2, 512) == "TokenOutOfRange"
    assert d(3, 34, 32, 1, None, 0, 0) == "Ok"
    assert d(2, 210, 256, 1, None, 1, 256) == "InvalidArgument"
