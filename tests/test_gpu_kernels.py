"""GPU parity of the kernel-level entry points against the CPU oracle.

Every comparison is bit-exact: the oracle restates the reference's AVX2 path
(and its scalar path for Q8_K), and the CUDA kernels reproduce that float
order.  All calls go through the C ABI (ramvamp_b200 wraps it with ctypes).
"""
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


def dev(a):
    return torch.from_numpy(np.array(a, copy=True)).cuda()


def q8k_dev(blocks):
    return dev(blocks.view(np.uint8))


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


# ---------------------------------------------------------------- Q8_K
def q8k_rows(orc):
    rng = np.random.default_rng(11)
    rows = [rng.standard_normal(256 * 64).astype(np.float32)]
    rows.append((rng.standard_normal(256 * 16) * 1e-30).astype(np.float32))
    rows.append((rng.standard_normal(256 * 16) * 1e30).astype(np.float32))
    t = np.zeros(256 * 8, np.float32)
    t[::5] = 1.0
    t[2::7] = -1.0
    rows.append(t)
    rows.append(np.zeros(256 * 4, np.float32))
    rows.append(np.full(256 * 4, -0.125, np.float32))
    rows.append(rng.integers(-127, 128, 256 * 32).astype(np.float32) / 2.0)
    for sign in (1.0, -1.0):
        x = np.zeros(256, np.float32)
        x[10] = -3.0 * sign
        x[20] = 1.5 * sign
        rows.append(x)
    rows.append(orc.Lcg(9).fill(768, 5.0))
    return rows


def test_quantize_q8k_bit_exact(rv, orc):
    """quantize.rs:68-103 incl. its KATs (:301-338) and tie/flat/zero rows."""
    for x in q8k_rows(orc):
        want = orc.quantize_row_q8_k(x)
        got = host(rv.quantize_row_q8_k(dev(x)))
        assert got.tobytes() == want.view(np.uint8).tobytes()


# ---------------------------------------------------------------- GEMV
FORMATS = [0, 1, 2]


def make_matrix(orc, fmt, in_dim, out_dim, seed, scale=1.0):
    w = orc.quantize_weights(fmt, orc.Lcg(seed).fill(in_dim * out_dim, scale))
    return w


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("in_dim,out_dim", [(256, 40), (768, 96), (2048, 72), (4096, 24)])
def test_gemv_bit_identical_to_avx2(rv, orc, fmt, in_dim, out_dim):
    """gemv.rs:347 via avx2.rs dots: every output bit equals the reference."""
    w = make_matrix(orc, fmt, in_dim, out_dim, 100 + fmt * 7 + in_dim)
    acts = orc.quantize_row_q8_k(orc.Lcg(5 + in_dim).fill(in_dim, 3.0))
    want = orc.gemv(fmt, w, in_dim, out_dim, acts, impl=orc.default_impl())
    lanes = orc.gemv(fmt, w, in_dim, out_dim, acts, impl=orc.LANES)
    assert bits(want).tobytes() == bits(lanes).tobytes()
    out = torch.empty(out_dim, dtype=torch.float32, device="cuda")
    rv.gemv_q8_k(fmt, dev(w), in_dim, out_dim, q8k_dev(acts), out)
    assert bits(host(out)).tobytes() == bits(want).tobytes()


@pytest.mark.parametrize("fmt", FORMATS)
def test_gemv_rows_partition_is_bit_identical(rv, orc, fmt):
    """gemv.rs:386: any partition of the rows reproduces the whole matrix."""
    in_dim, out_dim = 768, 83
    w = make_matrix(orc, fmt, in_dim, out_dim, 77 + fmt)
    acts = orc.quantize_row_q8_k(orc.Lcg(8).fill(in_dim, 2.0))
    want = orc.gemv(fmt, w, in_dim, out_dim, acts)
    wd, ad = dev(w), q8k_dev(acts)
    pieces = []
    for lo, hi in [(0, 1), (1, 17), (17, 40), (40, 41), (41, 83)]:
        out = torch.empty(hi - lo, dtype=torch.float32, device="cuda")
        rv.gemv_q8_k_rows(fmt, wd, in_dim, out_dim, ad, range(lo, hi), out)
        pieces.append(host(out))
    assert bits(np.concatenate(pieces)).tobytes() == bits(want).tobytes()


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("n_acts", [1, 3, 4, 9, 17])
def test_gemv_batched_bit_identical(rv, orc, fmt, n_acts):
    """gemv.rs:444 and the 4-row tiles (avx2.rs:162-192): out[i*n+a]."""
    in_dim, out_dim = 2048 if fmt != 2 else 768, 37
    w = make_matrix(orc, fmt, in_dim, out_dim, 300 + fmt)
    acts = orc.quantize_row_q8_k(orc.Lcg(9 + n_acts).fill(in_dim * n_acts, 2.5))
    want = orc.gemv(fmt, w, in_dim, out_dim, acts, n_acts=n_acts, rows=(3, 37), threads=4)
    out = torch.empty(34 * n_acts, dtype=torch.float32, device="cuda")
    rv.gemv_q8_k_batched(fmt, dev(w), in_dim, out_dim, q8k_dev(acts), n_acts, range(3, 37), out)
    assert bits(host(out)).tobytes() == bits(want).tobytes()


@pytest.mark.parametrize("fmt", FORMATS)
def test_gemv_misaligned_weights(rv, orc, fmt):
    """avx2.rs:1645: weight rows need only byte alignment."""
    in_dim, out_dim = 768, 20
    w = make_matrix(orc, fmt, in_dim, out_dim, 55 + fmt)
    acts = orc.quantize_row_q8_k(orc.Lcg(3).fill(in_dim, 1.0))
    want = orc.gemv(fmt, w, in_dim, out_dim, acts)
    for shift in (1, 2, 3, 5):
        buf = torch.zeros(w.size + 16, dtype=torch.uint8, device="cuda")
        buf[shift:shift + w.size] = dev(w)
        out = torch.empty(out_dim, dtype=torch.float32, device="cuda")
        rv.gemv_q8_k(fmt, buf[shift:shift + w.size], in_dim, out_dim, q8k_dev(acts), out)
        assert bits(host(out)).tobytes() == bits(want).tobytes(), shift


def test_gemv_fused_rows(rv, orc):
    """gemv.rs:747: concatenated row spaces, each part with its own acts."""
    parts, ref = [], []
    for j, (fmt, in_dim, out_dim) in enumerate([(0, 2048, 30), (0, 2048, 11), (2, 768, 25), (1, 256, 9)]):
        w = make_matrix(orc, fmt, in_dim, out_dim, 900 + j)
        a = orc.quantize_row_q8_k(orc.Lcg(40 + j).fill(in_dim, 2.0))
        parts.append(rv.FusedPart(fmt, dev(w), in_dim, out_dim, q8k_dev(a)))
        ref.append(orc.gemv(fmt, w, in_dim, out_dim, a))
    ref = np.concatenate(ref)
    for lo, hi in [(0, 75), (5, 50), (29, 31), (40, 41)]:
        out = torch.empty(hi - lo, dtype=torch.float32, device="cuda")
        rv.gemv_q8_k_fused_rows(parts, range(lo, hi), out)
        assert bits(host(out)).tobytes() == bits(ref[lo:hi]).tobytes()


@pytest.mark.parametrize("fmt", FORMATS)
def test_block_integer_sums_bit_exact(rv, orc, fmt):
    """Per-block AVX2 lane sums and min lanes: the integer contract."""
    from test_oracle_kat import adversarial_blocks
    in_dim = 2048
    w = make_matrix(orc, fmt, in_dim, 1, 4000 + fmt)
    acts = orc.quantize_row_q8_k(orc.Lcg(41).fill(in_dim, 3.0))
    lanes, mins = rv.debug_block_sums(fmt, dev(w), q8k_dev(acts))
    lanes, mins = host(lanes), host(mins)
    bb = orc.BLOCK_BYTES[fmt]
    for b in range(in_dim // 256):
        l8, m4, sumi, smin = orc.block_int_sums(fmt, w[b * bb:(b + 1) * bb], acts[b:b + 1])
        assert (lanes[b] == l8).all() and lanes[b].sum() == sumi
        assert (mins[b] == m4).all()
    a1 = orc.quantize_row_q8_k(orc.Lcg(0xD6).fill(256, 2.0))
    for blk in adversarial_blocks(orc)[fmt]:
        l, m = rv.debug_block_sums(fmt, dev(blk), q8k_dev(a1))
        l8, m4, _, _ = orc.block_int_sums(fmt, blk, a1)
        assert (host(l)[0] == l8).all() and (host(m)[0] == m4).all()


@pytest.mark.parametrize("fmt", FORMATS)
def test_adversarial_blocks_dot(rv, orc, fmt):
    from test_oracle_kat import adversarial_blocks
    acts = orc.quantize_row_q8_k(orc.Lcg(0xD4 + fmt).fill(256, 2.0))
    for blk in adversarial_blocks(orc)[fmt]:
        want = orc.vec_dot(fmt, blk, acts)
        out = torch.empty(1, dtype=torch.float32, device="cuda")
        rv.gemv_q8_k(fmt, dev(blk), 256, 1, q8k_dev(acts), out)
        assert bits(host(out)).tobytes() == bits(np.float32(want)).tobytes()


# --------------------------------------------------------- primitives
def test_rmsnorm_bit_exact(rv, orc):
    """norm.rs:17-60: f64 mean of squares, f32 scale."""
    rng = np.random.default_rng(3)
    for n, scale in [(2048, 1.0), (768, 30.0), (128, 1e-20), (4096, 1e15), (2048, 1e-3)]:
        x = (rng.standard_normal((3, n)) * scale).astype(np.float32)
        w = rng.uniform(0.5, 1.5, n).astype(np.float32)
        out = torch.empty(3 * n, dtype=torch.float32, device="cuda")
        rv.rmsnorm(dev(x), dev(w), 1e-6, out)
        got = host(out).reshape(3, n)
        for r in range(3):
            assert bits(got[r]).tobytes() == bits(orc.rmsnorm(x[r], w, 1e-6)).tobytes()


def test_softmax_bit_exact(rv, orc):
    """softmax.rs:18-40 (f64 exp and sum)."""
    rng = np.random.default_rng(4)
    for n in (1, 3, 128, 1000):
        x = (rng.standard_normal((5, n)) * 4).astype(np.float32)
        t = dev(x)
        rv.softmax(t)
        got = host(t)
        for r in range(5):
            assert bits(got[r]).tobytes() == bits(orc.softmax(x[r])).tobytes()


def test_swiglu_bit_exact_random(rv, orc):
    """activation.rs:14-42 with the host libm's expf."""
    rng = np.random.default_rng(5)
    g = np.concatenate([rng.uniform(-20, 20, 200_000), rng.standard_normal(200_000) * 0.05,
                        [-1e30, -100, -88, -10, -1e-40, 0, 1e-40, 10, 88, 100, 1e30, -87.5, 103.9]]
                       ).astype(np.float32)
    u = rng.uniform(-3, 3, g.size).astype(np.float32)
    want = orc.swiglu_combine(g, u)
    gt = dev(g)
    rv.swiglu_combine(gt, dev(u))
    assert bits(host(gt)).tobytes() == bits(want).tobytes()


def test_swiglu_bit_exact_on_every_misrounded_input(rv, orc):
    """Every input where glibc expf is not correctly rounded (the exception
    table), as SiLU arguments: exp(-g) for g = -x."""
    import os
    import re
    inc = os.path.join(os.path.dirname(rv.__file__), "csrc", "_gen", "expf_exceptions.inc")
    keys = np.array([int(k, 16) for k in re.findall(r"\{0x([0-9a-f]{8})u,", open(inc).read())],
                    dtype=np.uint32)
    x = keys.view(np.float32)
    g = -x
    u = np.ones_like(g)
    want = orc.swiglu_combine(g, u)
    gt = dev(g)
    rv.swiglu_combine(gt, dev(u))
    assert bits(host(gt)).tobytes() == bits(want).tobytes()


# ------------------------------------------------ weight quantizers
@pytest.mark.parametrize("fmt", FORMATS)
def test_gpu_weight_quantizers_match_reference(rv, orc, fmt):
    """test_support.rs:106-219, byte for byte."""
    rng = np.random.default_rng(6 + fmt)
    xs = [rng.standard_normal(256 * 512).astype(np.float32) * 0.02,
          orc.Lcg(42).fill(256 * 64, 8.0),
          np.zeros(256 * 2, np.float32),
          np.full(256 * 2, 3.0, np.float32),
          np.abs(rng.standard_normal(256 * 8)).astype(np.float32),
          -np.abs(rng.standard_normal(256 * 8)).astype(np.float32)]
    for ci, x in enumerate(xs):
        want = orc.quantize_weights(fmt, x)
        got = host(rv.quantize_weights(fmt, dev(x)))
        bad = np.nonzero(got != want)[0]
        assert bad.size == 0, (ci, bad.size, bad[:12].tolist(), got[bad[:12]].tolist(),
                               want[bad[:12]].tolist())


def test_synth_normal_deterministic(rv):
    a = host(rv.synth_normal(7, 0, 1.0, 1 << 20))
    b = host(rv.synth_normal(7, 1000, 1.0, 1 << 20))
    assert a[1000:].tobytes() == b[:-1000].tobytes()
    assert abs(a.mean()) < 5e-3 and abs(a.std() - 1.0) < 5e-3
    c = host(rv.synth_normal(8, 0, 0.02, 1 << 16))
    assert abs(c.std() - 0.02) < 1e-3
