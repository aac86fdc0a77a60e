"""GPU parity of the attention / lm_head / embedding GEMV family (Q8_0
quantizer, Q8_0 GEMV, k-quant GEMV at the lm_head shape, row
dequantization) against the CPU oracle.  Bit-exact, through the C ABI."""
import struct

import numpy as np
import pytest

from test_oracle_q8_0 import DIMS, _adversarial, _q8_0_batch, quantizer_inputs

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


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def q8_0_dev(blocks):
    return dev(blocks.view(np.uint8))


# ------------------------------------------------------------ quantizer
def test_quantize_row_q8_0_bytes_identical(rv, orc):
    """quantize.rs:37-54 on the reference's quantizer inputs (avx2.rs:
    1568-1601), very small / large / non-finite blocks, and rows that are
    not a multiple of 8 blocks."""
    rows = []
    for n in DIMS:
        rows += quantizer_inputs(orc, n, 0xC0 ^ n)
    rng = np.random.default_rng(3)
    rows.append((rng.standard_normal(32 * 40) * 1e-37).astype(np.float32))  # 1/d overflows
    rows.append((rng.standard_normal(32 * 40) * 1e-41).astype(np.float32))  # subnormal inputs
    rows.append((rng.standard_normal(32 * 40) * 3e38).astype(np.float32))
    odd = rng.standard_normal(32 * 13).astype(np.float32)
    odd[5], odd[40], odd[77] = np.nan, np.inf, -np.inf
    odd[96:128] = np.nan
    rows.append(odd)
    rows.append(rng.integers(-254, 255, 32 * 24).astype(np.float32) / 2.0)
    for x in rows:
        want = orc.quantize_row_q8_0(x, orc.SCALAR)
        got = host(rv.quantize_row_q8_0(dev(x)))
        assert got.tobytes() == want.tobytes()


# --------------------------------------------------------------- GEMV
def _w_q8_0(orc, in_dim, out_dim, seed, scale=1.0):
    return orc.quantize_weights(orc.Q8_0, orc.Lcg(seed).fill(in_dim * out_dim, scale))


@pytest.mark.parametrize("in_dim,out_dim", [(2048, 512), (32, 1), (96, 7), (4096, 1000), (2080, 300)])
def test_gemv_q8_0_bit_identical(rv, orc, in_dim, out_dim):
    """gemv.rs:544-565 with avx2.rs:942-963 as the dot."""
    w = _w_q8_0(orc, in_dim, out_dim, in_dim + out_dim)
    acts = orc.quantize_row_q8_0(orc.Lcg(0xAC7).fill(in_dim, 3.0))
    want = orc.gemv_q8_0(w, in_dim, out_dim, acts, impl=orc.LANES, threads=8)
    out = torch.empty(out_dim, dtype=torch.float32, device="cuda")
    rv.gemv_q8_0(dev(w), in_dim, out_dim, q8_0_dev(acts), out)
    assert host(out).tobytes() == want.tobytes()
    if orc.has_avx2():
        assert want.tobytes() == orc.gemv_q8_0(w, in_dim, out_dim, acts, impl=orc.AVX2).tobytes()


def test_gemv_q8_0_rows_batched_and_unaligned(rv, orc):
    """gemv.rs:579-640: row ranges and batches against the oracle, and a
    weight matrix starting on a 2-byte (not 16-byte) boundary."""
    in_dim, out_dim = 2048, 512
    w = _w_q8_0(orc, in_dim, out_dim, 0x8A)
    wd = dev(w)
    for n_acts in (1, 2, 5, 8, 9, 17):
        batch = _q8_0_batch(orc, in_dim, n_acts, 0xBA70)
        for r0, r1 in ((0, 512), (3, 67), (511, 512), (100, 100)):
            want = orc.gemv_q8_0(w, in_dim, out_dim, batch, n_acts=n_acts, rows=(r0, r1), impl=orc.LANES,
                                 threads=8)
            out = torch.full(((r1 - r0) * n_acts,), np.nan, dtype=torch.float32, device="cuda")
            if n_acts == 1:
                rv.gemv_q8_0_rows(wd, in_dim, out_dim, q8_0_dev(batch), range(r0, r1), out)
            else:
                rv.gemv_q8_0_batched(wd, in_dim, out_dim, q8_0_dev(batch), n_acts, range(r0, r1), out)
            assert host(out).tobytes() == want.tobytes(), (n_acts, r0, r1)
    buf = torch.zeros(w.size + 2, dtype=torch.uint8, device="cuda")
    buf[2:] = wd
    acts = orc.quantize_row_q8_0(orc.Lcg(5).fill(in_dim, 2.0))
    out = torch.empty(out_dim, dtype=torch.float32, device="cuda")
    rv.gemv_q8_0(buf[2:], in_dim, out_dim, q8_0_dev(acts), out)
    assert host(out).tobytes() == orc.gemv_q8_0(w, in_dim, out_dim, acts, impl=orc.LANES).tobytes()


def test_gemv_q8_0_adversarial_and_backend(rv, orc):
    """quants/tests.rs:324-344 on the GPU, through the Backend mirror."""
    wb, acts = _adversarial(orc)
    out = torch.empty(1, dtype=torch.float32, device="cuda")
    rv.CudaBackend().gemv_q8_0(dev(wb), 32, 1, q8_0_dev(acts), out)
    assert host(out).tobytes() == np.float32(orc.vec_dot_q8_0(wb, acts, orc.LANES)).tobytes()
    rv.gemv_q8_0(dev(wb), 32, 1, q8_0_dev(np.zeros(1, orc.Q8_0_DTYPE)), out)
    assert host(out)[0] == 0.0


def test_attn_k_quantize_then_gemv(rv, orc):
    """attn_k as the decode step runs it (forward.rs:2575-2651): Q8_0 of the
    normed row on the GPU, then the Q8_0 GEMV."""
    x = orc.Lcg(0x77).fill(2048, 2.5)
    w = _w_q8_0(orc, 2048, 512, 0x78, 0.05)
    acts = rv.quantize_row_q8_0(dev(x))
    out = torch.empty(512, dtype=torch.float32, device="cuda")
    rv.gemv_q8_0(dev(w), 2048, 512, acts, out)
    want = orc.gemv_q8_0(w, 2048, 512, orc.quantize_row_q8_0(x, orc.SCALAR), impl=orc.LANES)
    assert host(out).tobytes() == want.tobytes()


# ------------------------------------------------------ lm_head (Q6_K)
def test_lm_head_shape_q6_k(rv, orc):
    """output.weight, Q6_K 151,936 x 2048 (model/shapes.rs:14-35), through
    the k-quant GEMV: 4,096 sampled rows against the oracle, and the whole
    matrix equal to its row partitions."""
    vocab, hidden = 151936, 2048
    w = rv.quantize_weights(rv.QuantFormat.Q6_K, rv.synth_normal(0x1A, 0, 0.02, vocab * hidden))
    x = orc.Lcg(0x1B).fill(hidden, 2.0)
    acts = orc.quantize_row_q8_k(x)
    ad = dev(acts.view(np.uint8))
    out = torch.empty(vocab, dtype=torch.float32, device="cuda")
    rv.gemv_q8_k(rv.QuantFormat.Q6_K, w, hidden, vocab, ad, out)
    got = host(out)
    rb = hidden // 256 * 210
    rows = np.sort(np.random.default_rng(1).choice(vocab, 4096, replace=False))
    rows[-1] = vocab - 1
    wsel = torch.cat([w[r * rb:(r + 1) * rb] for r in rows.tolist()]).cpu().numpy()
    want = orc.gemv(orc.Q6_K, wsel, hidden, len(rows), acts, impl=orc.LANES, threads=8)
    assert got[rows].tobytes() == want.tobytes()
    part = torch.empty(vocab, dtype=torch.float32, device="cuda")
    for r0, r1 in ((0, 1), (1, 77777), (77777, vocab)):
        rv.gemv_q8_k_rows(rv.QuantFormat.Q6_K, w, hidden, vocab, ad, range(r0, r1), part[r0:r1])
    assert host(part).tobytes() == got.tobytes()


# ------------------------------------------------------- dequantization
@pytest.mark.parametrize("fmt", [0, 1, 2, 3])
def test_dequantize_rows_bit_identical(rv, orc, fmt):
    """dequant.rs:28-147 for every weight format, whole matrices and chosen
    rows (repeats allowed)."""
    in_dim, out_dim = (2048, 96) if fmt != 3 else (2080, 96)
    x = orc.Lcg(0xDE + fmt).fill(in_dim * out_dim, 1.5)
    w = orc.quantize_weights(fmt, x)
    rb = w.size // out_dim
    want = np.concatenate([orc.dequantize_row(fmt, w[r * rb:(r + 1) * rb]) for r in range(out_dim)])
    wd = dev(w)
    got = host(rv.dequantize_rows(fmt, wd, in_dim, out_dim))
    assert got.tobytes() == want.tobytes()
    ids = np.array([5, 0, 95, 5, 17], np.int32)
    got = host(rv.dequantize_rows(fmt, wd, in_dim, out_dim, rows=dev(ids))).reshape(len(ids), in_dim)
    for i, r in enumerate(ids):
        assert got[i].tobytes() == want[r * in_dim:(r + 1) * in_dim].tobytes()


def test_dequantize_adversarial_blocks(rv, orc):
    """quants/tests.rs:251-321's extreme blocks through the dequantizers."""
    from test_oracle_kat import adversarial_blocks

    for fmt, blocks in adversarial_blocks(orc).items():
        for blk in blocks:
            got = host(rv.dequantize_rows(fmt, dev(blk), 256, 1))
            assert got.tobytes() == orc.dequantize_row(fmt, blk).tobytes()
    q8 = np.frombuffer(struct.pack("<H", 0x7BFF) + bytes(range(0x70, 0x90)), np.uint8)
    assert host(rv.dequantize_rows(3, dev(q8), 32, 1)).tobytes() == orc.dequantize_row(3, q8).tobytes()


def test_embed_tokens(rv, orc):
    """Weights::embed (model/weights.rs:371-384) at the Qwen3 embedding
    shape (Q4_K, 151,936 x 2048), token ids on the device; an id past the
    vocabulary zeroes its row and reports TokenOutOfRange."""
    vocab, hidden = 151936, 2048
    table = rv.quantize_weights(rv.QuantFormat.Q4_K, rv.synth_normal(0xE1, 0, 0.5, vocab * hidden))
    toks = np.array([0, 151935, 42, 42, 100000], np.int32)
    got = host(rv.embed(table, hidden, vocab, dev(toks))).reshape(len(toks), hidden)
    rb = hidden // 256 * 144
    for i, t in enumerate(toks.tolist()):
        want = orc.dequantize_row(orc.Q4_K, table[t * rb:(t + 1) * rb].cpu().numpy())
        assert got[i].tobytes() == want.tobytes()
    rv.device_status(0)
    bad = host(rv.embed(table, hidden, vocab, dev(np.array([7, vocab], np.int32)))).reshape(2, hidden)
    with pytest.raises(rv.KernelError) as e:
        rv.device_status(0)
    assert e.value.kind == "TokenOutOfRange"
    assert (bad[1] == 0).all()
    assert bad[0].tobytes() == orc.dequantize_row(orc.Q4_K, table[7 * rb:8 * rb].cpu().numpy()).tobytes()
    rv.device_status(0)  # cleared


def _random_kquant_matrix(orc, fmt, in_dim, out_dim, seed):
    """Arbitrary block bytes (negative Q6_K scales included) with finite f16
    scale fields, so every integer path of the dot is exercised."""
    rng = np.random.default_rng(seed)
    bb = orc.BLOCK_BYTES[fmt]
    nblk = in_dim // 256 * out_dim
    w = rng.integers(0, 256, (nblk, bb), dtype=np.uint8)
    for off in ((208,) if fmt == orc.Q6_K else (0, 2)):
        h = (rng.integers(0x0400, 0x3C00, nblk) | (rng.integers(0, 2, nblk) << 15)).astype("<u2")
        w[:, off:off + 2] = h.view(np.uint8).reshape(nblk, 2)
    return w.reshape(-1)


@pytest.mark.parametrize("fmt,in_dim", [(2, 2048), (0, 2048), (1, 2048), (0, 1024)])
def test_streaming_gemv_random_blocks(rv, orc, fmt, in_dim):
    """Arbitrary blocks through the k-quant GEMV: for Q6_K at hidden 2048 the
    persistent lm_head kernel (one activation row, 6,007 rows = 376 tiles of
    16), for the others the tiled kernel; whole matrix and rows starting at
    an offset."""
    out_dim = 6007
    w = _random_kquant_matrix(orc, fmt, in_dim, out_dim, 17 + fmt)
    acts = orc.quantize_row_q8_k(orc.Lcg(0x5E + fmt).fill(in_dim, 3.0))
    want = orc.gemv(fmt, w, in_dim, out_dim, acts, impl=orc.LANES, threads=8)
    wd, ad = dev(w), dev(acts.view(np.uint8))
    out = torch.empty(out_dim, dtype=torch.float32, device="cuda")
    rv.gemv_q8_k(fmt, wd, in_dim, out_dim, ad, out)
    assert host(out).tobytes() == want.tobytes()
    part = torch.empty(out_dim - 5, dtype=torch.float32, device="cuda")
    rv.gemv_q8_k_rows(fmt, wd, in_dim, out_dim, ad, range(5, out_dim), part)
    assert host(part).tobytes() == want[5:].tobytes()
