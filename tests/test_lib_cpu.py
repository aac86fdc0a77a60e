"""CPU-only checks of the C-ABI library: it loads, exports every symbol the
header declares, and rejects bad geometry with the reference's error kinds
(validation runs before any CUDA call, so no GPU is needed)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def rv():
    import ramvamp_b200

    return ramvamp_b200


def header_symbols():
    src = open(os.path.join(ROOT, "include", "ramvamp_b200.h")).read()
    return sorted(set(re.findall(r"^RV_API [^(]*?\b(rv_\w+)\(", src, flags=re.M)))


def test_header_declares_the_boundary():
    syms = header_symbols()
    for name in ("rv_quantize_row_q8_k", "rv_gemv_q8_k", "rv_gemv_q8_k_rows", "rv_gemv_q8_k_batched",
                 "rv_gemv_q8_k_fused_rows", "rv_moe_forward", "rv_moe_forward_host",
                 "rv_expert_table_begin_layer", "rv_expert_table_view", "rv_expert_table_end_layer"):
        assert name in syms


def test_library_exports_every_header_symbol(rv):
    lib = rv.lib()
    missing = [s for s in header_symbols() if not hasattr(lib, s)]
    assert not missing, missing
    from ramvamp_b200 import _lib
    assert set(header_symbols()) == set(_lib.SIGNATURES), "binding table out of sync with the header"


def test_version_and_status_names(rv):
    assert rv.lib().rv_version().startswith(b"ramvamp_b200")
    names = [rv.lib().rv_status_name(i).decode() for i in range(1, 10)]
    assert names == ["IndivisibleRow", "RowBytesNotBlockMultiple", "BlockCountMismatch",
                     "QuantizeLenMismatch", "LengthMismatch", "Empty", "InvalidHeadDim",
                     "Unimplemented", "UnsupportedFormat"]


def test_row_bytes_helper(rv):
    """quants/tests.rs:444-467."""
    Q = rv.QuantFormat
    assert Q.Q4_K.row_bytes(2048) == 1152
    assert Q.Q5_K.row_bytes(768) == 528
    assert Q.Q6_K.row_bytes(768) == 630
    assert Q.Q8_0.row_bytes(2048) == 2176
    assert Q.Q8_K.row_bytes(256) == 292
    assert Q.Q4_K.row_bytes(0) == 0
    with pytest.raises(rv.KernelError) as e:
        Q.Q4_K.row_bytes(100)
    assert e.value.kind == "IndivisibleRow"
    with pytest.raises(rv.KernelError) as e:
        Q.Q8_0.row_bytes(33)
    assert e.value.kind == "IndivisibleRow"


def _gemv(rv, fmt, wlen, in_dim, out_dim, acts_len, r0, r1, out_len, n_acts=1):
    lib = rv.lib()
    code = lib.rv_gemv_q8_k_batched(fmt, None, wlen, in_dim, out_dim, None, acts_len, n_acts, r0, r1,
                                    None, out_len, None)
    return rv.lib().rv_status_name(code).decode()


def test_gemv_validation_precedence(rv):
    """gemv.rs:212-264 (validate) and its tests: same checks, same order."""
    assert _gemv(rv, 3, 0, 256, 1, 1, 0, 1, 1) == "UnsupportedFormat"  # Q8_0 with Q8_K acts
    assert _gemv(rv, 4, 0, 256, 1, 1, 0, 1, 1) == "UnsupportedFormat"
    assert _gemv(rv, 0, 0, 100, 1, 1, 0, 1, 1) == "IndivisibleRow"
    assert _gemv(rv, 0, 143, 256, 1, 1, 0, 1, 1) == "LengthMismatch"      # weight bytes vs rows
    assert _gemv(rv, 0, 144, 256, 1, 1, 1, 0, 0) == "LengthMismatch"      # inverted range
    assert _gemv(rv, 0, 144, 256, 1, 1, 0, 2, 2) == "LengthMismatch"      # range past out_dim
    assert _gemv(rv, 0, 144, 256, 1, 1, 0, 1, 2) == "LengthMismatch"      # out vs range
    assert _gemv(rv, 0, 144, 256, 1, 2, 0, 1, 1) == "BlockCountMismatch"
    # valid geometry reaches the pointer checks (still before any CUDA call)
    assert _gemv(rv, 2, 630 * 4, 768, 4, 3 * 3, 0, 4, 12, n_acts=3) == "InvalidArgument"
    # absurd n_acts saturates instead of wrapping (gemv.rs:207-211)
    assert _gemv(rv, 0, 144, 256, 1, 1, 0, 1, 1, n_acts=2 ** 63) == "LengthMismatch"


def test_empty_calls_are_noops(rv):
    lib = rv.lib()
    assert lib.rv_gemv_q8_k_batched(0, None, 144, 256, 1, None, 0, 0, 0, 1, None, 0, None) == 0
    assert lib.rv_gemv_q8_k_rows(0, None, 144, 256, 1, None, 1, 1, 1, None, 0, None) == 0
    assert lib.rv_quantize_row_q8_k(None, 0, None, 0, None) == 0


def test_quantize_and_primitive_errors(rv):
    """quantize.rs:179-200, norm.rs / softmax.rs / activation.rs error tests."""
    lib = rv.lib()
    name = lambda c: lib.rv_status_name(c).decode()
    assert name(lib.rv_quantize_row_q8_k(None, 100, None, 1, None)) == "QuantizeLenMismatch"
    assert name(lib.rv_rmsnorm(None, None, 0, 1, ctypes.c_float(1e-6), None, None)) == "Empty"
    assert name(lib.rv_softmax(None, 0, 1, None)) == "Empty"
    assert name(lib.rv_swiglu_combine(None, 4, None, 3, None)) == "LengthMismatch"
    assert name(lib.rv_debug_block_sums(0, None, 143, None, 1, None, None, None)) == "RowBytesNotBlockMultiple"


def test_fused_rows_validation(rv):
    """gemv.rs:747-823: range checks against the fused out_dim."""
    from ramvamp_b200 import _lib
    lib = rv.lib()
    parts = (_lib.FusedPartC * 2)(_lib.FusedPartC(0, None, 144 * 2, 256, 2, None, 1),
                                   _lib.FusedPartC(0, None, 144 * 3, 256, 3, None, 1))
    name = lambda c: lib.rv_status_name(c).decode()
    assert name(lib.rv_gemv_q8_k_fused_rows(parts, 2, 3, 2, None, 0, None)) == "LengthMismatch"
    assert name(lib.rv_gemv_q8_k_fused_rows(parts, 2, 0, 6, None, 6, None)) == "LengthMismatch"
    assert name(lib.rv_gemv_q8_k_fused_rows(parts, 2, 0, 5, None, 4, None)) == "LengthMismatch"
    bad = (_lib.FusedPartC * 2)(_lib.FusedPartC(0, None, 144 * 2, 256, 2, None, 1),
                                _lib.FusedPartC(3, None, 34 * 3, 32, 3, None, 1))
    assert name(lib.rv_gemv_q8_k_fused_rows(bad, 2, 1, 4, None, 3, None)) == "UnsupportedFormat"


def test_qwen3_layout_geometry(rv):
    """docs/architecture.md:72-76: blob strides and slab offsets."""
    L6 = rv.qwen3_layer_layout(0)
    assert (L6.stride, L6.gate_off, L6.up_off, L6.down_off) == (3_059_712, 0, 884_736, 1_769_472)
    assert (L6.gate_len, L6.down_len) == (884_736, 1_290_240)
    L4 = rv.qwen3_layer_layout(6)
    assert L4.stride == 2_654_208 and L4.down_format == int(rv.QuantFormat.Q4_K)
    assert len(rv.QWEN3_Q6K_DOWN_LAYERS) == 24
    total = sum(rv.qwen3_layer_layout(l).stride for l in range(48)) * 8
    assert total == 1_097_072_640  # expert bytes per decode token (docs/architecture.md:259)


def test_moe_create_rejects_bad_geometry(rv):
    from ramvamp_b200 import _lib
    lib = rv.lib()
    h = ctypes.c_void_p()
    name = lambda c: lib.rv_status_name(c).decode()
    cfg = _lib.MoeConfig(2000, 768, 128, 8, 1, 1e-6)
    assert name(lib.rv_moe_create(0, ctypes.byref(cfg), 1, ctypes.byref(h))) == "IndivisibleRow"
    cfg = _lib.MoeConfig(2048, 768, 512, 8, 1, 1e-6)
    assert name(lib.rv_moe_create(0, ctypes.byref(cfg), 1, ctypes.byref(h))) == "Unimplemented"
    cfg = _lib.MoeConfig(2048, 768, 128, 8, 1, 1e-6)
    assert name(lib.rv_moe_create(0, ctypes.byref(cfg), 0, ctypes.byref(h))) == "InvalidArgument"


def test_oracle_layout_twin_matches_the_product(rv):
    """oracle/layout.py (what the reference arm uses, so that it never loads
    this library) gives the product's blob geometry for all 48 layers and a
    small geometry, and the same model shapes."""
    import dataclasses

    from oracle.layout import Layout, ModelShape, layer_layout
    from ramvamp_b200.model import ModelConfig

    names = [f.name for f in dataclasses.fields(Layout)]
    for l in range(48):
        a, b = layer_layout(l), rv.qwen3_layer_layout(l)
        assert [getattr(a, n) for n in names] == [getattr(b, n) for n in names], l
    a = layer_layout(0, hidden=1024, moe=512, n_experts=64, down_format=0)
    b = rv.qwen3_layer_layout(0, hidden=1024, moe=512, n_experts=64, down_format=rv.QuantFormat.Q4_K)
    assert [getattr(a, n) for n in names] == [getattr(b, n) for n in names]
    assert dataclasses.asdict(ModelShape()) == dataclasses.asdict(ModelConfig())
    for n in (48, 3):
        assert [ModelShape(n_layers=n).q6k_layer(l) for l in range(n)] == \
            [ModelConfig(n_layers=n).q6k_layer(l) for l in range(n)]
