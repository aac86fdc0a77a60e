"""The install reader's validation (format/layout.rs:71-203), re-expressing
the reference's layout tests (format/layout.rs:206-339) on its sample
fixtures (format/mod.rs:100-250)."""
import copy
import json

import pytest

pytest.importorskip("torch")
from ramvamp_b200 import rvmp  # noqa: E402

ZERO_SHA = "0" * 64


def sample_layout():
    def proj(name, off, n, q):
        return rvmp.Projection(name, off, n, q)

    return rvmp.ExpertsLayout([
        rvmp.LayerEntry("experts/layer_00.bin", 12288, 4,
                        [proj("gate", 0, 1024, "q4_k"), proj("up", 4096, 1024, "q4_k"), proj("down", 8192, 2048, "q6_k")]),
        rvmp.LayerEntry("experts/layer_01.bin", 16384, 4,
                        [proj("gate", 0, 2048, "q4_k"), proj("up", 4096, 2048, "q4_k"), proj("down", 8192, 4096, "q6_k")]),
    ])


def sample_manifest():
    files = {"common.bin": {"size": 4096, "sha256": ZERO_SHA},
             "experts/layout.json": {"size": 2, "sha256": ZERO_SHA},
             "experts/layer_00.bin": {"size": 4 * 12288, "sha256": ZERO_SHA},
             "experts/layer_01.bin": {"size": 4 * 16384, "sha256": ZERO_SHA}}
    return {"arch": {"n_layers": 2, "n_experts": 4, "top_k": 2, "hidden": 64, "moe_intermediate": 96},
            "files": files}


def kind_of(fn, *a):
    with pytest.raises(rvmp.FormatError) as e:
        fn(*a)
    return e.value


def test_json_roundtrip():
    layout = sample_layout()
    back = rvmp.parse_layout(json.loads(json.dumps(layout.to_json())))
    assert back == layout


def test_projection_names_lowercase_and_unknown_fields_rejected():
    obj = sample_layout().to_json()
    assert obj["layers"][0]["projections"][2]["name"] == "down"
    bad = copy.deepcopy(obj)
    bad["layers"][0]["extra"] = 1
    assert kind_of(rvmp.parse_layout, bad).kind == "InvalidLayout"
    bad = copy.deepcopy(obj)
    bad["layers"][0]["projections"][0]["name"] = "Gate"
    assert kind_of(rvmp.parse_layout, bad).kind == "InvalidLayout"


def test_validates_sample_standalone_and_against_manifest():
    layout = sample_layout()
    rvmp.validate_layout(layout)
    rvmp.validate_against(layout, sample_manifest())


def test_rejects_stride_not_page_multiple():
    layout = sample_layout()
    layout.layers[0].stride = 12000
    e = kind_of(rvmp.validate_layout, layout)
    assert e.kind == "Misaligned" and e.what == "expert blob stride" and e.value == 12000


def test_rejects_unaligned_projection_offset():
    layout = sample_layout()
    layout.layers[1].projections[1].offset_in_blob = 4100
    e = kind_of(rvmp.validate_layout, layout)
    assert e.kind == "Misaligned" and e.what == "projection offset" and e.value == 4100


def test_rejects_projection_past_stride():
    layout = sample_layout()
    layout.layers[0].projections[2].len = 5000  # 8192 + 5000 > 12288
    assert kind_of(rvmp.validate_layout, layout).kind == "InvalidLayout"


def test_rejects_overlapping_projections():
    layout = sample_layout()
    layout.layers[0].projections[0].len = 4097  # gate spills into up's slab
    assert kind_of(rvmp.validate_layout, layout).kind == "InvalidLayout"


def test_rejects_duplicate_projection_name():
    layout = sample_layout()
    layout.layers[0].projections[1].name = "gate"
    assert kind_of(rvmp.validate_layout, layout).kind == "InvalidLayout"


def test_rejects_zero_stride_experts_and_projections():
    for mutate in (lambda l: setattr(l.layers[0], "stride", 0), lambda l: setattr(l.layers[0], "n_experts", 0),
                   lambda l: setattr(l.layers[0], "projections", []),
                   lambda l: setattr(l.layers[0].projections[0], "len", 0),
                   lambda l: setattr(l.layers[0].projections[0], "quant", "")):
        layout = sample_layout()
        mutate(layout)
        assert kind_of(rvmp.validate_layout, layout).kind == "InvalidLayout"
    assert kind_of(rvmp.validate_layout, rvmp.ExpertsLayout([])).kind == "InvalidLayout"


@pytest.mark.parametrize("name", ["", "/abs/layer.bin", "../layer.bin", "experts/../x.bin", "experts/./x.bin"])
def test_rejects_unsafe_file_names(name):
    layout = sample_layout()
    layout.layers[0].file = name
    assert kind_of(rvmp.validate_layout, layout).kind == "UnsafeFileName"


def test_cross_check_rejects_layer_count_mismatch():
    layout = sample_layout()
    layout.layers.pop()
    assert kind_of(rvmp.validate_against, layout, sample_manifest()).kind == "InvalidLayout"


def test_cross_check_rejects_file_size_mismatch():
    manifest = sample_manifest()
    manifest["files"]["experts/layer_00.bin"]["size"] -= 1
    assert kind_of(rvmp.validate_against, sample_layout(), manifest).kind == "InvalidLayout"


def test_cross_check_rejects_missing_file_entry():
    layout = sample_layout()
    layout.layers[1].file = "experts/other.bin"
    assert kind_of(rvmp.validate_against, layout, sample_manifest()).kind == "MissingFileEntry"


def test_cross_check_rejects_expert_count_mismatch_and_reused_file():
    layout = sample_layout()
    layout.layers[0].n_experts = 8
    assert kind_of(rvmp.validate_against, layout, sample_manifest()).kind == "InvalidLayout"
    layout = sample_layout()
    layout.layers[1].file = layout.layers[0].file
    assert kind_of(rvmp.validate_against, layout, sample_manifest()).kind == "InvalidLayout"


def test_qwen3_install_maps_to_the_table_layouts():
    """A Qwen3-30B-A3B layout.json (slabs at 0 / 884,736 / 1,769,472; Q6_K
    down on the pinned layers) gives the table's layer layouts."""
    import ramvamp_b200 as rv

    layers = []
    for li in range(48):
        L = rv.qwen3_layer_layout(li)
        down_q = "q6_k" if li in rv.QWEN3_Q6K_DOWN_LAYERS else "q4_k"
        layers.append(rvmp.LayerEntry(f"experts/layer_{li:02d}.bin", L.stride, 128, [
            rvmp.Projection("gate", L.gate_off, L.gate_len, "q4_k"),
            rvmp.Projection("up", L.up_off, L.up_len, "q4_k"),
            rvmp.Projection("down", L.down_off, L.down_len, down_q)]))
    layout = rvmp.ExpertsLayout(layers)
    rvmp.validate_layout(layout)
    got = rvmp.layer_layouts(layout, 2048, 768)
    for li, g in enumerate(got):
        want = rv.qwen3_layer_layout(li)
        assert bytes(g) == bytes(want), li
    assert got[0].stride == 3059712 and got[6].stride == 2654208


def test_unsupported_quant_for_the_gpu_path():
    layout = sample_layout()
    layout.layers[0].projections[2].quant = "q8_0"
    rvmp.validate_layout(layout)  # a valid install ...
    with pytest.raises(rvmp.FormatError):  # ... whose experts the GPU path cannot run
        rvmp.layer_layouts(layout, 64, 96)
