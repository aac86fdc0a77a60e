"""Loading an install's expert files into the HBM table (the native file
loader behind rvmp.load_expert_table), then the MoE block on those bytes
against the oracle, bit for bit."""
import json
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

H, M, E, K = 256, 512, 8, 2


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


def write_install(rv, root):
    """Two layers (Q6_K and Q4_K down) of synthetic experts as an install:
    manifest.json, experts/layout.json, experts/layer_XX.bin."""
    from ramvamp_b200 import rvmp

    lays = [rv.qwen3_layer_layout(0, hidden=H, moe=M, n_experts=E, down_format=rv.QuantFormat.Q6_K),
            rv.qwen3_layer_layout(1, hidden=H, moe=M, n_experts=E, down_format=rv.QuantFormat.Q4_K)]
    src = rv.ExpertTable(lays, device=0)
    os.makedirs(os.path.join(root, "experts"), exist_ok=True)
    layers, files, blobs = [], {}, []
    for li, L in enumerate(lays):
        src.fill_synthetic(li, seed=300 + li, sigma=0.02)
        b = host(rv.alias(src.view(li, 0).blob, E * L.stride, torch.uint8))
        name = f"experts/layer_{li:02d}.bin"
        b.tofile(os.path.join(root, name))
        blobs.append(b)
        files[name] = {"size": int(b.size), "sha256": "0" * 64}
        q = {0: "q4_k", 1: "q5_k", 2: "q6_k"}
        layers.append(rvmp.LayerEntry(name, L.stride, E, [
            rvmp.Projection("gate", L.gate_off, L.gate_len, q[L.gate_format]),
            rvmp.Projection("up", L.up_off, L.up_len, q[L.up_format]),
            rvmp.Projection("down", L.down_off, L.down_len, q[L.down_format])]))
    with open(os.path.join(root, "experts/layout.json"), "w") as f:
        json.dump(rvmp.ExpertsLayout(layers).to_json(), f)
    with open(os.path.join(root, "manifest.json"), "w") as f:
        json.dump({"arch": {"n_layers": 2, "n_experts": E, "top_k": K, "hidden": H, "moe_intermediate": M},
                   "files": files}, f)
    src.close()
    return lays, blobs


def test_install_loads_byte_for_byte_and_runs(rv, orc, tmp_path):
    from ramvamp_b200 import rvmp

    lays, blobs = write_install(rv, str(tmp_path))
    table = rvmp.load_expert_table(str(tmp_path), device=0)
    assert table.n_layers == 2
    for li, L in enumerate(lays):
        got = host(rv.alias(table.view(li, 0).blob, E * L.stride, torch.uint8))
        assert got.tobytes() == blobs[li].tobytes()
    router = rv.synth_normal(7, 0, 0.02, E * H).view(E, H).contiguous()
    norm = torch.ones(H, dtype=torch.float32, device="cuda")
    eng = rv.MoeEngine(H, M, E, K, True, 1e-6, max_tokens=4, device=0)
    for li, L in enumerate(lays):
        x = rv.synth_normal(40 + li, 0, 1.0, 3 * H).view(3, H).contiguous()
        res = x.clone()
        eng.forward(table, li, norm, router, res)
        ol = orc.make_layer(H, M, E, K, 1e-6, host(norm), host(router), blobs[li], L.stride, L.gate_off,
                            L.up_off, L.down_off, L.gate_format, L.up_format, L.down_format)
        want, _, _, _ = orc.moe_decode(ol, host(x), threads=4)
        assert bits(host(res)).tobytes() == bits(want).tobytes()


def test_load_file_errors(rv, tmp_path):
    lays, blobs = write_install(rv, str(tmp_path))
    table = rv.ExpertTable(lays, device=0)
    short = os.path.join(str(tmp_path), "short.bin")
    blobs[0][:-16].tofile(short)
    with pytest.raises(rv.KernelError) as e:
        table.load_file(0, short)
    assert e.value.kind == "LengthMismatch"
    with pytest.raises(rv.KernelError) as e:
        table.load_file(0, os.path.join(str(tmp_path), "missing.bin"))
    assert e.value.kind == "Io"
    with pytest.raises(rv.KernelError) as e:
        table.load_file(5, short)
    assert e.value.kind == "LayerOutOfRange"
    # a file with a header in front of the blobs
    padded = os.path.join(str(tmp_path), "padded.bin")
    np.concatenate([np.zeros(4096, np.uint8), blobs[1]]).tofile(padded)
    table.load_file(1, padded, offset=4096)
    got = host(rv.alias(table.view(1, 0).blob, E * lays[1].stride, torch.uint8))
    assert got.tobytes() == blobs[1].tobytes()
