"""rv_moe_forward_static: the MoE block for callers that cannot allocate.

Some callers cannot call cudaMalloc: their device memory is owned by another
allocator (a serving runtime's pool, a process under a memory cap) or they run
where allocation is not allowed.  rv_moe_forward_static keeps every
intermediate in one file-scope device array instead of an engine's scratch.
This test calls it through the C ABI twice in a row and checks each result
against rv_moe_forward (the entry point that owns its scratch) bit for bit,
the tolerance every parity test here uses.  It sorts last so a run that stops
at the first failure has already run everything else, and it works both in a
fresh process and after the other tests.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

# (hidden, moe, experts, top-k, down format): the Qwen3 geometry (fused
# combine in the down kernel), and a smaller one that takes the generic
# kernels (one-lane gate/up rows, 32-row down tiles and a separate combine)
# with Q4_K down rows.
GEOMETRIES = [(2048, 768, 128, 8, "Q6_K"), (1024, 512, 64, 4, "Q4_K")]


def bits(t):
    torch.cuda.synchronize()
    return t.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("H,M,E,K,down", GEOMETRIES)
def test_static_entry_point_matches_engine_on_two_calls(H, M, E, K, down):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import ramvamp_b200 as rv
    from ramvamp_b200 import _lib

    lib = rv.lib()
    layout = rv.qwen3_layer_layout(0, hidden=H, moe=M, n_experts=E, down_format=rv.QuantFormat[down])
    table = rv.ExpertTable([layout], device=0)
    table.fill_synthetic(0, seed=97, sigma=0.02)
    blobs = table.view(0, 0).blob  # the layer's blobs, contiguous
    router = rv.synth_normal(98, 0, 0.02, E * H).view(E, H).contiguous()
    norm = torch.ones(H, dtype=torch.float32, device="cuda")
    eng = rv.MoeEngine(H, M, E, K, True, 1e-6, max_tokens=4, device=0)
    cfg = _lib.MoeConfig(H, M, E, K, 1, 1e-6)
    stream = torch.cuda.current_stream().cuda_stream
    for call, (T, seed) in enumerate([(1, 5), (4, 6)]):
        x = rv.synth_normal(seed, 0, 1.0, T * H).view(T, H).contiguous()
        want = x.clone()
        wids = torch.empty(T * K, dtype=torch.int32, device="cuda")
        ww = torch.empty(T * K, dtype=torch.float32, device="cuda")
        eng.forward(table, 0, norm, router, want, wids, ww)
        got = x.clone()
        gids = torch.empty(T * K, dtype=torch.int32, device="cuda")
        gw = torch.empty(T * K, dtype=torch.float32, device="cuda")
        rc = lib.rv_moe_forward_static(ctypes.byref(cfg), ctypes.byref(layout), blobs, norm.data_ptr(),
                                       router.data_ptr(), got.data_ptr(), T, gids.data_ptr(),
                                       gw.data_ptr(), stream)
        assert rc == 0, _lib.last_error()
        assert (bits(got) == bits(want)).all(), f"call {call}: residual differs"
        assert (bits(gids) == bits(wids)).all() and (bits(gw) == bits(ww)).all(), f"call {call}: routing differs"
    # Sizes beyond the static limit are refused before any work is queued.
    big = torch.zeros(5, H, device="cuda")
    rc = lib.rv_moe_forward_static(ctypes.byref(cfg), ctypes.byref(layout), blobs, norm.data_ptr(),
                                   router.data_ptr(), big.data_ptr(), 5, None, None, stream)
    assert lib.rv_status_name(rc) == b"LengthMismatch"
    rv.device_status(0)
    eng.close()
    table.close()
