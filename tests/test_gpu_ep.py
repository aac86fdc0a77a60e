"""Expert-parallel MoE on GPUs.

The library's exchange (rv_ep_*, ramvamp_b200.ExpertParallel): with one rank
it runs every stage and equals rv_moe_forward bit for bit, also captured in a
CUDA graph and with empty calls; handles that are not the group's are
refused; on two GPUs (one process each) every rank's result equals the
single-GPU forward and the oracle bit for bit.

The host-collective harness (ramvamp_b200/ep.py, torch.distributed
all-to-alls over rv_moe_route / rv_ep_plan / rv_moe_experts /
rv_moe_combine) is checked the same way at world 1 and 2.  Two-GPU tests
are skipped with fewer than two GPUs.
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

H, M, E, K = 2048, 768, 128, 8


@pytest.fixture(scope="module")
def rv():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import ramvamp_b200

    return ramvamp_b200


def bits(t):
    torch.cuda.synchronize()
    return t.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("flags_name,T", [("EXACT", 5), ("EXACT", 40), ("TENSOR", 40)])
def test_ep_world1_equals_forward(rv, flags_name, T):
    from ramvamp_b200.ep import EngineBackend, ExpertParallelMoe

    flags = getattr(rv, flags_name)
    lay = rv.qwen3_layer_layout(0)
    table = rv.ExpertTable([lay], device=0)
    table.fill_synthetic(0, seed=71, sigma=0.02)
    router = rv.synth_normal(72, 0, 0.02, E * H).view(E, H).contiguous()
    norm = torch.ones(H, device="cuda")
    eng = rv.MoeEngine(H, M, E, K, True, 1e-6, max_tokens=64, device=0)
    x = rv.synth_normal(73 + T, 0, 1.0, T * H).view(T, H).contiguous()
    want = x.clone()
    eng.forward(table, 0, norm, router, want, flags=flags)
    got = x.clone()
    ep = ExpertParallelMoe(EngineBackend(eng, table, [norm], [router], flags), 1, 0)
    ep.forward(0, got)
    assert (bits(got) == bits(want)).all()
    rv.device_status(0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    try:
        import datetime

        import torch.distributed as dist

        import ramvamp_b200 as rv
        from ramvamp_b200.ep import EngineBackend, ExpertParallelMoe

        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        T = 96
        full = rv.ExpertTable([rv.qwen3_layer_layout(6)], device=rank)
        full.fill_synthetic(0, seed=81, sigma=0.02)
        shard = rv.ExpertTable([rv.qwen3_layer_layout(6, n_experts=E // world)], device=rank)
        shard.fill_synthetic(0, seed=81, sigma=0.02, first_expert=rank, expert_step=world)
        router = rv.synth_normal(82, 0, 0.02, E * H).view(E, H).contiguous()
        norm = torch.ones(H, device="cuda")
        eng = rv.MoeEngine(H, M, E, K, True, 1e-6, max_tokens=T * world, device=rank)
        x = rv.synth_normal(83 + rank, 0, 1.0, T * H).view(T, H).contiguous()
        results = []
        for flags in (rv.EXACT, rv.TENSOR):
            want = x.clone()
            eng.forward(full, 0, norm, router, want, flags=flags)
            got = x.clone()
            ExpertParallelMoe(EngineBackend(eng, shard, [norm], [router], flags), world, rank).forward(0, got)
            torch.cuda.synchronize()
            results.append(bool(torch.equal(got.view(torch.int32), want.view(torch.int32))))
        rv.device_status(rank)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, results))
    except Exception as exc:  # reported to the parent
        q.put((rank, repr(exc)))


def test_ep_two_gpus_bit_identical(rv):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    for rank, res in results:
        assert res == [True, True], f"rank {rank}: {res}"


# ------------------------------------------- the library's exchange (rv_ep_*)
def _layers(rv, world=1, rank=0, device=0):
    """Layers 0 (Q6_K down) and 6 (Q4_K down): this rank's experts (strided)."""
    lays = [rv.qwen3_layer_layout(l, n_experts=E // world) for l in (0, 6)]
    table = rv.ExpertTable(lays, device=device)
    for i, seed in enumerate((91, 96)):
        table.fill_synthetic(i, seed=seed, sigma=0.02, first_expert=rank, expert_step=world)
    return table


def _full_layers(rv, device=0):
    return _layers(rv, 1, 0, device)


def _routers(rv):
    return [rv.synth_normal(92 + i, 0, 0.02, E * H).view(E, H).contiguous() for i in range(2)]


@pytest.mark.parametrize("flags_name,T", [("EXACT", 1), ("EXACT", 37), ("TENSOR", 5), ("TENSOR", 300)])
def test_library_ep_world1_equals_forward(rv, flags_name, T):
    """rv_moe_ep_forward with one rank: every stage of the exchange runs
    (dispatch into the window, receive index, down rows stored through the
    output map, flags, combine) and the layer equals rv_moe_forward bit for
    bit through two layers, routing included."""
    flags = getattr(rv, flags_name)
    table = _full_layers(rv)
    routers = _routers(rv)
    norm = torch.ones(H, device="cuda")
    eng = rv.MoeEngine(H, M, E, K, True, 1e-6, max_tokens=max(T, 8), device=0)
    ref = rv.MoeEngine(H, M, E, K, True, 1e-6, max_tokens=max(T, 8), device=0)
    ep = rv.ExpertParallel(eng, 1, 0, max(T, 8))
    ep.connect([ep.handle_bytes()])
    x = rv.synth_normal(400 + T, 0, 1.0, T * H).view(T, H).contiguous()
    got, want = x.clone(), x.clone()
    for li in range(2):
        gi = torch.empty(T * K, dtype=torch.int32, device="cuda")
        wi = torch.empty(T * K, dtype=torch.int32, device="cuda")
        gw = torch.empty(T * K, device="cuda")
        ww = torch.empty(T * K, device="cuda")
        ep.forward(table, li, norm, routers[li], got, gi, gw, flags=flags)
        ref.forward(table, li, norm, routers[li], want, wi, ww, flags=flags)
        assert (bits(gi) == bits(wi)).all() and (bits(gw) == bits(ww)).all(), f"layer {li}: routing"
        assert (bits(got) == bits(want)).all(), f"layer {li}: residual"
    assert ep.received() == [T * K]
    rv.device_status(0)
    ep.close()


def test_library_ep_world1_with_a_placement(rv):
    """A placement that permutes the local ids (the table filled in that
    order) gives the same bits as rv_moe_forward on the natural order."""
    from ramvamp_b200.ep import placement_tensor

    T = 96
    rng = np.random.default_rng(11)
    order = [int(e) for e in rng.permutation(E)]
    lays = [rv.qwen3_layer_layout(l) for l in (0, 6)]
    table = rv.ExpertTable(lays, device=0)
    for i, seed in enumerate((91, 96)):
        table.fill_synthetic_list(i, seed, 0.02, order)
    place = placement_tensor([order], "cuda:0")
    full = _full_layers(rv)
    routers = _routers(rv)
    norm = torch.ones(H, device="cuda")
    eng = rv.MoeEngine(H, M, E, K, True, 1e-6, max_tokens=T, device=0)
    ref = rv.MoeEngine(H, M, E, K, True, 1e-6, max_tokens=T, device=0)
    ep = rv.ExpertParallel(eng, 1, 0, T)
    ep.connect([ep.handle_bytes()])
    x = rv.synth_normal(450, 0, 1.0, T * H).view(T, H).contiguous()
    for flags in (rv.EXACT, rv.TENSOR):
        got, want = x.clone(), x.clone()
        for li in range(2):
            ep.forward(table, li, norm, routers[li], got, flags=flags, placement=place)
            ref.forward(full, li, norm, routers[li], want, flags=flags)
        assert (bits(got) == bits(want)).all(), flags
    rv.device_status(0)
    ep.close()


def test_library_ep_graph_capture_and_empty_calls(rv):
    """Two layers of rv_moe_ep_forward captured in one CUDA graph replay to
    the eager result (the flags count layers on the device, so replays keep
    the protocol); calls with no tokens keep it too."""
    T = 64
    table = _full_layers(rv)
    routers = _routers(rv)
    norm = torch.ones(H, device="cuda")
    eng = rv.MoeEngine(H, M, E, K, True, 1e-6, max_tokens=T, device=0)
    ep = rv.ExpertParallel(eng, 1, 0, T)
    ep.connect([ep.handle_bytes()])
    ref = rv.MoeEngine(H, M, E, K, True, 1e-6, max_tokens=T, device=0)
    res = torch.empty(T, H, device="cuda")
    empty = torch.empty(0, H, device="cuda")

    def body():
        for li in range(2):
            ep.forward(table, li, norm, routers[li], res, flags=rv.TENSOR)
        ep.forward(table, 0, norm, routers[0], empty, flags=rv.TENSOR)

    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        res.copy_(rv.synth_normal(500, 0, 1.0, T * H).view(T, H))
        body()  # eager once (lazy set-up)
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        body()
    for seed in (501, 502, 503):
        x = rv.synth_normal(seed, 0, 1.0, T * H).view(T, H).contiguous()
        with torch.cuda.stream(s):
            res.copy_(x)
            g.replay()
        s.synchronize()
        want = x.clone()
        for li in range(2):
            ref.forward(table, li, norm, routers[li], want, flags=rv.TENSOR)
        assert (bits(res) == bits(want)).all(), seed
    rv.device_status(0)
    del g
    ep.close()


def test_library_ep_connect_checks_handles(rv):
    """rv_ep_connect refuses handles that are not this group's, before
    mapping anything; forward before connect is a protocol error."""
    eng = rv.MoeEngine(H, M, E, K, True, 1e-6, max_tokens=16, device=0)
    other = rv.MoeEngine(H, M, E, K, True, 1e-6, max_tokens=16, device=0)
    ep0 = rv.ExpertParallel(eng, 2, 0, 8)
    ep1 = rv.ExpertParallel(other, 2, 1, 8)  # the same GPU: refused as a peer
    h0, h1 = ep0.handle_bytes(), ep1.handle_bytes()
    table = _layers(rv, 2, 0)
    norm = torch.ones(H, device="cuda")
    x = torch.zeros(4, H, device="cuda")
    with pytest.raises(rv.KernelError) as e:
        ep0.forward(table, 0, norm, _routers(rv)[0], x)
    assert e.value.kind == "Protocol"
    bad = bytearray(h1)
    bad[0] ^= 0xFF
    cases = [([h0, bytes(bad)], "Peer"),            # not an exchange handle
             ([h0, h0], "Peer"),                    # rank 0 twice
             ([h1, h0], "Peer"),                    # wrong order
             ([h0, h1], "Peer"),                    # two ranks on one GPU
             ([h0], "LengthMismatch")]              # one handle for two ranks
    small = rv.ExpertParallel(rv.MoeEngine(H, M, E, K, True, 1e-6, max_tokens=16, device=0), 2, 1, 4)
    cases.append(([h0, small.handle_bytes()], "Peer"))  # another capacity
    for handles, kind in cases:
        with pytest.raises(rv.KernelError) as e:
            ep0.connect(handles)
        assert e.value.kind == kind, (kind, str(e.value))
    with pytest.raises(rv.KernelError) as e:
        rv.ExpertParallel(eng, 3, 0, 4)  # 128 experts do not split over 3 ranks
    assert e.value.kind == "Unimplemented"
    with pytest.raises(rv.KernelError) as e:
        rv.ExpertParallel(eng, 4, 0, 8)  # the engine holds 16 rows, not 4 x 8
    assert e.value.kind == "LengthMismatch"
    rv.device_status(0)


def _lib_rank_main(rank, world, port, tokens, out_dir, q):
    try:
        import datetime

        import torch.distributed as dist

        import ramvamp_b200 as rv
        from ramvamp_b200.ep import connect_group

        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        from ramvamp_b200.ep import balanced_placement, placement_tensor

        T = tokens[rank]
        cap = max(tokens)
        # Layer 0 by id mod world; layer 1 by a placement from skewed loads.
        ranks1 = balanced_placement(list(np.random.default_rng(5).zipf(1.5, E).astype(float)), world)
        lays = [rv.qwen3_layer_layout(l, n_experts=E // world) for l in (0, 6)]
        table = rv.ExpertTable(lays, device=rank)
        table.fill_synthetic(0, seed=91, sigma=0.02, first_expert=rank, expert_step=world)
        table.fill_synthetic_list(1, 96, 0.02, ranks1[rank])
        places = [None, placement_tensor(ranks1, f"cuda:{rank}")]
        routers = _routers(rv)
        norm = torch.ones(H, device="cuda")
        eng = rv.MoeEngine(H, M, E, K, True, 1e-6, max_tokens=world * cap, device=rank)
        ep = rv.ExpertParallel(eng, world, rank, cap)
        connect_group(ep)
        x = rv.synth_normal(600 + rank, 0, 1.0, T * H).view(T, H).contiguous()
        empty = torch.empty(0, H, device="cuda")
        for name, flags in (("exact", rv.EXACT), ("tensor", rv.TENSOR)):
            res = x.clone()
            for li in range(2):
                ep.forward(table, li, norm, routers[li], res, flags=flags, placement=places[li])
                # Every rank joins every call; in this extra one rank 0 sends
                # 16 other tokens and the last rank brings none.
                extra = rv.synth_normal(700 + li, 0, 1.0, 16 * H).view(16, H).contiguous()
                ep.forward(table, li, norm, routers[li], extra if rank == 0 else empty, flags=flags,
                           placement=places[li])
            torch.cuda.synchronize()
            np.save(os.path.join(out_dir, f"{name}_{rank}.npy"), res.cpu().numpy())
        rv.device_status(rank)
        dist.barrier()
        ep.close()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as exc:  # reported to the parent
        q.put((rank, repr(exc)))


def test_library_ep_two_gpus_matches_single_gpu_and_oracle(rv, orc, tmp_path):
    """Two ranks on two GPUs (one process each; handles exchanged over gloo,
    NVLS unused): each rank's tokens through two layers equal the
    single-GPU forward bit for bit on both paths, and the oracle's arms
    (lane model for the exact path, scalar for the tensor path)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    world, tokens = 2, [300, 212]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_lib_rank_main, args=(r, world, port, tokens, str(tmp_path), q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, res in results:
        assert res == "ok", f"rank {rank}: {res}"
    table = _full_layers(rv)
    routers = _routers(rv)
    norm = torch.ones(H, device="cuda")
    eng = rv.MoeEngine(H, M, E, K, True, 1e-6, max_tokens=max(tokens), device=0)
    lays = [rv.qwen3_layer_layout(l) for l in (0, 6)]
    blobs = [rv.alias(table.view(i, 0).blob, E * lays[i].stride).cpu().numpy() for i in range(2)]
    for name, flags, impl in (("exact", rv.EXACT, 2), ("tensor", rv.TENSOR, 0)):
        for rank in range(world):
            T = tokens[rank]
            x = rv.synth_normal(600 + rank, 0, 1.0, T * H).view(T, H).contiguous()
            want = x.clone()
            for li in range(2):
                eng.forward(table, li, norm, routers[li], want, flags=flags)
            got = np.load(str(tmp_path / f"{name}_{rank}.npy"))
            assert (got.view(np.uint32) == bits(want)).all(), (name, rank)
        # The oracle on the last rank's tokens.
        xr = x.cpu().numpy()
        for li in range(2):
            L = lays[li]
            OL = orc.make_layer(H, M, E, K, 1e-6, np.ones(H, np.float32), routers[li].cpu().numpy(), blobs[li],
                                L.stride, L.gate_off, L.up_off, L.down_off, L.gate_format, L.up_format,
                                L.down_format)
            xr, _, _ = orc.moe_prefill(OL, xr, impl=impl, threads=max(1, min(32, os.cpu_count() or 1)))
        assert (xr.view(np.uint32) == got.view(np.uint32)).all(), (name, "oracle")
    rv.device_status(0)
