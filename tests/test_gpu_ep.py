"""Expert-parallel MoE on GPUs (ramvamp_b200/ep.py with the CUDA engine).

world 1: ExpertParallelMoe over rv_moe_route / rv_ep_plan / rv_moe_experts /
rv_moe_combine equals rv_moe_forward bit for bit (exact and tensor paths).
world 2 (two GPUs, NCCL): each rank holds half the experts (strided) and its
own home tokens; every rank's result equals the single-GPU forward of its
tokens bit for bit.  Skipped with fewer than two GPUs.
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
