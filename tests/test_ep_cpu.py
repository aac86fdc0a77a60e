"""Expert-parallel exchange on CPU ranks (gloo), world sizes 1 and 2.

ExpertParallelMoe (ramvamp_b200/ep.py) drives the dispatch/combine
collectives; here its local compute is the CPU oracle (the reference's
AVX2-arm arithmetic), so the test checks the exchange logic itself: the
plan, the count exchange, the all-to-all-v of ids and Q8_K rows, the
return of the expert outputs and the top-k-order combine.  Every rank's
result must equal the single-process oracle forward (prefill.rs:2136-2263)
bit for bit.
"""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch

H, M, E, K, T = 512, 256, 8, 4, 5
HB, MB = H // 256, M // 256
ACT_STRIDE = (HB * 292 + 15) & ~15
SEED = 4242


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def make_layer(orc):
    import ramvamp_b200 as rv

    lay = rv.qwen3_layer_layout(0, hidden=H, moe=M, n_experts=E)
    blobs = orc.fill_layer_synthetic(lay, SEED, 0.02, 1)
    router = orc.synth_normal(SEED + 1, 0, 0.02, E * H).reshape(E, H)
    norm = np.ones(H, np.float32)
    return lay, blobs, router, norm


class OracleBackend:
    """The local compute of one rank on the CPU oracle (tests only)."""

    def __init__(self, orc, lay, blobs, router, norm, rank, world):
        self.orc, self.lay, self.blobs, self.router, self.norm = orc, lay, blobs, router, norm
        self.rank, self.world = rank, world
        self.hidden = H

    def route(self, layer, residual):
        x = residual.numpy()
        ids = np.zeros((x.shape[0], K), np.int32)
        w = np.zeros((x.shape[0], K), np.float32)
        acts = np.zeros((x.shape[0], ACT_STRIDE), np.uint8)
        for t in range(x.shape[0]):
            normed = self.orc.rmsnorm(x[t:t + 1], self.norm, 1e-6)[0]
            q = self.orc.quantize_row_q8_k(normed)
            acts[t, :HB * 292] = q.view(np.uint8)
            _, i, ww = self.orc.route(normed, self.router, K)
            ids[t], w[t] = i, ww
        return torch.from_numpy(ids), torch.from_numpy(w), torch.from_numpy(acts)

    def plan(self, topk_ids, acts, world):
        ids = topk_ids.numpy().reshape(-1)
        dest = ids % world
        order = np.argsort(dest, kind="stable")
        pos_of = np.empty_like(order)
        pos_of[order] = np.arange(order.size)
        counts = np.bincount(dest, minlength=world).astype(np.int32)
        send_local = (ids[order] // world).astype(np.int32)
        send_acts = acts.numpy()[order // K]
        return (torch.from_numpy(counts), torch.from_numpy(pos_of.astype(np.int32)), torch.from_numpy(send_local),
                torch.from_numpy(np.ascontiguousarray(send_acts)))

    def experts(self, layer, local_ids, acts):
        L, orc = self.lay, self.orc
        rb_gu = 144 * HB
        rb_dn = {0: 144, 1: 176, 2: 210}[L.down_format] * MB
        out = np.zeros((local_ids.numel(), H), np.float32)
        for row, le in enumerate(local_ids.tolist()):
            e = le * self.world + self.rank
            blob = self.blobs[e * L.stride:(e + 1) * L.stride]
            a = acts[row].numpy()[:HB * 292].view(orc.Q8K_DTYPE)
            gate = orc.gemv(L.gate_format, blob[L.gate_off:L.gate_off + M * rb_gu], H, M, a)
            up = orc.gemv(L.up_format, blob[L.up_off:L.up_off + M * rb_gu], H, M, a)
            h = orc.swiglu_combine(gate, up)
            hq = orc.quantize_row_q8_k(h)
            out[row] = orc.gemv(L.down_format, blob[L.down_off:L.down_off + H * rb_dn], M, H, hq)
        return torch.from_numpy(out)

    def combine(self, residual, topk_weights, expert_out, pos_of):
        x = residual.numpy()
        w = topk_weights.numpy()
        out = expert_out.numpy()
        pos = pos_of.numpy()
        for t in range(x.shape[0]):
            acc = np.zeros(H, np.float32)
            for k in range(K):
                acc = acc + w[t, k] * out[pos[t * K + k]]  # float32: separate multiply and add
            x[t] = x[t] + acc
        return residual


def expected(orc, rank):
    lay, blobs, router, norm = make_layer(orc)
    L = orc.make_layer(H, M, E, K, 1e-6, norm, router, blobs, lay.stride, lay.gate_off, lay.up_off, lay.down_off,
                       lay.gate_format, lay.up_format, lay.down_format)
    x = orc.synth_normal(SEED + 10 + rank, 0, 1.0, T * H).reshape(T, H)
    want, _, _ = orc.moe_prefill(L, x)
    return x, want


def _rank_main(rank, world, port, q):
    try:
        import torch.distributed as dist

        from oracle import oracle as orc
        from ramvamp_b200.ep import ExpertParallelMoe

        orc.build()
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        lay, blobs, router, norm = make_layer(orc)
        x, want = expected(orc, rank)
        ep = ExpertParallelMoe(OracleBackend(orc, lay, blobs, router, norm, rank, world), world, rank)
        res = torch.from_numpy(x.copy())
        ep.forward(0, res)
        ok = res.numpy().view(np.uint32).tobytes() == want.view(np.uint32).tobytes()
        q.put((rank, ok, ep.last_counts, ep.last_received))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # reported to the parent
        q.put((rank, repr(exc), None, None))


def test_ep_world1_equals_single_process(orc):
    lay, blobs, router, norm = make_layer(orc)
    from ramvamp_b200.ep import ExpertParallelMoe

    x, want = expected(orc, 0)
    ep = ExpertParallelMoe(OracleBackend(orc, lay, blobs, router, norm, 0, 1), 1, 0)
    res = torch.from_numpy(x.copy())
    ep.forward(0, res)
    assert res.numpy().view(np.uint32).tobytes() == want.view(np.uint32).tobytes()
    assert ep.last_counts == [T * K]


def test_ep_two_gloo_ranks_bit_identical():
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, counts, received in sorted(results, key=lambda r: r[0]):
        assert ok is True, f"rank {rank}: {ok}"
        assert sum(counts) == T * K
    # every pair sent was received somewhere
    sent = np.sum([r[2] for r in results], axis=0)
    assert sorted(r[3] for r in results) == sorted(sent.tolist())


def test_balanced_placement_spreads_hot_experts():
    """Experts in decreasing load go to the least-loaded rank with room:
    every rank holds n/world experts, the Zipf-skewed load ends near even,
    and the entries pass the library's placement check."""
    import math

    import ramvamp_b200 as rv
    from ramvamp_b200 import _lib
    from ramvamp_b200.ep import balanced_placement, placement_entries

    rng = np.random.default_rng(3)
    loads = [1.0 / (r + 1) ** 1.1 for r in rng.permutation(128)]
    for world in (1, 2, 4, 8):
        ranks = balanced_placement(loads, world)
        assert sorted(e for r in ranks for e in r) == list(range(128))
        assert all(len(r) == 128 // world for r in ranks)
        tot = [sum(loads[e] for e in r) for r in ranks]
        mean = sum(tot) / world
        # Near the floor set by the mean and by the hottest expert alone.
        assert max(tot) <= 1.25 * max(mean, max(loads))
        strided = [sum(loads[e] for e in range(r, 128, world)) for r in range(world)]
        assert max(tot) <= max(strided) + 1e-12
        entries = placement_entries(ranks)
        arr = (ctypes.c_uint32 * 128)(*entries)
        assert rv.lib().rv_ep_check_placement(128, world, arr, 128) == 0
    # The checker refuses a rank holding too many experts and duplicates.
    bad = [0] * 128  # every expert on rank 0, local 0
    arr = (ctypes.c_uint32 * 128)(*bad)
    assert rv.lib().rv_ep_check_placement(128, 2, arr, 128) != 0
    entries = placement_entries(balanced_placement(loads, 4))
    entries[5] = (9 << 16) | 0  # rank 9 of 4
    arr = (ctypes.c_uint32 * 128)(*entries)
    assert _lib.STATUS_NAMES[rv.lib().rv_ep_check_placement(128, 4, arr, 128)] == "RoutedExpertOutOfRange"
    assert not math.isnan(sum(loads))
