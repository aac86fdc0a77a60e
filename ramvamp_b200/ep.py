"""Expert parallelism: joining a group, and a host-collective harness.

The product path is ``ramvamp_b200.ExpertParallel`` (rv_ep_* in the C ABI):
dispatch and combine run through GPU memory inside the library, with no host
synchronization.  ``connect_group`` below is its set-up over a
torch.distributed group (the handles are small host byte strings).

``ExpertParallelMoe`` is the same layer with the exchange written as
torch.distributed all-to-alls.  It is kept as the harness of the CPU tests,
which check the exchange logic on gloo ranks with the oracle as the local
compute.

The 128 experts of a layer are spread over the G ranks of a group by expert
id modulo G: rank r holds experts r, r+G, r+2G, ... as its local experts
0, 1, 2, ... (the strided map keeps the load of a Zipf-skewed router close
to even).  Each rank routes its own ("home") tokens, then per layer:

  1. route: RMSNorm, Q8_K, router, top-k, renormalization (exact);
  2. plan: the (token, slot) pairs laid out rank by rank (counting sort on
     the GPU), each with its expert's local id and its token's Q8_K row;
  3. exchange counts (all_to_all of G integers), then the local ids and
     the Q8_K rows (all-to-all-v);
  4. experts: every rank runs its local experts on the rows it received;
  5. the expert output rows go back (all-to-all-v) in the order they came;
  6. combine: w_k * out_k summed in top-k order per home token.

Every pair's expert output is computed by the same kernels on the same
Q8_K row as on one GPU and the reduction order is the same, so the result
is bit-identical for every group size (prefill.rs:2734-2778).

The collective steps are the same on every rank in the same order.  The
backend object supplies the local compute: EngineBackend runs the CUDA
kernels of this package; tests substitute a CPU backend to check the
exchange logic on gloo ranks.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch
import torch.distributed as dist

from . import EXACT, ExpertTable, MoeEngine


def connect_group(ep, group=None) -> None:
    """rv_ep_connect for every rank of `group` (None: the default group):
    all-gathers each rank's handle and connects.  Collective: every rank
    calls it, after creating its ExpertParallel."""
    handles = [None] * dist.get_world_size(group)
    dist.all_gather_object(handles, ep.handle_bytes(), group=group)
    ep.connect(handles)


def balanced_placement(loads: Sequence[float], world: int) -> List[List[int]]:
    """Experts per rank for one layer, n_experts / world each, evening out
    the measured loads (pairs routed to each expert): experts in decreasing
    load (ties: lower id first) go to the rank with the least load so far
    among those with room (ties: lower rank).  Returns per rank its global
    expert ids in local-id order."""
    n = len(loads)
    if n % world:
        raise ValueError(f"{n} experts do not split over {world} ranks")
    per = n // world
    order = sorted(range(n), key=lambda e: (-float(loads[e]), e))
    ranks: List[List[int]] = [[] for _ in range(world)]
    total = [0.0] * world
    for e in order:
        r = min((r for r in range(world) if len(ranks[r]) < per), key=lambda r: (total[r], r))
        ranks[r].append(e)
        total[r] += float(loads[e])
    return ranks


def placement_entries(ranks: Sequence[Sequence[int]]) -> List[int]:
    """rank << 16 | local id per global expert (rv_moe_ep_forward's map)."""
    n = sum(len(r) for r in ranks)
    out = [0] * n
    for r, experts in enumerate(ranks):
        for local, e in enumerate(experts):
            out[e] = (r << 16) | local
    return out


def placement_tensor(ranks: Sequence[Sequence[int]], device) -> torch.Tensor:
    """The device map of a placement, checked by rv_ep_check_placement."""
    import ctypes

    from . import _lib

    entries = placement_entries(ranks)
    arr = (ctypes.c_uint32 * len(entries))(*entries)
    _lib.check(_lib.load().rv_ep_check_placement(len(entries), len(ranks), arr, len(entries)))
    return torch.tensor(entries, dtype=torch.int32, device=device)


def expert_owner(expert: int, world: int) -> int:
    """Rank holding global expert `expert`."""
    return expert % world


def local_experts(rank: int, world: int, n_experts: int) -> List[int]:
    """Global ids of the experts rank `rank` holds, in local-id order."""
    return list(range(rank, n_experts, world))


class EngineBackend:
    """Local compute of one rank on its GPU: routing for the home tokens
    and the experts this rank holds (`table` has only those, in local-id
    order)."""

    def __init__(self, engine: MoeEngine, table: ExpertTable, ffn_norms: Sequence[torch.Tensor],
                 routers: Sequence[torch.Tensor], flags: int = EXACT):
        self.engine, self.table, self.flags = engine, table, flags
        self.ffn_norms, self.routers = ffn_norms, routers

    @property
    def hidden(self) -> int:
        return self.engine.cfg.hidden

    @property
    def act_stride(self) -> int:
        return self.engine.act_stride

    def route(self, layer: int, residual: torch.Tensor):
        return self.engine.route(self.ffn_norms[layer], self.routers[layer], residual)

    def plan(self, topk_ids: torch.Tensor, acts: torch.Tensor, world: int):
        return self.engine.ep_plan(topk_ids, acts, world)

    def experts(self, layer: int, local_ids: torch.Tensor, acts: torch.Tensor) -> torch.Tensor:
        return self.engine.experts(self.table, layer, local_ids, acts, self.flags)

    def combine(self, residual: torch.Tensor, topk_weights: torch.Tensor, expert_out: torch.Tensor,
                pos_of: torch.Tensor) -> torch.Tensor:
        return self.engine.combine(residual, topk_weights, expert_out, pos_of)


class ExpertParallelMoe:
    """The MoE block of a layer with experts sharded over a process group.

    world == 1 (or no process group) runs the same steps without the
    exchange.  `group` is a torch.distributed group (None: the default
    group); NCCL for CUDA tensors, gloo for CPU tensors."""

    def __init__(self, backend, world: int = 1, rank: int = 0, group=None):
        self.backend, self.world, self.rank, self.group = backend, world, rank, group
        self.last_counts: Optional[List[int]] = None  # pairs sent to each rank by the last forward
        self.last_received: int = 0                   # pairs this rank's experts ran in the last forward

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits: List[int], in_splits: List[int]) -> None:
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def forward(self, layer: int, residual: torch.Tensor) -> torch.Tensor:
        """In place: residual (this rank's home tokens, [T, hidden]) +=
        MoE(residual)."""
        b = self.backend
        ids, w, acts = b.route(layer, residual)
        counts, pos_of, send_local, send_acts = b.plan(ids, acts, self.world)
        send = [int(c) for c in counts.tolist()]
        self.last_counts = send
        if self.world == 1:
            out = b.experts(layer, send_local, send_acts)
            self.last_received = send[0]
            return b.combine(residual, w, out, pos_of)
        counts64 = counts.to(torch.int64)
        recv_counts = torch.empty_like(counts64)
        self._a2a(recv_counts, counts64, [1] * self.world, [1] * self.world)
        recv = [int(c) for c in recv_counts.tolist()]
        n_recv = sum(recv)
        self.last_received = n_recv
        recv_local = torch.empty(n_recv, dtype=send_local.dtype, device=send_local.device)
        self._a2a(recv_local, send_local, recv, send)
        recv_acts = torch.empty(n_recv, send_acts.shape[1], dtype=send_acts.dtype, device=send_acts.device)
        self._a2a(recv_acts, send_acts, recv, send)
        out = b.experts(layer, recv_local, recv_acts)
        back = torch.empty(sum(send), b.hidden, dtype=out.dtype, device=out.device)
        self._a2a(back, out, send, recv)
        return b.combine(residual, w, back, pos_of)
