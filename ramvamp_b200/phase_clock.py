"""Phase timelines of the GPU MoE block (the GPU counterpart of the
reference's PhaseClock, model/prefill.rs:414-520).

Needs the instrumented build (`make -C ramvamp_b200/csrc phase`), in which
every kernel stamps %globaltimer (nanoseconds, common to all SMs) at its
phases; the normal build compiles the stamps out.

    python -m ramvamp_b200.phase_clock decode [layers]   # one decode layer, CTA phases
                                                         # (RV_DECODE_SPEC=0: without speculation)
    python -m ramvamp_b200.phase_clock tensor [tokens]   # tensor-path GEMM: per-CTA phases + one CTA's stages

Output: microseconds from the first stamp of the traced layer.
"""
from __future__ import annotations

import ctypes
import os
import sys

import numpy as np

from . import _lib

PHASE_LIB = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libramvamp_b200_phase.so")
CTAS, PHASES = 8192, 10
H, M, E, K = 2048, 768, 128, 8


def _open():
    if not os.path.exists(PHASE_LIB):
        raise ImportError(f"{PHASE_LIB} is missing: run make -C ramvamp_b200/csrc phase")
    _lib.LIB_PATH = PHASE_LIB
    import ramvamp_b200 as rv

    lib = rv.lib()
    lib.rv_debug_phase_clock.argtypes = [ctypes.c_int, ctypes.c_void_p]
    lib.rv_debug_phase_clock.restype = ctypes.c_int
    return rv, lib


def _read(lib, k):
    b = np.zeros((CTAS, PHASES), np.int64)
    lib.rv_debug_phase_clock(k, b.ctypes.data)
    return b


def _print_phases(name, b, t0, labels):
    used = b[:, 0] != 0
    print(f"{name}: {int(used.sum())} CTAs")
    for i, lab in enumerate(labels):
        if not lab:
            continue
        v = b[used, i]
        v = v[(v != 0) & (v >= t0) & (v < t0 + 10**7)]
        if v.size:
            d = (v - t0) / 1e3
            print(f"   {lab:16s} n={v.size:5d}  first {d.min():8.2f}  p50 {np.median(d):8.2f}  last {d.max():8.2f}")


def decode(n_layers: int = 4) -> None:
    """Phases of the last layer of an n-layer batch-1 decode graph."""
    import torch

    rv, lib = _open()
    table = rv.ExpertTable([rv.qwen3_layer_layout(l) for l in range(n_layers)], 0)
    for l in range(n_layers):
        table.fill_synthetic(l, 100 + l, 0.02)
    routers = [rv.synth_normal(200 + l, 0, 0.02, E * H).view(E, H).contiguous() for l in range(n_layers)]
    norm = torch.ones(H, device="cuda")
    eng = rv.MoeEngine(H, M, E, K, True, 1e-6, 1, 0)
    toks = rv.synth_normal(5, 0, 1.0, 16 * H).view(16, H)
    res = torch.empty(1, H, device="cuda")
    s = torch.cuda.Stream()

    def body():
        for l in range(n_layers):
            eng.forward(table, l, norm, routers[l], res)

    with torch.cuda.stream(s):
        res.copy_(toks[0:1])
        body()
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        body()
    for i in range(16):
        with torch.cuda.stream(s):
            res.copy_(toks[i:i + 1])
            g.replay()
    s.synchronize()
    bufs = [_read(lib, k) for k in range(6)]
    first = bufs[0][:, 0]
    t0 = first[first != 0].min()
    if os.environ.get("RV_DECODE_SPEC", "1") != "0":
        _print_phases("route (norm, bounds)", bufs[0], t0, ["start", "pdl_wait", "residual", "norm", "bounds",
                                                            "q8k", "norm:squares", "", "", "norm:inv"])
        _print_phases("exact chains", bufs[5], t0, ["start", "pdl_wait", "rows", "chain done", "LAST:start",
                                                    "LAST:routed", "LAST:index"])
    else:
        _print_phases("route", bufs[0], t0, ["start", "pdl_wait", "residual", "norm", "rows", "chain done",
                                             "LAST:start", "LAST:routed", "LAST:index"])
    b0 = bufs[0]
    used = (b0[:, 7] != 0) & (b0[:, 8] != 0) & (b0[:, 3] > b0[:, 2])
    if used.any():
        mhz = (b0[used, 8] - b0[used, 7]) / (b0[used, 3] - b0[used, 2]) * 1e3
        print(f"   SM clock during the norm (clock64 / globaltimer): p50 {np.median(mhz):.0f} MHz")
    _print_phases("gate_up", bufs[1], t0, ["start", "unit", "data", "compute", "LAST:quant", "row dots (thread 0)"])
    _print_phases("down", bufs[2], t0, ["start", "weights issued", "pdl_wait", "data", "compute", "LAST:combine"])
    tail = bufs[3][0]
    names = ["logits+max(warp)", "max(block)", "exp+sum(warp)", "sum(block)", "probs+finite", "rank", "sync",
             "weights"]
    print("routing tail (last CTA):")
    for i, n in enumerate(names):
        if tail[i]:
            print(f"   {n:16s} {(tail[i] - t0) / 1e3:8.2f}")


def tensor(tokens: int = 512) -> None:
    """Per-CTA phases of the two tensor-path GEMM kernels for one prefill
    layer, and the stage-by-stage events of one CTA of each."""
    import torch

    rv, lib = _open()
    table = rv.ExpertTable([rv.qwen3_layer_layout(0)], 0)
    table.fill_synthetic(0, 100, 0.02)
    router = rv.synth_normal(200, 0, 0.02, E * H).view(E, H).contiguous()
    norm = torch.ones(H, device="cuda")
    eng = rv.MoeEngine(H, M, E, K, True, 1e-6, tokens, 0)
    x = rv.synth_normal(5, 0, 1.0, tokens * H).view(tokens, H)
    for _ in range(3):
        r = x.clone()
        eng.forward(table, 0, norm, router, r, flags=rv.TENSOR)
    torch.cuda.synchronize()
    for k in range(5):
        _read(lib, k)
    r = x.clone()
    eng.forward(table, 0, norm, router, r, flags=rv.TENSOR)
    torch.cuda.synchronize()
    labels = ["start", "setup", "raw block 0", "first MMA", "last MMA", "first produced", "last produced",
              "first drained", "last drained", "end"]
    for k, name in ((1, "gate/up"), (2, "down")):
        b = _read(lib, k)
        used = b[:, 0] != 0
        v = b[used]
        t0 = v[:, 0].min()
        print(f"{name}: {int(used.sum())} CTAs, span {(v[:, 9].max() - t0) / 1e3:.1f} us; per CTA since its start:")
        rel = (v - v[:, :1]) / 1e3
        for i in range(1, PHASES):
            col = rel[:, i][v[:, i] != 0]
            if col.size:
                print(f"   {labels[i]:15s} p10 {np.percentile(col, 10):7.2f}  p50 {np.median(col):7.2f}  "
                      f"p90 {np.percentile(col, 90):7.2f}")
    ev = ["slot free", "produced", "A ready", "B ready", "committed", "B issued", "raw issued", "drained",
          "raw ready", "MMAs issued"]
    for k, name in ((3, "gate/up"), (4, "down")):
        b = _read(lib, k)
        rows = np.nonzero(b.max(1))[0]
        if rows.size == 0:
            continue
        t0 = b[rows][b[rows] > 0].min()
        print(f"{name} CTA 20, stage events (us):")
        for st in rows[:16]:
            print(f"  stage {st:2d}: " + "  ".join(f"{ev[i]} {(b[st, i] - t0) / 1e3:.2f}" for i in range(PHASES)
                                                    if b[st, i]))


if __name__ == "__main__":
    what = sys.argv[1] if len(sys.argv) > 1 else "decode"
    arg = int(sys.argv[2]) if len(sys.argv) > 2 else None
    if what == "decode":
        decode(arg or 4)
    elif what == "tensor":
        tensor(arg or 512)
    else:
        raise SystemExit(__doc__)
