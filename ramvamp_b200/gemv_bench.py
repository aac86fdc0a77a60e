"""Throughput of the dense-layer GEMVs of one Qwen3-30B-A3B decode step
(model/shapes.rs:14-35), each timed alone on one GPU:

    python -m ramvamp_b200.gemv_bench [--iters N]

attn_q Q4_K 4096x2048, attn_k Q8_0 512x2048 (with its Q8_0 quantizer),
attn_v Q6_K 512x2048, attn_output Q5_K 2048x4096, lm_head Q6_K
151936x2048, and one token's Q4_K embedding row.  Every launch is preceded
by a read of a buffer larger than L2 (which leaves only clean lines there:
a write would leave up to 126 MB of dirty lines whose write-back lands in
the timed launch) and timed with CUDA events on the launching stream; the
line per shape gives the median launch time, the
algorithmic bytes (weights + activations + output) and the HBM roofline
fraction against the measured copy bandwidth.  Weights are synthetic
(seeded normal values through the reference's quantizers).
"""
from __future__ import annotations

import argparse
import json
import os

import torch

import ramvamp_b200 as rv

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
Q = rv.QuantFormat


def hbm_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def time_launches(fn, iters, flush):
    """Median and best launch time in us, L2 flushed before each launch."""
    s = torch.cuda.current_stream()
    for _ in range(3):
        fn()
    ts = []
    for _ in range(iters):
        flush.sum()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(s)
        fn()
        b.record(s)
        b.synchronize()
        ts.append(a.elapsed_time(b) * 1e3)
    ts.sort()
    return ts[len(ts) // 2], ts[0]


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--only", default=None, help="time only the shapes whose name starts with this")
    args = ap.parse_args(argv)
    torch.cuda.init()
    flush = torch.zeros(64 << 20, dtype=torch.float32, device="cuda")
    peak, kind = hbm_peak()
    hidden, vocab = 2048, 151936
    x = rv.synth_normal(7, 0, 1.0, 4096)
    acts_k = {n: rv.quantize_row_q8_k(x[:n]) for n in (2048, 4096)}
    rows = []

    def kquant(name, fmt, out_dim, in_dim):
        w = rv.quantize_weights(fmt, rv.synth_normal(11, 0, 0.02, out_dim * in_dim))
        out = torch.empty(out_dim, dtype=torch.float32, device="cuda")
        a = acts_k[in_dim]
        fn = lambda: rv.gemv_q8_k(fmt, w, in_dim, out_dim, a, out)
        rows.append((name, fn, w.numel() + a.numel() + 4 * out_dim))

    kquant("attn_q Q4_K 4096x2048", Q.Q4_K, 4096, hidden)
    # attn_k: Q8_0 weights from the Q8_0 quantizer's blocks (f32 d -> f16 d).
    blocks = rv.quantize_row_q8_0(rv.synth_normal(12, 0, 0.02, 512 * hidden)).view(-1, 36)
    d16 = blocks[:, :4].contiguous().view(torch.float32).half().view(torch.uint8)
    wk = torch.cat([d16, blocks[:, 4:]], dim=1).contiguous().view(-1)
    outk = torch.empty(512, dtype=torch.float32, device="cuda")
    xk = x[:hidden]
    ak = rv.quantize_row_q8_0(xk)
    rows.append(("attn_k Q8_0 512x2048", lambda: rv.gemv_q8_0(wk, hidden, 512, ak, outk),
                 wk.numel() + ak.numel() + 4 * 512))
    rows.append(("attn_k Q8_0 quantize + GEMV", lambda: rv.gemv_q8_0(wk, hidden, 512, rv.quantize_row_q8_0(xk, ak), outk),
                 wk.numel() + 4 * hidden + 2 * ak.numel() + 4 * 512))
    kquant("attn_v Q6_K 512x2048", Q.Q6_K, 512, hidden)
    kquant("attn_output Q5_K 2048x4096", Q.Q5_K, hidden, 4096)
    kquant("lm_head Q6_K 151936x2048", Q.Q6_K, vocab, hidden)
    table = rv.quantize_weights(Q.Q4_K, rv.synth_normal(13, 0, 0.5, vocab * hidden))
    tok = torch.tensor([123456], dtype=torch.int32, device="cuda")
    emb = torch.empty(hidden, dtype=torch.float32, device="cuda")
    rows.append(("embed Q4_K 1 token", lambda: rv.embed(table, hidden, vocab, tok, out=emb),
                 hidden // 256 * 144 + 4 + 4 * hidden))
    torch.cuda.synchronize()
    print(f"peak {peak:.0f} GB/s ({kind}); a 256 MB read before every launch; {args.iters} launches each")
    for name, fn, nbytes in rows:
        if args.only and not name.startswith(args.only):
            continue
        med, best = time_launches(fn, args.iters, flush)
        gbs = nbytes / (med * 1e-6) / 1e9
        print(f"{name:32s} {nbytes / 1e6:9.3f} MB  median {med:8.2f} us  best {best:8.2f} us  "
              f"{gbs:8.1f} GB/s  {gbs / peak:6.3f} of {kind}")
    rv.device_status(0)


if __name__ == "__main__":
    main()
