#!/usr/bin/env python3
"""Benchmark of the B200 routed-expert FFN (ramvamp's MoE block).

Default workload (expert-FFN half): batch-1 greedy decode
of Qwen3-30B-A3B through all 48 MoE layers with every expert resident in HBM
(17.5 GB of Q4_K/Q6_K blobs).  A step is one token through the 48 MoE
blocks (RMSNorm, router, top-8, Q8_K, gate/up/SwiGLU/down, combine); the
attention half of the model is not part of this path.  Each step decodes a
different seeded token, and a step streams 1.1 GB of expert weights, far
more than the 126 MB L2, so nothing is served from L2 between steps.

Arms:
  default            the CUDA path (one CUDA graph per step, replayed)
  --impl reference   the reference's CPU algorithm (the C oracle restating
                     ramvamp's AVX2 path) on this host's cores, on a bounded
                     sample of layers, scaled to 48 layers

Prints one JSON line (rank 0).  On one GPU the line also carries config 4
at N=1 ("ep_prefill", the base point of the multi-GPU curve), config 2
("prefill", with the tensor-pipe fraction of its gate/up stage), config 3
("batch": 64 Zipf-skewed sequences through 48 MoE layers) and the whole
model of config 1 ("model": attention, MoE and lm_head, greedy decode
after a 512-token prompt), each measured in the same run.

Multi-GPU (torchrun, N>1): batch-1 decode does not shard, so the default
workload there is config 4, expert-parallel prefill of 4096 tokens through
48 MoE layers with the 128 experts spread over the N GPUs and the exchange
done by the library through GPU memory (rv_moe_ep_forward); strong scaling,
timed as the max over ranks.  `--workload decode` under torchrun runs
independent decode replicas instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, M, E, K, LAYERS = 2048, 768, 128, 8, 48
SEED = 20261201
METRIC = "decode tok/s (expert FFN, 48 MoE layers, batch 1)"


WORKLOADS = ("decode", "prefill", "batch", "ep", "model")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--impl", choices=["cuda", "reference"], default="cuda")
    ap.add_argument("--workload", choices=WORKLOADS, default=None,
                    help="decode: config 1's expert FFN (the default on one GPU); prefill: config 2; batch: "
                         "config 3; ep: config 4 (the default under torchrun with N > 1); model: config 1 "
                         "whole model (attention + MoE + lm_head, greedy)")
    ap.add_argument("--no-extras", action="store_true",
                    help="decode: skip the config-4 (N=1) and config-2 measurements added to the line")
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--exact", action="store_true", help="prefill/batch/ep: the exact (AVX2-order) path")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    a = ap.parse_args()
    if a.workload is None:
        a.workload = "ep" if int(os.environ.get("WORLD_SIZE", "1")) > 1 else "decode"
    steps, warmup = {"decode": (30, 5), "prefill": (20, 5), "batch": (10, 3), "ep": (10, 3),
                     "model": (64, 3)}[a.workload]
    a.steps = steps if a.steps is None else a.steps
    a.warmup = warmup if a.warmup is None else a.warmup
    return a


def layouts(rv, n_layers):
    return [rv.qwen3_layer_layout(l) for l in range(n_layers)]


def expert_bytes_per_token(lays):
    return sum(K * (L.gate_len + L.up_len + L.down_len) for L in lays)


# ------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples during the timed region (read-only queries)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.idx = gpu_id
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def start(self, wait_s: float = 10.0):
        """Starts sampling and returns once the first sample is written (so
        a short timed region right after still gets samples)."""
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.proc = None
            return
        t0 = time.time()
        while time.time() - t0 < wait_s and self.proc.poll() is None:
            if os.path.getsize(self.file.name) > 0:
                break
            time.sleep(0.05)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.file.read().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        os.unlink(self.file.name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "samples": len(sm), "reasons": sorted(reasons)}


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def measured_tensor_peak():
    """Dense bf16 TFLOP/s (burst, kernel timed alone); f16 runs at the same rate."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def ncu_traffic(kernel: str):
    """DRAM bytes per launch from the committed ncu summary, if one exists."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        return json.load(f).get(kernel)


# ------------------------------------------------------- CPU baseline
def cpu_baseline_sample(orc, lays, blobs_by_layer, routers, norm, tokens, threads):
    """The oracle (AVX2 restatement of the reference) on a sample of layers:
    returns seconds per token scaled to len(lays) layers."""
    sample_layers = sorted(blobs_by_layer)
    oracle_layers = {}
    for l in sample_layers:
        L = lays[l]
        oracle_layers[l] = orc.make_layer(H, M, E, K, 1e-6, norm, routers[l], blobs_by_layer[l], L.stride,
                                          L.gate_off, L.up_off, L.down_off, L.gate_format, L.up_format,
                                          L.down_format)
    x = tokens[:1].copy()
    for l in sample_layers:  # warm-up
        x, _, _, _ = orc.moe_decode(oracle_layers[l], x, threads=threads)
    t0 = time.perf_counter()
    n_tok = 0
    while True:
        for i in range(tokens.shape[0]):
            x = tokens[i:i + 1].copy()
            for l in sample_layers:
                x, _, _, _ = orc.moe_decode(oracle_layers[l], x, threads=threads)
            n_tok += 1
        if time.perf_counter() - t0 > 10.0 or n_tok >= 64:
            break
    dt = time.perf_counter() - t0
    return dt / n_tok * len(lays) / len(sample_layers), n_tok, sample_layers


# ----------------------------------------------------------- CUDA arm
def run_cuda(args):
    import torch
    import torch.distributed as dist

    import ramvamp_b200 as rv

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", init_method="env://", timeout=__import__("datetime").timedelta(seconds=120))
    dev = local if world > 1 else 0
    torch.cuda.set_device(dev)
    n_layers = args.layers
    lays = layouts(rv, n_layers)
    table = rv.ExpertTable(lays, device=dev)
    for l in range(n_layers):
        table.fill_synthetic(l, SEED + l, 0.02)
    routers = [rv.synth_normal(SEED + 1000 + l, 0, 0.02, E * H).view(E, H).contiguous() for l in range(n_layers)]
    norm = torch.ones(H, dtype=torch.float32, device="cuda")
    eng = rv.MoeEngine(H, M, E, K, True, 1e-6, max_tokens=1, device=dev)
    n_steps = args.warmup + args.steps
    tokens = rv.synth_normal(SEED + 7 + rank, 0, 1.0, n_steps * H).view(n_steps, H).contiguous()
    resid = torch.empty(1, H, dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()

    def step_body():
        for l in range(n_layers):
            eng.forward(table, l, norm, routers[l], resid)

    # Capture one decode step (48 MoE blocks) into a CUDA graph.
    with torch.cuda.stream(stream):
        resid.copy_(tokens[0:1])
        step_body()  # eager run: also initializes everything
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step_body()
    torch.cuda.synchronize()

    # Parity spot-check of the graph against the eager path on token 0.
    with torch.cuda.stream(stream):
        resid.copy_(tokens[0:1])
        graph.replay()
        g_out = resid.clone()
        resid.copy_(tokens[0:1])
        step_body()
    stream.synchronize()
    assert torch.equal(g_out, resid), "graph replay differs from eager forward"

    def run_steps(lo, hi):
        with torch.cuda.stream(stream):
            for i in range(lo, hi):
                resid.copy_(tokens[i:i + 1])
                graph.replay()

    stream.synchronize()
    if world > 1:
        dist.barrier()
    props = torch.cuda.get_device_properties(dev)
    uuid = str(getattr(props, "uuid", ""))
    clocks = ClockSampler(("GPU-" + uuid if uuid and not uuid.startswith("GPU-") else uuid) or str(dev))
    clocks.start()
    time.sleep(0.3)
    run_steps(0, args.warmup)  # warm-up right before the timed steps
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev0.record(stream)
    run_steps(args.warmup, n_steps)
    ev1.record(stream)
    ev1.synchronize()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    ms_per_step = ms / args.steps
    tok_s = world * args.steps / (ms / 1e3)

    # Per-kernel durations, measured with events baked into a profiling graph
    # (back-to-back launches, no host gaps), over the same steps.
    eng.profile_enable(n_layers)
    pgraph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        eng.profile_rewind()
        resid.copy_(tokens[0:1])
    stream.synchronize()
    with torch.cuda.graph(pgraph, stream=stream):
        step_body()
    stage = []
    for i in range(args.warmup, n_steps):
        with torch.cuda.stream(stream):
            resid.copy_(tokens[i:i + 1])
            pgraph.replay()
        stream.synchronize()
        stage.append(eng.profile_read())
    stage = np.stack(stage)  # [steps][layers][4]
    gu_ms = float(stage[:, :, 1].mean())
    dn_ms = float(stage[:, :, 2].mean())
    route_ms = float(stage[:, :, 0].mean())
    comb_ms = float(stage[:, :, 3].mean())
    del pgraph

    gu_bytes = K * (lays[0].gate_len + lays[0].up_len)  # same for every layer
    peak, peak_kind = measured_peaks()
    achieved = gu_bytes / (gu_ms * 1e-3) / 1e9
    tb = ncu_traffic("k_gate_up")

    # e2e through the public C-ABI calls, host buffers in and out every step.
    # (1) A caller that owns the decode step: the token's row from pinned
    # host memory, 48 rv_moe_forward calls (eager, one per layer) on the
    # device residual, the result back to pinned host memory, one
    # synchronization per token.  (2) A caller that holds each layer's
    # residual on the host: rv_moe_forward_host per layer (a copy in, a copy
    # out and a synchronization per layer).
    import torch as _t
    host_tok = _t.empty(n_steps, H, dtype=_t.float32).pin_memory()
    host_tok.copy_(tokens.cpu())
    hres = _t.empty(1, H, dtype=_t.float32).pin_memory()

    def e2e_step(i):
        with torch.cuda.stream(stream):
            resid.copy_(host_tok[i:i + 1], non_blocking=True)
            step_body()
            hres.copy_(resid, non_blocking=True)
        stream.synchronize()

    def e2e_step_host(i):
        hres.copy_(host_tok[i:i + 1])
        for l in range(n_layers):
            eng.forward_host(table, l, norm, routers[l], hres)

    def timed(fn):
        for i in range(min(3, args.warmup)):
            fn(i)
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for i in range(args.warmup, n_steps):
            fn(i)
        dt = time.perf_counter() - t0
        if world > 1:
            t = torch.tensor([dt], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dt = float(t.item())
        return world * args.steps / dt

    e2e_tok_s = timed(e2e_step)
    e2e_host_tok_s = timed(e2e_step_host)

    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        from oracle import oracle as orc
        orc.build()
        sample = [0, 6] if n_layers > 6 else [0]
        blobs = {l: rv.alias(table.view(l, 0).blob, E * lays[l].stride).cpu().numpy() for l in sample}
        rnp = {l: routers[l].cpu().numpy() for l in sample}
        threads = os.cpu_count() or 1
        s_per_tok, n_tok, used = cpu_baseline_sample(orc, lays, blobs, rnp, norm.cpu().numpy(),
                                                     tokens[:8].cpu().numpy(), threads)
        cpu = {"value": round(1.0 / s_per_tok, 3), "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"{n_tok} tokens through layers {used} (one Q6_K-down, one Q4_K-down) on the "
                         f"C oracle's AVX2 arm, time scaled to {n_layers} layers"}

    extras = {}
    if world == 1 and not args.no_extras:
        import copy

        a4 = copy.copy(args)
        a4.workload, a4.steps, a4.warmup, a4.exact = "ep", 10, 3, False
        l4 = run_ep(a4, table=table, quiet=True)
        extras["ep_prefill"] = {k: l4[k] for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup",
                                                   "ms_per_step", "scaling", "parity", "load", "roofline", "e2e",
                                                   "gpu_launches")}
        extras["ep_prefill"]["note"] = ("config 4 at N=1 through the same exchange code (one rank); the N>1 "
                                        "points are the torchrun lines of the same metric")
        a2 = copy.copy(args)
        a2.workload, a2.steps, a2.warmup, a2.exact, a2.no_cpu_baseline = "prefill", 20, 5, False, True
        l2 = run_cuda_batched(a2, quiet=True)
        extras["prefill"] = {k: l2.get(k) for k in ("metric", "value", "unit", "ms_per_step", "stage_ms_per_layer",
                                                    "tensor", "roofline", "e2e")}
        extras["prefill"]["config"] = l2["config"]["workload"]
        a3 = copy.copy(args)
        a3.workload, a3.steps, a3.warmup, a3.exact, a3.no_cpu_baseline = "batch", 10, 3, False, True
        l3 = run_cuda_batched(a3, quiet=True, table=table)
        extras["batch"] = {k: l3.get(k) for k in ("metric", "value", "unit", "ms_per_step", "tensor", "e2e")}
        extras["batch"]["config"] = l3["config"]["workload"]
        a1 = copy.copy(args)
        a1.workload, a1.steps, a1.warmup, a1.no_cpu_baseline = "model", 64, 3, True
        l1 = run_cuda_model(a1, quiet=True)
        extras["model"] = {k: l1[k] for k in ("metric", "value", "unit", "ms_per_step", "prompt_tok_s", "e2e",
                                              "roofline", "generated_ids_head")}
        extras["model"]["config"] = l1["config"]["workload"]

    if rank == 0:
        step_bytes = expert_bytes_per_token(lays)
        line = {
            "metric": METRIC, "value": round(tok_s, 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 (dp4a) + f32",
            "data": "synthetic: seeded N(0,1) tokens, N(0,0.02) router and expert weights quantized by the "
                    "reference's Q4_K/Q6_K quantizers",
            "config": {"workload": f"config1 expert FFN: batch-1 decode through {n_layers} MoE layers of "
                                   "Qwen3-30B-A3B (hidden 2048, moe 768, 128 experts, top-8), all experts "
                                   "resident in HBM",
                       "layers": n_layers, "tokens_per_step": 1, "router": "exact (serial f32 chains)",
                       "numerics": "bit-identical to the reference AVX2 path",
                       "l2": "inputs larger than L2: each step streams %.2f GB of expert weights" % (step_bytes / 1e9),
                       "parallelism": "replicas" if world > 1 else "single GPU", "cuda_graph": True},
            "expert_hbm_gbs": round(step_bytes / (ms_per_step * 1e-3) / 1e9, 1),
            "stage_ms_per_layer": {"routing": round(route_ms, 5), "gate_up": round(gu_ms, 5),
                                   "down": round(dn_ms, 5), "combine": round(comb_ms, 5)},
            "roofline": {"kernel": "k_gate_up", "bound": "hbm", "achieved": round(achieved, 1),
                         "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_source": f"{peak_kind} hbm_gbs", "bytes_per_launch": gu_bytes,
                         "traffic": tb},
            "e2e": {"value": round(e2e_tok_s, 2), "unit": "tok/s",
                    "h2d_bytes_per_step": H * 4, "d2h_bytes_per_step": H * 4,
                    "path": "per token: pinned host row in, 48 rv_moe_forward calls (eager) on the device "
                            "residual, row out, one synchronization"},
            "e2e_per_layer_host": {"value": round(e2e_host_tok_s, 2), "unit": "tok/s",
                                   "h2d_bytes_per_step": n_layers * H * 4, "d2h_bytes_per_step": n_layers * H * 4,
                                   "path": "rv_moe_forward_host per layer (pinned host residual in, result out, "
                                           "a synchronization per layer)"},
            # per layer: k_route_spec, k_route_chain, k_gate_up, k_down (the speculative pipeline)
            "gpu_launches": args.steps * n_layers * 4,
            "clocks": clk,
            "cpu_baseline": cpu,
        }
        line.update(extras)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        del graph
        dist.destroy_process_group()


# ------------------------------------------------------- reference arm
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle as orc
    from oracle.layout import layer_layout

    orc.build()
    n_layers = args.layers
    lays = [layer_layout(l) for l in range(n_layers)]
    threads = os.cpu_count() or 1
    sample = [0, 6] if n_layers > 6 else [0]
    blobs = {l: orc.fill_layer_synthetic(lays[l], SEED + l, 0.02, threads) for l in sample}
    routers = {l: orc.synth_normal(SEED + 1000 + l, 0, 0.02, E * H).reshape(E, H) for l in sample}
    norm = np.ones(H, np.float32)
    n_steps = args.warmup + args.steps
    tokens = orc.synth_normal(SEED + 7, 0, 1.0, n_steps * H).reshape(n_steps, H)
    oracle_layers = {l: orc.make_layer(H, M, E, K, 1e-6, norm, routers[l], blobs[l], lays[l].stride,
                                       lays[l].gate_off, lays[l].up_off, lays[l].down_off,
                                       lays[l].gate_format, lays[l].up_format, lays[l].down_format)
                     for l in sample}

    def step(i):
        x = tokens[i:i + 1].copy()
        for l in sample:
            x, _, _, _ = orc.moe_decode(oracle_layers[l], x, threads=threads)

    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    for i in range(args.warmup, n_steps):
        step(i)
    dt = time.perf_counter() - t0
    s_per_tok = dt / args.steps * n_layers / len(sample)
    v = 1.0 / s_per_tok
    sample_desc = (f"each step: one token through layers {sample} (one Q6_K-down, one Q4_K-down) on the C "
                   f"oracle's AVX2 arm with {threads} threads, time scaled to {n_layers} layers")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(s_per_tok * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 + f32",
        "data": "synthetic (same seeds and weights as the CUDA arm)",
        "config": {"workload": f"config1 expert FFN: batch-1 decode through {n_layers} MoE layers of "
                               "Qwen3-30B-A3B (sampled layers, scaled)", "layers": n_layers,
                   "tokens_per_step": 1},
        "cpu_baseline": {"value": round(v, 3), "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": sample_desc},
        "e2e": {"value": round(v, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ================================================ config 1, whole model
# Qwen3-30B-A3B, 48 layers, random-init weights through the reference's
# quantizers; a 512-token prompt of seeded uniform-random ids, then greedy
# decoding.  A step is one token through the whole model (embedding, 48 x
# (attention half + MoE block), final norm, lm_head, argmax), replayed from
# one captured CUDA graph with the token, position and sampled id in device
# memory.  W untimed generated tokens after the prompt, then K timed.
MODEL_PROMPT = 512
MODEL_SEED = SEED % 1000 + 1
MODEL_METRIC = "decode tok/s (whole model, greedy, batch 1, after a 512-token prompt)"


def model_launches_per_step(n_layers):
    # embedding; per layer: attn_norm, Q8_K, Q8_0, q/k/v GEMVs, attention
    # (prep, scores, softmax+out), Q8_K, attn_output, residual add, MoE (4);
    # final norm, Q8_K, lm_head, argmax, advance
    return 1 + n_layers * 17 + 5


def run_cuda_model(args, quiet=False):
    import torch
    import torch.distributed as dist

    import ramvamp_b200 as rv
    from ramvamp_b200.model import Decoder, ModelConfig, Qwen3Weights

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", init_method="env://", timeout=__import__("datetime").timedelta(seconds=300))
    dev = local if world > 1 else 0
    torch.cuda.set_device(dev)
    cfg = ModelConfig(n_layers=args.layers)
    w = Qwen3Weights.synthetic(cfg, seed=MODEL_SEED, device=dev)
    n_gen = args.warmup + args.steps
    e2e_steps = min(args.steps, 16)
    # room for the prompt, the warm-up and timed tokens and the e2e tokens
    dec = Decoder(w, max_positions=MODEL_PROMPT + n_gen + e2e_steps + 1, device=dev)
    dec.capture()
    prompt = np.random.default_rng(SEED + rank).integers(0, cfg.vocab, MODEL_PROMPT).astype(np.int32)
    prompt_d = torch.from_numpy(prompt).cuda()
    stream = torch.cuda.current_stream()
    dec.reset()
    dec.token.copy_(prompt_d[:1])
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    ev[0].record(stream)
    for i in range(MODEL_PROMPT):
        dec.step()
        if i + 1 < MODEL_PROMPT:
            dec.token.copy_(prompt_d[i + 1:i + 2])
    ev[1].record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    props = torch.cuda.get_device_properties(dev)
    uuid = str(getattr(props, "uuid", ""))
    clocks = ClockSampler(("GPU-" + uuid if uuid and not uuid.startswith("GPU-") else uuid) or str(dev))
    clocks.start()
    time.sleep(0.3)
    # warm-up right before the timed steps, so the GPU is not coming out of
    # the idle pause above
    for _ in range(args.warmup):
        dec.step()
    torch.cuda.synchronize()
    ev[2].record(stream)
    for _ in range(args.steps):
        dec.step()
    ev[3].record(stream)
    ev[3].synchronize()
    clk = clocks.stop()
    ms = ev[2].elapsed_time(ev[3])
    prompt_ms = ev[0].elapsed_time(ev[1])
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ids = dec.ids[MODEL_PROMPT - 1:MODEL_PROMPT - 1 + n_gen].cpu().numpy().tolist()
    rv.device_status(dev)

    # lm_head roofline, live: the same GEMV launched alone after a clean
    # (read) L2 flush, CUDA events on its stream.
    flush = torch.zeros(64 << 20, dtype=torch.float32, device="cuda")
    lm_ms = []
    for i in range(12):
        flush.sum()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        rv.gemv_q8_k(rv.QuantFormat.Q6_K, w.lm_head, cfg.hidden, cfg.vocab, dec.acts_k, dec.logits)
        b.record(stream)
        b.synchronize()
        if i >= 2:
            lm_ms.append(a.elapsed_time(b))
    lm_ms = statistics.median(lm_ms)
    lm_bytes = w.lm_head.numel()
    peak, peak_kind = measured_peaks()
    achieved = lm_bytes / (lm_ms * 1e-3) / 1e9
    del flush

    # e2e: a host-driven loop through the public API: each token's id goes
    # in from pinned host memory (4 B) and the sampled id comes back (4 B).
    # The cache continues from the timed run, so positions stay in range.
    tok_h = torch.zeros(1, dtype=torch.int32).pin_memory()
    out_h = torch.zeros(1, dtype=torch.int32).pin_memory()
    tok_h[0] = ids[-1]
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        dec.token.copy_(tok_h, non_blocking=True)
        dec.step()
        out_h.copy_(dec.next_token, non_blocking=True)
        stream.synchronize()
        tok_h[0] = out_h[0]
    e2e_s = time.perf_counter() - t0
    rv.device_status(dev)  # every step stayed inside the cache
    if world > 1:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())

    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        cpu = model_cpu_baseline(cfg)
    if rank == 0:
        line = {
            "metric": MODEL_METRIC, "value": round(world * args.steps / (ms / 1e3), 2), "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 (dp4a) + f32 + f16 KV",
            "data": "synthetic: random-init weights (seeded N(0,0.02), embedding N(0,1)) through the reference's "
                    "quantizers (Q4_K/Q8_0/Q6_K/Q5_K as Q4_K_M), 512 seeded uniform-random prompt ids",
            "config": {"workload": f"config1 whole model: Qwen3-30B-A3B ({cfg.n_layers} layers, 32/4 heads, "
                                   "head_dim 128, 128 experts top-8, vocab 151936), batch-1 greedy decode after "
                                   "a 512-token prompt, all weights resident in HBM",
                       "layers": cfg.n_layers, "prompt": MODEL_PROMPT, "generated": n_gen,
                       "numerics": "bit-identical to the reference's step (f64 exp caveat)",
                       "l2": "inputs larger than L2: each step reads ~1.9 GB of weights",
                       "parallelism": "replicas" if world > 1 else "single GPU", "cuda_graph": True},
            "prompt_tok_s": round(MODEL_PROMPT / (prompt_ms / 1e3), 2),
            "generated_ids_head": ids[:8],
            "roofline": {"kernel": "k_gemv_lm_head", "bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4), "peak_source": f"{peak_kind} hbm_gbs",
                         "bytes_per_launch": lm_bytes, "traffic": ncu_traffic("k_gemv_lm_head")},
            "e2e": {"value": round(world * e2e_steps / e2e_s, 2), "unit": "tok/s", "h2d_bytes_per_step": 4,
                    "d2h_bytes_per_step": 4, "path": "Decoder.step with the token id from pinned host memory "
                                                     "and the sampled id read back, one sync per token"},
            "gpu_launches": args.steps * model_launches_per_step(cfg.n_layers),
            "clocks": clk,
            "cpu_baseline": cpu,
        }
        if not quiet:
            print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return line if rank == 0 else None


def model_cpu_baseline(cfg, sample_layers=(0, 6), positions=64):
    """The reference's step on this host's cores (C oracle), bounded: one
    token at position `positions` through two sampled layers (a Q6_K and a
    Q4_K layer) plus the lm_head, scaled to all layers.  The weights are the
    CUDA arm's (same seeds through the CPU restatement of the generator and
    quantizers)."""
    from oracle import oracle as orc
    from oracle.model_ref import RefModel, synthetic_host

    orc.build()
    threads = os.cpu_count() or 1
    layers = [l for l in sample_layers if l < cfg.n_layers]
    weights, moe = synthetic_host(cfg, MODEL_SEED, layers, threads)
    import dataclasses

    sub = dataclasses.replace(cfg, n_layers=len(layers))
    impl = orc.default_impl()  # the arm the reference dispatches to on this host
    ref = RefModel(sub, weights, moe, positions + 2, threads, impl=impl)
    for p in range(positions):  # fill the caches (untimed)
        ref.step(p % cfg.vocab, p)
    t0 = time.perf_counter()
    ref.step(7, positions)
    t1 = time.perf_counter()
    # lm_head alone, to split the fixed part from the per-layer part
    normed = orc.rmsnorm(np.ones(cfg.hidden, np.float32), weights["output_norm"], cfg.eps)
    t2 = time.perf_counter()
    orc.gemv(orc.Q6_K, weights["lm_head"], cfg.hidden, cfg.vocab, orc.quantize_row_q8_k(normed), impl=impl,
             threads=threads)
    t3 = time.perf_counter()
    per_layer = max((t1 - t0) - (t3 - t2), 0.0) / len(layers)
    s_tok = per_layer * cfg.n_layers + (t3 - t2)
    return {"value": round(1.0 / s_tok, 3), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"one token at position {positions} through layers {layers} and the lm_head on the C "
                      f"oracle ({'AVX2' if impl == orc.AVX2 else 'scalar'} arm, {threads} threads), per-layer "
                      f"time scaled to {cfg.n_layers} layers"}


def run_reference_model(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle.layout import ModelShape

    cfg = ModelShape(n_layers=args.layers)
    cpu = model_cpu_baseline(cfg)
    line = {
        "impl": "reference", "metric": MODEL_METRIC, "value": cpu["value"], "unit": "tok/s", "n_gpus": args.gpus,
        "steps": 1, "warmup": 64, "ms_per_step": round(1e3 / cpu["value"], 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8 + f32 + f16 KV",
        "data": "synthetic (same seeds and weights as the CUDA arm)",
        "config": {"workload": "config1 whole model (sampled layers, scaled)", "layers": cfg.n_layers},
        "cpu_baseline": cpu,
        "e2e": {"value": cpu["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ===================================================== configs 2, 3, 4
# prefill (config 2): 512 tokens through one MoE layer (Q4_K gate/up, Q6_K
#   down), near-uniform routing from N(0,1) rows and an N(0,0.02) router.
# batch (config 3): 64 sequences, one token each, through all 48 MoE layers;
#   router logits biased so expert popularity follows Zipf s=1.1.
# ep (config 4): 4096 tokens (8 x 512) through all 48 MoE layers with the
#   Zipf skew, experts spread over the N GPUs by a load-balanced placement,
#   dispatch and combine through peer memory inside the library (run_ep).
# The Zipf skew: every token carries a shared component c*u (u a fixed unit
# vector, c = sqrt(H)/2) and router row e gets s_e*u/C added, s_e =
# -1.1*ln(rank_e + 1) over a seeded permutation of the experts and C the
# component's size after RMSNorm, so logit e is its N(0,0.02)-router logit
# (the noise, std ~0.9) plus s_e: Plackett-Luce sampling with Zipf weights.
ZIPF_S = 1.1


def zipf_parts(seed, perm_seed=None):
    """(u [H], s [E]) of the Zipf bias (numpy, host): u from `seed`, the
    expert popularity order from `perm_seed` (default: the same generator)."""
    rng = np.random.default_rng(seed)
    u = rng.standard_normal(H).astype(np.float64)
    u /= np.linalg.norm(u)
    rank = rng.permutation(E) if perm_seed is None else np.random.default_rng(perm_seed).permutation(E)
    s = -ZIPF_S * np.log(rank + 1.0)
    return u.astype(np.float32), s.astype(np.float32)


def zipf_inputs(base_router, tokens, seed, perm_seed=None):
    """Bias an [E,H] router and [T,H] token rows (numpy float32 in, out).
    Layers that share `seed` share the direction u the tokens carry, so the
    skew holds in every layer; perm_seed gives each layer its own popular
    experts."""
    u, s = zipf_parts(seed, perm_seed)
    c = 0.5 * np.sqrt(H)
    C = c / np.sqrt(1.0 + c * c / H)
    router = (base_router + (s / C)[:, None] * u[None, :]).astype(np.float32)
    x = (tokens + c * u[None, :]).astype(np.float32)
    return np.ascontiguousarray(router), np.ascontiguousarray(x)


def workload_shape(args):
    n_layers = 1 if args.workload == "prefill" else args.layers
    tokens = {"prefill": 512, "batch": 64, "ep": 4096}[args.workload]
    return n_layers, tokens


def workload_metric(args):
    return {"prefill": "prefill tok/s (one MoE layer, 512 tokens)",
            "batch": "batched decode tok/s (64 sequences, 48 MoE layers)",
            "ep": "expert-parallel prefill tok/s (4096 tokens, 48 MoE layers)"}[args.workload]


def workload_desc(args, n_layers, tokens, world):
    d = {"prefill": f"config2 prefill: {tokens} tokens through one Qwen3-30B-A3B MoE layer (Q4_K gate/up, "
                    "Q6_K down), near-uniform routing",
         "batch": f"config3 batched decode: {tokens} sequences x 1 token through {n_layers} MoE layers, "
                  "router biased to Zipf s=1.1 expert popularity",
         "ep": f"config4 expert-parallel prefill: {tokens} tokens (8 x 512) through {n_layers} MoE layers, "
               "Zipf s=1.1, " + (f"128 experts sharded over {world} GPUs by measured load, "
                                   f"{128 // world} per GPU" if world > 1 else "128 experts on one GPU")}
    return d[args.workload]


def run_cuda_batched(args, quiet=False, table=None):
    import datetime

    import torch
    import torch.distributed as dist

    import ramvamp_b200 as rv

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = local if world > 1 else 0
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", init_method="env://", timeout=datetime.timedelta(seconds=120))
    n_layers, n_tok = workload_shape(args)
    flags = rv.EXACT if args.exact else rv.TENSOR
    assert args.workload in ("prefill", "batch"), "config 4 runs through run_ep"
    # On N>1 every rank runs an independent replica.  `table`: the decode
    # run's table (the same seeds) to reuse.
    lays = [rv.qwen3_layer_layout(l) for l in range(n_layers)]
    if table is None:
        table = rv.ExpertTable(lays, device=dev)
        for l in range(n_layers):
            table.fill_synthetic(l, SEED + l, 0.02)
    zipf = args.workload in ("batch", "ep")
    routers_np = []
    for l in range(n_layers):
        r = rv.synth_normal(SEED + 1000 + l, 0, 0.02, E * H).view(E, H).cpu().numpy()
        if zipf:
            r, _ = zipf_inputs(r, np.zeros((1, H), np.float32), SEED + 77, perm_seed=SEED + 77 + l)
        routers_np.append(r)
    routers = [torch.from_numpy(r).cuda() for r in routers_np]
    norm = torch.ones(H, dtype=torch.float32, device="cuda")
    home = n_tok
    n_batches = 4
    xs = rv.synth_normal(SEED + 7 + rank, 0, 1.0, n_batches * home * H).view(n_batches, home, H).cpu().numpy()
    if zipf:
        xs = np.stack([zipf_inputs(routers_np[0], xs[i], SEED + 77)[1] for i in range(n_batches)])
    tokens = torch.from_numpy(np.ascontiguousarray(xs)).cuda()
    eng = rv.MoeEngine(H, M, E, K, True, 1e-6, max_tokens=home, device=dev)
    resid = torch.empty(home, H, dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()

    def step_body():
        for l in range(n_layers):
            eng.forward(table, l, norm, routers[l], resid, flags=flags)

    with torch.cuda.stream(stream):
        resid.copy_(tokens[0])
        step_body()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step_body()
    torch.cuda.synchronize()

    def run_steps(lo, hi):
        with torch.cuda.stream(stream):
            for i in range(lo, hi):
                resid.copy_(tokens[i % n_batches])
                graph.replay() if graph is not None else step_body()

    stream.synchronize()
    if world > 1:
        dist.barrier()
    props = torch.cuda.get_device_properties(dev)
    uuid = str(getattr(props, "uuid", ""))
    clocks = ClockSampler(("GPU-" + uuid if uuid and not uuid.startswith("GPU-") else uuid) or str(dev))
    clocks.start()
    time.sleep(0.3)
    run_steps(0, args.warmup)  # warm-up right before the timed steps
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev0.record(stream)
    run_steps(args.warmup, args.warmup + args.steps)
    ev1.record(stream)
    ev1.synchronize()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    total_tok = home * world
    tok_s = total_tok * args.steps / (ms / 1e3)

    # Per-stage durations on the profile events (single-GPU forward path,
    # outside the timed region): the expert GEMM stages bound the roofline.
    eng.profile_enable(n_layers)
    sets = []
    for i in range(3):
        eng.profile_rewind()
        with torch.cuda.stream(stream):
            resid.copy_(tokens[i % n_batches])
            for l in range(n_layers):
                eng.forward(table, l, norm, routers[l], resid, flags=flags)
        stream.synchronize()
        sets.append(eng.profile_read())
    stage = np.stack(sets).mean(0)  # [layers][4] ms
    eng.profile_enable(0)
    # e2e: host rows in, host rows out, through the public call a caller makes
    host_tok = torch.empty(n_batches, home, H, dtype=torch.float32).pin_memory()
    host_tok.copy_(tokens.cpu())
    hres = torch.empty(home, H, dtype=torch.float32).pin_memory()
    if world > 1:
        dist.barrier()
    n_e2e = max(2, min(args.steps, 5))
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(n_e2e):
        hres.copy_(host_tok[i % n_batches])
        for l in range(n_layers):
            eng.forward_host(table, l, norm, routers[l], hres, flags=flags)
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_tok_s = total_tok * n_e2e / e2e_s

    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_baseline_batched(args, rv, table, routers_np,
                                   tokens[0].cpu().numpy(), lays)

    if rank == 0:
        hbm, hbm_kind = measured_peaks()
        tpk, tpk_kind = measured_tensor_peak()
        line = {
            "metric": workload_metric(args), "value": round(tok_s, 1), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8/int4 levels as exact f16 integers on tcgen05, f32 accumulate" if flags == rv.TENSOR
            else "int8 (dp4a) + f32",
            "data": "synthetic: seeded N(0,1) rows, N(0,0.02) router and expert weights quantized by the "
                    "reference's Q4_K/Q6_K quantizers" + (", Zipf-biased router" if zipf else ""),
            "config": {"workload": workload_desc(args, n_layers, n_tok, world), "layers": n_layers,
                       "tokens_per_step": total_tok,
                       "path": "tensor (bit-identical to the reference's scalar arm)" if flags == rv.TENSOR
                       else "exact (bit-identical to the reference's AVX2 arm)",
                       "l2": "inputs larger than L2: each step streams every touched expert's weights "
                             "(%.0f MB per layer resident)" % (sum(L.stride for L in lays[:1]) * lays[0].n_experts / 1e6),
                       "parallelism": "replicas" if world > 1 else "single GPU",
                       "cuda_graph": graph is not None},
            "e2e": {"value": round(e2e_tok_s, 1), "unit": "tok/s",
                    "h2d_bytes_per_step": home * H * 4 * n_layers,
                    "d2h_bytes_per_step": home * H * 4 * n_layers,
                    "path": "rv_moe_forward_host per layer (pinned host rows in, result out)"},
            "gpu_launches": args.steps * n_layers * (10 if flags == rv.TENSOR else 7),
            "clocks": clk,
            "cpu_baseline": cpu,
        }
        if stage is not None:
            gu_ms, dn_ms = float(stage[:, 1].mean()), float(stage[:, 2].mean())
            L0 = lays[0]
            gu_bytes = L0.n_experts * (L0.gate_len + L0.up_len)
            pairs = home * K
            gu_flop = 2.0 * pairs * 2 * M * H
            line["stage_ms_per_layer"] = {"routing": round(float(stage[:, 0].mean()), 4),
                                          "gate_up": round(gu_ms, 4), "down": round(dn_ms, 4),
                                          "combine": round(float(stage[:, 3].mean()), 4)}
            achieved = gu_bytes / (gu_ms * 1e-3) / 1e9
            line["roofline"] = {"kernel": "k_tc_gemm gate/up (stage incl. SwiGLU+Q8_K)" if flags == rv.TENSOR
                                else "k_gate_up", "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm,
                                "unit": "GB/s", "frac": round(achieved / hbm, 4),
                                "peak_source": f"{hbm_kind} hbm_gbs",
                                "bytes_per_launch": gu_bytes, "traffic": ncu_traffic("k_tc_gemm_gate_up"),
                                "upper_bound_if_every_expert_is_touched": True}
            line["tensor"] = {"achieved_tflops": round(gu_flop / (gu_ms * 1e-3) / 1e12, 2), "peak": tpk,
                              "frac": round(gu_flop / (gu_ms * 1e-3) / 1e12 / tpk, 4),
                              "peak_source": f"{tpk_kind} bf16_tflops (dense f16 runs at the same rate)",
                              "flops": "2 * pairs * (gate + up) * hidden, useful products only"}
        if not quiet:
            print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return line if rank == 0 else None


# ============================= config 4 through the library's exchange
EP_TOKENS = 4096
EP_METRIC = "expert-parallel prefill tok/s (4096 tokens, 48 MoE layers)"


def ep_launches_per_layer(tensor: bool) -> int:
    # routing (k_prologue, k_router_logits, k_route), k_ep_dispatch,
    # k_ep_receive, the expert stage (tensor: k_tc_tiles, k_tc_gather,
    # k_tc_gemm, k_tc_quant, k_tc_gemm; exact: k_gate_up, k_down),
    # k_ep_signal, k_ep_combine
    return 3 + 2 + (5 if tensor else 2) + 2


def run_ep(args, table=None, quiet=False):
    """Config 4: 4096 tokens (8 x 512) with Zipf s=1.1 routing through all
    48 MoE layers, the 128 experts spread over the N ranks by the load a
    calibration batch measures through each layer's router
    (`balanced_placement`, 128/N experts per rank).  Each rank routes 4096/N
    home tokens; dispatch, expert outputs and the per-layer flags go through GPU memory (rv_moe_ep_forward), and a step
    (48 layers) is one captured CUDA graph.  Strong scaling: the total work
    is fixed.  `table`: the full 48-layer table to reuse at N=1.  Returns the
    JSON line (rank 0), printed unless quiet."""
    import datetime

    import torch
    import torch.distributed as dist

    import ramvamp_b200 as rv
    from ramvamp_b200.ep import balanced_placement, connect_group, placement_tensor

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = local if world > 1 else 0
    torch.cuda.set_device(dev)
    if world > 1 and not dist.is_initialized():
        dist.init_process_group("nccl", init_method="env://", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", dev))
    n_layers = args.layers
    home = EP_TOKENS // world
    flags = rv.EXACT if args.exact else rv.TENSOR
    routers_np = []
    for l in range(n_layers):
        r = rv.synth_normal(SEED + 1000 + l, 0, 0.02, E * H).view(E, H).cpu().numpy()
        r, _ = zipf_inputs(r, np.zeros((1, H), np.float32), SEED + 77, perm_seed=SEED + 77 + l)
        routers_np.append(r)
    routers = [torch.from_numpy(r).cuda() for r in routers_np]
    norm = torch.ones(H, dtype=torch.float32, device="cuda")
    eng = rv.MoeEngine(H, M, E, K, True, 1e-6, max_tokens=EP_TOKENS, device=dev)
    # Expert placement (N > 1): route a calibration batch of 512 rows of the
    # workload's distribution (the same on every rank, so every rank derives
    # the same placement) through each layer's router and spread the
    # experts by measured load, n_experts / N per rank.
    placements, loads = [None] * n_layers, None
    if world > 1:
        cal = rv.synth_normal(SEED + 99, 0, 1.0, 512 * H).view(512, H).cpu().numpy()
        cal = torch.from_numpy(zipf_inputs(routers_np[0], cal, SEED + 77, perm_seed=SEED + 77)[1]).cuda()
        ranks_of = []
        for l in range(n_layers):
            ids, _, _ = eng.route(norm, routers[l], cal)
            cnt = torch.bincount(ids.reshape(-1).long(), minlength=E).cpu().numpy()
            ranks = balanced_placement(cnt.tolist(), world)
            ranks_of.append(ranks)
            placements[l] = placement_tensor(ranks, f"cuda:{dev}")
    if table is None or world > 1:
        lays = [rv.qwen3_layer_layout(l, n_experts=E // world) for l in range(n_layers)]
        table = rv.ExpertTable(lays, device=dev)
        for l in range(n_layers):
            if world > 1:
                table.fill_synthetic_list(l, SEED + l, 0.02, ranks_of[l][rank])
            else:
                table.fill_synthetic(l, SEED + l, 0.02)
    n_batches = 2
    xs = rv.synth_normal(SEED + 7 + rank, 0, 1.0, n_batches * home * H).view(n_batches, home, H).cpu().numpy()
    xs = np.stack([zipf_inputs(routers_np[0], xs[i], SEED + 77, perm_seed=SEED + 77)[1] for i in range(n_batches)])
    tokens = torch.from_numpy(np.ascontiguousarray(xs)).cuda()
    ep = rv.ExpertParallel(eng, world, rank, home)
    if world > 1:
        connect_group(ep)
    else:
        ep.connect([ep.handle_bytes()])
    resid = torch.empty(home, H, dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()

    def step_body():
        for l in range(n_layers):
            ep.forward(table, l, norm, routers[l], resid, flags=flags, placement=placements[l])

    # Every rank runs the same exchange steps in the same order: eager once,
    # capture (no steps run), replays.
    with torch.cuda.stream(stream):
        resid.copy_(tokens[0])
        step_body()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step_body()
    torch.cuda.synchronize()
    # Parity 1: the captured step equals the eager one.
    with torch.cuda.stream(stream):
        resid.copy_(tokens[1])
        graph.replay()
        g_out = resid.clone()
        resid.copy_(tokens[1])
        step_body()
    stream.synchronize()
    same_graph = bool(torch.equal(g_out.view(torch.int32), resid.view(torch.int32)))
    # Parity 2: one layer through the exchange equals this rank's own
    # single-GPU forward of its tokens (layer 0's full table on this GPU).
    full0 = rv.ExpertTable([rv.qwen3_layer_layout(0)], device=dev)
    full0.fill_synthetic(0, SEED, 0.02)
    with torch.cuda.stream(stream):
        resid.copy_(tokens[0])
        ep.forward(table, 0, norm, routers[0], resid, flags=flags, placement=placements[0])
        ep_l0 = resid.clone()
        resid.copy_(tokens[0])
        eng.forward(full0, 0, norm, routers[0], resid, flags=flags)
    stream.synchronize()
    same_1gpu = bool(torch.equal(ep_l0.view(torch.int32), resid.view(torch.int32)))
    # Parity 3 (rank 0): 16 rows of that layer against the oracle's arm.
    same_oracle = None
    if rank == 0:
        from oracle import oracle as orc

        orc.build()
        L0 = rv.qwen3_layer_layout(0)
        blobs = rv.alias(full0.view(0, 0).blob, E * L0.stride).cpu().numpy()
        OL = orc.make_layer(H, M, E, K, 1e-6, np.ones(H, np.float32), routers_np[0], blobs, L0.stride,
                            L0.gate_off, L0.up_off, L0.down_off, L0.gate_format, L0.up_format, L0.down_format)
        want, _, _ = orc.moe_prefill(OL, np.ascontiguousarray(xs[0][:16]), impl=0 if flags == rv.TENSOR else 2,
                                     threads=os.cpu_count() or 1)
        same_oracle = bool((ep_l0[:16].cpu().numpy().view(np.uint32) == want.view(np.uint32)).all())
    full0.close()
    ok = torch.tensor([int(same_graph and same_1gpu)], device="cuda")
    if world > 1:
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)

    if world > 1:
        dist.barrier()
    props = torch.cuda.get_device_properties(dev)
    uuid = str(getattr(props, "uuid", ""))
    clocks = ClockSampler(("GPU-" + uuid if uuid and not uuid.startswith("GPU-") else uuid) or str(dev))
    clocks.start()

    def run_steps(lo, hi):
        with torch.cuda.stream(stream):
            for i in range(lo, hi):
                resid.copy_(tokens[i % n_batches])
                graph.replay()

    run_steps(0, args.warmup)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0.record(stream)
    run_steps(args.warmup, args.warmup + args.steps)
    ev1.record(stream)
    ev1.synchronize()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    tok_s = EP_TOKENS * args.steps / (ms / 1e3)
    # Load: the pairs each rank's experts ran in the last layer.
    recv = [int(sum(ep.received()))]
    if world > 1:
        allr = [None] * world
        dist.all_gather_object(allr, recv[0])
        recv = allr
    # e2e through the public call: pinned host rows in, 48 rv_moe_ep_forward
    # calls (eager), the result back to the host, every step.
    host_tok = torch.empty(n_batches, home, H, dtype=torch.float32).pin_memory()
    host_tok.copy_(tokens.cpu())
    hres = torch.empty(home, H, dtype=torch.float32).pin_memory()
    n_e2e = max(2, min(args.steps, 5))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(n_e2e):
        with torch.cuda.stream(stream):
            resid.copy_(host_tok[i % n_batches], non_blocking=True)
            step_body()
            hres.copy_(resid, non_blocking=True)
        stream.synchronize()
    e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_tok_s = EP_TOKENS * n_e2e / e2e_s

    line = None
    if rank == 0:
        tpk, tpk_kind = measured_tensor_peak()
        flops = 2.0 * 3 * M * H * EP_TOKENS * K * n_layers  # useful products of gate, up and down
        achieved = flops / (ms_per_step * 1e-3) / 1e12 / world  # per GPU
        line = {
            "metric": EP_METRIC, "value": round(tok_s, 1), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int8/int4 levels as exact f16 integers on tcgen05, f32 accumulate" if flags == rv.TENSOR
            else "int8 (dp4a) + f32",
            "data": "synthetic: seeded N(0,1) rows and N(0,0.02) router and expert weights quantized by the "
                    "reference's Q4_K/Q6_K quantizers; router and rows biased to Zipf s=1.1 expert popularity",
            "config": {"workload": f"config4 expert-parallel prefill: {EP_TOKENS} tokens (8 x 512) through "
                                   f"{n_layers} MoE layers, Zipf s=1.1, 128 experts over {world} GPU(s) by id "
                                   f"mod {world}", "layers": n_layers, "tokens_per_step": EP_TOKENS,
                       "path": "tensor (bit-identical to the reference's scalar arm)" if flags == rv.TENSOR
                       else "exact (bit-identical to the reference's AVX2 arm)",
                       "parallelism": f"ep{world}", "exchange": "rv_moe_ep_forward: peer stores over NVLink + "
                       "release/acquire flags, no host synchronization", "cuda_graph": True,
                       "placement": "per layer, experts spread by load measured on a 512-row calibration batch "
                                    "(n_experts/N per rank)" if world > 1 else "all experts local",
                       "l2": "inputs larger than L2: each step streams every touched expert's weights (17.5 GB "
                             "over all ranks)"},
            "parity": {"graph_equals_eager": same_graph, "ep_equals_single_gpu_layer0": bool(ok.item()),
                       "oracle_rank0_16_rows_layer0": same_oracle},
            "load": {"pairs_per_rank_last_layer": recv,
                     "max_over_mean": round(max(recv) / (sum(recv) / len(recv)), 3) if sum(recv) else None},
            "roofline": {"kernel": "whole EP step (routing, exchange, tcgen05 expert GEMMs, combine)",
                         "bound": "tensor", "achieved": round(achieved, 2), "peak": tpk, "unit": "TFLOP/s",
                         "frac": round(achieved / tpk, 4), "peak_source": f"{tpk_kind} bf16_tflops",
                         "flops_per_step": flops, "traffic": None},
            "e2e": {"value": round(e2e_tok_s, 1), "unit": "tok/s", "h2d_bytes_per_step": EP_TOKENS * H * 4,
                    "d2h_bytes_per_step": EP_TOKENS * H * 4,
                    "path": "per rank: pinned home rows in, 48 rv_moe_ep_forward calls, rows out"},
            "gpu_launches": args.steps * n_layers * ep_launches_per_layer(flags == rv.TENSOR),
            "clocks": clk,
            "cpu_baseline": None,
        }
        if not quiet:
            print(json.dumps(line), flush=True)
    del graph
    ep.close()
    if world > 1:
        dist.barrier()
    return line


def cpu_baseline_batched(args, rv, table, routers_np, x0, lays):
    """The oracle (AVX2 restatement of the reference) on a bounded sample of
    the workload: up to 32 rows through layer 0 on every host core, scaled
    to the workload's layers and tokens."""
    from oracle import oracle as orc

    import torch

    orc.build()
    threads = os.cpu_count() or 1
    L = lays[0]
    if table is not None and L.n_experts == E:
        blobs = rv.alias(table.view(0, 0).blob, E * L.stride).cpu().numpy()
    else:
        full = rv.qwen3_layer_layout(0)
        blobs = orc.fill_layer_synthetic(full, SEED, 0.02, threads)
        L = full
    norm = np.ones(H, np.float32)
    OL = orc.make_layer(H, M, E, K, 1e-6, norm, routers_np[0], blobs, L.stride, L.gate_off, L.up_off, L.down_off,
                        L.gate_format, L.up_format, L.down_format)
    n = min(32, x0.shape[0])
    x = np.ascontiguousarray(x0[:n])
    orc.moe_prefill(OL, x[:2], threads=threads)  # warm-up
    t0 = time.perf_counter()
    reps = 0
    while True:
        orc.moe_prefill(OL, x, threads=threads)
        reps += 1
        if time.perf_counter() - t0 > 8.0:
            break
    dt = (time.perf_counter() - t0) / reps  # one layer, n rows
    n_layers, _ = workload_shape(args)
    tok_s = n / (dt * n_layers)
    return {"value": round(tok_s, 3), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{n} rows through one Q6_K-down layer on the C oracle's AVX2 arm ({reps} repetitions), "
                      f"time scaled to {n_layers} layer(s)"}


def run_reference_batched(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle as orc
    from oracle.layout import layer_layout

    orc.build()
    threads = os.cpu_count() or 1
    n_layers, n_tok = workload_shape(args)
    full = layer_layout(0)
    blobs = orc.fill_layer_synthetic(full, SEED, 0.02, threads)
    router = orc.synth_normal(SEED + 1000, 0, 0.02, E * H).reshape(E, H)
    x = orc.synth_normal(SEED + 7, 0, 1.0, 32 * H).reshape(32, H)
    if args.workload in ("batch", "ep"):
        router, x = zipf_inputs(router, x, SEED + 77, perm_seed=SEED + 77)  # layer 0 of the CUDA arm
    OL = orc.make_layer(H, M, E, K, 1e-6, np.ones(H, np.float32), router, blobs, full.stride, full.gate_off,
                        full.up_off, full.down_off, full.gate_format, full.up_format, full.down_format)
    sample = 64 if args.workload == "batch" else 128
    xs = np.ascontiguousarray(x[:sample])
    for _ in range(args.warmup):
        orc.moe_prefill(OL, xs[:2], threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        orc.moe_prefill(OL, xs, threads=threads)
    dt = (time.perf_counter() - t0) / args.steps
    v = sample / (dt * n_layers)
    line = {
        "impl": "reference", "metric": workload_metric(args), "value": round(v, 3), "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * n_layers * n_tok / sample * 1e3, 3), "higher_is_better": True,
        "scaling": "strong" if args.workload == "ep" else "weak", "vs_baseline": None, "dtype": "int8 + f32",
        "data": "synthetic (same seeds as the CUDA arm)",
        "config": {"workload": workload_desc(args, n_layers, n_tok, 1) + " (sampled rows, scaled)",
                   "layers": n_layers, "tokens_per_step": n_tok},
        "cpu_baseline": {"value": round(v, 3), "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": f"each step: {sample} rows through one Q6_K-down layer on the C oracle's "
                                   f"AVX2 arm with {threads} threads, time scaled to {n_layers} layer(s)"},
        "e2e": {"value": round(v, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.workload == "model":
        (run_reference_model if args.impl == "reference" else run_cuda_model)(args)
        return
    if args.workload == "ep" and args.impl != "reference":
        run_ep(args)
        import torch.distributed as dist

        if dist.is_available() and dist.is_initialized():
            dist.destroy_process_group()
        return
    if args.workload != "decode":
        (run_reference_batched if args.impl == "reference" else run_cuda_batched)(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_cuda(args)


if __name__ == "__main__":
    main()
