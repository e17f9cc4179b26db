#!/usr/bin/env python
"""Benchmark: Qwen3.8-Flash-Next-shaped NVFP4 MoE layer decode over a VRAM expert-slot cache.

Workload (one "step" = one decode batch through a stack of MoE layers):
  hidden 2048, 512 experts, top-10 softmax routing with Zipf(1.1) skew (N(0,1) + ln p router
  logits, per-layer rank permutation), expert intermediate 512, one always-on shared expert,
  NVFP4 weights (E2M1 codes uniform, E4M3 per-16 scales 2^U(-8,-2), fp32 global 1/448),
  128 slots per layer prewarmed with each layer's most frequent experts; 48 layers with
  distinct slot pools (10.9 GB of pools: inputs larger than L2 between steps); misses refill
  from a pinned host tier holding all 512 experts (shared by the layers' pools).
  Layers depend on each other (the headline): per layer the residual add, RMSNorm and router
  gate GEMV (bf16 gate [512, 2048], logit bias ln p of Zipf(1.1)) -> router top-k -> slot
  remap (LRU, miss list) -> fused FFN (gate/up SwiGLU, down, weighted combine, shared expert)
  that also copies the misses in from pinned host memory; attention is omitted.
  Reported beside it ("independent_layers"): every layer routes precomputed N(0,1) + ln p
  logits of the same tokens, so a layer's routing and remap overlap the previous layer's FFN.

metric: layer tokens/s = batch * layers / step time (device CUDA events, max over ranks).
N > 1: expert parallelism (weak scaling): every rank holds 512 / N experts of each layer in its
128-slot pools and a batch of its own; each layer dispatches the tokens to the experts' owners
and combines the outputs by NCCL all-to-all (graph-captured with the kernels).  The prefill
object at N > 1 is the 4096-token layer under expert parallelism (strong scaling).
--impl reference times the CPU oracle port of the same step on the host cores.
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
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "MoE-layer decode tokens/s (Qwen3.8-shaped NVFP4 layer, 128-slot VRAM expert cache)"
UNIT = "layer-tokens/s"
FP4_TERMS = 3              # NVFP4 residual terms per activation row in the FP4 prefill
FP4_NOMINAL_TFLOPS = 9000.0  # B200 dense FP4, nominal


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="nvmoe", choices=["nvmoe", "reference"])
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--cpu-baseline-seconds", type=float, default=12.0)
    ap.add_argument("--prefill-tokens", type=int, default=4096,
                    help="also time one prefill layer of this many tokens (0: skip)")
    ap.add_argument("--only-prefill", action="store_true",
                    help="time the prefill layer alone on one GPU and print its object")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-config3", action="store_true", help="skip the Q2_K stack object")
    return ap.parse_args()


def config_dict(a, world):
    return {
        "workload": f"Qwen3.8-shaped NVFP4 MoE layer decode, batch {a.batch}, {a.layers}-layer "
                    "stack of dependent layers (residual + RMSNorm + router gate in front of "
                    "each), 512 experts top-10 + shared, H2048 I512, 128 slots/layer",
        "model": "Qwen3.8-Flash-Next MoE layer (synthetic NVFP4)",
        "global_batch": a.batch * world,
        "seq_len": 1,
        "layers": a.layers,
        "experts": 512, "top_k": 10, "hidden": 2048, "inter": 512, "slots_per_layer": 128,
        "parallelism": f"expert parallel x{world}" if world > 1 else "single GPU",
        "l2": "inputs larger than L2 (10.9 GB of distinct per-layer slot pools)",
        "routing": "softmax top-10 of the gate logits (RMS-normalised tokens x N(0, 1/H) gate "
                   "rows, about N(0,1)) + ln Zipf(1.1), seed 0",
    }


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0: float | None = None) -> dict:
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[4:]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in rows:
            for n, v in zip(names, r[3][1:]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        loaded = [r for r in rows if r[2] > 200.0] or rows
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": rows[0][1],
                "reasons": sorted(reasons), "samples": len(rows)}


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    return json.loads(p.read_text()) if p.exists() else None


# ------------------------------------------------------------------ GPU arm
def run_nvmoe(a, rank, world, local_rank):
    import numpy as np
    import torch

    from nvmoe_b200 import ops
    from nvmoe_b200.engine import MoEStack, StackConfig
    from nvmoe_b200.synth import layer_log_bias

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    L, B = a.layers, a.batch
    cfg = StackConfig(n_layers=L)
    E, k, H, I, S = cfg.n_experts, cfg.top_k, cfg.hidden, cfg.inter, cfg.cache_size
    stack = MoEStack(cfg, device=dev, seed=0)
    bias = layer_log_bias(L, E, 1.1, seed=0)
    ranking = np.argsort(-bias, axis=1, kind="stable")
    stack.prewarm(ranking)
    # dependent layers: the routing skew enters as the gate's logit bias ln p (Zipf 1.1)
    stack.init_router(logit_bias=bias, seed=5)

    # fresh tokens (and, for the independent stack, fresh logits) every step; the last
    # E2E_WARM + e2e_steps rounds are only seen by the end-to-end leg
    R = a.warmup + a.steps
    e2e_steps = 0 if a.no_e2e else max(10, a.steps)
    E2E_WARM = a.warmup
    RT = R + (E2E_WARM + e2e_steps if e2e_steps else 0)
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    bias_t = torch.from_numpy(bias).to(dev)
    logits = torch.randn((R, L, B, E), generator=g, device=dev) + bias_t[None, :, None, :]
    xs = torch.randn((RT, B, H), generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty((L, B, H), dtype=torch.bfloat16, device=dev)
    hout = torch.empty((B, H), dtype=torch.bfloat16, device=dev)
    cap_stream = torch.cuda.Stream(dev)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    def distinct(plans):
        return np.array([len(np.unique(p.slot_ids.cpu().numpy())) for p in plans])

    def timed(step, plans, clocks: bool):
        """Captures one graph per round, replays every graph once (the first launch of a
        graph uploads it) recording the distinct experts each layer step routes, puts the
        cache back in its prewarmed state, runs the warm-up rounds and times the rest."""
        step(0)  # eager pass: kernel attributes, allocations
        torch.cuda.synchronize()
        stack.prewarm(ranking)
        graphs = []
        for r in range(R):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=cap_stream):
                step(r)
            graphs.append(gr)
        torch.cuda.synchronize()
        U = np.zeros((R, L), np.int64)
        for r, gr in enumerate(graphs):
            gr.replay()
            U[r] = distinct(plans)  # the same routing the timed replay of round r sees
        stack.prewarm(ranking)
        for i in range(a.warmup):
            graphs[i].replay()
        barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        clk = ClockSampler(local_rank) if clocks else None
        if clk:
            clk.__enter__()
        t0.record()
        for i in range(a.steps):
            graphs[a.warmup + i].replay()
        t1.record()
        torch.cuda.synchronize()
        if clk:
            clk.__exit__(None, None, None)
        barrier()
        el = t0.elapsed_time(t1)
        if world > 1:
            tt = torch.tensor([el], device=dev)
            torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
            el = float(tt.item())
        del graphs
        return el / a.steps, U, (clk.summary() if clk else None)

    # headline: layers that depend on each other (residual + RMSNorm + router gate GEMV in
    # front of every layer's routing): per layer nvmoe_router_gate + nvmoe_decode_layer
    chain = stack.chain_buffers(B)
    ms_chain, U_chain, clocks = timed(lambda r: stack.forward_chain(xs[r], hout), chain["plans"],
                                      clocks=True)
    misses_last = int(stack.misses.counts[1].item())
    # beside it: independent layers (every layer routes precomputed logits of the same tokens,
    # so a layer's routing overlaps the previous layer's FFN)
    plans = stack.plans(B)
    ms_ind, U_ind, _ = timed(lambda r: stack.forward(xs[r], logits[r], out), plans, clocks=False)
    value = B * L * world / (ms_chain / 1e3)

    # roofline kernel: ffn_fused of every layer on the slot ids of the final dependent step,
    # timed per launch with CUDA events
    ffn_graph = torch.cuda.CUDAGraph()
    evs = [(torch.cuda.Event(enable_timing=True, external=True),
            torch.cuda.Event(enable_timing=True, external=True)) for _ in range(L)]
    ws = ops.FfnWorkspace(dev)
    yb = torch.empty((L, B, H), dtype=torch.bfloat16, device=dev)
    cp = chain["plans"]
    xr = chain["xn"]
    for l in range(L):  # eager once (attributes)
        ops.moe_ffn(stack.pools[l], xr[l], cp[l].slot_ids, cp[l].weights,
                    shared=stack.shared[l], out=yb[l], workspace=ws)
    torch.cuda.synchronize()
    # events bracket the fused expert kernel alone (ffn_fused); the grouping launch before it
    # (nvmoe_moe_ffn_prepare) sits outside them
    with torch.cuda.graph(ffn_graph, stream=cap_stream):
        for l in range(L):
            ops.moe_ffn(stack.pools[l], xr[l], cp[l].slot_ids, cp[l].weights,
                        shared=stack.shared[l], out=yb[l], workspace=ws, phase="prepare")
            evs[l][0].record()
            ops.moe_ffn(stack.pools[l], xr[l], cp[l].slot_ids, cp[l].weights,
                        shared=stack.shared[l], out=yb[l], workspace=ws, phase="execute")
            evs[l][1].record()
    Ulast = distinct(cp)
    ffn_ms, reps = 0.0, 5
    for _ in range(reps):
        ffn_graph.replay()
        torch.cuda.synchronize()
        ffn_ms += sum(evs[l][0].elapsed_time(evs[l][1]) for l in range(L))
    n_ffn = reps * L
    ffn_bytes = reps * float(((Ulast + 1) * stack.bytes_per_expert).sum() +
                             L * (2 * B * H * 2 + B * k * 8))
    del ffn_graph

    # e2e through the public API (MoEStack.forward_chain) with host buffers: per step the H2D
    # copy of the step's tokens and the D2H read of the stack's output, on fresh tokens
    e2e_ms = None
    if e2e_steps:
        xh = xs[R:].cpu().pin_memory()
        yh = torch.empty((B, H), dtype=torch.bfloat16).pin_memory()
        xin = torch.empty((B, H), dtype=torch.bfloat16, device=dev)
        gr_e2e = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr_e2e, stream=cap_stream):
            stack.forward_chain(xin, hout)
        torch.cuda.synchronize()
        # the same starting cache state as the timed leg: prewarmed, then the warm-up rounds
        stack.prewarm(ranking)
        for i in range(E2E_WARM):
            xin.copy_(xh[i], non_blocking=True)
            gr_e2e.replay()
            yh.copy_(hout, non_blocking=True)
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(E2E_WARM, E2E_WARM + e2e_steps):
            xin.copy_(xh[i], non_blocking=True)
            gr_e2e.replay()
            yh.copy_(hout, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / e2e_steps
        if world > 1:
            tt = torch.tensor([e2e_ms], device=dev)
            torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
            e2e_ms = float(tt.item())
        del gr_e2e

    peaks = load_peaks()
    hbm_peak = peaks["hbm_gbs"] if peaks else 6650.0
    achieved = (ffn_bytes / n_ffn) / ((ffn_ms / n_ffn) / 1e3) / 1e9
    step_bytes = float(((U_chain[a.warmup:] + 1) * stack.bytes_per_expert).sum()) / a.steps
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms_chain, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "nvfp4/f16",
        "data": "synthetic (seeded; random-init NVFP4 expert weights and bf16 router gates)",
        "config": config_dict(a, world),
        "e2e": None if e2e_ms is None else {
            "value": round(B * L * world / (e2e_ms / 1e3), 1), "unit": UNIT,
            "h2d_bytes_per_step": B * H * 2, "d2h_bytes_per_step": B * H * 2},
        # per layer step: router gate (gate GEMV + top-k) + decode_front_kernel (pre-routed)
        # + ffn_fused (misses are copied in by the FFN), plus the final residual add
        "gpu_launches": a.steps * (3 * L + 1),
        "roofline": {"bound": "hbm", "kernel": "ffn_fused (the fused expert kernel of one layer)",
                     "achieved": round(achieved, 1),
                     "peak": hbm_peak, "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)" if peaks else
                     "fallback 6650 GB/s",
                     "traffic": _traffic_from_profiles(B),
                     "bytes_per_launch": round(ffn_bytes / n_ffn),
                     "avg_launch_us": round(1e3 * ffn_ms / n_ffn, 3)},
        "breakdown": {"layer_step_us": round(1e3 * ms_chain / L, 3),
                      "layer_step_hbm_gbs": round(step_bytes / (ms_chain / 1e3) / 1e9, 1),
                      "distinct_experts_per_layer": round(float(U_chain.mean()), 2),
                      "misses_last_layer_step": misses_last},
        "independent_layers": {
            "value": round(B * L * world / (ms_ind / 1e3), 1), "unit": UNIT,
            "ms_per_step": round(ms_ind, 4), "layer_step_us": round(1e3 * ms_ind / L, 3),
            "distinct_experts_per_layer": round(float(U_ind.mean()), 2),
            "gpu_launches": a.steps * 2 * L,
            "what": "same stack and tokens, every layer routing precomputed N(0,1) + ln Zipf "
                    "logits: no gate GEMV, and a layer's routing overlaps the previous FFN"},
        "clocks": clocks,
    }
    if a.prefill_tokens > 0:
        line["prefill"] = run_prefill(a, dev, peaks)
    if not a.no_config3:
        line["config3_q2k_stack"] = run_config3(a, dev)
        line["config3_q2k_stack"]["bounded_host_tier"] = run_config3_bounded(dev)
    return line


def run_ep(a, rank, world, local_rank):
    """Expert-parallel decode (the N-GPU line): every rank holds E / world experts of each layer
    (128-slot pools, its own host tier) and B tokens of its own; the same dependent-layer stack
    as the 1-GPU line, with the tokens dispatched to the experts' owners by NCCL all-to-all."""
    import numpy as np
    import torch

    from nvmoe_b200.engine import StackConfig
    from nvmoe_b200.ep import EPMoEStack
    from nvmoe_b200.formats import random_experts
    from nvmoe_b200.synth import layer_log_bias

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    L, B = a.layers, a.batch
    cfg = StackConfig(n_layers=L)
    E, k, H = cfg.n_experts, cfg.top_k, cfg.hidden
    host = random_experts("nvfp4", E, H, cfg.inter, seed=0)
    shared = random_experts("nvfp4", 1, H, cfg.inter, seed=2)
    bias = layer_log_bias(L, E, 1.1, seed=0)
    ranking = np.argsort(-bias, axis=1, kind="stable")
    st = EPMoEStack(cfg, B, rank, world, host, shared, device=dev, seed=1 + rank, logit_bias=bias)
    st.prewarm(ranking)
    R = a.warmup + a.steps
    e2e_steps = 0 if a.no_e2e else max(10, a.steps)
    E2E_WARM = 3
    RT = R + (E2E_WARM + e2e_steps if e2e_steps else 0)
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    xs = torch.randn((RT, B, H), generator=g, device=dev).to(torch.bfloat16)
    hout = torch.empty((B, H), dtype=torch.bfloat16, device=dev)
    cap = torch.cuda.Stream(dev)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    st.forward(xs[0], hout)  # eager pass: kernel attributes, allocations
    torch.cuda.synchronize()
    st.prewarm(ranking)
    graphs = []
    for r in range(R):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=cap):
            st.forward(xs[r], hout)
        graphs.append(gr)
    torch.cuda.synchronize()
    U = np.zeros((R, L), np.int64)  # distinct local experts each layer step ran
    for r, gr in enumerate(graphs):
        gr.replay()
        torch.cuda.synchronize()
        for l, p in enumerate(st.plans):
            s = p.slot_ids.cpu().numpy()
            U[r, l] = len(np.unique(s[s >= 0]))
    st.prewarm(ranking)
    for i in range(a.warmup):
        graphs[i].replay()
    barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        t0.record()
        for i in range(a.steps):
            graphs[a.warmup + i].replay()
        t1.record()
        torch.cuda.synchronize()
    barrier()
    el = t0.elapsed_time(t1)
    tt = torch.tensor([el], device=dev)
    torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
    ms = float(tt.item()) / a.steps
    graphs = None
    torch.cuda.synchronize()

    e2e_ms = None
    if e2e_steps:
        xh = xs[R:].cpu().pin_memory()
        yh = torch.empty((B, H), dtype=torch.bfloat16).pin_memory()
        xin = torch.empty((B, H), dtype=torch.bfloat16, device=dev)
        gr_e2e = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr_e2e, stream=cap):
            st.forward(xin, hout)
        torch.cuda.synchronize()
        for i in range(E2E_WARM):
            xin.copy_(xh[i], non_blocking=True)
            gr_e2e.replay()
            yh.copy_(hout, non_blocking=True)
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(E2E_WARM, E2E_WARM + e2e_steps):
            xin.copy_(xh[i], non_blocking=True)
            gr_e2e.replay()
            yh.copy_(hout, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        tt = torch.tensor([e0.elapsed_time(e1) / e2e_steps], device=dev)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(tt.item())
        gr_e2e = None
        torch.cuda.synchronize()

    peaks = load_peaks()
    hbm_peak = peaks["hbm_gbs"] if peaks else 6650.0
    step_bytes = float(((U[a.warmup:] + 0) * st.local.bytes_per_expert).sum()) / a.steps
    achieved = step_bytes / (ms / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": round(B * L * world / (ms / 1e3), 1), "unit": UNIT,
        "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "nvfp4/f16",
        "data": "synthetic (seeded; random-init NVFP4 expert weights and bf16 router gates)",
        "config": dict(config_dict(a, world),
                       parallelism=f"expert parallel x{world} ({E // world} experts per GPU, "
                                   "NCCL all-to-all dispatch / combine)"),
        "e2e": None if e2e_ms is None else {
            "value": round(B * L * world / (e2e_ms / 1e3), 1), "unit": UNIT,
            "h2d_bytes_per_step": B * H * 2, "d2h_bytes_per_step": B * H * 2},
        # per layer: router gate (with the top-k), two dispatch kernels, decode front,
        # ffn_fused, combine (NCCL's all-to-all kernels not counted), plus the final residual add
        "gpu_launches": a.steps * (6 * L + 1),
        "roofline": {"bound": "hbm", "kernel": "expert-parallel layer step (one rank's expert "
                                               "bytes per layer step / layer step time)",
                     "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4),
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)" if peaks else
                     "fallback 6650 GB/s", "traffic": None},
        "breakdown": {"layer_step_us": round(1e3 * ms / L, 3),
                      "distinct_local_experts_per_layer": round(float(U.mean()), 2),
                      "tokens_per_rank": B},
        "clocks": clk.summary(),
    }
    return line


def run_ep_prefill(a, rank, world, local_rank, peaks):
    """The prefill layer under expert parallelism: a.prefill_tokens tokens in all (strong
    scaling), a.prefill_tokens / world per rank, E / world experts resident per rank."""
    import numpy as np
    import torch

    from nvmoe_b200 import ops
    from nvmoe_b200.ep import EPPrefill
    from nvmoe_b200.formats import random_experts
    from nvmoe_b200.synth import layer_log_bias, router_logits

    dev = torch.device("cuda", local_rank)
    E, k, H, I = 512, 10, 2048, 512
    T = a.prefill_tokens
    Tr = T // world
    host = random_experts("nvfp4", E, H, I, seed=11)
    shared = random_experts("nvfp4", 1, H, I, seed=12)
    rng = np.random.default_rng(7)
    lg = torch.from_numpy(router_logits(T, layer_log_bias(1, E, 1.1, seed=0)[0], rng))
    lg = lg[rank * Tr:(rank + 1) * Tr].contiguous().to(dev)
    ids, w = ops.router_topk(lg, k)
    x = torch.randn((T, H), generator=torch.Generator().manual_seed(13))[rank * Tr:(rank + 1) * Tr]
    x = x.to(torch.bfloat16).to(dev)
    out = torch.empty((Tr, H), dtype=torch.bfloat16, device=dev)
    ep = EPPrefill(E, k, Tr, rank, world, host, shared, device=dev)
    del host
    for _ in range(3):
        ep.forward(x, ids, w, out)
    torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 10
    e0.record()
    for _ in range(n):
        ep.forward(x, ids, w, out)
    e1.record()
    torch.cuda.synchronize()
    tt = torch.tensor([e0.elapsed_time(e1) / n], device=dev)
    torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
    ms = float(tt.item())
    flop = 6.0 * T * (k + 1) * H * I
    tf = flop / (ms / 1e3) / 1e12
    return {"tokens": T, "tokens_per_rank": Tr, "ms_per_layer": round(ms, 4),
            "tokens_per_s": round(T / (ms / 1e3), 1), "algorithmic_tflops": round(tf, 1),
            "mma_tflops_fp4": round(tf * FP4_TERMS, 1),
            "frac_of_fp4_nominal_dense": round(tf * FP4_TERMS / FP4_NOMINAL_TFLOPS, 4),
            "parallelism": f"expert parallel x{world}, strong scaling (NCCL all-to-all)",
            "kernel": "nvmoe_ep_dispatch -> all-to-all -> tcgen05 kind::mxf4nvf4 grouped GEMM "
                      "(pre-routed) -> all-to-all -> nvmoe_ep_combine"}


def pcie_h2d_gbs(dev, nbytes=256 << 20):
    """Pinned host -> device copy bandwidth of this box (one 256 MiB cudaMemcpyAsync, best of 5)."""
    import torch
    src = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    dst = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    best = 0.0
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        dst.copy_(src, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        best = max(best, nbytes / (e0.elapsed_time(e1) / 1e3) / 1e9)
    return best


def run_config3(a, dev, batches=(1, 8, 16), steps=20, warmup=3):
    """The Q2_K 48-layer stack: Qwen3.8 shape, Q2_K weights, dependent layers (RMSNorm + router
    gate in front of each), slot pools of 128 of the 512 experts (25 %), misses refilled from the
    pinned host tier by the FFN (SM copies over PCIe).  Per batch: layer-tokens/s, the refill
    bytes per step and the time those bytes need at this box's pinned H2D bandwidth."""
    import numpy as np
    import torch

    from nvmoe_b200.engine import MoEStack, StackConfig
    from nvmoe_b200.synth import layer_log_bias

    L = a.layers
    cfg = StackConfig(n_layers=L, quant="q2_k")
    stack = MoEStack(cfg, device=dev, seed=30)
    bias = layer_log_bias(L, cfg.n_experts, 1.1, seed=0)
    ranking = np.argsort(-bias, axis=1, kind="stable")
    stack.init_router(logit_bias=bias, seed=31)
    bw = pcie_h2d_gbs(dev)
    per_expert = stack.bytes_per_expert
    res = []
    cap = torch.cuda.Stream(dev)
    for B in batches:
        R = warmup + steps
        g = torch.Generator(device=dev)
        g.manual_seed(3000 + B)
        xs = torch.randn((R, B, cfg.hidden), generator=g, device=dev).to(torch.bfloat16)
        out = torch.empty((B, cfg.hidden), dtype=torch.bfloat16, device=dev)
        stack.forward_chain(xs[0], out)
        torch.cuda.synchronize()
        stack.prewarm(ranking)
        graphs = []
        for r in range(R):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=cap):
                stack.forward_chain(xs[r], out)
            graphs.append(gr)
        plans = stack.chain_buffers(B)["plans"]
        # misses per step: each miss installs a new expert in one slot of its layer (one remap
        # per layer step), so they are the slots whose occupant changed over the step
        miss = np.zeros(R, np.int64)
        for r, gr in enumerate(graphs):
            before = torch.stack([t.real_in_slot for t in stack.tables]).clone()
            gr.replay()
            after = torch.stack([t.real_in_slot for t in stack.tables])
            miss[r] = int((before != after).sum().item())
        stack.prewarm(ranking)
        for i in range(warmup):
            graphs[i].replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(warmup, R):
            graphs[i].replay()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        refill = float(miss[warmup:].mean()) * per_expert
        res.append({"batch": B, "layer_tokens_per_s": round(B * L / (ms / 1e3), 1),
                    "ms_per_step": round(ms, 4), "layer_step_us": round(1e3 * ms / L, 3),
                    "misses_per_step": round(float(miss[warmup:].mean()), 2),
                    "refill_bytes_per_step": round(refill),
                    "refill_pcie_us_per_step": round(refill / (bw * 1e9) * 1e6, 1)})
        del graphs
    del stack
    torch.cuda.empty_cache()
    return {"workload": f"Q2_K {L}-layer stack of dependent layers (RMSNorm + router gate), "
                        "512 experts top-10 + shared, H2048 I512, 128 slots/layer (25 %)",
            "pinned_h2d_gbs": round(bw, 1), "bytes_per_expert": per_expert, "batches": res}


def run_config3_bounded(dev, layers=8, host_frac=0.5, batch=8, steps=10, warmup=3):
    """The Q2_K stack with a bounded host tier: pinned host tiers of host_frac of the experts per
    layer in front of a backing store (pageable host memory standing in for the NVMe tier), the
    host tier placed by the native SLRU from each layer step's miss list read back by the host,
    misses copied by cudaMemcpyAsync on a side stream (copy engine).  Eager, one host read per
    layer step, as the reference's eval_cb; fewer layers than the stack above (its pinned tiers
    are per layer)."""
    import torch

    from nvmoe_b200.engine import StackConfig
    from nvmoe_b200.synth import layer_log_bias
    from nvmoe_b200.tier import BoundedTierStack

    cfg = StackConfig(n_layers=layers, quant="q2_k")
    hs = int(cfg.n_experts * host_frac)
    st = BoundedTierStack(cfg, hs, device=dev, seed=40)
    st.init_router(logit_bias=layer_log_bias(layers, cfg.n_experts, 1.1, seed=0), seed=41)
    g = torch.Generator(device=dev)
    g.manual_seed(4000)
    xs = torch.randn((warmup + steps, batch, cfg.hidden), generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty((batch, cfg.hidden), dtype=torch.bfloat16, device=dev)
    for i in range(warmup):
        st.forward(xs[i], out)
    torch.cuda.synchronize()
    s0 = dict(st.stats)
    t0 = time.perf_counter()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(warmup, warmup + steps):
        st.forward(xs[i], out)
    e1.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    ms = e0.elapsed_time(e1) / steps
    d = {k: st.stats[k] - s0[k] for k in st.stats}
    return {"workload": f"Q2_K {layers}-layer dependent stack, 128 GPU slots and {hs} pinned host "
                        f"slots per layer of 512 experts, batch {batch}",
            "layer_tokens_per_s": round(batch * layers / (ms / 1e3), 1),
            "ms_per_step": round(ms, 3), "host_wall_ms_per_step": round(1e3 * wall / steps, 3),
            "gpu_misses_per_step": round(d["gpu_misses"] / steps, 2),
            "host_hits_per_step": round(d["host_hits"] / steps, 2),
            "backing_loads_per_step": round(d["host_loads"] / steps, 2),
            "refill_bytes_per_step": round(d["refill_bytes"] / steps),
            "refill": "cudaMemcpyAsync per bank on a side stream, event-joined (copy engine)"}


def run_prefill(a, dev, peaks):
    """One Qwen3.8-shaped NVFP4 MoE layer over a.prefill_tokens bf16 tokens (the prefill
    config: 512 experts all resident, top-10 Zipf routing, shared expert) through
    nvmoe_moe_ffn_prefill; device time per layer with CUDA events over 10 launches."""
    import numpy as np
    import torch

    from nvmoe_b200 import ops
    from nvmoe_b200.formats import random_experts
    from nvmoe_b200.synth import layer_log_bias, router_logits
    from nvmoe_b200.engine import StackConfig

    cfg = StackConfig(n_layers=1)
    T, E, k, H, I = a.prefill_tokens, cfg.n_experts, cfg.top_k, cfg.hidden, cfg.inter
    pool = random_experts("nvfp4", E, H, I, seed=11, device=dev)
    shared = random_experts("nvfp4", 1, H, I, seed=12, device=dev)
    rng = np.random.default_rng(7)
    lg = torch.from_numpy(router_logits(T, layer_log_bias(1, E, 1.1, seed=0)[0], rng)).to(dev)
    ids, w = ops.router_topk(lg, k)
    x = torch.randn((T, H), device=dev).to(torch.bfloat16)
    out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    for _ in range(3):
        ops.moe_ffn_prefill(pool, x, ids, w, shared=shared, out=out)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 10
    e0.record()
    for _ in range(n):
        ops.moe_ffn_prefill(pool, x, ids, w, shared=shared, out=out)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / n
    flop = 6.0 * T * (k + 1) * H * I
    tf = flop / (ms / 1e3) / 1e12
    del shared
    fp4 = os.environ.get("NVMOE_PREFILL_KERNEL", "fp4") != "f16"
    # HBM floor of the layer: the distinct experts' banks (+ tokens in, y out)
    n_used = int(torch.unique(ids).numel()) + 1
    floor_bytes = n_used * pool.bytes_per_slot + 2 * T * H * 2
    hbm = peaks["hbm_gbs"] if peaks else 6650.0
    out = {"tokens": T, "ms_per_layer": round(ms, 4), "tokens_per_s": round(T / (ms / 1e3), 1),
           "algorithmic_tflops": round(tf, 1),
           "hbm_floor_ms": round(floor_bytes / (hbm * 1e9) * 1e3, 4),
           "frac_of_hbm_floor": round(floor_bytes / (hbm * 1e9) * 1e3 / ms, 4),
           "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)" if peaks else "fallback"}
    if fp4:
        # the activations enter the MMA as FP4_TERMS residual NVFP4 terms: the tensor cores do
        # FP4_TERMS x the algorithmic products; the FP4 peak is this GPU's measured mxf4nvf4 rate
        # at the kernel's MMA shape (nvmoe_probe_fp4_mma), the nominal 9 PFLOP/s beside it
        mma_tf = tf * FP4_TERMS
        fp4_peak = ops.fp4_mma_tflops(device=dev)
        out.update({"kernel": "tcgen05 kind::mxf4nvf4 block-scaled FP4 grouped GEMM (weights "
                              "unchanged from the slot banks, activations as %d NVFP4 terms)" % FP4_TERMS,
                    "mma_tflops_fp4": round(mma_tf, 1),
                    "fp4_peak_measured_tflops": round(fp4_peak, 1),
                    "frac_of_fp4_measured": round(mma_tf / fp4_peak, 4),
                    "algorithmic_frac_of_fp4_measured": round(tf / fp4_peak, 4),
                    "frac_of_fp4_nominal_dense": round(mma_tf / FP4_NOMINAL_TFLOPS, 4)})
    else:
        out["kernel"] = "tcgen05 kind::f16 grouped GEMM, weights dequantised into tensor memory"
    del pool
    return out


def _traffic_from_profiles(batch):
    """DRAM bytes per ffn_fused launch (dram__bytes_read.sum + dram__bytes_write.sum) from the
    ncu capture of this bench's roofline launches, kept with its command in the profile summary
    profiles/ffn_fused_nvfp4_decode_b<batch>.txt (None when no capture exists for this batch)."""
    p = ROOT / "profiles" / f"ffn_fused_nvfp4_decode_b{batch}.txt"
    if not p.exists():
        return None
    for ln in p.read_text().splitlines():
        if ln.startswith("dram_bytes_per_launch:"):
            try:
                return float(ln.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


# ------------------------------------------------------------------ CPU (oracle port)
def cpu_oracle_sample(batch: int, seconds: float, layers_cap: int = 48):
    """Times the CPU restatement of one layer step (router, remap, dequant + FFN in fp32) on
    this host's cores; returns (layer-tokens/s, cores, description)."""
    import numpy as np
    import torch

    from nvmoe_b200.formats import random_experts
    from nvmoe_b200.synth import layer_log_bias, router_logits
    from oracle import ref_numpy as R
    from oracle.native import OracleLayer

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    E, k, H, I, S = 512, 10, 2048, 512, 128
    rng = np.random.default_rng(0)
    host = random_experts("nvfp4", E, H, I, seed=0)
    shared = random_experts("nvfp4", 1, H, I, seed=2)
    bias = layer_log_bias(1, E, 1.1, seed=0)[0]
    lay = OracleLayer(E, S)
    for e in np.argsort(-bias)[:S]:
        lay.eval(np.array([e], np.int32), is_decode=False)

    def dense(w, which, s):
        m = w.gate_up if which != "down" else w.down
        rows = slice(0, I) if which == "gate" else (slice(I, 2 * I) if which == "up" else slice(None))
        return R.dequant_nvfp4(m.data[s, rows].numpy(), m.scale[s, rows].numpy(), m.glob[s].item())

    done, t_start = 0, time.perf_counter()
    while True:
        lg = router_logits(batch, bias, rng)
        ids, w = R.router_topk_softmax(lg, k)
        lay.eval(ids.reshape(-1), is_decode=True)  # slot bookkeeping; weights come from host
        x = R.f32_to_bf16(rng.standard_normal((batch, H)).astype(np.float32))
        # every expert used by the step (shared one included) is dequantised from its packed
        # bytes, as a CPU implementation of the quantised path has to
        sh = (dense(shared, "gate", 0), dense(shared, "up", 0), dense(shared, "down", 0))
        R.moe_ffn(x, ids, w, lambda s: dense(host, "gate", s), lambda s: dense(host, "up", s),
                  lambda s: dense(host, "down", s), shared=sh)
        done += 1
        el = time.perf_counter() - t_start
        if el >= seconds or done >= layers_cap:
            break
    return batch * done / el, cores, f"{done} layer steps of batch {batch} (oracle port: numpy " \
                                     f"dequant + fp32 FFN, torch/BLAS threads={cores})"


def reference_host_code(batch: int, seconds: float = 1.5, n_expert: int = 512, top_k: int = 10,
                        cache_size: int = 128) -> dict:
    """The reference's own host code for the step this library moves to the device, timed on
    the host cores: eval_cb's remap + host-tier block (scripts/moe_cache_probe.cpp:627-753,
    955-970, compiled from the reference tree into oracle/_ref by oracle/Makefile) over
    Zipf(1.1)-routed decode steps of the benchmark's shape.  Routing is drawn before the timed
    loop; one call per layer step, through a preallocated-buffer binding."""
    import ctypes as C
    import numpy as np
    try:
        from oracle import ref_numpy as R
        from oracle.native import RefEvalCb
        from nvmoe_b200.synth import layer_log_bias, router_logits
        ref = RefEvalCb(n_expert, cache_size, 0, host_cache_size=n_expert)
    except (OSError, ImportError) as e:  # the reference build is not on this machine
        return {"unavailable": f"oracle/_ref not loadable ({type(e).__name__})"}
    rng = np.random.default_rng(17)
    bias = layer_log_bias(1, n_expert, 1.1, seed=0)[0]
    steps = [np.ascontiguousarray(R.router_topk_softmax(router_logits(batch, bias, rng),
                                                         top_k)[0].reshape(-1), np.int32)
             for _ in range(256)]
    n = batch * top_k
    bufs = [np.empty(n, np.int32) for _ in range(7)] + [np.zeros(1, np.int32), np.zeros(1, np.int32)]
    out, hg, hh, li, lg, lh, _, nh, nl = bufs
    fn, h = ref.L.ref_evalcb_step, ref.h
    for ids in steps[:32]:  # warm: the pool fills with the hot experts
        fn(h, ids, batch, top_k, 1, out, hg, hh, nh, li, lg, lh, nl)
    count, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        for ids in steps:
            fn(h, ids, batch, top_k, 1, out, hg, hh, nh, li, lg, lh, nl)
        count += len(steps)
    dt = time.perf_counter() - t0
    return {"eval_cb_remap_us_per_layer_step": round(1e6 * dt / count, 3), "cores": 1,
            "steps": count,
            "what": f"the reference's eval_cb remap + host-tier block (moe_cache_probe.cpp:"
                    f"627-753,955-970) per layer step, {n_expert} experts, top-{top_k}, "
                    f"{cache_size} slots, batch {batch}, one host thread (ctypes call "
                    f"overhead included); on the GPU this step runs inside the decode front "
                    f"kernel"}


def run_reference(a):
    """Reference arm: the CPU implementation of the path (oracle port; the reference's own FFN
    lives in FreeToken / ggml, which are not in the reference tree) on the host cores."""
    per_step = max(0.5, min(3.0, 120.0 / max(1, a.steps + a.warmup)))
    vals = []
    for i in range(a.warmup + a.steps):
        v, cores, desc = cpu_oracle_sample(a.batch, per_step, layers_cap=4)
        if i >= a.warmup:
            vals.append(v)
    value = statistics.median(vals)
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": UNIT,
        "n_gpus": 0, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": round(1e3 * a.batch / value, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (oracle port)",
        "data": "synthetic (seeded)", "config": config_dict(a, 1),
        "cpu_baseline": {"value": round(value, 2), "unit": UNIT, "cores": cores,
                         "kind": "port", "sample": desc,
                         "reference_host_code": reference_host_code(a.batch)},
        "e2e": {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main():
    a = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if a.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(a)), flush=True)
        return
    import torch
    if a.only_prefill:
        dev = torch.device("cuda", local_rank)
        torch.cuda.set_device(dev)
        if rank == 0:
            print(json.dumps({"prefill": run_prefill(a, dev, load_peaks())}), flush=True)
        return
    if world > 1:
        import datetime
        # rank 0's stdout carries exactly one JSON line: no NCCL version banner on it
        if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION"):
            os.environ["NCCL_DEBUG"] = "WARN"
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local_rank))
    if world > 1:
        line = run_ep(a, rank, world, local_rank)
        if a.prefill_tokens > 0:
            line["prefill"] = run_ep_prefill(a, rank, world, local_rank, load_peaks())
    else:
        line = run_nvmoe(a, rank, world, local_rank)
    if rank == 0:
        if not a.no_cpu and world == 1:
            v, cores, desc = cpu_oracle_sample(a.batch, a.cpu_baseline_seconds)
            line["cpu_baseline"] = {"value": round(v, 2), "unit": UNIT, "cores": cores,
                                    "kind": "port", "sample": desc,
                                    "reference_host_code": reference_host_code(a.batch)}
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
