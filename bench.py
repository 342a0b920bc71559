#!/usr/bin/env python
"""MoE expert-layer benchmark on B200: the Qwen3.6-35B-A3B-shaped decode configuration (40 stacked layers, every expert
resident in HBM, IQ3_XXS routed experts + Q8_0 shared expert, T tokens per step).

One step = one decode step through all 40 MoE layers for T tokens (router GEMV + top-8 + grouping + grouped expert
GEMVs + shared expert + gated combine + the next layer's RMS/q8_1), replayed as one CUDA graph.  The metric is
MoE-layer tokens/s (T / mean layer time) with microseconds per layer beside it.  Decode does not shard: with --gpus N
each rank runs its own replica (weak scaling) and `value` sums the replicas.

The same line carries the other configurations as keys: decode_sweep (T = 2, 4, 16), prefill_c2 (Gemma-4-shaped Q4_0
layer, T = 8192) and prefill_c3 (LFM2.5-shaped Q4_K / Q6_K layer, T = 2048) on one GPU, each with its CPU baseline
where one exists, gemma_lfm_decode (the Gemma 4 / LFM2 decode layer, layer by layer and in one launch), and ep_c4
(the Qwen IQ3 layer over T = 65536 tokens, experts sharded over every rank of the run).
--workload selects one of them alone.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--tokens T] [--impl tsb|reference]
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_LAYERS = 40   # --layers changes it for profiling captures only (a smaller device footprint); the bench is 40
# DRAM bytes (read + write) per layer of k_decode_layers at T = 1 from one ncu capture of a 4-layer launch (61.79 MB
# per launch); traffic grows with the layer count, so a launch of N layers moves N times this.
TRAFFIC_PER_LAYER_T1 = (60848896 + 938496) / 4
METRIC = "MoE-layer tokens/s (decode, Qwen3.6-35B-A3B-shaped IQ3_XXS layer, 40 layers resident)"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


class Clocks:
    """nvidia-smi samples during the timed region: median SM clock, max clock, throttle reasons seen."""

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self.proc = None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if len(r) > 3 + i and r[3 + i] == "Active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def reference_arm(args):
    """The reference's own CPU expert path (oracle/_ref) on this host's cores, same metric and config."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    from oracle import oracle as O
    from tinystrata_b200 import synth
    cfg = synth.QWEN
    vals = []
    per = max(3.0, 60.0 / max(1, args.steps + args.warmup))
    for i in range(args.warmup + args.steps):
        r = O.cpu_baseline_decode(cfg, seconds=per, seed=1 + i)
        if i >= args.warmup:
            vals.append(r)
    v = float(np.mean([r["value"] for r in vals]))
    line = {"metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": N_LAYERS * args.tokens / v * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8 dp (q8_1/Q8_K x IQ3_XXS)", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": f"decode T={args.tokens}, 1 layer x 256 IQ3_XXS experts in host memory "
                                   f"(routed experts; the reference runs the shared expert on the GPU)",
                       "model": "qwen3.6-35b-a3b-shaped MoE layer", "tokens": args.tokens},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": vals[0]["cores"], "kind": "reference",
                             "sample": vals[0]["sample"]},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def decode_priors(cfg, T, device):
    """C1 at T > 1: each token's top-8 distinct and disjoint across the step's tokens (T * 8 distinct experts per
    layer).  The routing prior adds 30 to the logits of token t's experts {(8 t + k + 37 l) mod 256} in layer l (the
    natural logits spread about 1 on RMS-normed inputs), through the decode path's logit_prior input; T = 1 routes
    without a prior.  Returns [L][T][E] fp32 or None."""
    import torch
    if T == 1:
        return None
    E, K = cfg["n_expert"], cfg["n_used"]
    pr = torch.zeros((N_LAYERS, T, E), dtype=torch.float32)
    for l in range(N_LAYERS):
        for t in range(T):
            for k in range(K):
                pr[l, t, (t * K + k + 37 * l) % E] = 30.0
    return pr.to(device)


def verify_decode(cfg, D, layers, x0_dev, priors, stream):
    """The fused step checked layer by layer (teacher-forced): layer l of the layer-by-layer entry points (MoELayer,
    whose pieces the GPU parity tests pin to the reference's kernels) runs on the fused step's own input to layer l
    (x after layer l - 1, recorded by the step), and its routing and MoE output (x_l - x_{l-1}) are compared with the
    fused step's.  Tolerance as the layer parity tests: max-abs <= 1e-2 of the output RMS, cosine >= 0.9999."""
    import torch
    import tinystrata_b200 as TS
    T, H = x0_dev.shape
    with torch.cuda.stream(stream):
        x = x0_dev.clone()
        D.forward(x, stream=stream)
    stream.synchronize()
    assert D.error() == 0 and TS.device_error() == 0, D.error_detail
    worst, min_cos, same = 0.0, 1.0, True
    h = torch.empty((T, H), device=x0_dev.device)
    hq = torch.empty((T, H // 32 * 36), dtype=torch.uint8, device=x0_dev.device)
    for l, M in enumerate(layers):
        xin = x0_dev if l == 0 else D.x_rec[l - 1]
        with torch.cuda.stream(stream):
            x1 = xin.clone()
            TS.rms_norm_q8_1(x1, h, hq, stream=stream)
            M.forward(x1, h, hq, stream=stream, prior=priors[l] if priors is not None else None)
        stream.synchronize()
        ref = (x1 - xin).double()
        got = (D.x_rec[l] - xin).double()
        rms = float(ref.pow(2).mean().sqrt())
        err = float((got - ref).abs().max()) / rms
        cos = float((got * ref).sum() / (got.norm() * ref.norm()))
        worst, min_cos = max(worst, err), min(min_cos, cos)
        same &= bool(torch.equal(D.ids[l], M.ids[:T]))
    assert torch.isfinite(D.x_rec).all(), "non-finite layer output"
    return {"layers": len(layers), "max_abs_over_rms": worst, "min_cosine": min_cos, "same_routing": same,
            "teacher_forced": True, "tolerance": {"max_abs_over_rms": 1e-2, "cosine": 0.9999}}


PREFILL_METRIC = "MoE-layer tokens/s (prefill, Gemma-4-26B-A4B-shaped Q4_0 layer, T=8192)"
PREFILL_LFM_METRIC = "MoE-layer tokens/s (prefill, LFM2.5-24B-A2B-shaped Q4_K/Q6_K layer, T=2048)"
# int8 operations per layer of the C2 configuration: 2 T (K 3 H F + 3 H FS) + router 2 T H E (algorithmic: the
# reference's MMQ work, one int8 multiply-add per weight value and routed row, whatever the kernels issue)
def prefill_ops(T, H, F, FS, K, E):
    return 2.0 * T * (K * 3 * H * F + 3 * H * FS) + 2.0 * T * H * E


INT8_SPEC_TOPS = 4500.0   # B200 dense int8 tensor-core rate (NVIDIA's 9 POP/s figure is with 2:4 sparsity)


def prefill_measure(lfm: bool, T: int, steps: int, warmup: int, local: int = 0) -> dict:
    """C2: one Gemma-4-26B-A4B-shaped layer (128 Q4_0 experts, top-8, dense Q4_0 shared FFN 2112, GELU-tanh) over
    T = 8192 prompt tokens; C3 (lfm): one LFM2.5-24B-A2B-shaped layer (64 experts, top-4 by sigmoid, SwiGLU 1792,
    Q4_K gate/up, Q6_K down, no shared expert) over T = 2048 with router logits near N(0, 2): router GEMM, routing,
    q8_1, dispatch, grouped gate/up + down on tcgen05, shared FFN, combine, replayed as one CUDA graph."""
    import torch
    import tinystrata_b200 as TS
    from tinystrata_b200 import synth
    from tinystrata_b200.layer import PrefillLayer

    device = torch.device("cuda", local)
    # C3's router logits N(0, 2): weights of sd 2 / sqrt(H) on RMS-normed inputs
    cfg = dict(synth.LFM, router_sd=2.0 / np.sqrt(synth.LFM["n_embd"])) if lfm else synth.GEMMA
    seed = 3 if lfm else 2
    H, F, FS, K, E = cfg["n_embd"], cfg["n_ff"], cfg["sh_n_ff"], cfg["n_used"], cfg["n_expert"]
    st = synth.device_layers(cfg, 1, seed=seed, device=device)
    escale = None if lfm else torch.ones(E, dtype=torch.float32, device=device)
    P = PrefillLayer(cfg, st["blobs"][0], st["routers"][0], None if lfm else st["sh_blobs"][0], max_tokens=T,
                     escale=escale)
    rng = np.random.default_rng(seed)
    x0 = synth.rms_normed(rng, T, H)
    x0_dev = torch.from_numpy(x0).to(device)
    x0_host = torch.from_numpy(x0).pin_memory()
    out_host = torch.empty((T, H), dtype=torch.float32).pin_memory()
    x = torch.empty_like(x0_dev)
    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        x.copy_(x0_dev)
        P.forward(x, x0_dev, stream=stream)   # eager pass (allocations, kernel attributes)
    stream.synchronize()
    assert TS.device_error() == 0
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        x.copy_(x0_dev)
        P.forward(x, x0_dev, stream=stream)
    ge = torch.cuda.CUDAGraph()   # end to end: host input in, result out, each step
    with torch.cuda.graph(ge, stream=stream):
        x0_dev.copy_(x0_host, non_blocking=True)
        x.copy_(x0_dev)
        P.forward(x, x0_dev, stream=stream)
        out_host.copy_(x, non_blocking=True)

    def timed(gr, n):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(n):
                gr.replay()
            e1.record(stream)
        stream.synchronize()
        return e0.elapsed_time(e1) / n

    timed(g, max(3, warmup))
    with Clocks(local) as clk:
        ms = timed(g, steps)
    ms_e2e = timed(ge, max(3, steps // 2))
    # the grouped gate/up kernel alone (the dominant kernel), CUDA events on its stream
    n = T * K
    with torch.cuda.stream(stream):
        kev = []
        for _ in range(4):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            TS.moe_prefill_gu(P.L, P.blobs, P.stride, P.bounds, E, n, P.xa, cfg["act"], h=P.ha, stream=stream)
            b.record(stream)
            kev.append((a, b))
    stream.synchronize()
    gu_ms = float(np.mean([a.elapsed_time(b) for a, b in kev[1:]]))
    assert TS.device_error() == 0
    ops = prefill_ops(T, H, F, FS, K, E)
    gu_ops = 2.0 * n * 2 * H * F
    bf16_peak = None
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            bf16_peak = float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        pass
    achieved = ops / (ms * 1e-3) / 1e12
    wbytes = int(st["blobs"][0].numel())
    del g, ge
    return {
        "metric": PREFILL_LFM_METRIC if lfm else PREFILL_METRIC, "value": T / (ms * 1e-3), "unit": "tokens/s",
        "n_gpus": 1, "ms_per_step": ms, "us_per_layer": ms * 1e3,
        "dtype": ("q8_1 x " + ("Q4_K / Q6_K" if lfm else "Q4_0") +
                  " exact int32 block sums on tcgen05.mma.kind::i8 (TMA-staged activations), fp32 block scaling"),
        "config": {"workload": f"prefill T={T} through one " +
                               ("LFM2.5-24B-A2B" if lfm else "Gemma-4-26B-A4B") + "-shaped MoE layer",
                   "tokens": T, "hidden": H, "experts": E, "top_k": K, "n_ff": F, "shared_n_ff": FS,
                   "weights": "Q4_K gate/up, Q6_K down" if lfm else "Q4_0",
                   "l2": f"expert weights {wbytes / 1e6:.0f} MB (" +
                         ("larger" if wbytes > 126e6 else "smaller") + " than L2); no flush between steps"},
        "roofline": {"bound": "tensor", "kernel": "k_mmq<gate/up> (grouped gate/up + activation, the top kernel)",
                     "achieved": gu_ops / (gu_ms * 1e-3) / 1e12, "peak": INT8_SPEC_TOPS,
                     "unit": "TOP/s (int8, algorithmic)", "frac": gu_ops / (gu_ms * 1e-3) / 1e12 / INT8_SPEC_TOPS,
                     "peak_kind": "B200 dense int8 spec (4.5 POP/s; no measured int8 peak on this pool)",
                     "traffic": None, "avg_launch_ms": gu_ms, "algorithmic_ops_per_launch": gu_ops,
                     "layer_achieved": achieved, "layer_frac": achieved / INT8_SPEC_TOPS,
                     "layer_frac_of_measured_bf16": achieved / bf16_peak if bf16_peak else None,
                     "algorithmic_ops_per_layer": ops},
        "e2e": {"value": T / (ms_e2e * 1e-3), "unit": "tokens/s", "ms_per_step": ms_e2e,
                "h2d_bytes_per_step": int(x0_host.numel() * 4), "d2h_bytes_per_step": int(out_host.numel() * 4)},
        "gpu_launches_per_step": 11 if not lfm else 8,
        "clocks": clk.summary(),
    }


def prefill_cpu_baseline(lfm: bool) -> dict | None:
    """C2's routed experts through a C restatement of the reference's CPU expert path (gemma4/cpu_experts.cpp:145-235,
    oracle/cpu_experts_port.c) on this host's cores, for about 10 s (None for C3, which has no CPU port)."""
    if lfm:
        return None
    try:
        from oracle import oracle as O
        from tinystrata_b200 import synth
        return O.cpu_baseline_prefill(synth.GEMMA, seconds=10.0)
    except Exception as e:  # the baseline is reported, never required
        return {"value": None, "unit": "tokens/s", "cores": 0, "kind": "port", "sample": f"unavailable: {e}"}


def bench_prefill(args):
    import torch
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    lfm = args.workload == "prefill_lfm"
    r = prefill_measure(lfm, args.tokens, args.steps, args.warmup, local)
    cpu = None
    if not args.no_cpu_baseline:
        cpu = prefill_cpu_baseline(lfm)
    line = dict(r, steps=args.steps, warmup=args.warmup, higher_is_better=True, scaling="weak", vs_baseline=None,
                data="synthetic", cpu_baseline=cpu, gpu_launches=r["gpu_launches_per_step"] * args.steps)
    print(json.dumps(line), flush=True)
    return 0


EP_METRIC = "EP prefill MoE-layer tokens/s (Gemma-4-26B-A4B-shaped Q4_0 layer, T=8192 per GPU, experts sharded)"
EPQ_METRIC = "EP prefill MoE-layer tokens/s (Qwen3.6-35B-A3B-shaped IQ3_XXS/IQ3_S layer, T=65536, experts sharded)"


def ep_qwen_measure(args, steps: int, warmup: int, micro_batches: int = 2, bf16: bool = False,
                    own_group: bool = True) -> dict | None:
    """C4: the Qwen3.6-35B-A3B-shaped layer (256 experts, IQ3_XXS gate/up, IQ3_S down, top-8 softmax, Q8_0 shared
    expert gated by a sigmoid of the 257th router row) over T = 65536 prompt tokens split evenly over the ranks
    (strong scaling), experts sharded 256 / N per GPU in cyclic placement (expert e on rank e % N: the skewed head
    spreads over the ranks), router logits skewed by a Zipf(1.1) prior over the experts (log p_e added to expert
    e's logit) so that the expert load is imbalanced.  Per step: router GEMM, routing, q8_1, the device expert-parallel
    path (tsb_ep_dispatch: plan, pack, counts exchange -- the step's one host synchronisation -- and the micro-batched
    dispatch exchanges over NCCL; the shared expert on a second stream meanwhile; tsb_ep_combine: local experts on the
    tensor cores per micro-batch, partial rows back, the rank-ordered gated sum).  Timed with CUDA events between
    barriers, max over ranks.  Returns rank 0's result (None on the other ranks)."""
    import datetime
    import torch
    import torch.distributed as dist
    import tinystrata_b200 as TS
    from tinystrata_b200 import synth
    from tinystrata_b200.ep import ExpertParallel

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if own_group:
        if ws > 1:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
        else:
            import tempfile
            dist.init_process_group("gloo", init_method="file://" + tempfile.mktemp(), rank=0, world_size=1)
    cfg = synth.QWEN_EP
    T_all = 65536
    T = T_all // ws
    H, F, FS, K, E = cfg["n_embd"], cfg["n_ff"], cfg["sh_n_ff"], cfg["n_used"], cfg["n_expert"]
    per = E // ws
    st = synth.device_layers(cfg, 1, seed=4, device=device)   # every rank draws the same layer, keeps its experts
    blobs = st["blobs"][0][rank::ws].contiguous()
    router, sh = st["routers"][0], st["sh_blobs"][0]
    del st
    L = TS.native_expert_layout(cfg["gu_type"], cfg["d_type"], H, F)
    Ls = TS.native_expert_layout(cfg["sh_gu_type"], cfg["sh_d_type"], H, FS)
    zipf = torch.tensor(-1.1 * np.log(np.arange(1, E + 1)), dtype=torch.float32, device=device)
    x0_np = synth.rms_normed(np.random.default_rng(4 + rank), T, H)
    x0 = torch.from_numpy(x0_np).to(device)
    ep = ExpertParallel(L, blobs, int(L.bytes), E, K, cfg["act"], max_tokens=T, cyclic=True)
    logits = torch.empty((T, E + 1), dtype=torch.float32, device=device)
    ids = torch.empty((T, K), dtype=torch.int32, device=device)
    w = torch.empty((T, K), dtype=torch.float32, device=device)
    xq = torch.empty((T, H // 32 * 36), dtype=torch.uint8, device=device)
    xs = TS.MmqAct(T, H, device)
    hs = TS.MmqAct(T, FS, device)
    shared = torch.empty((T, H), dtype=torch.float32, device=device)
    out = torch.empty((T, H), dtype=torch.float32, device=device)
    main = torch.cuda.current_stream(device)
    side = torch.cuda.Stream(device)

    def step(x):
        TS.router_logits_f32(router, x, logits, ld=E + 1)       # [T, E + 1]: the experts, then the shared gate
        logits[:, :E].add_(zipf)
        TS.native_router_topk(logits, K, E, ids, w)             # softmax top-8, renormalised (the Qwen router)
        TS.quantize_q8_1_rows(x, xq)
        ready = torch.cuda.Event()
        ready.record(main)
        side.wait_event(ready)
        with torch.cuda.stream(side):                            # the shared expert while the rows travel
            TS.mmq_quantize(x, out=xs, stream=side)
            TS.moe_prefill_gu(Ls, sh, 0, None, 1, T, xs, cfg["act"], h=hs, stream=side)
            TS.moe_prefill_down(Ls, sh, 0, None, 1, T, hs, out=shared, stream=side)
        done = torch.cuda.Event()
        done.record(side)
        ep.dispatch(xq, ids, w, micro_batches=micro_batches)
        main.wait_event(done)
        ep.combine(out, accumulate=False, shared=shared, sgate=logits[:, E:], sg_stride=E + 1, bf16=bf16)
        return out

    for _ in range(max(3, warmup)):
        step(x0)
    ep.synchronize()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        e0.record(main)
        for _ in range(steps):
            step(x0)
        e1.record(main)
        ep.synchronize()   # bounded: a peer that stops answering ends the run with an error, not a hang
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    # end to end: the step's tokens from pinned host memory, the layer output back, every step
    x_host = torch.from_numpy(x0_np).pin_memory()
    o_host = torch.empty((T, H), dtype=torch.float32).pin_memory()
    xin = torch.empty_like(x0)
    dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(main)
    for _ in range(max(2, steps // 2)):
        xin.copy_(x_host, non_blocking=True)
        step(xin)
        o_host.copy_(out, non_blocking=True)
    b.record(main)
    ep.synchronize()
    torch.cuda.synchronize()
    ms_e2e = a.elapsed_time(b) / max(2, steps // 2)
    stats = ep.stats()
    t = torch.tensor([ms, ms_e2e, float(stats["picks"])], device=device)
    if ws > 1:
        dist.all_reduce(t[:2], op=dist.ReduceOp.MAX)
    ms, ms_e2e = float(t[0]), float(t[1])
    ep.close()
    assert TS.device_error() == 0
    res = None
    if rank == 0:
        ops = prefill_ops(T_all, H, F, FS, K, E + 1)
        res = {
            "metric": EPQ_METRIC, "value": T_all / (ms * 1e-3), "unit": "tokens/s", "n_gpus": ws,
            "steps": steps, "warmup": warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": "q8_1 x IQ3_XXS / IQ3_S / Q8_0 exact integer block dots on tcgen05, fp32 block scaling",
            "data": "synthetic (Zipf(1.1)-skewed router logits)",
            "config": {"workload": f"expert-parallel prefill, {T_all} tokens over {ws} GPU(s), {per} of {E} "
                                   "experts per GPU", "tokens": T_all, "tokens_per_gpu": T, "experts_per_gpu": per,
                       "placement": "cyclic (expert e on rank e % N)", "parallelism": f"ep{ws}",
                       "micro_batches": micro_batches, "return": "bf16" if bf16 else "fp32",
                       "collectives": "NCCL send/recv on the library's communicator (counts; q8_1 rows, local "
                                      "picks, weights; partial rows back), one host synchronisation per step"},
            "us_per_layer": ms * 1e3,
            "rank0_rows": stats,
            "roofline": {"bound": "tensor", "achieved": ops / (ms * 1e-3) / 1e12 / ws, "unit": "TOP/s per GPU",
                         "peak": INT8_SPEC_TOPS, "frac": ops / (ms * 1e-3) / 1e12 / ws / INT8_SPEC_TOPS,
                         "peak_kind": "B200 dense int8 spec (4.5 POP/s); no measured int8 peak",
                         "note": "int8-op/s, algorithmic"},
            "e2e": {"value": T_all / (ms_e2e * 1e-3), "unit": "tokens/s", "ms_per_step": ms_e2e,
                    "h2d_bytes_per_step": int(x_host.numel() * 4) * ws,
                    "d2h_bytes_per_step": int(o_host.numel() * 4) * ws},
            "clocks": clk.summary(),
        }
    if own_group:
        dist.destroy_process_group()
    return res


def bench_ep_qwen(args):
    res = ep_qwen_measure(args, args.steps, args.warmup)
    if res is not None:
        print(json.dumps(res), flush=True)
    return 0


def bench_ep(args):
    """Expert-parallel prefill: the C2 layer's 128 experts sharded 128/N per GPU, T tokens per GPU (weak scaling);
    per step every rank routes its tokens, the dispatch / return all-to-alls run over NCCL, the local experts on the
    tensor cores, the dense shared FFN on the rank's own tokens.  Eager (host-synchronising counts), timed with CUDA
    events between barriers, max over ranks."""
    import datetime
    import torch
    import torch.distributed as dist
    import tinystrata_b200 as TS
    from tinystrata_b200 import synth
    from tinystrata_b200.ep import ep_forward, gpu_expert_fn

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    else:
        import tempfile
        dist.init_process_group("nccl", init_method="file://" + tempfile.mktemp(), rank=0, world_size=1,
                                device_id=device)
    cfg = synth.GEMMA
    T, H, F, FS, K, E = args.tokens, cfg["n_embd"], cfg["n_ff"], cfg["sh_n_ff"], cfg["n_used"], cfg["n_expert"]
    per = E // ws
    st = synth.device_layers(cfg, 1, seed=2, device=device)   # every rank draws the same layer, keeps its slice
    blobs = st["blobs"][0][rank * per:(rank + 1) * per].contiguous()
    router, sh = st["routers"][0], st["sh_blobs"][0]
    del st
    L = TS.native_expert_layout(cfg["gu_type"], cfg["d_type"], H, F)
    Ls = TS.native_expert_layout(cfg["sh_gu_type"], cfg["sh_d_type"], H, FS)
    escale = torch.ones(E, dtype=torch.float32, device=device)
    x0 = torch.from_numpy(synth.rms_normed(np.random.default_rng(2 + rank), T, H)).to(device)
    fn = gpu_expert_fn(L, blobs, int(L.bytes), cfg["act"])

    def step():
        logits = TS.router_logits_f32(router, x0)
        ids, w = TS.route_rows(logits, K, 0, cfg["in_scale"], None, escale, True, 0.0)
        xq = TS.quantize_q8_1_rows(x0)
        out = ep_forward(xq, ids, w, E, H, fn)
        hs = TS.moe_prefill_gu(Ls, sh, 0, None, 1, T, TS.mmq_quantize(x0), cfg["act"])
        shared = TS.moe_prefill_down(Ls, sh, 0, None, 1, T, hs)
        return out.add_(shared)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    t = torch.tensor([ms], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    assert TS.device_error() == 0
    if rank == 0:
        ops = prefill_ops(T, H, F, FS, K, E) * ws
        line = {
            "metric": EP_METRIC, "value": ws * T / (ms * 1e-3), "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "q8_1 x Q4_0 exact block dots on tcgen05, fp32 block scaling",
            "data": "synthetic",
            "config": {"workload": f"expert-parallel prefill, {T} tokens per GPU, {per} of {E} experts per GPU",
                       "tokens_per_gpu": T, "experts_per_gpu": per, "parallelism": f"ep{ws}",
                       "collectives": "NCCL all_to_all_single (counts, q8_1 rows, picks; fp32 partial rows back)"},
            "us_per_layer": ms * 1e3,
            "roofline": {"bound": "tensor", "achieved": ops / (ms * 1e-3) / 1e12 / ws, "unit": "TFLOP/s per GPU",
                         "note": "int8-op/s, algorithmic"},
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    dist.destroy_process_group()
    return 0


def act_decode_measure(device, steps: int = 30, warmup: int = 5) -> dict:
    """The Gemma 4 and LFM2 decode MoE layer (one layer, every expert resident) at T = 1 and 4: the layer-by-layer
    entry points (route_rows, grouping, grouped experts, moe_sum, the dense shared MLP) and the one-launch block
    (tsb_moe_decode_act), each as a CUDA graph with the input's q8_1, a new token per step and L2 flushed (a 256 MB
    write) between steps; CUDA events around each replay.  The two paths' outputs are compared bit for bit first."""
    import torch
    import tinystrata_b200 as TS
    from tinystrata_b200 import synth

    res = {}
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    s = torch.cuda.Stream(device)
    for name, cfg in (("gemma", synth.GEMMA), ("lfm", synth.LFM)):
        st = synth.device_layers(cfg, 1, seed=31, device=device)
        H, E, K = cfg["n_embd"], cfg["n_expert"], cfg["n_used"]
        kw = ({"escale": torch.ones(E, device=device)} if cfg["router_mode"] == "softmax_scaled"
              else {"bias": torch.zeros(E, device=device)})
        sh = st["sh_blobs"][0] if cfg.get("sh_n_ff") else None
        blob_bytes = int(st["blobs"].shape[-1])
        sh_bytes = int(sh.numel()) if sh is not None else 0
        for T in (1, 4):
            M = TS.MoELayer(cfg, st["blobs"][0], st["routers"][0], sh, max_tokens=T, **kw)
            n_in = warmup + steps
            rng = np.random.default_rng(T)
            xs = torch.from_numpy(np.stack([synth.rms_normed(rng, T, H) for _ in range(n_in)])).to(device)
            hd = torch.empty((T, H), device=device)
            hq = torch.empty((T, H // 32 * 36), dtype=torch.uint8, device=device)
            x = torch.zeros((T, H), device=device)
            # bit-for-bit check of the two paths on the first input
            hd.copy_(xs[0])
            TS.quantize_q8_1_rows(hd, hq)
            xa, xb = torch.zeros_like(x), torch.zeros_like(x)
            M.forward(xa, hd, hq)
            M.forward_fused(xb, hd, hq)
            torch.cuda.synchronize()
            same = bool(torch.equal(xa, xb))
            out = {"bitwise_equal": same}
            for path in ("layerwise", "fused"):
                fwd = M.forward if path == "layerwise" else M.forward_fused
                with torch.cuda.stream(s):
                    TS.quantize_q8_1_rows(hd, hq, stream=s)
                    fwd(x, hd, hq, stream=s)
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    TS.quantize_q8_1_rows(hd, hq, stream=s)
                    fwd(x, hd, hq, stream=s)
                times, bytes_ = [], []
                for i in range(n_in):
                    with torch.cuda.stream(s):
                        hd.copy_(xs[i])
                        flush.fill_(i & 255)
                        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        a.record(s)
                        g.replay()
                        b.record(s)
                    torch.cuda.synchronize()
                    if i >= warmup:
                        times.append(a.elapsed_time(b) * 1e3)
                        n_dist = len(np.unique(M.ids[:T].cpu().numpy()))
                        bytes_.append(E * H * 4 + n_dist * blob_bytes + sh_bytes)
                del g
                us = float(np.mean(times))
                out[f"{path}_us_per_layer"] = us
                if path == "fused":
                    out["fused_hbm_gbs"] = float(np.mean(bytes_)) / (us * 1e-6) / 1e9
                    out["algorithmic_bytes_per_layer"] = float(np.mean(bytes_))
            assert TS.device_error() == 0
            res[f"{name}_T{T}"] = out
        del st
    return res


def bench_staged(args):
    """Host-staged experts: one Qwen-shaped decode layer (256 IQ3_XXS experts) whose experts all sit in pinned host
    memory, 64 of them in HBM slots; T tokens a step.  The layer-by-layer step (router, top-8, staged grouping with the
    missed experts pulled over the host link by the GPU, experts, shared expert, combine) as a CUDA graph, timed
    beside the same step on the resident layer, and the grouping + fetch alone (CUDA events on its stream) for the
    host-link rate.  Per step a new token: its picks miss the slots about 3 times in 4."""
    import torch
    import tinystrata_b200 as TS
    from tinystrata_b200 import synth
    from tinystrata_b200.layer import MoELayer, StagedExperts

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    cfg = synth.QWEN
    T, H, K, E = args.tokens, cfg["n_embd"], cfg["n_used"], cfg["n_expert"]
    n_slots = 64
    st = synth.device_layers(cfg, 1, seed=5, device=device)
    blobs, router, sh = st["blobs"][0], st["routers"][0], st["sh_blobs"][0]
    nb = blobs.shape[1]
    stride = (nb + 15) // 16 * 16
    host = torch.zeros((E, stride), dtype=torch.uint8).pin_memory()
    host[:, :nb].copy_(blobs.cpu())
    S = StagedExperts(host, nb, n_slots, T * K, device)
    R = MoELayer(cfg, blobs, router, sh, max_tokens=T)
    M = MoELayer(cfg, None, router, sh, max_tokens=T, staged=S)
    n_in = args.steps + args.warmup
    rng = np.random.default_rng(5)
    xs_all = torch.from_numpy(np.stack([synth.rms_normed(rng, T, H) for _ in range(n_in)])).to(device)
    hd = torch.empty((T, H), device=device)
    hq = torch.empty((T, H // 32 * 36), dtype=torch.uint8, device=device)
    x = torch.zeros((T, H), device=device)
    s = torch.cuda.Stream()
    graphs = {}
    for name, layer in (("staged", M), ("resident", R)):
        with torch.cuda.stream(s):
            hd.copy_(xs_all[0])
            TS.quantize_q8_1_rows(hd, hq, stream=s)
            layer.forward(x, hd, hq, stream=s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            TS.quantize_q8_1_rows(hd, hq, stream=s)
            layer.forward(x, hd, hq, stream=s)
        graphs[name] = g
    res = {}
    with Clocks(0) as clk:
        for name in ("staged", "resident"):
            g = graphs[name]
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n_in)]
            with torch.cuda.stream(s):
                for i in range(n_in):
                    hd.copy_(xs_all[i])
                    evs[i][0].record(s)
                    g.replay()
                    evs[i][1].record(s)
            torch.cuda.synchronize()
            res[name] = float(np.mean([a.elapsed_time(b) for a, b in evs[args.warmup:]])) * 1e3
        # the grouping + fetch alone, on the routing of each step's token
        fetch_us, fetched = [], 0
        for i in range(n_in):
            with torch.cuda.stream(s):
                hd.copy_(xs_all[i])
                TS.quantize_q8_1_rows(hd, hq, stream=s)
                M.forward(x, hd, hq, stream=s)
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(s)
                S.group(M.ids[:T], M.groups, stream=s)
                b.record(s)
            torch.cuda.synchronize()
            if i >= args.warmup:
                fetch_us.append(a.elapsed_time(b) * 1e3)
                fetched += sum(1 for e in np.unique(M.ids[:T].cpu().numpy()) if S.slot_of[e] < 0)
    assert TS.device_error() == 0
    f_us = float(np.mean(fetch_us))
    per_step = fetched / args.steps
    line = {
        "metric": "staged decode layer time", "value": res["staged"], "unit": "us per layer", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": False, "dtype": "q8_1 x IQ3_XXS",
        "data": "synthetic",
        "config": {"workload": f"decode T={T}, one Qwen3.6-shaped layer, 256 IQ3_XXS experts in pinned host memory, "
                               f"{n_slots} in HBM slots", "slots": n_slots, "tokens": T},
        "resident_us_per_layer": res["resident"],
        "fetch": {"us_per_step": f_us, "experts_per_step": per_step, "blob_bytes": int(nb),
                  "host_link_GBps": per_step * nb / (f_us * 1e-6) / 1e9},
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--impl", default="tsb", choices=["tsb", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true", help="only the headline token count (profiling captures)")
    ap.add_argument("--no-extras", action="store_true",
                    help="decode only: without the C2 / C3 prefill and C4 expert-parallel keys")
    ap.add_argument("--layers", type=int, default=40, help="profiling captures only: fewer resident layers")
    ap.add_argument("--trace", action="store_true", help="print the fused kernel's per-phase timeline (stderr)")
    ap.add_argument("--workload", default="decode",
                    choices=["decode", "prefill", "prefill_lfm", "ep", "ep_qwen", "staged", "decode_act"],
                    help="decode: the headline C1 line; prefill: the C2 Gemma-shaped prefill layer (--tokens 8192); "
                         "prefill_lfm: the C3 LFM2-shaped layer (--tokens 2048); ep: the C2 layer expert-parallel "
                         "over the launched ranks; ep_qwen: the C4 Qwen IQ3 layer expert-parallel (65536 tokens); "
                         "staged: a decode layer with its experts in host memory, 64 of 256 in HBM slots; "
                         "decode_act: the Gemma 4 / LFM2 decode layer, layer by layer and in one launch")
    args = ap.parse_args()
    if args.workload == "staged":
        return bench_staged(args)
    if args.workload == "decode_act":
        import torch
        torch.cuda.set_device(0)
        with Clocks(0) as clk:
            r = act_decode_measure(torch.device("cuda", 0), args.steps, args.warmup)
        print(json.dumps({"workload": "gemma / lfm decode layer", **r, "clocks": clk.summary()}), flush=True)
        return 0
    if args.workload == "ep_qwen":
        return bench_ep_qwen(args)
    if args.workload in ("prefill", "prefill_lfm", "ep"):
        if args.tokens == 1:
            args.tokens = 2048 if args.workload == "prefill_lfm" else 8192
        return bench_prefill(args) if args.workload != "ep" else bench_ep(args)
    global N_LAYERS
    N_LAYERS = args.layers
    if args.impl == "reference":
        return reference_arm(args)
    return bench_decode(args)


def bench_decode(args):
    """C1: the Qwen-shaped decode step through 40 resident layers (the headline line), at T = args.tokens, plus the
    other C1 token counts (2, 4, 16) as extra keys.  Every configuration is verified layer by layer before it is
    timed; a broken tolerance or routing ends the run with an error instead of a number."""
    import torch
    import torch.distributed as dist
    import tinystrata_b200 as TS
    from tinystrata_b200 import synth

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if ws > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)

    def barrier():
        if ws > 1:
            dist.barrier()

    def max_over_ranks(v):
        if ws > 1:
            t = torch.tensor([v], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())
        return v

    cfg = synth.QWEN
    H, K, E = cfg["n_embd"], cfg["n_used"], cfg["n_expert"]
    st = synth.device_layers(cfg, N_LAYERS, 1, device)
    layers = [TS.MoELayer(cfg, st["blobs"][l], st["routers"][l], st["sh_blobs"][l], max_tokens=16)
              for l in range(N_LAYERS)]
    x_c1 = synth.rms_normed(np.random.default_rng(1), 16, H)   # C1 inputs: RMS-normed N(0, 1), seed 1
    stream = torch.cuda.Stream(device)
    L0, Ls = layers[0].L, layers[0].Ls
    peak, peak_kind = peaks()

    def timed(g, n):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(n):
                g.replay()
            e1.record(stream)
        stream.synchronize()
        return e0.elapsed_time(e1) / n

    def point(T, headline):
        priors = decode_priors(cfg, T, device)
        x0_dev = torch.from_numpy(x_c1[:T].copy()).to(device)
        Dv = TS.DecodeStack(cfg, st["blobs"], st["routers"], st["sh_blobs"], n_tok=T, priors=priors, record_x=True)
        check = verify_decode(cfg, Dv, layers, x0_dev, priors, stream)
        del Dv
        if not (check["same_routing"] and check["max_abs_over_rms"] <= 1e-2 and check["min_cosine"] >= 0.9999):
            raise SystemExit(f"decode T={T}: the fused step does not match the layer-by-layer path: {check}")
        D = TS.DecodeStack(cfg, st["blobs"], st["routers"], st["sh_blobs"], n_tok=T, priors=priors)
        x = torch.empty((T, H), device=device)
        with torch.cuda.stream(stream):
            x.copy_(x0_dev)
            D.forward(x, stream=stream)
        stream.synchronize()
        distinct = [int(torch.unique(D.ids[l]).numel()) for l in range(N_LAYERS)]
        bytes_layer = [d * L0.bytes + Ls.bytes + (E + 1) * H * 4 for d in distinct]
        if headline and args.trace:   # per-phase timeline of the fused kernel (mean / max over CTAs, us from start)
            with torch.cuda.stream(stream):
                x.copy_(x0_dev)
            stream.synchronize()
            tr = D.trace(x, stream=stream).double()
            names = ["start", "P0", "P1", "routed", "sh_q", "P2", "hq", "P3", "end", "logits_in", "topk", "-", "-"]
            rows = []
            for l in range(1, N_LAYERS):
                t0 = tr[l, 0].min()
                rows.append([((tr[l, e] - t0) / 1e3).mean().item() for e in range(13)] +
                            [((tr[l, e] - t0) / 1e3).max().item() for e in range(13)])
            m = np.array(rows).mean(0)
            print("phase (us from layer start): " + "  ".join(f"{n}={m[i]:.2f}/{m[13 + i]:.2f}" for i, n in
                                                            enumerate(names)), file=sys.stderr, flush=True)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                x.copy_(x0_dev)
                D.forward(x, stream=stream)
        stream.synchronize()
        timed(g, max(3, args.warmup))
        barrier()
        torch.cuda.synchronize()
        clk = Clocks(local) if headline else None
        if clk:
            clk.__enter__()
        ms = timed(g, args.steps)
        if clk:
            clk.__exit__()
        torch.cuda.synchronize()
        barrier()
        assert D.error() == 0 and TS.device_error() == 0
        ms = max_over_ranks(ms)
        us_layer = ms * 1e3 / N_LAYERS
        res = {"tokens": T, "us_per_layer": us_layer, "tokens_per_s": ws * T / (us_layer * 1e-6),
               "ms_per_step": ms, "distinct_experts_per_layer": float(np.mean(distinct)),
               "layer_algorithmic_bytes": float(np.mean(bytes_layer)),
               "hbm_frac": float(np.mean(bytes_layer)) / (us_layer * 1e-6) / 1e9 / peak, "verify": check}
        if not headline:
            del g
            return res
        res["clocks"] = clk.summary()
        # end to end through the public API: pinned host x in, the fused step, x back to the host, every step
        x0_host = torch.from_numpy(x_c1[:T].copy()).pin_memory()
        out_host = torch.empty((T, H), dtype=torch.float32).pin_memory()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(args.steps):
                x.copy_(x0_host, non_blocking=True)
                D.forward(x, stream=stream)
                out_host.copy_(x, non_blocking=True)
            e1.record(stream)
        stream.synchronize()
        barrier()
        ms_e2e = max_over_ranks(e0.elapsed_time(e1) / args.steps)
        res["e2e"] = {"value": ws * T / (ms_e2e * 1e3 / N_LAYERS * 1e-6), "unit": "tokens/s", "ms_per_step": ms_e2e,
                      "h2d_bytes_per_step": int(x0_host.numel() * 4), "d2h_bytes_per_step": int(out_host.numel() * 4)}
        # the dominant (and only) kernel alone, CUDA events on its stream: k_decode_layers over the 40 layers
        kms = []
        with torch.cuda.stream(stream):
            for rep in range(4):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                x.copy_(x0_dev)
                a.record(stream)
                D.forward(x, stream=stream)
                b.record(stream)
                kms.append((a, b))
        stream.synchronize()
        k_avg_ms = float(np.mean([a.elapsed_time(b) for a, b in kms[1:]]))
        k_bytes = float(np.sum(bytes_layer))
        k_gbs = k_bytes / (k_avg_ms * 1e-3) / 1e9
        res["roofline"] = {"bound": "hbm", "kernel": "k_decode_layers (fused decode step, 40 layers)",
                           "achieved": k_gbs, "peak": peak, "unit": "GB/s", "frac": k_gbs / peak, "peak_kind": peak_kind,
                           "traffic": TRAFFIC_PER_LAYER_T1 * N_LAYERS if T == 1 else None,
                           "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of a 4-layer capture of "
                                             "k_decode_layers, scaled to the launch's layers" if T == 1 else None,
                           "algorithmic_bytes_per_launch": k_bytes, "avg_launch_ms": k_avg_ms}

        def layerwise_step():
            x.copy_(x0_dev)
            h = torch.empty((T, H), device=device)
            hq = torch.empty((T, H // 32 * 36), dtype=torch.uint8, device=device)
            TS.rms_norm_q8_1(x, h, hq, stream=stream)
            for l, M in enumerate(layers):
                M.forward(x, h, hq, h_next=h, hq_next=hq, stream=stream,
                          prior=priors[l] if priors is not None else None)

        gl = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(gl, stream=stream):
                layerwise_step()
        stream.synchronize()
        res["layerwise_us_per_layer"] = timed(gl, max(3, args.steps // 2)) * 1e3 / N_LAYERS
        del g, gl
        return res

    T = args.tokens
    head = point(T, headline=True)
    sweep = {}
    if not args.no_sweep:
        for Tx in (1, 2, 4, 16):
            if Tx != T:
                r = point(Tx, headline=False)
                sweep[f"T={Tx}"] = {k: r[k] for k in ("us_per_layer", "tokens_per_s", "hbm_frac",
                                                      "distinct_experts_per_layer", "layer_algorithmic_bytes")}
                sweep[f"T={Tx}"]["verify"] = {k: r["verify"][k] for k in ("max_abs_over_rms", "min_cosine",
                                                                         "same_routing")}
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        try:
            from oracle import oracle as O
            cpu = O.cpu_baseline_decode(cfg, seconds=10.0)
        except Exception as e:  # the baseline is reported, never required
            cpu = {"value": None, "unit": "tokens/s", "cores": 0, "kind": "reference", "sample": f"unavailable: {e}"}

    # the other headline configurations as extra keys: C2 / C3 prefill (one GPU) and C4 expert-parallel prefill
    # (every rank of the run, the sharded configuration)
    extras = {}
    if not args.no_extras:
        if ws == 1:
            for key, lfm, T_p in (("prefill_c2", False, 8192), ("prefill_c3", True, 2048)):
                r = prefill_measure(lfm, T_p, 10, 3, local)
                r["cpu_baseline"] = None if args.no_cpu_baseline else prefill_cpu_baseline(lfm)
                extras[key] = {k: r[k] for k in ("metric", "value", "unit", "us_per_layer", "ms_per_step", "dtype",
                                                 "config", "roofline", "e2e", "clocks", "cpu_baseline")}
                extras[key]["gpu_launches"] = r["gpu_launches_per_step"] * 10
            try:   # a failure here is recorded in the line; the headline does not depend on it
                extras["gemma_lfm_decode"] = act_decode_measure(device)
            except Exception as e:  # noqa: BLE001
                extras["gemma_lfm_decode"] = {"error": f"{type(e).__name__}: {e}"}
        r = ep_qwen_measure(args, 5, 3, own_group=(ws == 1))
        if r is not None:
            extras["ep_c4"] = {k: r[k] for k in ("metric", "value", "unit", "n_gpus", "us_per_layer", "ms_per_step",
                                                 "scaling", "config", "roofline", "e2e", "clocks", "rank0_rows")}

    if rank == 0:
        line = {
            "metric": METRIC, "value": head["tokens_per_s"], "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8 dp4a (q8_1 x IQ3_XXS / Q8_0), fp32 accumulate", "data": "synthetic",
            "config": {"workload": f"decode T={T} through 40 resident Qwen3.6-35B-A3B-shaped MoE layers",
                       "model": "qwen3.6-35b-a3b-shaped MoE layer x40", "tokens_per_step": T, "layers": N_LAYERS,
                       "hidden": H, "experts": E, "top_k": K, "n_ff": cfg["n_ff"], "routed": "IQ3_XXS",
                       "shared": "Q8_0", "parallelism": f"replicas x{ws}",
                       "inputs": "RMS-normed N(0,1), seed 1" + ("" if T == 1 else "; routing prior: disjoint experts"),
                       "distinct_experts_per_layer": head["distinct_experts_per_layer"],
                       "l2": "inputs larger than L2 (12.3 GB of expert weights, 40 distinct layers per step)"},
            "us_per_layer": head["us_per_layer"],
            "layer_hbm_gbs": head["layer_algorithmic_bytes"] / (head["us_per_layer"] * 1e-6) / 1e9,
            "layerwise_us_per_layer": head["layerwise_us_per_layer"],
            "verify": head["verify"],
            "roofline": head["roofline"],
            "e2e": head["e2e"],
            "gpu_launches": args.steps,   # one k_decode_layers per step
            "clocks": head["clocks"],
            "cpu_baseline": cpu,
            "decode_sweep": sweep,
            **extras,
        }
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
