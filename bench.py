#!/usr/bin/env python3
"""Benchmark of the routed-MoE hot path (BASELINE metric: routed-MoE tokens/s/layer).

Workload: Qwen3.6-35B-A3B MoE block, batch-1 decode, q4 expert
packs, k = 8 of 256, bf16 router / shared expert / gate vector, x bf16 [1, 2048].
One step = one decode token through the MoE blocks of all 40 layers (40 layer calls,
each with its own resident weights and its own input row). 40 layers x 256 experts of
q4 packs (18.1 GB) stay resident in HBM; each layer call reads its 8 routed experts
plus router and shared expert (21.5 MB), so a step touches ~860 MB, far above the
126 MB L2 (no flush needed; said in `config`).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  python bench.py --workload batched --tokens T     (T tokens a call)
  python bench.py --workload lm_head [--lm-dtypes q4,bf16]   (LM head alone)

ours: `value` = layer calls / s with inputs resident in HBM (CUDA graph of the 40
calls, timed with CUDA events, max over ranks); `e2e` = the same metric through the C
ABI with pinned host inputs copied in and outputs read back every step.
reference: the CPU restatement of the reference's block (oracle, OpenMP over all
host cores) on a bounded sample of the same workload.
N > 1: batch-1 decode does not shard (one token); each rank runs an independent
replica on its own GPU ("replicas only"), value = all ranks' layer calls / max time.

--workload batched (config 2): T tokens [T, 2048] bf16 through the MoE block of each
of --layers resident layers per step (nmoe_moe_forward_batched: routing, expert-order
permutation, tcgen05 grouped GEMMs with in-TMEM dequant, combine); value = tokens/s/layer.

--workload decode_step (config 3): the whole 40-layer decode step (nmoe_decoder_step:
embedding, attention layers with their q4 projections, MoE blocks, LM head), tokens/s;
the default run (N = 1) adds it to its line as `decode_step`.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "nano-metal-moe-qwen36_b200")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

METRIC = "routed-MoE tokens/s/layer (batch-1 decode)"
UNIT = "tokens/s/layer"
HIDDEN, INTER, EXPERTS = 2048, 512, 256
FALLBACK_HBM_GBS = 6650.0


def algorithmic_bytes(bits: int, k: int, router_dtype: int, shared_dtype: int, x_bytes: int = 2) -> int:
    """Bytes one batch-1 layer call must move: k expert packs + router + shared expert +
    gate vector + x in + out (fp32)."""
    esz = {4: 1769472, 2: 983040}[bits]
    bf16 = 1
    router = 256 * 2048 * 2 if router_dtype == bf16 else 256 * 1024 + 2 * 256 * 32 * 2
    shared = 3 * 512 * 2048 * 2 if shared_dtype == bf16 else 3 * (512 * 1024 + 2 * 512 * 32 * 2)
    gvec = 2048 * 2 if shared_dtype == bf16 else 1024 + 2 * 32 * 2
    return k * esz + router + shared + gvec + 2048 * x_bytes + 2048 * 4


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.dev), "-lms", "100"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic(name: str):
    """dram read+write bytes per launch recorded from ncu in profiles/<name>.md
    (line 'traffic_bytes_per_launch: N'), or None."""
    p = os.path.join(REPO, "profiles", name + ".md")
    try:
        for ln in open(p):
            if ln.startswith("traffic_bytes_per_launch:"):
                return int(float(ln.split(":", 1)[1].strip()))
    except Exception:
        pass
    return None


# ------------------------------------------------------------------ workload ----

def host_llc_bytes() -> int:
    try:
        v = open("/sys/devices/system/cpu/cpu0/cache/index3/size").read().strip()
        return int(v[:-1]) * 1024 if v.endswith("K") else int(v[:-1]) * 2**20 if v.endswith("M") else int(v)
    except Exception:
        return 0


def routing_mass_top20(logits: np.ndarray, k: int) -> float:
    """Share of the renormalised top-k routing mass (softmax -> top-k -> renormalise, per
    token) that the 20% most-used experts (51 of 256) receive over the sampled tokens."""
    z = logits - logits.max(axis=1, keepdims=True)
    top = np.argpartition(-z, k - 1, axis=1)[:, :k]
    p = np.exp(np.take_along_axis(z, top, axis=1))
    p /= p.sum(axis=1, keepdims=True)
    mass = np.zeros(logits.shape[1])
    np.add.at(mass, top.ravel(), p.ravel())
    return float(np.sort(mass)[::-1][: int(0.2 * logits.shape[1])].sum() / mass.sum())


def calibrate_router_skew(router_bf16: np.ndarray, k: int, seed: int, tokens: int = 1024):
    """Config 1's skewed router: logits = x . W_r + b_e, with a seeded per-expert
    log-popularity b_e = sigma * z_e (z ~ N(0,1)); sigma is bisected so that over `tokens`
    sampled x ~ N(0,1) the top 20% of experts receive 80% +- 1% of the renormalised routing
    mass. The bias enters the kernels as router column 2047, with x[2047] = 1."""
    from oracle import oracle as O
    rng = np.random.default_rng(seed + 77)
    z = rng.standard_normal(EXPERTS).astype(np.float32)
    x = O.bf16_to_f32(O.f32_to_bf16(rng.standard_normal((tokens, HIDDEN), dtype=np.float32)))
    x[:, HIDDEN - 1] = 1.0
    w = O.bf16_to_f32(router_bf16).astype(np.float32)
    w[:, HIDDEN - 1] = 0.0
    base = x @ w.T
    lo, hi, sigma, mass = 0.0, 64.0, 0.0, 0.0
    for _ in range(60):
        sigma = 0.5 * (lo + hi)
        b = O.bf16_to_f32(O.f32_to_bf16(sigma * z))
        mass = routing_mass_top20(base + b[None, :], k)
        if abs(mass - 0.8) <= 0.005:
            break
        lo, hi = (sigma, hi) if mass < 0.8 else (lo, sigma)
    b16 = O.f32_to_bf16(sigma * z)
    return b16, {"bias_sigma": sigma, "tau": 1.0, "top20_mass": mass, "tokens": tokens, "k": k,
                 "rule": "logits = x.W_r + b_e, b_e = sigma*z_e (seeded), x[2047] = 1 carries b_e"}


def build_workload(num_layers: int, bits: int, k: int, router_dtype: int, shared_dtype: int, pool: int, seed: int,
                   skew: bool = False):
    """Seeded synthetic layers: `pool` distinct q4 experts quantised by the restated
    convert_qwen36.py quantiser, placed in the 256 slots of each layer with a per-layer
    rotation (each layer's 256 slots are a separate copy in memory); per-layer bf16
    router / shared weights ~N(0, 0.02). skew: config 1's calibrated router skew
    (calibrate_router_skew) on every layer; returns (layers, xs, calibration)."""
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    esz = O.expert_size(bits)
    packs = np.stack([O.pack_expert(O.randn_bf16(rng, (1024, 2048), 0.02), O.randn_bf16(rng, (2048, 512), 0.02), bits)
                      for _ in range(pool)])
    layers = []
    for l in range(num_layers):
        order = (np.arange(EXPERTS) * 7 + l * 13) % pool
        experts = packs[order].reshape(-1)
        dense = {}
        for name, shape, dt in (("router", (256, 2048), router_dtype), ("shared_gate", (512, 2048), shared_dtype),
                                ("shared_up", (512, 2048), shared_dtype), ("shared_down", (2048, 512), shared_dtype),
                                ("shared_gate_vec", (1, 2048), shared_dtype)):
            w = O.randn_bf16(rng, shape, 0.02)
            if dt == 1:
                dense[name] = {"dtype": 1, "weight": w}
            else:
                p_, s_, b_ = O.quantize_rows(w, 4)
                dense[name] = {"dtype": 4, "weight": p_, "scales": s_, "biases": b_}
        layers.append(O.LayerWeights(bits, experts, EXPERTS, dense["router"], dense["shared_gate"],
                                     dense["shared_up"], dense["shared_down"], dense["shared_gate_vec"]))
    xs = O.f32_to_bf16(rng.standard_normal((num_layers, HIDDEN), dtype=np.float32))
    calib = None
    if skew:
        if router_dtype != 1:
            raise ValueError("the router skew is defined on the bf16 router")
        bias, calib = calibrate_router_skew(layers[0].router["weight"], k, seed)
        for lw in layers:
            r = lw.router["weight"].copy()
            r[:, HIDDEN - 1] = bias
            lw.router = {"dtype": 1, "weight": r}
        xs[:, HIDDEN - 1] = O.f32_to_bf16(np.ones(1, np.float32))[0]
        # the mass with the bias as the kernels see it (bf16 column, x[2047] = 1), fresh tokens
        xt = O.bf16_to_f32(O.f32_to_bf16(np.random.default_rng(seed + 78).standard_normal((1024, HIDDEN),
                                                                                       dtype=np.float32)))
        xt[:, HIDDEN - 1] = 1.0
        calib["top20_mass_checked"] = routing_mass_top20(xt @ O.bf16_to_f32(layers[0].router["weight"]).T, k)
    return layers, xs, calib


CPU_LAYERS = 8   # layers the CPU sample rotates over: 8 x 453 MB of expert slots >> host LLC


def cpu_sample(layers, xs, k, seconds: float):
    """The oracle's block forward (all host threads) over batch-1 calls rotating through
    `layers` (each with its own 256 expert slots in memory, so that the working set is far
    above the host's last-level cache), for about `seconds`. Returns (calls/s, threads,
    calls, seconds). The GPU arm's cpu_baseline and the reference arm both use it."""
    from oracle import oracle as O
    L = O.lib()
    n, t0 = 0, time.perf_counter()
    while True:
        l = n % len(layers)
        O.block_forward(layers[l], k, O.bf16_to_f32(xs[l % xs.shape[0]]))
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds and n >= 3:
            break
    return n / el, L.orc_get_threads(), n, el


def cpu_sample_text(n_layers, n, el, bits, k):
    llc = host_llc_bytes()
    return (f"{n} batch-1 layer calls in {el:.1f}s rotating over {n_layers} layers (q{bits}, k={k}, each layer "
            f"its own 256 expert slots: {n_layers * 256 * (1769472 if bits == 4 else 983040) / 2**20:.0f} MiB of "
            f"expert memory; host LLC {llc / 2**20:.0f} MiB), oracle port of the reference block, OpenMP")


# ---------------------------------------------------------------- reference ----

def run_reference(args, rank, world):
    if rank != 0:
        return None
    from oracle import oracle as O
    O.build()
    n_layers = CPU_LAYERS
    skew = args.bits == 2
    layers, xs, calib = build_workload(n_layers, args.bits, args.k, 1, 1, pool=args.pool, seed=args.seed, skew=skew)
    k = args.k

    def step():   # one step = one call per layer, as in the GPU arm's step over its layers
        for l in range(n_layers):
            O.block_forward(layers[l], k, O.bf16_to_f32(xs[l]))

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    calls = args.steps * n_layers
    value = calls / el
    cores = O.lib().orc_get_threads()
    res = {
        "metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded bf16 ~N(0,0.02) weights quantised by the reference quantiser rule)",
        "config": {"workload": workload_name(args.bits, n_layers, k), "layers": n_layers, "k": k,
                   "step": f"{n_layers} layer calls (one token through {n_layers} MoE blocks)"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": cpu_sample_text(n_layers, calls, el, args.bits, k)},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if calib is not None:
        res["config"]["router_skew"] = calib
    return res


def workload_name(bits, L, k):
    return (f"config{0 if bits == 4 else 1} batch-1 decode: {L} layers x 256 q{bits} experts resident, k={k}, "
            "bf16 router/shared/gate-vector, x bf16 [1,2048]"
            + ("; router skewed (top 20% of experts get 80% of routing mass)" if bits == 2 else ""))


# ------------------------------------------------------------------ batched ----

def batched_flops(T: int, k: int) -> float:
    """Algorithmic FLOPs of one T-token block: routed gate/up/down for k experts per
    token, the shared expert, the router."""
    return 2.0 * T * (k * 3 * INTER * HIDDEN + 3 * INTER * HIDDEN + EXPERTS * HIDDEN)


def run_batched(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import nmoe_b200 as N
    from oracle import oracle as O

    dev = local_rank
    torch.cuda.set_device(dev)
    bits, k, rdt, sdt = 4, 8, N.DTYPE_BF16, N.DTYPE_BF16
    T, L = args.tokens, args.batched_layers
    # one model on every rank: with expert parallelism each rank holds a slice of it
    layers, _, _ = build_workload(L, bits, k, rdt, sdt, pool=args.pool, seed=args.seed)
    uid = None
    if world > 1:   # experts sharded 256/world per rank, tokens exchanged by NCCL
        obj = [N.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        uid = obj[0]
    ctx = N.Context(quant_bits=bits, num_layers=L, router_dtype=rdt, shared_dtype=sdt, t_max=T, device=dev,
                    world_size=world, rank=rank, nccl_unique_id=uid)
    for l, lw in enumerate(layers):
        ctx.load_layer(l, lw.experts)
        ctx.set_dense(l, lw.router, lw.shared_gate, lw.shared_up, lw.shared_down, lw.shared_gate_vec)
    cpu_layer = layers[0]
    for lw in layers[1:]:
        lw.experts = None
    rng = np.random.default_rng(args.seed + 7)
    x_h = O.f32_to_bf16(np.random.default_rng(args.seed + 7 + 1000 * rank).standard_normal((T, HIDDEN),
                                                                                           dtype=np.float32))
    x = torch.from_numpy(x_h.view(np.int16)).to(f"cuda:{dev}")
    outs = torch.zeros((L, T, HIDDEN), dtype=torch.float32, device=f"cuda:{dev}")
    idx = torch.zeros((T, 8), dtype=torch.int32, device=f"cuda:{dev}")
    stream = torch.cuda.Stream(device=dev)

    def step(s):
        for l in range(L):
            ctx.forward_batched(l, T, k, x, outs[l], idx_out=idx if l == 0 else None, stream=s)

    with torch.cuda.stream(stream):
        step(stream.cuda_stream)
    stream.synchronize()
    rc, code = ctx.device_status()
    if rc != N.OK:
        raise RuntimeError(f"device error word {code} after the first step")
    distinct = int(np.unique(idx.cpu().numpy()[:, :k]).size)
    if world == 1:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step(torch.cuda.current_stream().cuda_stream)
        run_step = graph.replay
    else:   # the count exchange synchronises the host each call: no graph
        def run_step():
            step(stream.cuda_stream)
    for _ in range(max(args.warmup, 3)):
        run_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(dev)
    clocks.start()
    time.sleep(0.3)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(args.steps):
            run_step()
    ev1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        tm = torch.tensor([ms], dtype=torch.float64, device=f"cuda:{dev}")
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        ms = float(tm.item())
    per_call_s = ms / 1e3 / (args.steps * L)
    value = world * T / per_call_s

    # e2e: pinned host tokens in, outputs read back, every step, through the C ABI
    x_pin = torch.from_numpy(x_h.view(np.int16)).pin_memory()
    out_pin = torch.zeros((L, T, HIDDEN), dtype=torch.float32).pin_memory()
    e2e_steps = max(1, args.steps // 4)

    def step_e2e():
        with torch.cuda.stream(stream):
            x.copy_(x_pin, non_blocking=True)
            step(stream.cuda_stream)
            out_pin.copy_(outs, non_blocking=True)
        stream.synchronize()

    for _ in range(2):
        step_e2e()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        step_e2e()
    e2e_el = time.perf_counter() - t0
    if world > 1:
        te = torch.tensor([e2e_el], dtype=torch.float64, device=f"cuda:{dev}")
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_el = float(te.item())
    e2e_value = world * e2e_steps * L * T / e2e_el

    # correctness of the timed outputs: a sample of layer-0 tokens against the oracle on
    # the GPU's own logits
    sample = list(range(0, T, max(1, T // 8)))[:8]
    ctx.forward_batched(0, T, k, x, outs[0])
    torch.cuda.synchronize()
    lg = ctx.debug_logits(T)
    got = outs[0].cpu().numpy()
    errs = []
    for t in sample:
        ref = O.block_forward(cpu_layer, k, O.bf16_to_f32(x_h[t]), logits_override=lg[t])
        errs.append(float(np.linalg.norm(got[t] - ref["out"]) / np.linalg.norm(ref["out"])))
    rel = max(errs)
    if rel > 1e-2:
        raise RuntimeError(f"timed output disagrees with the oracle: rel_l2={rel}")

    esz = {4: 1769472, 2: 983040}[bits]
    dense = algorithmic_bytes(bits, 0, rdt, sdt) - HIDDEN * 2 - HIDDEN * 4
    abytes = distinct * esz + dense + T * HIDDEN * (2 + 4)
    flops = batched_flops(T, k)
    hbm, hbm_kind = peaks()
    try:
        tf = float(json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))["bf16_tflops"])
        tf_kind = "measured"
    except Exception:
        tf, tf_kind = 1590.0, "fallback"
    gbs = abytes / per_call_s / 1e9
    tfs = flops / per_call_s / 1e12
    if gbs / hbm >= tfs / tf:
        roof = {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                "peak_kind": hbm_kind, "algorithmic_bytes_per_launch": abytes}
    else:
        roof = {"bound": "tensor", "achieved": tfs, "peak": tf, "unit": "TFLOP/s", "frac": tfs / tf,
                "peak_kind": tf_kind, "algorithmic_flops_per_launch": flops}
    roof["traffic"] = profiled_traffic(f"batched_block_T{T}")
    roof["other_bound"] = {"hbm_frac": gbs / hbm, "tensor_frac": tfs / tf}
    cpu = None
    if rank == 0 and world == 1:
        n_cpu = min(T, 8)
        t0 = time.perf_counter()
        O.block_forward_batched(cpu_layer, k, O.bf16_to_f32(x_h[:n_cpu]))
        cel = time.perf_counter() - t0
        cpu = {"value": n_cpu / cel, "unit": "tokens/s/layer", "cores": O.lib().orc_get_threads(), "kind": "port",
               "sample": f"{n_cpu} tokens of the same block (oracle, OpenMP over tokens) in {cel:.2f}s"}
    result = {
        "metric": "routed-MoE tokens/s/layer (batched)", "value": value, "unit": "tokens/s/layer", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16 operands (q4 dequantised in TMEM), f32 accumulate",
        "data": "synthetic (seeded bf16 ~N(0,0.02) weights quantised by the reference quantiser rule; "
                f"{args.pool} distinct expert packs placed in 256 slots per layer; x ~N(0,1) bf16)",
        "config": {"workload": f"config2 batched MoE block, T={T}, q4 experts, k=8, bf16 router/shared",
                   "tokens": T, "tokens_per_rank": T, "layers": L, "distinct_experts_routed": distinct,
                   "parallelism": f"expert parallel: {EXPERTS // world} experts per GPU, NCCL all-to-all-v dispatch "
                                  "and combine" if world > 1 else "single GPU",
                   "l2": "weights of a step exceed L2 (each layer's experts are separate HBM copies)",
                   "timing": "CUDA graph of one step (all layers), CUDA events" if world == 1 else
                             "CUDA events around the step loop, max over ranks"},
        "roofline": roof,
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": "tokens/s/layer", "h2d_bytes_per_step": T * HIDDEN * 2,
                "d2h_bytes_per_step": L * T * HIDDEN * 4},
        "gpu_launches": args.steps * L * 9,
        "clocks": clk,
        "check": {"rel_l2_max_sample": rel, "tokens_checked": len(sample)},
    }
    ctx.close()
    return result if rank == 0 else None


# ---------------------------------------------------------------------- ours ----

def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import nmoe_b200 as N
    from oracle import oracle as O

    dev = local_rank
    torch.cuda.set_device(dev)
    bits, k, rdt, sdt = args.bits, args.k, N.DTYPE_BF16, N.DTYPE_BF16
    L = args.layers
    layers, xs_h, calib = build_workload(L, bits, k, rdt, sdt, pool=args.pool, seed=args.seed + rank, skew=bits == 2)
    flags = N.FLAG_PREFETCH_NEXT_LAYER if args.prefetch else 0
    ctx = N.Context(quant_bits=bits, num_layers=L, router_dtype=rdt, shared_dtype=sdt, device=dev, flags=flags)
    for l, lw in enumerate(layers):
        ctx.load_layer(l, lw.experts)
        ctx.set_dense(l, lw.router, lw.shared_gate, lw.shared_up, lw.shared_down, lw.shared_gate_vec)
    cpu_layers = layers[:CPU_LAYERS]
    fp32_layers = layers[:CPU_LAYERS]
    for lw in layers[CPU_LAYERS:]:
        lw.experts = None
    del layers

    xs = torch.from_numpy(xs_h.view(np.int16)).to(f"cuda:{dev}")
    outs = torch.zeros((L, HIDDEN), dtype=torch.float32, device=f"cuda:{dev}")
    stream = torch.cuda.Stream(device=dev)

    def step_direct(s):
        for l in range(L):
            ctx.forward(l, k, xs[l], outs[l], x_dtype=N.DTYPE_BF16, stream=s)

    # correctness gate on this box before timing: layer 0 against the oracle
    with torch.cuda.stream(stream):
        step_direct(stream.cuda_stream)
    stream.synchronize()
    rc, code = ctx.device_status()
    if rc != N.OK:
        raise RuntimeError(f"device error word {code} after the first step")

    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step_direct(torch.cuda.current_stream().cuda_stream)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    clocks = ClockSampler(dev)
    clocks.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(args.steps):
            graph.replay()
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    t = torch.tensor([ms], dtype=torch.float64, device=f"cuda:{dev}")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    calls = args.steps * L * world
    value = calls / (ms_max / 1e3)

    # e2e: public C ABI, pinned host inputs in, outputs read back, every step
    xs_pin = torch.from_numpy(xs_h.view(np.int16)).pin_memory()
    out_pin = torch.zeros((L, HIDDEN), dtype=torch.float32).pin_memory()
    e2e_steps = max(1, args.steps // 4)

    def step_e2e():
        with torch.cuda.stream(stream):
            xs.copy_(xs_pin, non_blocking=True)
            step_direct(stream.cuda_stream)
            out_pin.copy_(outs, non_blocking=True)
        stream.synchronize()

    for _ in range(3):
        step_e2e()
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        step_e2e()
    e2e_el = time.perf_counter() - t0
    te = torch.tensor([e2e_el], dtype=torch.float64, device=f"cuda:{dev}")
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = e2e_steps * L * world / float(te.item())

    # the fp32 routed-expert path (NMOE_FLAG_EXPERT_FP32), timed the same way on the first
    # CPU_LAYERS layers, reported beside the default half2 path
    fp32 = None
    if rank == 0:
        L8 = len(fp32_layers)
        cf = N.Context(quant_bits=bits, num_layers=L8, router_dtype=rdt, shared_dtype=sdt, device=dev,
                       flags=N.FLAG_EXPERT_FP32)
        for l, lw in enumerate(fp32_layers):
            cf.load_layer(l, lw.experts)
            cf.set_dense(l, lw.router, lw.shared_gate, lw.shared_up, lw.shared_down, lw.shared_gate_vec)
        outs_f = torch.zeros((L8, HIDDEN), dtype=torch.float32, device=f"cuda:{dev}")   # keeps `outs` the timed path's
        gf = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gf, stream=stream):
            for l in range(L8):
                cf.forward(l, k, xs[l], outs_f[l], x_dtype=N.DTYPE_BF16, stream=torch.cuda.current_stream().cuda_stream)
        for _ in range(3):
            gf.replay()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = max(5, args.steps)
        f0.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(reps):
                gf.replay()
        f1.record(stream)
        torch.cuda.synchronize()
        fms = f0.elapsed_time(f1)
        fp32 = {"value": reps * L8 / (fms / 1e3), "unit": UNIT, "layers": L8,
                "dtype": "fp32 products and accumulation (q weights, fp32 x and activations)"}
        del gf
        cf.close()

    # correctness of the timed outputs (layer 0 vs oracle, using the GPU's own routing)
    lg = torch.zeros(256, dtype=torch.float32, device=f"cuda:{dev}")
    ctx.route(0, k, xs[0], x_dtype=N.DTYPE_BF16, logits_out=lg)
    torch.cuda.synchronize()
    ref = O.block_forward(cpu_layers[0], k, O.bf16_to_f32(xs_h[0]), logits_override=lg.cpu().numpy())
    got = outs[0].cpu().numpy()
    rel = float(np.linalg.norm(got - ref["out"]) / np.linalg.norm(ref["out"]))
    if rel > 1e-2:
        raise RuntimeError(f"timed output disagrees with the oracle: rel_l2={rel}")

    result = None
    if rank == 0:
        per_launch_s = ms_max / 1e3 / (args.steps * L)
        abytes = algorithmic_bytes(bits, k, rdt, sdt)
        pk, pk_kind = peaks()
        achieved = abytes / per_launch_s / 1e9
        launches_per_call = 1   # one persistent kernel per layer call
        cpu = None
        if world == 1:
            v, cores, n, el = cpu_sample(cpu_layers, xs_h, k, args.cpu_seconds)
            cpu = {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
                   "sample": cpu_sample_text(len(cpu_layers), n, el, bits, k)}
        result = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": (f"routed experts: q{bits} weights x fp16-scaled x / activations, half2 partial sums over "
                      f"{4 if bits == 4 else 8} products flushed to fp32; router, shared expert, combine fp32"),
            "data": "synthetic (seeded bf16 ~N(0,0.02) weights quantised by the reference quantiser rule; "
                    f"{args.pool} distinct expert packs placed in 256 slots per layer)",
            "config": {"workload": workload_name(bits, L, k),
                       "layers": L, "k": k, "step": f"{L} layer calls (one token through {L} MoE blocks)",
                       "l2": f"inputs larger than L2: a step reads {L * abytes / 1e6:.0f} MB of weights "
                             f"({L} layers x {abytes / 1e6:.1f} MB) against a 126 MB L2; no flush",
                       "parallelism": "replicas only" if world > 1 else "single GPU",
                       "timing": "CUDA graph of one step, CUDA events, max over ranks",
                       "next_layer_prefetch": bool(args.prefetch)},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk, "unit": "GB/s", "frac": achieved / pk,
                         "peak_kind": pk_kind, "algorithmic_bytes_per_launch": abytes,
                         "traffic": profiled_traffic("decode_fused_cfg0") if (bits, k) == (4, 8) else None,
                         "traffic_source": "ncu dram__bytes_read+write of this kernel on this config, copied from "
                                           "profiles/decode_fused_cfg0.md (not measured in this run)"},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": L * HIDDEN * 2,
                    "d2h_bytes_per_step": L * HIDDEN * 4},
            "gpu_launches": args.steps * L * launches_per_call,
            "clocks": clk,
            "check": {"rel_l2_layer0": rel},
            "expert_fp32_path": fp32,
        }
        if calib is not None:
            result["config"]["router_skew"] = calib
    ctx.close()
    del outs, xs, cpu_layers, fp32_layers   # host copies of 8 layers' experts (3.6 GB)
    torch.cuda.empty_cache()
    if args.lm_head and rank == 0:
        result["lm_head"] = run_lm_head(args, dev)
        result["layer_crc32c"] = run_crc(args, dev)
        result["linear_attn"] = run_linear_attn(args, dev)
        result["full_attn"] = run_full_attn(args, dev)
        if world == 1:   # config 3 beside the per-layer line: 60 graphed steps
            try:
                result["decode_step"] = run_decode_step(argparse.Namespace(**{**vars(args), "steps": 60,
                                                                               "warmup": 5}), dev)
            except Exception as e:   # reported, never fatal to the headline line
                result["decode_step"] = {"error": f"{type(e).__name__}: {e}"}
            torch.cuda.empty_cache()
    if args.ep_tokens > 0:
        ep = run_ep_batched(args, rank, world, dev)
        if result is not None:
            result["ep_batched"] = ep
    return result


LM_VOCAB = 248320   # src/runtime.m:1911


def lm_head_bytes(dtype: int, vocab: int = LM_VOCAB) -> int:
    """Algorithmic bytes of one token-only LM head call: every weight byte once, plus x and
    the RMSNorm weight (the token is 4 bytes)."""
    per_row = HIDDEN // 2 + 2 * (HIDDEN // 64) * 2 if dtype == 4 else HIDDEN * 2
    return vocab * per_row + HIDDEN * 4 + HIDDEN * 2


def run_lm_head(args, dev):
    """The LM head (final RMSNorm + 248,320-row GEMV + top-1, one launch) at the reference's
    vocab, q4 (the reference's lm_head) and bf16: device time per call (CUDA graph of calls,
    each reading 0.29 / 1.02 GB, above L2), roofline against measured HBM, the oracle's time
    for one call on the host cores, and a parity check of one call against the oracle."""
    import torch
    import nmoe_b200 as N
    from oracle import oracle as O
    out = {}
    rng = np.random.default_rng(args.seed + 77)
    xh = rng.standard_normal(HIDDEN).astype(np.float32)
    nw = O.f32_to_bf16(rng.standard_normal(HIDDEN).astype(np.float32) * 0.1)
    pk, pk_kind = peaks()
    stream = torch.cuda.Stream(device=dev)
    want = [t.strip() for t in args.lm_dtypes.split(",")]
    for dt, name in ((N.DTYPE_Q4, "q4"), (N.DTYPE_BF16, "bf16")):
        if name not in want:
            continue
        head = O.make_lm_head(args.seed + 5, LM_VOCAB, dt)
        d = {"weight": torch.from_numpy(head.weight.view(np.int32) if dt == N.DTYPE_Q4 else head.weight.view(np.int16))
             .to(f"cuda:{dev}")}
        if dt == N.DTYPE_Q4:
            d["scales"] = torch.from_numpy(head.scales.view(np.int16)).to(f"cuda:{dev}")
            d["biases"] = torch.from_numpy(head.biases.view(np.int16)).to(f"cuda:{dev}")
        x = torch.from_numpy(xh).to(f"cuda:{dev}")
        nwd = torch.from_numpy(nw.view(np.int16)).to(f"cuda:{dev}")
        tok = torch.zeros(1, dtype=torch.int32, device=f"cuda:{dev}")
        ws = torch.zeros(N.lm_head_workspace_bytes() // 8, dtype=torch.int64, device=f"cuda:{dev}")
        lg = torch.empty(LM_VOCAB, dtype=torch.float32, device=f"cuda:{dev}")
        # parity of one call (logits requested) against the oracle
        N.lm_head_argmax(d, dt, LM_VOCAB, x, tok, ws, norm_weight=nwd, logits_out=lg, stream=stream.cuda_stream)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        otok, ol = O.lm_head_argmax(head, xh, nw)
        cpu_s = time.perf_counter() - t0
        glg = lg.cpu().numpy()
        err = float(np.abs(glg - ol).max() / np.abs(ol).max())
        gtok = int(tok.item())
        if err > 3e-6 or gtok != O.argmax_top1(glg):
            raise RuntimeError(f"lm head {name} disagrees with the oracle: rel err {err}, token {gtok} vs {otok}")
        reps = 20
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for _ in range(reps):
                N.lm_head_argmax(d, dt, LM_VOCAB, x, tok, ws, norm_weight=nwd,
                                 stream=torch.cuda.current_stream().cuda_stream)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_rep = 10
        e0.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(n_rep):
                g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (n_rep * reps)
        ab = lm_head_bytes(dt)
        ach = ab / (us * 1e-6) / 1e9
        out[name] = {"us_per_call": us, "calls_per_s": 1e6 / us, "token": gtok, "oracle_token": otok,
                     "logits_max_rel_err": err,
                     "roofline": {"bound": "hbm", "achieved": ach, "peak": pk, "unit": "GB/s", "frac": ach / pk,
                                  "peak_kind": pk_kind, "algorithmic_bytes_per_launch": ab},
                     "cpu_oracle_ms_per_call": cpu_s * 1e3, "cpu_oracle_threads": O.lib().orc_get_threads()}
        del g, d, x, lg, head
        torch.cuda.empty_cache()
    out["config"] = {"vocab": LM_VOCAB, "in_dim": HIDDEN, "norm": "model.norm RMSNorm fused (eps 1e-6, w+1)",
                     "timing": "CUDA graph of 20 token-only calls x 10 replays, CUDA events; weights above L2"}
    return out


def run_crc(args, dev):
    """Device CRC-32C of one q4 layer image (256 expert blobs, 453 MB, in HBM) against the
    host CRC-32C (SSE4.2, one core) of the same bytes; both checked against each other."""
    import torch
    import nmoe_b200 as N
    from oracle import oracle as O
    lw = O.make_layer(args.seed + 9, bits=4, distinct_experts=8)
    img = lw.experts.view(np.uint8)
    esz = N.expert_size(4)
    d = torch.from_numpy(img.view(np.int32)).to(f"cuda:{dev}")
    out = torch.zeros(256, dtype=torch.int32, device=f"cuda:{dev}")
    st = torch.cuda.Stream(device=dev)
    for _ in range(3):
        N.crc32c_device(d, esz, 256, out, stream=st.cuda_stream)
    torch.cuda.synchronize()
    reps = 10
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        N.crc32c_device(d, esz, 256, out, stream=st.cuda_stream)
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    t0 = time.perf_counter()
    host = N.expert_crcs(img, 4)
    host_s = time.perf_counter() - t0
    dev_crc = out.cpu().numpy().view(np.uint32)
    if not np.array_equal(dev_crc, host):
        raise RuntimeError("device CRC-32C disagrees with the host")
    pk, pk_kind = peaks()
    gbs = img.nbytes / (ms * 1e-3) / 1e9
    return {"bytes": int(img.nbytes), "device_ms": ms, "device_gbs": gbs, "frac_of_hbm": gbs / pk,
            "peak_kind": pk_kind, "host_sse42_one_core_ms": host_s * 1e3,
            "host_gbs": img.nbytes / host_s / 1e9,
            "note": "load-time integrity check (nmoe_moe_load_layer_checked), not on the decode path"}


def linear_attn_bytes() -> int:
    """Algorithmic bytes of one linear-attention step: the recurrent state read and written
    (32 x 128 x 128 f32), the conv state read and written, conv weights, qkv, z, out, and the
    per-head vectors."""
    state = 32 * 128 * 128 * 4
    conv = 3 * 8192 * 4
    return 2 * state + 2 * conv + 8192 * 4 * 2 + 8192 * 4 + 4096 * 4 * 2 + 32 * 4 * 3 + 32 * 2 + 128 * 2


def run_linear_attn(args, dev):
    """GatedDeltaNet decode-step core (nmoe_linear_attn_step) over 64 layers' states (134 MB,
    above L2): device time per call against the HBM roofline, and the oracle on the host."""
    import torch
    import nmoe_b200 as N
    from oracle import oracle as O
    L = 64
    w = O.make_linear_attn(args.seed + 11)
    dw = {k: torch.from_numpy(v.view(np.int16) if v.dtype == np.uint16 else v).to(f"cuda:{dev}") for k, v in w.items()}
    rng = np.random.default_rng(args.seed + 12)
    inp = O.linear_attn_inputs(rng)
    di = {k: torch.from_numpy(v).to(f"cuda:{dev}") for k, v in inp.items()}
    conv = torch.zeros((L, 3, 8192), device=f"cuda:{dev}")
    S = torch.zeros((L, 32, 128, 128), device=f"cuda:{dev}")
    out = torch.zeros(4096, device=f"cuda:{dev}")
    st = torch.cuda.Stream(device=dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for l in range(L):
            N.linear_attn_step(dw, di["qkv"], di["z"], di["alpha"], di["beta"], conv[l], S[l], out,
                               stream=torch.cuda.current_stream().cuda_stream)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    reps = 20
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    with torch.cuda.stream(st):
        for _ in range(reps):
            g.replay()
    e1.record(st)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * L)
    hc, hs = np.zeros((3, 8192), np.float32), np.zeros((32, 128, 128), np.float32)
    t0 = time.perf_counter()
    n = 0
    while time.perf_counter() - t0 < 1.0:
        O.linear_attn_step(w, inp, hc, hs)
        n += 1
    cpu_us = (time.perf_counter() - t0) / n * 1e6
    ab = linear_attn_bytes()
    pk, pk_kind = peaks()
    ach = ab / (us * 1e-6) / 1e9
    return {"us_per_call": us, "calls_per_s": 1e6 / us,
            "roofline": {"bound": "hbm", "achieved": ach, "peak": pk, "unit": "GB/s", "frac": ach / pk,
                         "peak_kind": pk_kind, "algorithmic_bytes_per_launch": ab},
            "cpu_oracle_us_per_call": cpu_us, "cpu_oracle_threads": 1,
            "config": {"layers_cycled": L, "state_bytes": L * (32 * 128 * 128 + 3 * 8192) * 4,
                       "timing": "CUDA graph of 64 calls (one per layer state) x 20 replays, CUDA events; "
                                 "states above L2"}}


def run_full_attn(args, dev):
    """Full-attention decode step (nmoe_full_attn_step) at positions 4095 and 32767: device
    time per call (CUDA graph of 20 calls x 5 replays), bytes = the K and V rows read plus
    the new rows written, against HBM; the oracle's time at position 4095 on one core."""
    import torch
    import nmoe_b200 as N
    from oracle import oracle as O
    rng = np.random.default_rng(args.seed + 21)
    w = {"q_norm": O.randn_bf16(rng, (256,), 0.1), "k_norm": O.randn_bf16(rng, (256,), 0.1)}
    dw = {k: torch.from_numpy(v.view(np.int16).copy()).to(f"cuda:{dev}") for k, v in w.items()}
    ws = torch.zeros(N.full_attn_workspace_bytes() // 4, dtype=torch.int32, device=f"cuda:{dev}")
    q = torch.randn(16, 512, device=f"cuda:{dev}")
    kn = torch.randn(2, 256, device=f"cuda:{dev}")
    vn = torch.randn(2, 256, device=f"cuda:{dev}")
    out = torch.zeros(16 * 256, device=f"cuda:{dev}")
    pk, pk_kind = peaks()
    res = {}
    st = torch.cuda.Stream(device=dev)
    for pos in (4095, 32767):
        cap = pos + 1
        kc = torch.randn(cap, 2, 256, device=f"cuda:{dev}") * 0.3
        vc = torch.randn(cap, 2, 256, device=f"cuda:{dev}")
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            for _ in range(20):
                N.full_attn_step(dw, q, kn, vn, kc, vc, pos, cap, out, ws,
                                 stream=torch.cuda.current_stream().cuda_stream)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        with torch.cuda.stream(st):
            for _ in range(5):
                g.replay()
        e1.record(st)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / 100
        ab = (pos + 1) * 2 * 256 * 4 * 2 + 16 * 512 * 4 + 16 * 256 * 4
        ach = ab / (us * 1e-6) / 1e9
        res[f"position_{pos}"] = {"us_per_call": us, "roofline": {"bound": "hbm", "achieved": ach, "peak": pk,
                                  "unit": "GB/s", "frac": ach / pk, "peak_kind": pk_kind,
                                  "algorithmic_bytes_per_launch": ab},
                                  "l2": "K and V of 32768 positions = 128 MB, about the L2 size"
                                        if pos > 8192 else "16 MB of K and V: L2-resident across calls"}
        del g, kc, vc
    hk = np.zeros((4096, 2, 256), np.float32)
    hv = np.zeros((4096, 2, 256), np.float32)
    t0 = time.perf_counter()
    O.full_attn_step(q.cpu().numpy(), kn.cpu().numpy(), vn.cpu().numpy(), w["q_norm"], w["k_norm"], hk, hv, 4095)
    res["cpu_oracle_ms_at_4095"] = (time.perf_counter() - t0) * 1e3
    return res


def run_full_attn_batched(args, dev):
    """Config 4's attention: nmoe_full_attn_step_batched for 64 sequences at position 32767
    over one layer's bf16 caches (64 x 32768 x 2 x 256 x 2 bytes each for K and V: 4.3 GB),
    device time per call (CUDA graph of 5 calls x 3 replays); bytes = the K and V rows read
    plus the new rows, against HBM."""
    import torch
    import nmoe_b200 as N
    from oracle import oracle as O
    B, cap = 64, 32768
    pos = cap - 1
    rng = np.random.default_rng(args.seed + 23)
    w = {"q_norm": O.randn_bf16(rng, (256,), 0.1), "k_norm": O.randn_bf16(rng, (256,), 0.1)}
    dw = {k: torch.from_numpy(v.view(np.int16).copy()).to(f"cuda:{dev}") for k, v in w.items()}
    ws = torch.zeros(N.full_attn_batched_workspace_bytes(B) // 4, dtype=torch.int32, device=f"cuda:{dev}")
    q = torch.randn(B, 16, 512, device=f"cuda:{dev}")
    kn = torch.randn(B, 2, 256, device=f"cuda:{dev}")
    vn = torch.randn(B, 2, 256, device=f"cuda:{dev}")
    out = torch.zeros(B, 16 * 256, device=f"cuda:{dev}")
    kc = (torch.randn(B, cap, 2, 256, device=f"cuda:{dev}") * 0.3).to(torch.bfloat16)
    vc = torch.randn(B, cap, 2, 256, device=f"cuda:{dev}").to(torch.bfloat16)
    positions = torch.full((B,), pos, dtype=torch.int32, device=f"cuda:{dev}")
    st = torch.cuda.Stream(device=dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for _ in range(5):
            N.full_attn_step_batched(dw, q, kn, vn, kc, vc, positions, cap, out, ws,
                                     stream=torch.cuda.current_stream().cuda_stream)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    with torch.cuda.stream(st):
        for _ in range(3):
            g.replay()
    e1.record(st)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / 15
    pk, pk_kind = peaks()
    ab = B * ((pos + 1) * 2 * 256 * 2 * 2 + 16 * 512 * 4 + 16 * 256 * 4)
    ach = ab / (us * 1e-6) / 1e9
    return {"batch": B, "position": pos, "us_per_call": us, "sequences_per_s": B / (us * 1e-6),
            "roofline": {"bound": "hbm", "achieved": ach, "peak": pk, "unit": "GB/s", "frac": ach / pk,
                         "peak_kind": pk_kind, "algorithmic_bytes_per_launch": ab},
            "l2": "4.3 GB of K and V per call: far above L2"}


def fast_decoder_weights(seed: int, num_layers: int, vocab: int):
    """Synthetic q4 attention / embedding / head weights of the 40-layer model, drawn
    directly in the packed format (uniform nibbles, scale 0.005, bias -0.0375: weights
    uniform in +-0.0375); norms and linear-attention parameters as the oracle's generator
    makes them. Generating 40 layers through the quantiser takes minutes of host time."""
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    s16 = O.f32_to_bf16(np.full(1, 0.005, np.float32))[0]
    b16 = O.f32_to_bf16(np.full(1, -0.0375, np.float32))[0]

    def q4(rows, cols):
        return {"weight": rng.integers(0, 1 << 32, (rows, cols // 8), dtype=np.uint32),
                "scales": np.full((rows, cols // 64), s16, np.uint16),
                "biases": np.full((rows, cols // 64), b16, np.uint16), "rows": rows, "cols": cols}
    layers = []
    for l in range(num_layers):
        norms = {"input_norm": O.randn_bf16(rng, (HIDDEN,), 0.02), "post_norm": O.randn_bf16(rng, (HIDDEN,), 0.02)}
        if (l + 1) % 4 == 0:
            layers.append({"kind": "full", **norms, "q": q4(8192, 2048), "k": q4(512, 2048), "v": q4(512, 2048),
                           "o": q4(2048, 4096), "q_norm": O.randn_bf16(rng, (256,), 0.02),
                           "k_norm": O.randn_bf16(rng, (256,), 0.02)})
        else:
            layers.append({"kind": "linear", **norms, "qkv": q4(8192, 2048), "z": q4(4096, 2048),
                           "beta": q4(32, 2048), "alpha": q4(32, 2048), "out": q4(2048, 4096),
                           **O.make_linear_attn(int(rng.integers(1 << 30)))})
    emb, head = q4(vocab, HIDDEN), q4(vocab, HIDDEN)
    g = {"vocab": vocab, "embed": {"dtype": 4, **emb}, "lm_head": {"dtype": 4, **head},
         "final_norm": O.randn_bf16(rng, (HIDDEN,), 0.02)}
    return layers, g


def run_decode_step(args, dev):
    """the whole decode step of the 40-layer model (nmoe_decoder_step:
    embedding, 30 linear-attention and 10 full-attention layers with their q4 projections,
    the MoE block of every layer, final norm and q4 LM head over 248320 rows), each step's
    token read on the device from the step before. Tokens per second over K steps at
    positions W..W+K-1, device time by CUDA events."""
    import torch
    import nmoe_b200 as N
    L = 40
    moe, _, _ = build_workload(L, 4, 8, N.DTYPE_BF16, N.DTYPE_BF16, pool=args.pool, seed=args.seed)
    ctx = N.Context(quant_bits=4, num_layers=L, router_dtype=N.DTYPE_BF16, shared_dtype=N.DTYPE_BF16, device=dev)
    for l, lw in enumerate(moe):
        ctx.load_layer(l, lw.experts)
        ctx.set_dense(l, lw.router, lw.shared_gate, lw.shared_up, lw.shared_down, lw.shared_gate_vec)
    del moe
    layers, g = fast_decoder_weights(args.seed + 5, L, LM_VOCAB)
    steps, warm = args.steps, args.warmup
    dec = N.Decoder(ctx, L, k=8, max_positions=steps + warm + 1)
    for l in range(L):
        dec.set_layer(l, layers[l])
    dec.set_globals(g)
    del layers, g
    st = torch.cuda.Stream(device=dev)
    sp = st.cuda_stream
    tok = torch.tensor([11], dtype=torch.int32, device=f"cuda:{dev}")
    with torch.cuda.stream(st):
        for p in range(warm):
            dec.step(tok, p, tok, stream=sp)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(dev)
    clk.start()
    e0.record(st)
    with torch.cuda.stream(st):
        for p in range(warm, warm + steps):
            dec.step(tok, p, tok, stream=sp)
    e1.record(st)
    torch.cuda.synchronize()
    clocks = clk.stop()
    ms = e0.elapsed_time(e1) / steps
    dec.close()
    ctx.close()
    return {"metric": "decode_tokens_per_s", "value": 1e3 / ms, "unit": "tokens/s", "ms_per_step": ms,
            "steps": steps, "warmup": warm, "higher_is_better": True, "dtype": "q4 weights, f32 activations",
            "data": "synthetic, random-init weights of the 40-layer architecture",
            "config": {"workload": "config3 decode step, 40 layers, q4 experts k=8, q4 attention projections, "
                                   "q4 LM head over 248320 rows, batch 1",
                       "positions": [warm, warm + steps - 1]},
            "clocks": clocks}


def run_ep_batched(args, rank, world, dev):
    """Config 2 beside the decode line, at every N: T tokens per rank (--ep-tokens) through
    --ep-layers resident layers per step, experts sharded 256/N per GPU with token rows
    exchanged over NVLink (one GPU: the plain batched path). Device-timed, max over ranks;
    with N > 1 also the device time of the two exchanges of one call."""
    import torch
    import torch.distributed as dist
    import nmoe_b200 as N
    T, L = args.ep_tokens, args.ep_layers
    layers, _, _ = build_workload(L, 4, 8, N.DTYPE_BF16, N.DTYPE_BF16, pool=args.pool, seed=args.seed)
    uid = None
    if world > 1:
        obj = [N.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        uid = obj[0]
        os.environ["NMOE_EP_TIMING"] = "1"
    ctx = N.Context(quant_bits=4, num_layers=L, t_max=T, device=dev, world_size=world, rank=rank, nccl_unique_id=uid)
    for l, lw in enumerate(layers):
        ctx.load_layer(l, lw.experts)
        ctx.set_dense(l, lw.router, lw.shared_gate, lw.shared_up, lw.shared_down, lw.shared_gate_vec)
    del layers
    from oracle import oracle as O
    xh = O.f32_to_bf16(np.random.default_rng(args.seed + 1000 + rank).standard_normal((T, HIDDEN), dtype=np.float32))
    x = torch.from_numpy(xh.view(np.int16)).to(f"cuda:{dev}")
    out = torch.zeros((T, HIDDEN), dtype=torch.float32, device=f"cuda:{dev}")
    stream = torch.cuda.Stream(device=dev)

    def step():
        for l in range(L):
            ctx.forward_batched(l, T, 8, x, out, stream=stream.cuda_stream)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    steps = max(5, args.steps // 2)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=f"cuda:{dev}")
    exch = None
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        d, r = ctx.debug_ep_times()
        ex = torch.tensor([d, r], dtype=torch.float64, device=f"cuda:{dev}")
        dist.all_reduce(ex, op=dist.ReduceOp.MAX)
        exch = {"dispatch_and_wait_ms": float(ex[0]), "return_and_wait_ms": float(ex[1]),
                "transport": "NVLink peer stores into IPC-mapped slabs (no NCCL on the call path)"}
    rc, code = ctx.device_status()
    ctx.close()
    if rc != N.OK:
        raise RuntimeError(f"expert-parallel device error word {code}")
    per_call_ms = float(ms.item()) / (steps * L)
    return {"metric": "routed-MoE tokens/s/layer (batched, config 2)", "value": world * T / (per_call_ms / 1e3),
            "unit": "tokens/s/layer", "per_rank_value": T / (per_call_ms / 1e3), "per_call_ms": per_call_ms,
            "tokens_per_rank": T, "layers": L, "ranks": world, "scaling": "weak",
            "parallelism": f"expert parallel, {EXPERTS // world} experts per GPU" if world > 1 else "single GPU",
            "exchange": exch, "timing": "CUDA events around the step loop, max over ranks"}


_JSON_OUT = sys.stdout


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=40)
    ap.add_argument("--pool", type=int, default=32, help="distinct expert packs generated on the host")
    ap.add_argument("--seed", type=int, default=2026)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--workload", choices=["decode", "batched", "lm_head", "crc", "linear_attn", "full_attn", "decode_step", "full_attn_batched"], default="decode")
    ap.add_argument("--lm-dtypes", default="q4,bf16", help="LM head weight types timed (q4, bf16)")
    ap.add_argument("--bits", type=int, choices=[2, 4], default=4, help="decode: expert packs (4: config 0, 2: config 1)")
    ap.add_argument("--k", type=int, default=8, help="decode: routed experts per token (config 1 sweeps 1..8)")
    ap.add_argument("--tokens", type=int, default=4096, help="T for --workload batched")
    ap.add_argument("--batched-layers", type=int, default=4, help="resident layers cycled by --workload batched")
    ap.add_argument("--ep-tokens", type=int, default=4096,
                    help="decode workload: also time config 2 at this many tokens per rank (0: skip)")
    ap.add_argument("--ep-layers", type=int, default=2)
    ap.add_argument("--lm-head", type=int, default=1, help="also time the LM head (rank 0) beside the decode line")
    ap.add_argument("--prefetch", action="store_true",
                    help="let each layer call prefetch the next layer's router/shared weights to L2")
    args = ap.parse_args()

    # stdout carries exactly one JSON line: libraries (NCCL's version banner, ...) write
    # to file descriptor 1, so it is pointed at stderr and the JSON goes to a saved copy
    global _JSON_OUT
    _JSON_OUT = os.fdopen(os.dup(1), "w")
    sys.stdout.flush()
    os.dup2(2, 1)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        res = run_reference(args, rank, world)
        if res is not None:
            print(json.dumps(res), file=_JSON_OUT, flush=True)
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", device_id=torch.device(f"cuda:{local_rank}"))
    if args.workload == "full_attn_batched":
        import torch
        torch.cuda.set_device(local_rank)
        res = {"workload": "full_attn_batched", **run_full_attn_batched(args, local_rank)} if rank == 0 else None
    elif args.workload == "decode_step":
        import torch
        torch.cuda.set_device(local_rank)
        res = {"workload": "decode_step", **run_decode_step(args, local_rank)} if rank == 0 else None
    elif args.workload == "full_attn":
        import torch
        torch.cuda.set_device(local_rank)
        res = {"workload": "full_attn", **run_full_attn(args, local_rank)} if rank == 0 else None
    elif args.workload == "linear_attn":
        import torch
        torch.cuda.set_device(local_rank)
        res = {"workload": "linear_attn", **run_linear_attn(args, local_rank)} if rank == 0 else None
    elif args.workload == "crc":
        import torch
        torch.cuda.set_device(local_rank)
        res = {"workload": "crc", **run_crc(args, local_rank)} if rank == 0 else None
    elif args.workload == "lm_head":
        import torch
        torch.cuda.set_device(local_rank)
        res = {"workload": "lm_head", **run_lm_head(args, local_rank)} if rank == 0 else None
    else:
        res = (run_batched if args.workload == "batched" else run_ours)(args, rank, world, local_rank)
    if res is not None:
        print(json.dumps(res), file=_JSON_OUT, flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
