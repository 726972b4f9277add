"""Benchmark: the 40-layer Q4_K/Q6_K expert stack decode step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch T] [--impl ours|reference]

Workload: 40 layers x (256 routed + 1 shared) experts, all
resident in HBM (20.97 GB of Q4_K gate/up and Q6_K down blocks, synthetic from a
seed with the benchmark value distributions), hidden 2048, expert inter 512,
top-8 softmax routing over an fp32 256 x 2048 router.  One step decodes T
tokens through all 40 MoE layers; each layer's input is the RMS-normalised
residual stream left by the previous layer (h <- h + moe_l(rmsnorm(h))), so
every layer waits for the previous layer's combine, as decode does.  With N
GPUs the experts are split expert-parallel (rank r holds experts
[r*256/N, (r+1)*256/N)) and each layer's partial outputs are combined over
NVLink.  Inputs cycle through 16 distinct seeded hidden states so routing
changes between steps; one step streams ~0.8 GB (T=1) to ~18 GB (T=64) of
distinct expert weights, far more than the 126 MB L2, so no flush is needed.

Prints one JSON line on rank 0.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Q4_K/Q6_K expert matvec HBM GB/s (% of peak); MoE-stack decode tok/s at 1/2/4/8 B200"
H, I, E, K_TOP, LAYERS = 2048, 512, 256, 8, 40
GATE_B = I * H // 256 * 144      # one expert's gate (= up) matrix, bytes
DOWN_B = H * I // 256 * 210      # one expert's down matrix, bytes
EXPERT_B = 2 * GATE_B + DOWN_B   # 2,039,808
N_INPUTS = 16
BATCH2 = 64                      # second batch size of config 5, reported beside the headline


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def layer_bytes(groups: int, pairs: int, T: int) -> dict:
    """Algorithmic bytes of one layer's three phases (each weight byte once)."""
    k1 = E * H * 4 + H * 2 + T * H * 4 + T * H * 2 + T * (H // 32) * 4 + T * E * 4
    k2 = groups * 2 * GATE_B + T * H * 2 + pairs * I * 2
    k3 = groups * DOWN_B + pairs * I * 2 + 2 * T * H * 4
    return {"route": k1, "gateup": k2, "down": k3, "combine": 0}


STAMP_POINTS = ["start", "logits", "router_barrier", "routed", "x_landed", "gateup_done", "gateup_barrier",
                "down_landed", "down_done", "end", "p_routed", "p_gateup_issued", "p_down_issued", "p_router_issued",
                "p_gateup_barrier", "p_down_all_issued", "quantised", "router_rows", "router_dots", "route_inputs",
                "topk", "tables", "down_stages", "down_stored"]


def layer_timeline(stamps) -> dict:
    """Timeline of a layer over all CTAs from the phase stamps [layers, ctas,
    24] (ns): median and max over CTAs of each phase point, in us from the
    earliest start of the layer, averaged over layers.  A point a CTA never
    reaches (no work of that kind) stays 0 and is left out of the median."""
    import warnings

    import numpy as np

    s = stamps.astype(np.float64)
    st0 = s[:, :, 0].min(axis=1)[:, None, None]
    rel = np.where(s > 0, (s - st0) * 1e-3, np.nan)
    with warnings.catch_warnings():  # (points no CTA reaches in some mode are NaN)
        warnings.simplefilter("ignore", RuntimeWarning)
        med = np.nanmean(np.nanmedian(rel, axis=1), axis=0)
        mx = np.nanmean(np.nanmax(rel, axis=1), axis=0)
    def r2(v):  # (strict JSON: a point no CTA reached is null)
        return round(float(v), 2) if v == v else None

    return {"points": STAMP_POINTS, "median_us": [r2(v) for v in med], "max_us": [r2(v) for v in mx]}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200", "-f", self.path],
                                         stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        try:
            with open(self.path) as f:
                for line in f:
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) >= 9:
                        rows.append(parts)
            os.unlink(self.path)
        except Exception:
            return None
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        pw = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        loaded = [s for s, p in zip(sm, pw) if p >= (max(pw) * 0.5 if pw else 0)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "power_w_max": max(pw) if pw else None}


# ---------------------------------------------------------------------------
# CPU side: the reference's own CPU path (oracle/_ref) or the oracle port
# ---------------------------------------------------------------------------
def host_info() -> dict:
    """Logical cores this process may use and the CPU model of the host."""
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"host_cores": n, "cpu_model": model}


class CpuLayerSampler:
    """Runs whole MoE layers of the benchmark stack on the host with the
    reference's CPU code: route_layer's arithmetic (one_layer.cu:937-992) and the
    expert block of expert_bench.cu:158-179 (OpenMP over the top-k experts +
    shared expert, cpu_tensor_matvec / cpu_swiglu, layer_ops.cu)."""

    def __init__(self, seed: int, threads: int):
        import numpy as np

        import oracle

        # inputs from the oracle's host restatement of the seeded generator
        # (the same bytes as the product library's), so this CPU leg loads no
        # product code
        self.np, self.oracle = np, oracle
        self.kind = "reference" if oracle.ref_available() else "port"
        self.seed, self.threads = seed, threads
        self.cache = {}

    def _sid(self, layer, kind, e):
        return (layer << 32) | (kind << 24) | e

    def _blocks(self, layer, kind, e, n, qt):
        key = (layer, kind, e)
        if key not in self.cache:
            self.cache[key] = self.oracle.synth_blocks(n, qt, self.seed, self._sid(layer, kind, e))
        return self.cache[key]

    def layer_inputs(self, layer):
        o = self.oracle
        W = o.synth_normal(E * H, 0.02, self.seed, self._sid(layer, 6, 0)).reshape(E, H)
        sg = o.synth_normal(H, 0.02, self.seed, self._sid(layer, 7, 0), half=True)
        return W, sg

    def run_layer(self, layer, h, W, sg):
        """One layer for T tokens: returns seconds spent in the reference code."""
        np, o = self.np, self.oracle
        # rmsnorm_inplace (one_layer.cu:158-180): x * rms * post_attention_norm.weight
        nw = o.synth_normal(H, 0.1, self.seed, self._sid(layer, 8, 0)) + np.float32(1.0)
        x = (h / np.sqrt((h.astype(np.float64) ** 2).mean(axis=1, keepdims=True) + 1e-6) * nw).astype(np.float32)
        t0 = time.perf_counter()
        if self.kind == "reference":
            idx, wt, sgw = o.ref_route(x, W, sg, K_TOP)
        else:
            idx, wt, sgw, _ = o.route(x, W, sg, K_TOP)
        t1 = time.perf_counter()
        nb_g, nb_d = I * H // 256, H * I // 256
        empty = np.zeros(1, np.uint8)
        gate, up, down = [empty] * E, [empty] * E, [empty] * E
        for e in set(idx.ravel().tolist()):
            gate[e] = self._blocks(layer, 0, e, nb_g, 12)
            up[e] = self._blocks(layer, 1, e, nb_g, 12)
            down[e] = self._blocks(layer, 2, e, nb_d, 14)
        sh = (self._blocks(layer, 3, 0, nb_g, 12), self._blocks(layer, 4, 0, nb_g, 12),
              self._blocks(layer, 5, 0, nb_d, 14))
        es = o.ExpertSet(gate, up, down, *sh)
        t2 = time.perf_counter()
        if self.kind == "reference":
            out = o.ref_moe_block(es, x, idx, wt, sgw, H, I, self.threads)
        else:
            out = o.moe_f32(es, x, idx, wt, sgw, H, I)
        t3 = time.perf_counter()
        return (t1 - t0) + (t3 - t2), h + out


def cpu_sample(T: int, seed: int, threads: int, budget_s: float = 15.0):
    """Time whole reference-CPU layers until ~budget_s of CPU work; returns
    (tok/s for the 40-layer stack, layers timed, kind)."""
    import oracle

    s = CpuLayerSampler(seed, threads)
    h = oracle.synth_normal(T * H, 1.0, seed, 777).reshape(T, H)
    spent, layers = 0.0, 0
    while layers < LAYERS and (layers == 0 or spent < budget_s):
        W, sg = s.layer_inputs(layers)
        dt, h = s.run_layer(layers, h, W, sg)
        spent += dt
        layers += 1
    per_layer = spent / layers
    return T / (per_layer * LAYERS), layers, s.kind, per_layer


def run_reference(args, rank: int, world: int) -> int:
    """--impl reference: the reference's CPU implementation of the path on the
    host cores, same metric and config; rank 0 only."""
    if rank != 0:
        return 0
    import oracle

    threads = host_info()["host_cores"]
    s = CpuLayerSampler(args.seed, threads)
    T = args.batch
    hs = [oracle.synth_normal(T * H, 1.0, args.seed, 900 + i).reshape(T, H) for i in range(N_INPUTS)]
    times = []
    for i in range(args.warmup + args.steps):
        layer = i % LAYERS
        W, sg = s.layer_inputs(layer)
        dt, _ = s.run_layer(layer, hs[i % N_INPUTS], W, sg)
        if i >= args.warmup:
            times.append(dt)
    per_layer = sum(times) / len(times)
    value = T / (per_layer * LAYERS)
    sample = f"{args.steps} timed layers (one MoE layer per step, cycling layers 0..39) at T={T}; tok/s = T / (40 x mean layer time)"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_layer * LAYERS * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_block(args, world),
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": s.kind, "sample": sample,
                         "threads": threads, **host_info()},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    # the reference's own GPU kernels on this box, beside its CPU path (extra key)
    try:
        import torch

        if torch.cuda.is_available() and oracle.refgpu_available():
            line["reference_gpu"] = reference_gpu_bar()
    except Exception as ex:
        line["reference_gpu"] = {"error": f"{type(ex).__name__}: {ex}"[:300]}
    print(json.dumps(line), flush=True)
    return 0


def reference_gpu_bar() -> dict:
    """The reference's OWN GPU path on this B200 (kernels.cu compiled for
    sm_100a from its sources, oracle/_ref/libbread_refgpu.so): its
    bread_matvec on configs 1 and 2 (a CUDA graph of back-to-back launches
    over 256 distinct weight copies, > L2, as our arm measures them) and the
    expert_bench.cu:182-194 serial launch loop for one MoE block at T = 1
    (8 routed + 1 shared expert: 5 launches each, fp16 activations), over 16
    distinct expert sets.  Timed with CUDA events; a measurement beside the
    CPU reference, not its value."""
    import ctypes

    import numpy as np
    import torch

    import oracle

    L = oracle.refgpu()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)

    def sp():  # the current stream at call time (the capture stream inside a graph)
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    out = {"kernel": "kernels.cu dequant_q4k/q6k_matvec (one CTA per row, 256 threads), sm_100a build"}
    peak = peaks()[0]

    def graph_us(fn, n):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for i in range(3):
                fn(i)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(n):
                fn(i)
        g.replay()
        torch.cuda.synchronize()
        best = None
        for _ in range(3):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            t = e0.elapsed_time(e1) * 1e3 / n
            best = t if best is None else min(best, t)
        return best

    ncopy = 256
    for name, qt, rows, cols, blk in (("config1_q4k_512x2048", 12, 512, 2048, 144),
                                      ("config2_q6k_2048x512", 14, 2048, 512, 210)):
        nb = rows * cols // 256
        wall = torch.from_numpy(oracle.synth_blocks(nb * ncopy, qt, 11, 20 + qt)).to(dev)
        x = torch.from_numpy(oracle.synth_normal(cols, 1.0, 11, 30).astype(np.float16)).to(dev)
        y = torch.empty(rows, dtype=torch.float16, device=dev)
        mb = nb * blk
        base = wall.data_ptr()

        def f(i, base=base, mb=mb, x=x, y=y, rows=rows, cols=cols, qt=qt):
            L.refgpu_matvec(ctypes.c_void_p(base + (i % ncopy) * mb), ctypes.c_void_p(x.data_ptr()),
                            ctypes.c_void_p(y.data_ptr()), rows, cols, qt, sp())

        us = graph_us(f, ncopy)
        gbs = (mb + 2 * cols + 2 * rows) / (us * 1e-6) / 1e9
        out[name] = {"us_per_launch": us, "GB_s": gbs, "frac": gbs / peak}
        del wall
    # one MoE block at T = 1: 9 experts (8 routed + shared) per call, 16 sets
    Hh, Ii = H, I
    nb_g, nb_d = Ii * Hh // 256, Hh * Ii // 256
    nexp = 16 * 9
    gate = torch.from_numpy(oracle.synth_blocks(nb_g * nexp, 12, 13, 1)).to(dev)
    up = torch.from_numpy(oracle.synth_blocks(nb_g * nexp, 12, 13, 2)).to(dev)
    down = torch.from_numpy(oracle.synth_blocks(nb_d * nexp, 14, 13, 3)).to(dev)
    x = torch.from_numpy(oracle.synth_normal(Hh, 1.0, 13, 4).astype(np.float16)).to(dev)
    hid = torch.empty(Hh, dtype=torch.float16, device=dev)
    eg = torch.empty(Ii, dtype=torch.float16, device=dev)
    eu = torch.empty(Ii, dtype=torch.float16, device=dev)
    eo = torch.empty(Hh, dtype=torch.float16, device=dev)
    wts = (ctypes.c_float * 9)(*([0.125] * 8 + [0.5]))
    sets = []
    for j in range(16):
        e = [9 * j + k for k in range(9)]
        sets.append(tuple((ctypes.c_void_p * 9)(*[t.data_ptr() + i * b for i in e])
                          for t, b in ((gate, nb_g * 144), (up, nb_g * 144), (down, nb_d * 210))))

    def blk(i):
        g_, u_, d_ = sets[i % 16]
        L.refgpu_expert_loop(g_, u_, d_, wts, 9, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(hid.data_ptr()),
                             ctypes.c_void_p(eg.data_ptr()), ctypes.c_void_p(eu.data_ptr()),
                             ctypes.c_void_p(eo.data_ptr()), Hh, Ii, sp())

    us = graph_us(blk, 32)
    nbytes = 9 * EXPERT_B
    out["config3_expert_loop_t1"] = {"us_per_block": us, "launches_per_block": 1 + 9 * 5,
                                     "GB_s": nbytes / (us * 1e-6) / 1e9, "frac": nbytes / (us * 1e-6) / 1e9 / peak,
                                     "note": "experts only (the reference routes on the host, one_layer.cu:937-992)"}
    del gate, up, down
    torch.cuda.empty_cache()
    return out


def config_block(args, world):
    return {"workload": "config 5: 40-layer Q4_K/Q6_K expert stack, 40 x (256 routed + 1 shared) experts resident "
                        "(20.97 GB), decode step of `batch` tokens",
            "layers": LAYERS, "hidden": H, "inter": I, "experts": E, "top_k": K_TOP, "shared_expert": True,
            "batch": args.batch, "global_batch": args.batch, "layer_input": "rmsnorm(residual), layers chained",
            "parallelism": f"ep{world}", "l2": "inputs larger than L2 (>= 0.8 GB of distinct weights per step)"}


# ---------------------------------------------------------------------------
# GPU: this library
# ---------------------------------------------------------------------------
def run_ours(args, rank: int, world: int, local_rank: int) -> int:
    import numpy as np
    import torch

    import breadv2_b200 as bb

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    T = args.batch
    T2 = BATCH2 if (T != BATCH2 and not args.quick) else None  # secondary batch size, same stack
    st = bb.ExpertStack(n_layers=args.layers, hidden=H, inter=I, n_experts=E, top_k=K_TOP,
                        max_tokens=max(T, T2 or 0),
                        shared_expert=True, norm_eps=1e-6, seed=args.seed, rank=rank, world=world)
    if world > 1:
        st.connect_peers(dist)
    parity = ep_parity(dist, rank, world, dev, args.seed) if world > 1 else None
    stream = torch.cuda.current_stream()
    inputs = [bb.synth_normal(T * H, 1.0, args.seed, 900 + i, device=dev).view(T, H) for i in range(N_INPUTS)]
    h = torch.empty(T, H, dtype=torch.float32, device=dev)

    def barrier():
        if dist is not None:
            dist.barrier()

    def one(i):
        h.copy_(inputs[i % N_INPUTS])
        st.step(h)

    for i in range(args.warmup):
        one(i)
    torch.cuda.synchronize()
    assert bb.device_error() == 0, "device-side wait timed out"

    clocks = ClockSampler(local_rank)
    if not args.quick:
        clocks.start()
    # keep the GPU loaded ~1 s before timing so the clock samples see steady state
    t_end = time.time() + (0.0 if args.quick else 1.0)
    i = 0
    while time.time() < t_end:
        one(i)
        i += 1
        if i % 8 == 0:
            torch.cuda.synchronize()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        one(i)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = e0.elapsed_time(e1)
    if args.quick:
        if rank == 0:
            print(json.dumps({"quick": True, "ms_per_step": ms / args.steps, "batch": T, "n_gpus": world}), flush=True)
        st.close()
        if dist is not None:
            dist.destroy_process_group()
        return 0

    # end to end through the host-buffer entry point (H2D + step + D2H per step)
    hin = [x.cpu().pin_memory() for x in inputs]
    hout = torch.empty(T, H, dtype=torch.float32).pin_memory()
    for i in range(2):
        st.step_host(hin[i], hout)
    torch.cuda.synchronize()
    barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for i in range(args.steps):
        st.step_host(hin[i % N_INPUTS], hout)
    e3.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms_e2e = e2.elapsed_time(e3)
    clk = clocks.stop()

    # the same stack at the second batch size (config 5 names batch 1 and 64)
    batch2 = None
    if T2:
        inputs2 = [bb.synth_normal(T2 * H, 1.0, args.seed, 950 + i, device=dev).view(T2, H) for i in range(4)]
        h2 = torch.empty(T2, H, dtype=torch.float32, device=dev)
        for i in range(3):
            h2.copy_(inputs2[i % 4])
            st.step(h2)
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n2 = max(3, args.steps // 5)
        f0.record(stream)
        for i in range(n2):
            h2.copy_(inputs2[i % 4])
            st.step(h2)
        f1.record(stream)
        torch.cuda.synchronize()
        barrier()
        ms2 = f0.elapsed_time(f1) / n2
        g2, p2 = st.routing_stats()
        b2 = sum(sum(layer_bytes(int(g), int(p), T2).values()) for g, p in zip(g2, p2))
        batch2 = {"batch": T2, "steps": n2, "ms_per_step": ms2, "tok_s": T2 / (ms2 * 1e-3),
                  "step_hbm_gbs": b2 / (ms2 * 1e-3) / 1e9, "experts_per_layer": float(np.mean(g2))}

    # phase durations (a profiled launch of the same step: every CTA records
    # %globaltimer at its phase points) and routing stats
    h.copy_(inputs[0])
    kms = st.profile_step(h)
    stamps = st.profile_stamps()
    groups, pairs = st.routing_stats()
    assert bb.device_error() == 0, "device-side wait timed out"

    if dist is not None:
        t = torch.tensor([ms, ms_e2e, batch2["ms_per_step"] if batch2 else 0.0], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_e2e = float(t[0]), float(t[1])
        if batch2:
            batch2["ms_per_step"] = float(t[2])
            batch2["tok_s"] = T2 / (batch2["ms_per_step"] * 1e-3)
    if rank != 0:
        st.close()
        dist.destroy_process_group()
        return 0

    hbm_peak, peak_kind = peaks()
    launches = args.steps * st.launches_per_step(T)
    ms_step = ms / args.steps
    value = T / (ms_step * 1e-3)
    bytes_per_layer = [layer_bytes(int(g), int(p), T) for g, p in zip(groups, pairs)]
    names = ["route", "gateup", "down", "combine"]
    tot_ms = {n: float(kms[:, j].sum()) for j, n in enumerate(names)}
    step_bytes = sum(sum(b.values()) for b in bytes_per_layer)
    # The step is ONE kernel launch (moe_step_kernel): achieved = algorithmic
    # bytes of the step / its CUDA-event duration from the timed loop.
    achieved = step_bytes / (ms_step * 1e-3) / 1e9
    # instantiation that runs: 0 = tagged-word decode on one GPU (T <= 8),
    # 1 = grid barriers at T <= 8 (BREAD_NO_FLAGGED=1), 2 = T > 8,
    # 3 = tagged-word decode with expert parallelism; one-token launches of
    # modes 0 and 3 use the one-token instantiation (fourth argument true)
    if T > 8:
        mode = 2
    elif os.environ.get("BREAD_NO_FLAGGED") == "1":
        mode = 1
    else:
        mode = 3 if world > 1 else 0
    kname = f"moe_step_kernel<{H // 256},{I // 256},{mode}{',true' if T == 1 and mode in (0, 3) else ''}>"
    traffic = None
    tfile = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tfile):
        try:
            traffic = json.load(open(tfile)).get(f"{kname}@T{T}")
        except Exception:
            traffic = None
    timeline = layer_timeline(stamps)

    matvec = configs = None
    if world == 1:
        st.close()  # free the stack before the GEMV weights
        matvec = matvec_bench(dev, hbm_peak)
        try:
            configs = configs_bench(dev, hbm_peak)
        except Exception as ex:  # a side measurement: never lose the headline line to it
            configs = {"error": f"{type(ex).__name__}: {ex}"[:300]}

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        threads = min(8, host_info()["host_cores"])
        v, layers, kind, per_layer = cpu_sample(T, args.seed, threads)
        cpu = {"value": v, "unit": "tok/s", "cores": threads, "threads": threads, **host_info(), "kind": kind,
               "sample": f"{layers} of 40 MoE layers at T={T} on the host ({per_layer * 1e3:.1f} ms/layer, "
                         f"OpenMP over experts as expert_bench.cu:158-179); tok/s = T / (40 x layer time)"}

    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "i32+f32", "data": "synthetic",
        "config": config_block(args, world),
        "roofline": {"bound": "hbm", "kernel": kname, "achieved": achieved, "peak": hbm_peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / hbm_peak, "traffic": traffic,
                     "algorithmic_bytes_per_launch": step_bytes, "avg_launch_us": ms_step * 1e3},
        "phases_us_per_layer": {n: tot_ms[n] / LAYERS * 1e3 for n in names},
        "layer_timeline": timeline,
        "experts_per_layer": float(np.mean(groups)),
        "cpu_baseline": cpu,
        "e2e": {"value": T / (ms_e2e / args.steps * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": T * H * 4,
                "d2h_bytes_per_step": T * H * 4},
        "gpu_launches": launches,
        "clocks": clk,
        "batch2": batch2,
        "matvec": matvec,
        "configs_1_4": configs,
        "ep_parity": parity,
    }
    print(json.dumps(line), flush=True)
    st.close()
    if dist is not None:
        dist.destroy_process_group()
    return 0


def graph_time_us(fn, n_iter: int, reps: int = 3) -> float:
    """Device time per call of `fn(i)` (i = 0..n_iter-1), captured into one CUDA
    graph and replayed (launch gaps of a Python loop would dominate kernels of
    a few microseconds): best of `reps` replays, CUDA events on the stream."""
    import torch

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for i in range(3):
            fn(i)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(n_iter):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    best = None
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) * 1e3 / n_iter
        best = t if best is None else min(best, t)
    del g
    return best


def configs_bench(dev, hbm_peak) -> dict:
    """BASELINE configs 1-4 on one GPU (each a separate measurement beside the
    config-5 headline):
      1  Q4_K 512 x 2048 expert gate GEMV,  2  Q6_K 2048 x 512 expert down GEMV:
         a CUDA graph of back-to-back bread_matvec_f32 launches over 256 distinct
         weight copies (151 / 220 MB, > L2); bytes = weights + x + y;
      3  one MoE block at T = 1 (router + 8 routed + shared expert) and
      4  the same block for k in {1, 2, 4, 8, 16} tokens (speculative verify):
         bread_moe_ffn over one resident layer of 256 + 1 experts, 16 distinct
         seeded inputs cycled (~144 distinct experts, > L2); bytes = distinct
         experts touched x 2,039,808 + the fp32 router + activations."""
    import numpy as np
    import torch

    import breadv2_b200 as bb

    out = {}
    ncopy = 256
    for name, qt, rows, cols, blk in (("config1_q4k_512x2048", 12, 512, 2048, 144),
                                      ("config2_q6k_2048x512", 14, 2048, 512, 210)):
        nb = rows * cols // 256
        wall = bb.synth_blocks(nb * ncopy, qt, 11, 20 + qt, device=dev)
        x = bb.synth_normal(cols, 1.0, 11, 30, device=dev)
        y = torch.empty(rows, device=dev)
        mb = nb * blk

        def f(i, wall=wall, x=x, y=y, mb=mb, rows=rows, cols=cols, qt=qt):
            bb.matvec_f32(wall[(i % ncopy) * mb:(i % ncopy + 1) * mb], x, rows, cols, qt, y=y)

        us = graph_time_us(f, ncopy)
        gbs = (mb + 4 * cols + 4 * rows) / (us * 1e-6) / 1e9
        out[name] = {"shape": [rows, cols], "us_per_launch": us, "GB_s": gbs, "frac": gbs / hbm_peak,
                     "launches": ncopy, "note": "CUDA graph of back-to-back launches, distinct weights each"}
        del wall
    torch.cuda.empty_cache()

    # one resident MoE layer: 256 routed experts + shared, router, shared gate
    Hh, Ii, Ee, Kk = H, I, E, K_TOP
    nb_g, nb_d = Ii * Hh // 256, Hh * Ii // 256
    gate = bb.synth_blocks(nb_g * Ee, 12, 12, 1, device=dev)
    up = bb.synth_blocks(nb_g * Ee, 12, 12, 2, device=dev)
    down = bb.synth_blocks(nb_d * Ee, 14, 12, 3, device=dev)
    gb_, db_ = nb_g * 144, nb_d * 210
    tabs = [bb.pointer_table([t.data_ptr() + e * b for e in range(Ee)], dev) for t, b in ((gate, gb_), (up, gb_),
                                                                                             (down, db_))]
    shared = (bb.synth_blocks(nb_g, 12, 12, 4, device=dev), bb.synth_blocks(nb_g, 12, 12, 5, device=dev),
              bb.synth_blocks(nb_d, 14, 12, 6, device=dev))
    W_r = bb.synth_normal(Ee * Hh, 0.02, 12, 7, device=dev).view(Ee, Hh)
    w_sg = bb.synth_normal(Hh, 0.02, 12, 8, half=True, device=dev)
    sweep = {}
    for k in (1, 2, 4, 8, 16):
        xs = [bb.synth_normal(k * Hh, 1.0, 12, 100 + 17 * k + i, device=dev).view(k, Hh) for i in range(16)]
        outb = torch.zeros(k, Hh, device=dev)
        ws = bb.alloc_workspace(k, Hh, Ii, Ee, Kk, device=dev)
        distinct = []
        for i in range(16):
            idx, _, _ = bb.moe_ffn(*tabs, W_r, w_sg, shared, xs[i], outb, Ii, Kk, workspace=ws, want_routing=True)
            distinct.append(len(set(idx.cpu().numpy().ravel().tolist())))

        def f(i, xs=xs, outb=outb, ws=ws):
            bb.moe_ffn(*tabs, W_r, w_sg, shared, xs[i % 16], outb, Ii, Kk, workspace=ws)

        us = graph_time_us(f, 64)
        groups = float(np.mean(distinct)) + 1
        nbytes = groups * EXPERT_B + Ee * Hh * 4 + Hh * 2 + 2 * k * Hh * 4
        sweep[str(k)] = {"tokens": k, "us_per_block": us, "tok_s_per_layer": k / (us * 1e-6),
                         "experts_touched": groups, "GB_s": nbytes / (us * 1e-6) / 1e9,
                         "frac": nbytes / (us * 1e-6) / 1e9 / hbm_peak}
    out["config3_moe_block_t1"] = sweep["1"]
    out["config4_verify_sweep"] = sweep
    del gate, up, down
    torch.cuda.empty_cache()
    return out


def ep_parity(dist, rank: int, world: int, dev, seed: int) -> dict:
    """Expert-parallel correctness on the box that runs the scaling bench: a
    3-layer stack at the full config shape split over the N ranks, one step at
    T = 1 and one at T = 24, against a one-GPU stack from the same seed (rank
    0).  Every rank must hold the same bits (all-gather)."""
    import torch

    import breadv2_b200 as bb
    import oracle

    res = {}
    st = bb.ExpertStack(n_layers=3, max_tokens=24, seed=seed, rank=rank, world=world)
    st.connect_peers(dist)
    one = bb.ExpertStack(n_layers=3, max_tokens=24, seed=seed) if rank == 0 else None
    for T in (1, 24):
        h0 = bb.synth_normal(T * H, 1.0, seed, 4242 + T, device=dev).view(T, H)
        h = h0.clone()
        torch.cuda.synchronize()
        dist.barrier()  # every rank launches the step together
        st.step(h)
        torch.cuda.synchronize()
        allh = [torch.empty_like(h) for _ in range(world)]
        dist.all_gather(allh, h)
        if rank == 0:
            h1 = h0.clone()
            one.step(h1)
            torch.cuda.synchronize()
            res[f"T{T}"] = {"rel_l2_vs_one_gpu": oracle.rel_l2(h.cpu().numpy(), h1.cpu().numpy()),
                            "ranks_bitwise_equal": all(torch.equal(a, allh[0]) for a in allh)}
    assert bb.device_error() == 0, "device-side wait timed out"
    dist.barrier()
    st.close()
    if one is not None:
        one.close()
    if rank == 0:
        res["layers"], res["config"] = 3, "H=2048 I=512 E=256 top-8 + shared, experts split over the ranks"
    return res


def matvec_bench(dev, hbm_peak) -> dict:
    """The expert matvec kernels on their largest benchmark shape (config 2's
    248320 x 2048 output head, Q6_K and Q4_K): CUDA-event time of back-to-back
    bread_matvec_f32 launches alternating between two weight copies (417 MB /
    286 MB each, > L2), algorithmic bytes = weights + x + y."""
    import torch

    import breadv2_b200 as bb

    out = {}
    rows, cols = 248320, 2048
    x = bb.synth_normal(cols, 1.0, 7, 8, device=dev)
    y = torch.empty(rows, device=dev)
    for name, qt, bb_ in (("q6k_head", 14, 210), ("q4k_head", 12, 144)):
        nb = rows * cols // 256
        ws = [bb.synth_blocks(nb, qt, 7, 10 + i, device=dev) for i in range(2)]
        for i in range(3):
            bb.matvec_f32(ws[i % 2], x, rows, cols, qt, y=y)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = 10
        e0.record()
        for i in range(n):
            bb.matvec_f32(ws[i % 2], x, rows, cols, qt, y=y)
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) / n * 1e3
        gbs = (nb * bb_ + 4 * cols + 4 * rows) / (us * 1e-6) / 1e9
        out[name] = {"shape": [rows, cols], "us": us, "GB_s": gbs, "frac": gbs / hbm_peak}
        del ws
    torch.cuda.empty_cache()
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=1, help="tokens per decode step (T)")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="layers in the stack (profiling of small cases only; the benchmark is 40)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--quick", action="store_true",
                    help="profiler runs: timed steps only (no load phase, end-to-end pass, kernel events or CPU baseline)")
    ap.add_argument("--gemv", action="store_true",
                    help="profiler runs: only the output-head GEMV measurement (Q6_K then Q4_K, 3 + 10 launches each)")
    args = ap.parse_args(argv)
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and "WORLD_SIZE" in os.environ:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.gemv:
        import torch

        dev = torch.device("cuda", local_rank)
        torch.cuda.set_device(dev)
        print(json.dumps({"matvec": matvec_bench(dev, peaks()[0])}), flush=True)
        return 0
    return run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    sys.exit(main())
