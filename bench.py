#!/usr/bin/env python3
"""Benchmark of the block-FP8 MoE expert path on B200.

Workload (config 2, "c2"): a Qwen3-30B-A3B-shaped MoE layer — hidden
2048, 128 experts, moe_intermediate 768, top-8 with normalised probabilities,
E4M3 weights with 128x128 f32 block scales, f32 router — decoding a batch of
`--tokens` bf16 tokens (default 1; the config also lists 4 and 16).  One step =
one MoE-layer forward over one batch.  Data are seeded synthetic tensors with
the configured distributions (no checkpoint is available).

Steps cycle through `--layers` distinct registered layers (default 16, 9.7 GB of
expert weights) with a fresh token batch each step, so a layer's weights come
back only after ~16 x 39 MB of other traffic: inputs larger than L2, no L2 reuse
between timed iterations.

value = tokens/s over all ranks, device-timed (CUDA events on the launch
stream, max over ranks), inputs resident in HBM.  e2e = the same metric through
the C ABI with host buffers (pinned H2D of the tokens and D2H of the outputs
inside the timed region).  --gpus N > 1 runs one process per GPU (torchrun) as
expert parallelism: every layer's experts are partitioned over the GPUs, the
router runs replicated, and the GPUs' outputs are summed inside the decode
kernel (peer stores over NVLink; prefill-sized batches: one NCCL all-reduce per
layer call); each GPU contributes --tokens tokens to the step's batch (N x
--tokens tokens per step, weak scaling).

--impl reference times the reference path's CPU implementation (the oracle's C
restatement of the Zig AVX2 path, all host threads) on the same config.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

EXPERT_BYTES = {}  # per config: bytes of one expert (3 projections + scales)


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one
# moe_decode_kernel launch, from an ncu capture of the same workload; other
# (config, tokens) pairs report null until captured.
NCU_TRAFFIC = {("c2", 1): 39.02e6, ("c3", 2048): 535.5e6}


def expert_bytes(d) -> int:
    nb = lambda x: (x + 127) // 128
    return 3 * d.inter * d.hidden + 4 * (2 * nb(d.inter) * nb(d.hidden) + nb(d.hidden) * nb(d.inter))


def shared_bytes(d) -> int:
    if not d.shared_inter:
        return 0
    nb = lambda x: (x + 127) // 128
    return 3 * d.shared_inter * d.hidden + 4 * 3 * nb(d.shared_inter) * nb(d.hidden) + 4 * d.hidden


PREFILL_MIN_TOKENS = 32  # the library's switch to the prefill path (grouped tcgen05 GEMMs)


def gen_tokens(args, d, T, seed, device, synth, dtype=None):
    import torch

    dt = dtype or torch.bfloat16
    if args.config == "c3":
        return synth.zipf_tokens(T, d.hidden, seed, device=device, dtype=dt)
    return synth.make_tokens(T, d.hidden, seed, device=device, dtype=dt)


def gen_layer(args, d, seed, device, synth):
    w = synth.make_layer(d, seed=seed, device=device)
    if args.config == "c3":
        synth.zipf_router(w, seed)
    return w


def algorithmic_bytes(d, T: int, U: float) -> float:
    """Bytes one layer call must move (survey 8d): U distinct experts' weights +
    scales, the f32 router, the shared expert, bf16 tokens in, f32 outputs out."""
    return U * expert_bytes(d) + shared_bytes(d) + d.experts * d.hidden * 4 + T * d.hidden * (2 + 4)


def algorithmic_flops(d, T: int) -> float:
    return T * (d.topk * 6 * d.hidden * d.inter + 2 * d.experts * d.hidden +
                (6 * d.hidden * d.shared_inter if d.shared_inter else 0))


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        j = json.load(open(p))
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def native_host_forwards(L, layer_ids, xh, T, oh, ih, gh, steps):
    """Seconds for `steps` synchronous host-pointer forwards (bf16 tokens), called
    from the native loop in libcz_hostbench.so, after one warm-up pass over every
    layer twice; None when the helper is not built."""
    import ctypes

    path = os.path.join(ROOT, "colizig_b200", "libcz_hostbench.so")
    if not os.path.exists(path):
        return None
    hb = ctypes.CDLL(path)
    hb.cz_hostbench_forwards.restype = ctypes.c_double
    hb.cz_hostbench_forwards.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                         ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                         ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]
    fn = ctypes.cast(L.colizig_cuda_moe_forward, ctypes.c_void_p).value
    lids = (ctypes.c_uint32 * len(layer_ids))(*layer_ids)
    xs = (ctypes.c_void_p * len(xh))(*[x.data_ptr() for x in xh])
    rc = ctypes.c_int(0)
    args = (lids, len(layer_ids), xs, len(xh), 1, T, oh.data_ptr(), ih.data_ptr(), gh.data_ptr(), ctypes.byref(rc))
    hb.cz_hostbench_forwards(fn, 2 * len(layer_ids), *args)  # warm-up: direct, then captured, per layer
    dt = hb.cz_hostbench_forwards(fn, steps, *args)
    if dt < 0:
        raise RuntimeError(f"colizig_cuda_moe_forward returned {rc.value} in the native loop")
    return dt


def timed_replays(torch, graph, stream, dev, reps):
    """Device time (ms) of `reps` replays of a captured graph, each between its own
    CUDA event pair on the launching stream, with L2 flushed (a 256 MB write, more
    than the 126 MB L2) before each replay, outside the event pair."""
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    ev = []
    for r in range(reps):
        flush.fill_(r & 0xFF)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        ev.append((e0, e1))
    torch.cuda.synchronize()
    del flush
    return [a.elapsed_time(b) for a, b in ev]


# Arithmetic of the decode kernel: gate/up multiply the stored E4M3 weights by the
# token split exactly into E4M3 terms (bf16 tokens: 2 terms, exact); down multiplies
# the weights (converted exactly to f16) by h carried as f16 hi + lo terms (22 bits);
# every sum is f32.
DECODE_DTYPE = "e4m3 x e4m3 token terms (gate/up), f16 x f16 hi/lo h terms (down), f32 sums"

REPLAYS = 7  # timed replays of the K-step graph; the reported time is their median


def cpu_sample(args, d, layers_np, T, seconds, threads):
    """Time the CPU oracle (restatement of the reference AVX2 path) on a bounded
    sample of the workload: as many steps as fit in ~`seconds`."""
    import torch

    import oracle
    from colizig_b200 import synth

    oracle_layer = oracle.layer_from_dict
    oracle.set_threads(threads)
    od = oracle.Dims(d.hidden, d.experts, d.topk, d.inter, d.shared_inter, d.norm_topk)
    ols = [oracle_layer(w) for w in layers_np]
    toks = [synth.tokens_f32(gen_tokens(args, d, T, 5000 + i, "cpu", synth)) for i in range(8 if T > 1 else 64)]
    oracle.moe_forward(ols[0], od, toks[0])  # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        oracle.moe_forward(ols[n % len(ols)], od, toks[n % len(toks)])
        n += 1
        dt = time.perf_counter() - t0
        if dt >= seconds or n >= 100000:
            break
    oracle.set_threads(1)
    return n * T / dt, n, dt


def reference_arm(args):
    import torch

    from colizig_b200 import synth

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if args.config == "c4":
        reference_stack(args)
        return
    if args.config == "attn":
        attn_reference(args)
        return
    d = synth.CONFIGS[args.config]
    T = args.tokens
    Ts = min(T, 64)  # each step: a bounded sample of the batch (prefill batches are thousands of tokens)
    cores = os.cpu_count() or 1
    layers = [synth.to_numpy_layer(gen_layer(args, d, i, "cpu", synth)) for i in range(args.cpu_layers)]
    import oracle

    oracle_layer = oracle.layer_from_dict
    oracle.set_threads(cores)
    od = oracle.Dims(d.hidden, d.experts, d.topk, d.inter, d.shared_inter, d.norm_topk)
    ols = [oracle_layer(w) for w in layers]
    toks = [synth.tokens_f32(gen_tokens(args, d, Ts, 9000 + i, "cpu", synth)) for i in range(args.steps + args.warmup)]
    for i in range(args.warmup):
        oracle.moe_forward(ols[i % len(ols)], od, toks[i])
    t0 = time.perf_counter()
    for i in range(args.steps):
        oracle.moe_forward(ols[i % len(ols)], od, toks[args.warmup + i])
    dt = time.perf_counter() - t0
    value = args.steps * Ts / dt
    line = {
        "impl": "reference", "metric": metric_name(args, T), "value": value,
        "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_block(args, d),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{args.steps} steps, each the {args.config} layer forward of {Ts} of the step's "
                                   f"{T} tokens, over {args.cpu_layers} layers (C restatement of the reference AVX2 "
                                   f"path, {cores} threads)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def stack_metric(NL, T):
    return f"MoE-stack ({NL} layers) {'prefill' if T >= PREFILL_MIN_TOKENS else 'decode'} tokens/s (c4, T={T})"


def stack_config(args, d, NL, T, world):
    return {"workload": f"c4: {NL} config-2 MoE layers, attention = identity, {T} f32 token(s)/step "
                        "through colizig_cuda_moe_stack_forward (rms + MoE + residual per layer)",
            "hidden": d.hidden, "experts": d.experts, "topk": d.topk, "moe_intermediate": d.inter,
            "layers": NL, "tokens_per_step": T, "tokens_per_gpu": args.tokens, "global_batch": T,
            "expert_weight_bytes": NL * d.experts * expert_bytes(d),
            "l2": "inputs larger than L2: each step streams every layer's routed experts",
            "parallelism": ep_label(world, T)}


def reference_stack(args):
    """--impl reference for config 4: the oracle's restatement of the reference's
    per-layer caller (model.zig:227-232: n = rms(h, w); h += moe(n)) over the
    stack, each step on a bounded sample of the batch (at most 64 tokens), the
    layers cycling through --cpu-layers distinct weight sets."""
    import torch

    import oracle
    from colizig_b200 import synth

    d = synth.CONFIGS["c2"]
    NL, T = args.layers, args.tokens * args.gpus
    Ts = min(T, 64)
    cores = os.cpu_count() or 1
    oracle.set_threads(cores)
    od = oracle.Dims(d.hidden, d.experts, d.topk, d.inter, d.shared_inter, d.norm_topk)
    ols = [oracle.layer_from_dict(synth.to_numpy_layer(synth.make_layer(d, seed=l, device="cpu")))
           for l in range(args.cpu_layers)]
    g = torch.Generator(device="cpu").manual_seed(77)
    norm_w = (1.0 + 0.05 * torch.randn(NL, d.hidden, generator=g)).numpy().astype(np.float32)

    def run(h):
        for l in range(NL):
            out, _, _ = oracle.moe_forward(ols[l % len(ols)], od, oracle.rms(h, norm_w[l], 1e-6))
            h = (h + out).astype(np.float32)
        return h

    toks = [synth.make_tokens(Ts, d.hidden, 30000 + i, device="cpu", dtype=torch.float32).numpy()
            for i in range(4)]
    for i in range(min(args.warmup, 3)):
        run(toks[i % 4])
    steps = max(1, min(args.steps, 5 if Ts > 1 else 20))  # bounded: a whole-stack step is 48 layer forwards
    t0 = time.perf_counter()
    for i in range(steps):
        run(toks[i % 4])
    dt = time.perf_counter() - t0
    value = steps * Ts / dt
    line = {
        "impl": "reference", "metric": stack_metric(NL, T), "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": steps, "warmup": min(args.warmup, 3), "ms_per_step": dt / steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": stack_config(args, d, NL, T, args.gpus),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{steps} steps, each the {NL}-layer stack (rms + MoE + residual per layer) over "
                                   f"{Ts} of the step's {T} tokens, layers cycling over {len(ols)} weight sets "
                                   f"(C restatement of the reference AVX2 path, {cores} threads)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def stack_main(args, world, rank, local, torch, dist, cz, _abi, moe, synth):
    """Config 4: the 48-layer stack of config-2 MoE layers (29 GB of E4M3 expert
    weights), attention = identity, through colizig_cuda_moe_stack_forward: per
    layer n = rms(h, w_l), h += moe_l(n) (model.zig:227-232).  One step = the
    whole stack over one batch of `--tokens` tokens per GPU."""
    d = synth.CONFIGS["c2"]
    NL = args.layers
    T = args.tokens * world
    dev = torch.device("cuda", local)
    layers = []
    for l in range(NL):
        w = synth.make_layer(d, seed=l, device=dev)
        layers.append(moe.Layer.from_weights(l, d, w, ep=world > 1))
        del w
    torch.cuda.empty_cache()
    g = torch.Generator(device="cpu").manual_seed(77)
    norm_w = (1.0 + 0.05 * torch.randn(NL, d.hidden, generator=g)).to(dev)
    n = args.warmup + args.steps
    xs = [synth.make_tokens(T, d.hidden, 30000 + i, device=dev, dtype=torch.float32) for i in range(n)]
    hs = torch.empty((n, T, d.hidden), dtype=torch.float32, device=dev)
    L = _abi.load()
    prefill = T >= PREFILL_MIN_TOKENS

    def step(i, sh):
        hs[i].copy_(xs[i])
        rc = L.colizig_cuda_moe_stack_forward(0, NL, norm_w.data_ptr(), 1e-6, hs[i].data_ptr(), T,
                                              _abi.COLIZIG_PTR_DEVICE, sh)
        if rc:
            raise cz.ColizigError("colizig_cuda_moe_stack_forward", rc)

    stream = torch.cuda.current_stream()
    for i in range(args.warmup):
        step(i, stream.cuda_stream)
    torch.cuda.synchronize()
    moe.check()
    if prefill:
        moe.kernel_timer(2 * NL * args.steps)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=torch.cuda.Stream(device=dev)):
        gs = torch.cuda.current_stream()
        for k in range(args.steps):
            step(args.warmup + k, gs.cuda_stream)
    graph.replay()
    torch.cuda.synchronize()
    moe.check()
    sampler = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)
    t0e = torch.cuda.Event(enable_timing=True)
    t1e = torch.cuda.Event(enable_timing=True)
    t0e.record(stream)
    graph.replay()
    t1e.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    moe.check()
    elapsed_ms = t0e.elapsed_time(t1e)
    if world > 1:
        tt = torch.tensor([elapsed_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        elapsed_ms = float(tt.item())
    value = args.steps * T / (elapsed_ms / 1e3)
    gemm = {}
    if prefill:
        for kind, ms in moe.kernel_timer_read():
            gemm.setdefault(kind, []).append(ms)
        moe.kernel_timer(0)
    del graph

    # end to end: host h (pinned), the C ABI copies it in and the result out each step
    hh = [xs[i % 8].cpu().pin_memory() for i in range(min(n, 8))]

    # host norm weights for the host-pointer call
    nw_host = norm_w.cpu().contiguous()

    def e2e_step_h(i):
        rc = L.colizig_cuda_moe_stack_forward(0, NL, nw_host.data_ptr(), 1e-6, hh[i % len(hh)].data_ptr(), T, 0, None)
        if rc:
            raise cz.ColizigError("colizig_cuda_moe_stack_forward", rc)

    ke = max(1, min(args.steps, 20))
    for i in range(2):
        e2e_step_h(i)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for k in range(ke):
        e2e_step_h(k)
    e2e_s = time.perf_counter() - t0
    if world > 1:
        tt = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_s = float(tt.item())
    e2e = {"value": ke * T / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": T * d.hidden * 4 + NL * d.hidden * 4,
           "d2h_bytes_per_step": T * d.hidden * 4, "ms_per_step": e2e_s / ke * 1e3}

    hbm_peak, tf_peak, peak_kind = load_peaks()
    step_ms = elapsed_ms / args.steps
    if prefill:
        fp8_peak = 2.0 * tf_peak
        gu = float(np.mean(gemm[moe.TIMER_PREFILL_GATE_UP]))
        dn = float(np.mean(gemm[moe.TIMER_PREFILL_DOWN]))
        pairs = T * d.topk / world  # average pairs per rank and layer
        gu_flops = 2.0 * pairs * d.hidden * 2 * d.inter
        tf = gu_flops / (gu / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": tf, "peak": fp8_peak, "unit": "TFLOP/s", "frac": tf / fp8_peak,
                "traffic": None, "kernel": "pf_gemm_kernel (gate/up), per layer", "kernel_ms_avg": gu,
                "flops_per_launch": gu_flops,
                "peak_kind": f"FP8 dense = 2 x {peak_kind} bf16 (MEASURED_PEAKS.json bf16_tflops)",
                "down_gemm": {"kernel_ms_avg": dn, "achieved_tflops": gu_flops / 2 / (dn / 1e3) / 1e12},
                "step": {"ms": step_ms, "flops": NL * algorithmic_flops(d, T) / world,
                         "achieved_tflops": NL * algorithmic_flops(d, T) / world / (step_ms / 1e3) / 1e12}}
    else:
        # decode: every layer call moves its U = top-k distinct experts (T = 1) + router + token rows
        U = float(d.topk) if T == 1 else float(min(d.experts, T * d.topk))
        per_layer = algorithmic_bytes(d, T, U) + (world - 1) * d.experts * d.hidden * 4
        gbs = NL * per_layer / world / (step_ms / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
                "traffic": NCU_TRAFFIC.get(("c2", T)) if world == 1 else None,
                "traffic_unit": "DRAM bytes per moe_decode_kernel launch (ncu, config 2)",
                "kernel": "moe_decode_kernel, one launch per layer (rms and residual fused)",
                "kernel_ms_avg": step_ms / NL, "bytes_per_launch": per_layer / world,
                "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cores = os.cpu_count() or 1
        Tc = min(T, 64)
        host_layers = [synth.to_numpy_layer(synth.make_layer(d, seed=l, device="cpu")) for l in range(args.cpu_layers)]
        v, nsteps, dt = cpu_sample(args, d, host_layers, Tc, args.cpu_seconds, cores)
        cpu = {"value": v / NL, "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"{nsteps} config-2 layer forwards of T={Tc} in {dt:.1f} s (C restatement of the reference "
                         f"AVX2 path, {cores} threads); stack tokens/s = layer tokens/s / {NL} (rms and residual "
                         "not timed)"}
    if rank == 0:
        line = {
            "metric": stack_metric(NL, T),
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "e4m3 x e4m3 -> f32", "data": "synthetic",
            "config": stack_config(args, d, NL, T, world),
            "roofline": roof, "e2e": e2e, "cpu_baseline": cpu, "clocks": clocks,
            "gpu_launches": args.steps * NL * (12 if prefill else  # prefill: rms + 11
                                               -(-T // L.colizig_cuda_moe_decode_batch(layers[0].id, 0))),
        }
        print(json.dumps(line), flush=True)
    for lay in layers:
        lay.unregister()


def sharded_main(args, world, rank, local, torch, dist, cz, _abi, moe, synth):
    """Expert-parallel prefill with sharded tokens (N > 1): every rank routes its own
    --tokens rows, sends each row to the ranks holding its experts, runs the grouped
    GEMMs on the rows it receives and adds the partial sums of its own tokens.  The
    library reads the exchange's row counts on the host, so the steps are issued one
    by one (no CUDA graph) and timed with CUDA events around all of them."""
    from colizig_b200 import ep

    d = synth.CONFIGS[args.config]
    Tr = args.tokens
    T = Tr * world
    dev = torch.device("cuda", local)
    layers = []
    for l in range(args.layers):
        w = gen_layer(args, d, l, dev, synth)  # the same layer on every rank
        layers.append(moe.Layer.from_weights(l, d, w, ep=True))
        del w
    torch.cuda.empty_cache()
    n = args.warmup + args.steps
    # rank r's rows of step i: rows [r*Tr, (r+1)*Tr) of that step's job-wide batch
    xs = [gen_tokens(args, d, T, 20000 + i, dev, synth)[rank * Tr:(rank + 1) * Tr].contiguous() for i in range(n)]
    outs = torch.empty((n, Tr, d.hidden), dtype=torch.float32, device=dev)
    idx = torch.empty((n, Tr, d.topk), dtype=torch.int32, device=dev)
    gates = torch.empty((n, Tr, d.topk), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream()
    L = _abi.load()
    sh = stream.cuda_stream
    flags = _abi.COLIZIG_PTR_DEVICE | _abi.COLIZIG_EP_SHARDED

    def step(i):
        lay = layers[i % len(layers)]
        rc = L.colizig_cuda_moe_forward(lay.id, xs[i].data_ptr(), _abi.COLIZIG_X_BF16, Tr, outs[i].data_ptr(),
                                        idx[i].data_ptr(), gates[i].data_ptr(), flags, sh)
        if rc:
            raise cz.ColizigError("colizig_cuda_moe_forward", rc)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    moe.check()
    moe.kernel_timer(2 * args.steps)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    flush.fill_(1)
    del flush
    sampler = ClockSampler(local)
    dist.barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for k in range(args.steps):
        step(args.warmup + k)
    t_end.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    dist.barrier()
    moe.check()
    elapsed_ms = t_start.elapsed_time(t_end)
    gemm_ms = {}
    for kind, ms in moe.kernel_timer_read():
        gemm_ms.setdefault(kind, []).append(ms)
    moe.kernel_timer(0)
    tt = torch.tensor([elapsed_ms], device=dev)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    elapsed_ms = float(tt.item())
    value = args.steps * T / (elapsed_ms / 1e3)

    # pairs this rank's GEMMs processed: every rank's (token, expert) pairs on its experts
    lo, hi = ep.expert_range(rank, world, d.experts)
    hist = torch.stack([torch.bincount(idx[args.warmup + k].reshape(-1).long(), minlength=d.experts)
                        for k in range(args.steps)]).to(torch.float64)
    dist.all_reduce(hist)
    hist = hist.cpu().numpy()
    pairs_local = float(hist[:, lo:hi].sum(axis=1).mean())
    gu_flops = 2.0 * pairs_local * d.hidden * 2 * d.inter
    dn_flops = 2.0 * pairs_local * d.inter * d.hidden
    gu_ms = float(np.mean(gemm_ms.get(moe.TIMER_PREFILL_GATE_UP, [float("nan")])))
    dn_ms = float(np.mean(gemm_ms.get(moe.TIMER_PREFILL_DOWN, [float("nan")])))
    hbm_peak, tf_peak, peak_kind = load_peaks()
    fp8_peak = 2.0 * tf_peak
    tf = gu_flops / (gu_ms / 1e3) / 1e12
    step_tf = algorithmic_flops(d, T) * args.steps / (elapsed_ms / 1e3) / 1e12 / world
    U = (hist > 0).sum(axis=1)

    # end to end: this rank's rows from pinned host memory, outputs back to host memory
    xh = [x.cpu().pin_memory() for x in xs[:min(n, 64)]]
    oh = torch.empty((Tr, d.hidden), dtype=torch.float32).pin_memory()
    ih = torch.empty((Tr, d.topk), dtype=torch.int32).pin_memory()
    gh = torch.empty((Tr, d.topk), dtype=torch.float32).pin_memory()

    def e2e_step(i):
        lay = layers[i % len(layers)]
        rc = L.colizig_cuda_moe_forward(lay.id, xh[i % len(xh)].data_ptr(), _abi.COLIZIG_X_BF16, Tr, oh.data_ptr(),
                                        ih.data_ptr(), gh.data_ptr(), _abi.COLIZIG_EP_SHARDED, None)
        if rc:
            raise cz.ColizigError("colizig_cuda_moe_forward", rc)

    for i in range(args.warmup):
        e2e_step(i)
    dist.barrier()
    t0 = time.perf_counter()
    for k in range(args.steps):
        e2e_step(args.warmup + k)
    e2e_s = time.perf_counter() - t0
    tt = torch.tensor([e2e_s], device=dev)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    e2e_s = float(tt.item())
    e2e = {"value": args.steps * T / e2e_s, "unit": "tokens/s",
           "h2d_bytes_per_step": Tr * d.hidden * 2, "d2h_bytes_per_step": Tr * d.hidden * 4 + Tr * d.topk * 8,
           "bytes_are": "per rank (each rank copies its own rows)", "ms_per_step": e2e_s / args.steps * 1e3}

    if rank == 0:
        cfg = config_block(args, d)
        cfg["parallelism"] = (f"ep{world}, sharded tokens: each rank routes its own {Tr} rows, rows go to the ranks "
                              "holding their experts and partial sums come back over NCCL send/recv")
        cfg["l2"] = "inputs larger than L2: steps cycle through distinct layers; L2 flushed once before the timed steps"
        roof = {"bound": "tensor", "achieved": tf, "peak": fp8_peak, "unit": "TFLOP/s", "frac": tf / fp8_peak,
                "traffic": None, "traffic_unit": "DRAM bytes per gate/up GEMM launch (ncu; captured on one GPU only)",
                "peak_kind": (f"FP8 dense = 2 x {peak_kind} bf16 (MEASURED_PEAKS.json bf16_tflops)"
                              if peak_kind == "measured" else "FP8 dense = 2 x fallback 1.59 PFLOP/s"),
                "kernel": "pf_gemm_kernel (gate/up, tcgen05 grouped GEMM with the SiLU*up epilogue), rank 0",
                "kernel_ms_avg": gu_ms, "flops_per_launch": gu_flops,
                "down_gemm": {"kernel_ms_avg": dn_ms, "flops_per_launch": dn_flops,
                              "achieved_tflops": dn_flops / (dn_ms / 1e3) / 1e12,
                              "frac": dn_flops / (dn_ms / 1e3) / 1e12 / fp8_peak},
                "step": {"ms": elapsed_ms / args.steps, "flops": algorithmic_flops(d, T) / world,
                         "achieved_tflops": step_tf, "frac": step_tf / fp8_peak},
                "distinct_experts_avg": float(U.mean())}
        line = {
            "metric": metric_name(args, T), "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "e4m3 x e4m3 -> f32", "data": "synthetic",
            "config": cfg, "roofline": roof, "tflops": step_tf * world,
            "e2e": e2e, "cpu_baseline": None, "clocks": clocks,
            # route (logits, top-k), plan (mask, slots), pack, unpack, xexp, xterms, count, scan, place,
            # tokpos, dispatch, 2 GEMMs, combine, ep_combine (NCCL's own kernels not counted)
            "gpu_launches": args.steps * 17,
        }
        print(json.dumps(line), flush=True)
    for lay in layers:
        lay.unregister()


# ---- attention projections (config "attn") -----------------------------------
# The FP8 projections of Qwen3-30B-A3B's attention (src/qwen3moe/attn.zig:46-78):
# q [32*128, 2048], k and v [4*128, 2048], o [2048, 32*128], E4M3 with 128 x 128
# block scales, keyed by attnKey and computed by the per-matrix call
# colizig_cuda_matmul_fp8 (matmulFp8Keyed, src/ops/fp8.zig:165-188).  One step =
# the four projections of one layer for the step's tokens (the attention core
# between them is outside this path).
ATTN_SHAPES = ((32 * 128, 2048), (4 * 128, 2048), (4 * 128, 2048), (2048, 32 * 128))  # q, k, v, o: (O, I)


def attn_layer(l, synth, torch):
    gen = torch.Generator(device="cpu")
    gen.manual_seed(7000 + l)
    return [(synth._e4m3((O, I), gen, "cpu").numpy(), synth._scales(((O + 127) // 128, (I + 127) // 128), gen,
                                                                       "cpu").numpy()) for O, I in ATTN_SHAPES]


def attn_inputs(T, i):
    rng = np.random.default_rng(9100 + i)
    return (rng.standard_normal((T, ATTN_SHAPES[0][1])).astype(np.float32),
            rng.standard_normal((T, ATTN_SHAPES[3][1])).astype(np.float32))


def attn_bytes(T):
    nb = lambda x: (x + 127) // 128  # noqa: E731
    return sum(O * I + nb(O) * nb(I) * 4 + T * (I + O) * 4 for O, I in ATTN_SHAPES)


def attn_config(args):
    return {"workload": f"Qwen3-30B-A3B attention projections q/k/v/o (FP8 E4M3, 128x128 block scales), "
                        f"{args.tokens} token(s)/step, one layer's four keyed calls per step",
            "hidden": 2048, "q_heads": 32, "kv_heads": 4, "head_dim": 128, "tokens_per_step": args.tokens,
            "global_batch": args.tokens, "layers_cycled": args.layers,
            "l2": "inputs larger than L2: steps cycle through the layers' weights",
            "parallelism": "single GPU"}


def attn_main(args, torch, cz, moe, synth):
    """Our arm.  value: the four projections of every step as device-pointer
    launches (colizig_cuda_matmul_fp8_device) in one captured CUDA graph, timed by
    CUDA events (median of the replays, L2 flushed before each).  e2e: the keyed
    host-pointer calls the reference makes (colizig_cuda_matmul_fp8 with attnKey
    keys, synchronous, weights resident after the first call of each key)."""
    from colizig_b200 import _abi

    T, NL = args.tokens, args.layers
    L = [attn_layer(l, synth, torch) for l in range(NL)]
    xs = [attn_inputs(T, i) for i in range(16)]
    dev = torch.device("cuda", 0)
    lib = _abi.load()
    Wd = [[(torch.from_numpy(w).to(dev), torch.from_numpy(sc).to(dev)) for w, sc in L[l]] for l in range(NL)]
    xd = [(torch.from_numpy(x).to(dev), torch.from_numpy(a).to(dev)) for x, a in xs]
    outs = [torch.empty((T, O), dtype=torch.float32, device=dev) for O, _ in ATTN_SHAPES]

    def dstep(i, sh):
        x, a = xd[i % len(xd)]
        for r, (O, I) in enumerate(ATTN_SHAPES):
            w, sc = Wd[i % NL][r]
            rc = lib.colizig_cuda_matmul_fp8_device(outs[r].data_ptr(), (a if r == 3 else x).data_ptr(),
                                                    w.data_ptr(), sc.data_ptr(), T, I, O, sh)
            if rc:
                raise cz.ColizigError("colizig_cuda_matmul_fp8_device", rc)

    stream = torch.cuda.current_stream()
    for i in range(args.warmup):
        dstep(i, stream.cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=torch.cuda.Stream(device=dev)):
        gs = torch.cuda.current_stream().cuda_stream
        for k in range(args.steps):
            dstep(args.warmup + k, gs)
    graph.replay()
    torch.cuda.synchronize()
    sampler = ClockSampler(0)
    sampler.start()
    time.sleep(0.3)
    replay_ms = timed_replays(torch, graph, stream, dev, REPLAYS)
    clocks = sampler.stop()
    del graph
    step_ms = float(statistics.median(replay_ms)) / args.steps
    hbm_peak, _, peak_kind = load_peaks()
    gbs = attn_bytes(T) / (step_ms / 1e3) / 1e9

    # end to end: the reference's calls, host buffers, keyed residency
    cz.gpu.set_vram_budget(1 << 34)
    key = cz.fp8.attn_key

    def hstep(i):
        l = i % NL
        x, a = xs[i % len(xs)]
        for r in range(4):
            cz.fp8.matmul_fp8_keyed(a if r == 3 else x, *L[l][r], key=key(l, r))

    for i in range(max(args.warmup, NL)):  # every key uploaded once (misses), then hits
        hstep(i)
    h0, m0, _, _ = cz.gpu.stats()
    t0 = time.perf_counter()
    for k in range(args.steps):
        hstep(args.warmup + k)
    e2e_s = time.perf_counter() - t0
    h1, m1, _, _ = cz.gpu.stats()
    if (h1 - h0, m1 - m0) != (4 * args.steps, 0):
        raise RuntimeError(f"keyed store: {h1 - h0} hits, {m1 - m0} misses in the timed calls")
    cz.gpu.set_vram_budget(0)
    cpu = None
    if not args.no_cpu:
        import oracle

        cores = os.cpu_count() or 1
        oracle.set_threads(cores)
        n, c0 = 0, time.perf_counter()
        while time.perf_counter() - c0 < args.cpu_seconds / 3 and n < 10000:
            x, a = xs[n % len(xs)]
            for r in range(4):
                oracle.matmul_fp8(a if r == 3 else x, *L[n % NL][r])
            n += 1
        dt = time.perf_counter() - c0
        oracle.set_threads(1)
        cpu = {"value": n * T / dt, "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"{n} steps (4 projections of T={T}) in {dt:.1f} s over {NL} layers (C restatement of "
                         f"matmulFp8Cpu, {cores} threads)"}
    line = {
        "metric": f"attention-projection tokens/s (Qwen3-30B-A3B q/k/v/o, T={T})",
        "value": T / (step_ms / 1e3), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "e4m3 weights (f16 decode) x f32 tokens -> f32",
        "data": "synthetic", "config": attn_config(args),
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
                     "traffic": None, "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                     "kernel": "fp8_matmul_kernel (four launches a step)", "bytes_per_step": attn_bytes(T)},
        "e2e": {"value": args.steps * T / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": T * (3 * 2048 + 4096) * 4,
                "d2h_bytes_per_step": T * (4096 + 512 + 512 + 2048) * 4, "ms_per_step": e2e_s / args.steps * 1e3,
                "caller": "python ctypes, four synchronous host-pointer colizig_cuda_matmul_fp8 calls a step "
                          "(attnKey keys, resident)"},
        "cpu_baseline": cpu, "clocks": clocks,
        "timing": {"replays": REPLAYS, "replay_ms": replay_ms, "statistic": "median over replays",
                   "l2": f"flushed before each replay; steps cycle through {NL} layers ({NL * attn_bytes(0) >> 20} MiB)"},
        "gpu_launches": 4 * args.steps,
    }
    print(json.dumps(line), flush=True)


def attn_reference(args):
    """Reference arm: the oracle's restatement of matmulFp8Cpu on the same calls."""
    import torch

    import oracle
    from colizig_b200 import synth

    T, NL = args.tokens, min(args.layers, 4)
    L = [attn_layer(l, synth, torch) for l in range(NL)]
    xs = [attn_inputs(T, i) for i in range(16)]
    cores = os.cpu_count() or 1
    oracle.set_threads(cores)

    def step(i):
        x, a = xs[i % len(xs)]
        for r in range(4):
            oracle.matmul_fp8(a if r == 3 else x, *L[i % NL][r])

    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    for k in range(args.steps):
        step(args.warmup + k)
    dt = time.perf_counter() - t0
    value = args.steps * T / dt
    print(json.dumps({
        "impl": "reference", "metric": f"attention-projection tokens/s (Qwen3-30B-A3B q/k/v/o, T={T})",
        "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic", "config": attn_config(args),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{args.steps} steps of the four projections over {NL} layers (C restatement "
                                   f"of matmulFp8Cpu, {cores} threads)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}), flush=True)


def metric_name(args, T):
    mode = "prefill" if T >= PREFILL_MIN_TOKENS else "decode"
    return f"MoE-layer {mode} tokens/s ({args.config}, T={T})"


def ep_label(world, T):
    if world < 2:
        return "single GPU"
    if T >= PREFILL_MIN_TOKENS:
        return f"ep{world}: experts partitioned over the GPUs, router replicated, NCCL all-reduce of each layer's output"
    return (f"ep{world}: experts partitioned over the GPUs, router replicated, ranks summed inside the decode "
            "kernel (partial rows stored into every rank's peer-mapped buffer over NVLink)")


def config_block(args, d):
    g = args.tokens * args.gpus
    if g >= PREFILL_MIN_TOKENS:
        wl = (f"{args.config} MoE layer prefill, {g} tokens/step (config 3: Zipf-skewed routing)"
              if args.config == "c3" else f"{args.config} MoE layer prefill, {g} tokens/step")
    else:
        wl = f"{args.config} MoE layer decode, {g} token(s)/step (config 2)"
    return {"workload": wl,
            "hidden": d.hidden, "experts": d.experts, "topk": d.topk, "moe_intermediate": d.inter,
            "shared_intermediate": d.shared_inter, "tokens_per_step": g, "tokens_per_gpu": args.tokens,
            "global_batch": g, "layers_cycled": args.layers,
            "l2": "inputs larger than L2: steps cycle through distinct layers; L2 flushed once before the timed replay",
            "parallelism": ep_label(args.gpus, g)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c2")
    ap.add_argument("--tokens", type=int, default=None)
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--cpu-layers", type=int, default=4)
    ap.add_argument("--no-cpu", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    prefill_cfg = args.config == "c3"
    if args.tokens is None:
        args.tokens = 2048 if prefill_cfg else 1
    big = args.tokens * args.gpus >= PREFILL_MIN_TOKENS
    if args.steps is None:
        args.steps = 20 if big else 200
    if args.config == "c4":
        args.layers = args.layers or 48
    if args.layers is None:
        args.layers = 4 if big else 16

    if args.impl == "reference":
        reference_arm(args)
        return

    import torch
    import torch.distributed as dist

    import colizig_b200 as cz
    from colizig_b200 import _abi, moe, synth

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    cz.gpu.init(local)
    if world > 1:
        # expert parallelism: rank r holds experts [r*E/W, (r+1)*E/W) of every layer; the
        # ranks' outputs are summed inside the decode kernel (or by NCCL for prefill batches)
        from colizig_b200 import ep

        ep.init()
    if args.config == "attn":
        if world > 1:
            raise SystemExit("--config attn runs on one GPU")
        attn_main(args, torch, cz, moe, synth)
        return
    if args.config == "c4":
        stack_main(args, world, rank, local, torch, dist, cz, _abi, moe, synth)
        if world > 1:
            from colizig_b200 import ep

            torch.cuda.synchronize()
            ep.shutdown()
            dist.destroy_process_group()
        return
    if world > 1 and args.tokens >= PREFILL_MIN_TOKENS:
        sharded_main(args, world, rank, local, torch, dist, cz, _abi, moe, synth)
        from colizig_b200 import ep

        torch.cuda.synchronize()
        ep.shutdown()
        dist.destroy_process_group()
        return
    d = synth.CONFIGS[args.config]
    T = args.tokens * world  # tokens per step over the whole job (each rank contributes --tokens)
    dev = torch.device("cuda", local)

    layers, host_layers = [], []
    for l in range(args.layers):
        w = gen_layer(args, d, l, dev, synth)  # the same layer on every rank
        layers.append(moe.Layer.from_weights(l, d, w, ep=world > 1))
        if rank == 0 and world == 1 and l < args.cpu_layers and not args.no_cpu:
            host_layers.append(synth.to_numpy_layer(w))
        del w
    torch.cuda.empty_cache()

    n = args.warmup + args.steps
    xs = [gen_tokens(args, d, T, 20000 + i, dev, synth) for i in range(n)]
    outs = torch.empty((n, T, d.hidden), dtype=torch.float32, device=dev)
    idx = torch.empty((n, T, d.topk), dtype=torch.int32, device=dev)
    gates = torch.empty((n, T, d.topk), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream()
    L = _abi.load()
    sh = stream.cuda_stream

    def step(i, stream_handle=None):
        lay = layers[i % len(layers)]
        rc = L.colizig_cuda_moe_forward(lay.id, xs[i].data_ptr(), _abi.COLIZIG_X_BF16, T, outs[i].data_ptr(),
                                        idx[i].data_ptr(), gates[i].data_ptr(), _abi.COLIZIG_PTR_DEVICE,
                                        sh if stream_handle is None else stream_handle)
        if rc:
            raise cz.ColizigError("colizig_cuda_moe_forward", rc)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    moe.check()

    # The timed steps are captured once into a CUDA graph (one kernel node per
    # step) so the timing is not bounded by the host's launch rate.
    prefill = T >= PREFILL_MIN_TOKENS
    if prefill:
        # event pairs around the grouped GEMM launches of every captured step, so the
        # dominant kernel's own device time comes out of the timed replay itself
        moe.kernel_timer(2 * args.steps)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=torch.cuda.Stream(device=dev)):
        gs = torch.cuda.current_stream().cuda_stream
        for k in range(args.steps):
            step(args.warmup + k, gs)
    graph.replay()  # untimed replay: instantiation / first-upload costs
    torch.cuda.synchronize()
    moe.check()
    sampler = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)
    replay_ms = timed_replays(torch, graph, stream, dev, REPLAYS)
    clocks = sampler.stop()
    if world > 1:
        dist.barrier()
    moe.check()
    elapsed_ms = float(statistics.median(replay_ms))
    kernel_ms = [elapsed_ms / args.steps] * args.steps  # one kernel per step, back to back
    gemm_ms = {}
    if prefill:
        for kind, ms in moe.kernel_timer_read():
            gemm_ms.setdefault(kind, []).append(ms)
        moe.kernel_timer(0)
    if world > 1:
        tt = torch.tensor([elapsed_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        elapsed_ms = float(tt.item())
    value = args.steps * T / (elapsed_ms / 1e3)
    del graph

    # realised distinct experts per step -> algorithmic bytes
    ids = idx[args.warmup:].cpu().numpy()
    U = np.array([len(np.unique(ids[k])) for k in range(args.steps)], np.float64)
    # whole-job algorithmic bytes (the router is read on every rank), per GPU on average
    bytes_per = np.array([algorithmic_bytes(d, T, u) + (world - 1) * d.experts * d.hidden * 4 for u in U]) / world
    hbm_peak, tf_peak, peak_kind = load_peaks()
    achieved_gbs = float(bytes_per.sum() / (np.sum(kernel_ms) / 1e3) / 1e9)

    # end to end through the C ABI with host buffers (pinned), synchronous calls
    xh = [x.cpu().pin_memory() for x in xs[:min(n, 64)]]
    oh = torch.empty((T, d.hidden), dtype=torch.float32).pin_memory()
    ih = torch.empty((T, d.topk), dtype=torch.int32).pin_memory()
    gh = torch.empty((T, d.topk), dtype=torch.float32).pin_memory()

    def e2e_step(i):
        lay = layers[i % len(layers)]
        rc = L.colizig_cuda_moe_forward(lay.id, xh[i % len(xh)].data_ptr(), _abi.COLIZIG_X_BF16, T, oh.data_ptr(),
                                        ih.data_ptr(), gh.data_ptr(), 0, None)
        if rc:
            raise cz.ColizigError("colizig_cuda_moe_forward", rc)

    # warm-up: every layer twice, so that each (layer, batch) host call has been run
    # once directly and captured once (the library replays host-pointer decode calls
    # from a captured CUDA graph from the second call on)
    for i in range(max(args.warmup, 2 * len(layers))):
        e2e_step(i)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for k in range(args.steps):
        e2e_step(args.warmup + k)
    e2e_s = time.perf_counter() - t0
    if world > 1:
        tt = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_s = float(tt.item())
    py_e2e_s = e2e_s
    # The same calls from a native caller loop (the reference's host is a compiled
    # program calling the C ABI, src/backend/gpu.zig): no interpreter between calls.
    native_s = native_host_forwards(L, [lay.id for lay in layers], xh, T, oh, ih, gh, args.steps)
    if native_s is not None:
        if world > 1:
            tt = torch.tensor([native_s], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            native_s = float(tt.item())
        e2e_s = native_s
    e2e = {"value": args.steps * T / e2e_s, "unit": "tokens/s",
           "h2d_bytes_per_step": T * d.hidden * 2, "d2h_bytes_per_step": T * d.hidden * 4 + T * d.topk * 8,
           "ms_per_step": e2e_s / args.steps * 1e3,
           "caller": ("native C loop through colizig_cuda_moe_forward (libcz_hostbench.so)" if native_s is not None
                      else "python ctypes"),
           "python_ctypes_ms_per_step": py_e2e_s / args.steps * 1e3}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cores = os.cpu_count() or 1
        Tc = min(T, 64)  # bounded sample for prefill batches
        v, nsteps, dt = cpu_sample(args, d, host_layers, Tc, args.cpu_seconds, cores)
        v1, n1, dt1 = cpu_sample(args, d, host_layers, Tc, max(3.0, args.cpu_seconds / 3), 1)
        cpu = {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"{nsteps} layer forwards of {args.config} T={Tc} in {dt:.1f} s over {len(host_layers)} "
                         f"layers (C restatement of the reference AVX2 path, {cores} threads)",
               "single_thread": {"value": v1, "unit": "tokens/s", "cores": 1,
                                 "sample": f"{n1} layer forwards of {args.config} T={Tc} in {dt1:.1f} s, 1 thread"}}

    timing = {"replays": REPLAYS, "replay_ms": replay_ms, "statistic": "median over replays, max over ranks",
              "l2": "flushed (256 MB write) before each replay; steps cycle through "
                    f"{len(layers)} layers, so no step finds its weights in L2"}
    # prefill: logits, topk, xterms, count, scan, place, tokpos, dispatch, 2 GEMMs, combine;
    # decode: ceil(T / tokens per launch) launches of the decode kernel
    launches_per_step = 11 if prefill else -(-T // L.colizig_cuda_moe_decode_batch(layers[0].id, _abi.COLIZIG_X_BF16))
    if prefill:
        # tensor-bound.  Dominant kernel: the gate/up grouped GEMM.  Its algorithmic FLOPs
        # (2 x pairs x H x 2I routed + 2 x T x H x 2SI shared, pairs on this rank's
        # experts) over its own device time from the timer's event pairs, against the FP8
        # dense peak taken as 2 x the measured cuBLAS bf16 throughput.
        lo, hi = (0, d.experts) if world == 1 else ep.expert_range(rank, world, d.experts)
        ids_t = idx[args.warmup:].cpu().numpy()
        pairs_local = float(np.mean([((ids_t[k] >= lo) & (ids_t[k] < hi)).sum() for k in range(args.steps)]))
        sh_t = T if (d.shared_inter and rank == 0) else 0
        gu_flops = 2.0 * pairs_local * d.hidden * 2 * d.inter + 2.0 * sh_t * d.hidden * 2 * d.shared_inter
        dn_flops = 2.0 * pairs_local * d.inter * d.hidden + 2.0 * sh_t * d.shared_inter * d.hidden
        gu_ms = float(np.mean(gemm_ms[moe.TIMER_PREFILL_GATE_UP]))
        dn_ms = float(np.mean(gemm_ms[moe.TIMER_PREFILL_DOWN]))
        tf = gu_flops / (gu_ms / 1e3) / 1e12
        step_tf = algorithmic_flops(d, T) * args.steps / (elapsed_ms / 1e3) / 1e12 / world
        fp8_peak = 2.0 * tf_peak
        roof = {"bound": "tensor", "achieved": tf, "peak": fp8_peak, "unit": "TFLOP/s", "frac": tf / fp8_peak,
                "traffic": NCU_TRAFFIC.get((args.config, T)) if world == 1 else None,
                "traffic_unit": "DRAM bytes per gate/up GEMM launch (ncu)",
                "peak_kind": (f"FP8 dense = 2 x {peak_kind} bf16 (MEASURED_PEAKS.json bf16_tflops)"
                              if peak_kind == "measured" else "FP8 dense = 2 x fallback 1.59 PFLOP/s"),
                "kernel": "pf_gemm_kernel (gate/up, tcgen05 grouped GEMM with the SiLU*up epilogue)",
                "kernel_ms_avg": gu_ms, "flops_per_launch": gu_flops,
                "down_gemm": {"kernel_ms_avg": dn_ms, "flops_per_launch": dn_flops,
                              "achieved_tflops": dn_flops / (dn_ms / 1e3) / 1e12,
                              "frac": dn_flops / (dn_ms / 1e3) / 1e12 / fp8_peak},
                "step": {"ms": elapsed_ms / args.steps, "flops": algorithmic_flops(d, T) / world,
                         "achieved_tflops": step_tf, "frac": step_tf / fp8_peak},
                "distinct_experts_avg": float(U.mean()),
                "top_expert_pairs_avg": float(np.mean([np.bincount(ids[k].ravel()).max() for k in range(args.steps)]))}
    else:
        roof = None
    if rank == 0:
        line = {
            "metric": metric_name(args, T), "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "e4m3 x e4m3 -> f32" if prefill else DECODE_DTYPE, "data": "synthetic",
            "config": config_block(args, d),
            "hbm_gbs": achieved_gbs,
            "roofline": roof or {"bound": "hbm", "achieved": achieved_gbs, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved_gbs / hbm_peak, "traffic": NCU_TRAFFIC.get((args.config, T)),
                         "traffic_unit": "bytes per launch (ncu)",
                         "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback 6.65 TB/s",
                         "kernel": "moe_decode_kernel", "kernel_ms_avg": float(np.mean(kernel_ms)),
                         "bytes_per_launch_avg": float(bytes_per.mean()), "distinct_experts_avg": float(U.mean())},
            "tflops": algorithmic_flops(d, T) * args.steps / (np.sum(kernel_ms) / 1e3) / 1e12,
            "e2e": e2e, "cpu_baseline": cpu, "clocks": clocks, "timing": timing,
            "gpu_launches": args.steps * launches_per_step,
        }
        if world > 1:
            line["ep_combine"] = ("in the decode kernel (peer stores)" if ep.combine_mode() == 1 and not prefill
                                  else "NCCL all-reduce")
        print(json.dumps(line), flush=True)
    for lay in layers:
        lay.unregister()
    if world > 1:
        from colizig_b200 import ep

        torch.cuda.synchronize()
        ep.shutdown()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
