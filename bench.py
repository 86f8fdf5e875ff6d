"""Benchmark of the mixture-of-experts hot path on B200 (driver contract: one JSON line).

Workload (the metric's decode b=1 case): one MoE layer, H 2048, 512
routed experts, top-10 renormalised routing, one shared expert, expert intermediate 512,
Q2 packed blobs (uniform 2-bit codes, FP16 scales |N(0,0.02)|), F32 router N(0,0.02),
F32 activations N(0,1); seeded synthetic data. A step is one pass of the fused layer over
one batch. `--batch 8` and `--batch 64` are config 2's other decode sizes; `--batch 4096`
is config 3 (prefill, router logits biased by a Zipf(1.1) per-expert offset). Batches of 9 to
64 run the medium-batch layer (HBM roofline, like decode); batches above 64 run the
tensor-core prefill path, whose roofline is the grouped GEMMs' FLOP rate against the
measured sustained dense BF16 peak, timed by the library's phase profile in a second pass.
Steps cycle over `--layers` distinct layer replicas (default 24: every layer's
routed weights are evicted from the 126 MB L2 before the layer comes round again) with a
fresh activation batch per step, so no step reads weights left in L2 by the previous one.

  value   device time (CUDA events on the library's stream) of K fused steps, inputs
          resident in HBM; whole-job tokens/s (sum over ranks / max time over ranks).
  e2e     the same steps through the C-ABI with host buffers: strata_write of the batch
          from pinned memory, the layer call (replayed from its captured CUDA graph with
          strata_graph_launch; strata_moe_forward itself with --no-graph), strata_read of y,
          host-timed.
  roofline  algorithmic bytes of each step (the U+1 distinct expert blobs actually routed,
          router rows, shared gate, activations in and out) over the measured step time,
          against the measured HBM copy bandwidth.
  cpu_baseline / --impl reference  the reference's own kernels/strata.cu compiled natively
          (oracle/_ref, WASM-path host order, 8 threads) on a bounded sample of the same
          workload; falls back to the C restatement when the native build is absent.

Nested blocks (skipped with --headline-only): the line also carries the metric's other
configurations, each timed the same way on the same GPU(s):
  decode_b8, decode_b64   BASELINE config 2's other batch sizes: tokens/s and the HBM roofline
          from the experts each step actually routed to;
  prefill_4096            BASELINE config 3 (Zipf(1.1) router offsets): layer tokens/s, the
          grouped GEMMs' TFLOP/s against the measured sustained dense BF16 peak, phase split;
  ep                      BASELINE config 4 at this run's N: 16384 tokens split over the ranks,
          the 512 experts sharded, NCCL dispatch and return between the ranks when N >= 2;
          tokens/s (max over ranks), per-GPU TFLOP/s, rank 0's phase split, and
          efficiency_vs_n1 when an N=1 run on the same host left its number in /tmp;
  model48                 BASELINE config 5 (one GPU only): the 48-layer synthetic model through
          the whole engine, prompt 1920 prefilled in chunks of 64, 128 greedy decode tokens at
          batch 1 and at batch 64 (64 sequences from the prompt's state, each with its own
          seeded first token); decode ms per token or step and prefill tokens/s by the host clock.

Multi-GPU: the headline has every rank run its own replica of the layer stack (the reference
has no multi-GPU path); scaling is weak. The `ep` block (and `--ep`, which times BASELINE
config 4 alone) is strong scaling.
"""
from __future__ import annotations

import argparse
import json
import os
import pathlib
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "MoE-layer tokens/s (decode b=1 %HBM BW; prefill %TC peak) at 1/2/4/8 B200"
WIDTH, FF, EXPERTS, TOPK = 2048, 512, 512, 10
BLOB_BYTES = 884_736
ROUTER_BYTES = EXPERTS * WIDTH * 4
GATE_BYTES = WIDTH * 4


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            self.proc.wait(timeout=5)

    def summary(self):
        rows = [l.split(", ") for l in self.lines if l.count(",") >= 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    return world, rank, local


def dist_max(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def dist_barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ----------------------------------------------------------------------------- CPU reference leg

def cpu_reference_sample(budget_s: float = 12.0, max_tokens: int = 64):
    """Time the reference's CPU path (oracle/_ref, WASM-path order, 8 threads) on decode tokens
    of the bench's own layer 0 until the time budget is spent. Returns (tokens/s, info)."""
    from oracle.oracle import Oracle, moe_layer_port, moe_layer_wasm_path, route_port
    from stratacuda_b200 import synth
    try:
        o = Oracle("reference", threads=8)
        kind, cores = "reference", 8
    except (FileNotFoundError, OSError):
        o = Oracle("port")
        kind, cores = "port", 1
    router = synth.router_weights(1, 0, EXPERTS, WIDTH)
    gate = synth.shared_gate(1, 0, WIDTH)
    shared = synth.expert_blob(1, 0, 0, WIDTH, FF, shared=True)
    words = shared.size
    blobs = np.zeros((EXPERTS, words), np.uint32)
    filled = set()
    port = Oracle("port")
    done, spent = 0, 0.0
    while done < max_tokens and spent < budget_s:
        x = synth.activations(2, 1, WIDTH, start_token=done)
        _, ids, _ = route_port(port, x, router, TOPK)
        for e in set(ids.reshape(-1).tolist()) - filled:
            blobs[e] = synth.expert_blob(1, 0, e, WIDTH, FF)
            filled.add(e)
        t0 = time.perf_counter()
        if kind == "reference":
            moe_layer_wasm_path(o, x, router, gate, blobs, shared, TOPK)
        else:
            moe_layer_port(o, x, router, gate, blobs, shared, TOPK)
        spent += time.perf_counter() - t0
        done += 1
    return done / spent, {"kind": kind, "cores": cores, "tokens": done, "seconds": round(spent, 3)}


def run_reference_arm(args, world, rank):
    if rank != 0:
        return
    steps, warm = args.steps, args.warmup
    # a step is one decode token through the reference's CPU path; bound the whole run
    per_step_budget = max(0.5, min(4.0, 150.0 / max(1, steps + warm)))
    rate_w, _ = cpu_reference_sample(budget_s=per_step_budget * warm, max_tokens=max(1, warm))
    rate, info = cpu_reference_sample(budget_s=per_step_budget * steps, max_tokens=max(1, steps))
    line = {"metric": METRIC, "value": rate, "unit": "tokens/s", "impl": "reference", "n_gpus": args.gpus, "steps": info["tokens"],
            "warmup": warm, "ms_per_step": 1000.0 / rate, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded)", "config": workload_config(1, args.layers),
            "cpu_baseline": {"value": rate, "unit": "tokens/s", "cores": info["cores"], "kind": info["kind"],
                             "sample": f"{info['tokens']} decode tokens (B=1) of layer 0, WASM-path order, {info['seconds']} s"},
            "e2e": {"value": rate, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def workload_config(batch: int, layers: int, zipf=None, graph=None):
    kind = "prefill" if batch > 64 else "decode"
    skew = f", Zipf({zipf}) router bias" if zipf else ""
    return {"workload": f"MoE layer {kind} b={batch} (H2048, E512 top-10, F512, Q2 experts + shared expert{skew})", "batch": batch,
            "hidden": WIDTH, "experts": EXPERTS, "top_k": TOPK, "ff": FF, "layers_cycled": layers, "zipf": zipf,
            "l2": "inputs larger than L2: distinct layer replicas cycled, fresh activations per step", "parallelism": "replicas",
            **({} if graph is None else {"timing": "CUDA events around one CUDA-graph replay of the K steps" if graph
                                         else "CUDA events around K direct launches"})}


def peak_tflops():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["bf16_tflops_sustained"]), "measured (sustained dense bf16)"
    return 1400.0, "fallback (sustained)"


# ----------------------------------------------------------------------------- GPU arm

class LayerSteps:
    """Per-step device buffers of a batch size over a stack of layers: fresh activations every
    step (a ring of 8 batches above 64 tokens), one dedicated y/ids/weights slot per batch."""

    def __init__(self, b, B, n_x, seed):
        from stratacuda_b200.moe import synth_activations
        self.b, self.B, self.n_x = b, B, n_x
        x_all = synth_activations(b, seed, n_x * B, WIDTH)
        self.xs = [b.alloc(B * WIDTH, zero=False) for _ in range(n_x)]
        for s in range(n_x):
            b.copy(x_all, self.xs[s], B * WIDTH, s * B * WIDTH, 0)
        self.x_all = x_all
        self.ys = [b.alloc(B * WIDTH, zero=False) for _ in range(n_x)]
        self.idss = [b.alloc(B * TOPK, "i32") for _ in range(n_x)]
        self.wss = [b.alloc(B * TOPK, zero=False) for _ in range(n_x)]
        b.idle()

    def run(self, layers, s, mode):
        i = s % self.n_x
        layers[s % len(layers)].forward(self.xs[i], self.B, self.ys[i], self.idss[i], self.wss[i], mode=mode)

    def free(self):
        for buf in [self.x_all] + self.xs + self.ys + self.idss + self.wss:
            self.b.free(buf)


def time_layer_steps(b, layers, st, K, W, mode, world, local, graph=True, clocks=False):
    """W warm-up steps, then K steps captured once as a CUDA graph and replayed between CUDA
    events on the library's stream (K direct launches without `graph`); max over ranks."""
    import torch
    stream = torch.cuda.ExternalStream(b.stream_handle, device=torch.device("cuda", local))
    for s in range(W):
        st.run(layers, s, mode)
    b.idle()
    g = None
    if graph:
        b.capture_begin()
        for s in range(W, W + K):
            st.run(layers, s, mode)
        g = b.capture_end()
    dist_barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local) if clocks else None
    if sampler:
        sampler.__enter__()
    start.record(stream)
    if g is not None:
        b.graph_launch(g)
    else:
        for s in range(W, W + K):
            st.run(layers, s, mode)
    end.record(stream)
    b.idle()
    if sampler:
        sampler.__exit__(None, None, None)
    if g is not None:
        b.graph_free(g)
    torch.cuda.synchronize()
    dist_barrier(world)
    ms = dist_max(start.elapsed_time(end), world)
    return ms, (sampler.summary() if sampler else None)


def routed_bytes(b, st, B, K, W):
    """Algorithmic bytes per step from the routing that actually happened (the last n_x steps):
    the U + 1 distinct blobs read, router rows, shared gate, activations in and out."""
    out = []
    for s in range(max(W, W + K - st.n_x), W + K):
        U = len(set(b.read(st.idss[s % st.n_x]).tolist()))
        out.append((U + 1) * BLOB_BYTES + ROUTER_BYTES + GATE_BYTES + 2 * B * WIDTH * 4)
    return float(np.mean(out))


def decode_block(b, layers, B, K, W, mode, world, local):
    """A decode batch (BASELINE config 2's 8 and 64): tokens/s and the HBM roofline."""
    from stratacuda_b200 import _lib as LL
    st = LayerSteps(b, B, K + W, seed=20 + B)
    ms, _ = time_layer_steps(b, layers, st, K, W, mode, world, local)
    alg = routed_bytes(b, st, B, K, W)
    st.free()
    hbm, kind = peaks()
    step_s = ms / 1000.0 / K
    kernel = ("k_moe_decode1 (one launch of 8-CTA clusters per step)" if mode == LL.MOE_FAST and B == 1 else
              "k_moe_fast (one persistent launch per step)" if mode == LL.MOE_FAST and B <= 8 else
              "k_moe_medium (after the exact router kernels: 4 launches per step)" if mode == LL.MOE_FAST else "fused exact layer")
    return {"batch": B, "tokens_per_s": B * K * world / (ms / 1000.0), "ms_per_step": ms / K, "steps": K, "warmup": W,
            "roofline": {"bound": "hbm", "achieved": alg / step_s / 1e9, "peak": hbm, "unit": "GB/s", "frac": alg / step_s / 1e9 / hbm,
                         "peak_kind": kind, "algorithmic_bytes_per_step": alg, "kernel": kernel}}


def prefill_block(b, layers, K, W, mode, world, local, T=4096, zipf=1.1):
    """4096 tokens, Zipf(1.1) router offsets, tensor-core prefill path."""
    from stratacuda_b200 import synth
    bias = b.alloc(synth.zipf_bias(1, EXPERTS, zipf))
    for L in layers:
        L.router_bias = bias
    try:
        st = LayerSteps(b, T, 8, seed=40)
        ms, _ = time_layer_steps(b, layers, st, K, W, mode, world, local)
        roof = prefill_roofline(b, layers, st.xs, st.ys, st.idss, st.wss, T, len(layers), st.n_x, mode, K)
        st.free()
    finally:
        for L in layers:
            L.router_bias = None
        b.free(bias)
    flops = 2.0 * 3 * WIDTH * FF * (T * TOPK + T)
    peak, kind = peak_tflops()
    layer_tf = flops / (ms / 1000.0 / K) / 1e12
    return {"tokens": T, "zipf": zipf, "tokens_per_s": T * K * world / (ms / 1000.0), "ms_per_step": ms / K, "steps": K, "warmup": W,
            "layer_tflops": layer_tf, "layer_frac": layer_tf / peak, "gemm_tflops": roof["achieved"], "gemm_frac": roof["frac"],
            "peak_tflops": peak, "peak_kind": kind, "phase_ms_per_step": roof["phase_ms_per_step"],
            "kernel": roof["kernel"], "algorithmic_flops_per_step": flops}


def run_gpu_arm(args, world, rank, local):
    import torch

    from stratacuda_b200.backend import CudaBackend
    from stratacuda_b200.moe import MoeLayer

    torch.cuda.set_device(local)
    b = CudaBackend(local)
    B, K, W, NL = args.batch, args.steps, args.warmup, args.layers
    zipf = args.zipf if args.zipf is not None else (1.1 if B > 64 else None)
    layers = [MoeLayer.synthesize(b, seed=1, layer=l, width=WIDTH, ff=FF, experts=EXPERTS, top_k=TOPK, zipf=zipf) for l in range(NL)]
    # distinct activation batches: every step for small batches, a ring of 8 for large ones
    st = LayerSteps(b, B, K + W if B <= 64 else min(K + W, 8), seed=2 + rank)
    from stratacuda_b200 import _lib as LL
    mode = LL.MOE_FAST if args.mode == "fast" else LL.MOE_EXACT
    medium = mode == LL.MOE_FAST and 8 < B <= 64
    prefill = mode == LL.MOE_FAST and B > 64
    # kernels per step: decode 1; medium 4 (router tail rows, exact logits, top-k, the layer);
    # prefill 9; exact 6
    launches = 1 if (mode == LL.MOE_FAST and B <= 8) else 4 if medium else 9 if prefill else 6
    ms_max, clocks = time_layer_steps(b, layers, st, K, W, mode, world, local, graph=not args.no_graph, clocks=True)
    alg_bytes = routed_bytes(b, st, B, K, W)
    step_s = ms_max / 1000.0 / K
    hbm_peak, peak_kind = peaks()
    achieved = alg_bytes / step_s / 1e9
    if prefill:
        roofline = prefill_roofline(b, layers, st.xs, st.ys, st.idss, st.wss, B, NL, st.n_x, mode, K)
    else:
        roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak, "traffic": None,
                    "peak_kind": peak_kind,
                    "kernel": ("k_moe_decode1 (one launch of 8-CTA clusters per step)" if launches == 1 and B == 1
                               else "k_moe_fast (one persistent launch per step)" if launches == 1
                               else "k_moe_medium (after the exact router kernels: 4 launches per step)" if medium
                               else "fused exact MoE layer (6 launches per step)"),
                    "algorithmic_bytes_per_step": alg_bytes}

    # end to end through the C-ABI with host buffers (pinned), host-timed
    e2e_steps = min(K, max(20, K // 2)) if B <= 64 else min(K, 8)
    e2e_steps = min(e2e_steps, st.n_x)
    hx = torch.empty(e2e_steps, B * WIDTH, dtype=torch.float32, pin_memory=True)
    hx.copy_(torch.from_numpy(b.read(st.x_all, count=e2e_steps * B * WIDTH).reshape(e2e_steps, B * WIDTH)))
    hy = torch.empty(B * WIDTH, dtype=torch.float32, pin_memory=True)
    hx_np, hy_np = hx.numpy(), hy.numpy()
    lib, ctx = b.lib, b.ctx
    xbuf, ybuf = st.xs[0], st.ys[0]
    # Each layer's call is captured once (the decode-loop pattern of the graph API): a step is
    # strata_write of the batch from pinned memory, strata_graph_launch of that layer's call,
    # strata_read of y into pinned memory. --no-graph calls strata_moe_forward every step.
    e2e_graphs = []
    if not args.no_graph:
        for l in range(min(NL, e2e_steps)):
            b.capture_begin()
            layers[l].forward(xbuf, B, ybuf, st.idss[0], st.wss[0], mode=mode)
            e2e_graphs.append(b.capture_end())

    def e2e_step(s):
        b.write(xbuf, hx_np[s])
        if e2e_graphs:
            b.graph_launch(e2e_graphs[s % len(e2e_graphs)])
        else:
            layers[s % NL].forward(xbuf, B, ybuf, st.idss[0], st.wss[0], mode=mode)
        b._check(lib.strata_read(ctx, ybuf.handle, hy_np.ctypes.data, B * WIDTH, 0))

    for s in range(min(3, e2e_steps)):
        e2e_step(s)
    dist_barrier(world)
    t0 = time.perf_counter()
    for s in range(e2e_steps):
        e2e_step(s)
    e2e_s = time.perf_counter() - t0
    e2e_s = dist_max(e2e_s, world)
    for g in e2e_graphs:
        b.graph_free(g)
    st.free()

    # the metric's other configurations, nested in the same line (3, 4)
    blocks = {}
    if not args.headline_only:
        kb, wb = min(K, 40), max(3, min(W, 5))
        for bb in (8, 64):
            if bb != B:
                blocks[f"decode_b{bb}"] = decode_block(b, layers, bb, kb, wb, mode, world, local)
        if B != 4096:
            blocks["prefill_4096"] = prefill_block(b, layers, min(K, 10), 3, mode, world, local)
    for L in layers:
        L.free()
    if not args.headline_only:
        blocks["ep"] = ep_block(args, world, rank, local, b)
    if not args.headline_only and world == 1:
        blocks["model48"] = model_block(b)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        rate, info = cpu_reference_sample(budget_s=args.cpu_seconds)
        cpu = {"value": rate, "unit": "tokens/s", "cores": info["cores"], "kind": info["kind"],
               "sample": f"{info['tokens']} decode tokens (B=1) of layer 0 through the reference's WASM-path order, "
                         f"{info['seconds']} s on {info['cores']} host threads"}

    tp = ROOT / "profiles" / "traffic.json"
    if tp.exists() and roofline["bound"] == "hbm":
        roofline["traffic"] = json.loads(tp.read_text()).get(f"decode_b{B}")

    total_tokens = B * K * world
    line = {"metric": METRIC, "value": total_tokens / (ms_max / 1000.0), "unit": "tokens/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": ms_max / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded SplitMix64; BASELINE config 2 distributions)",
            "config": workload_config(B, NL, zipf, graph=not args.no_graph),
            "roofline": roofline,
            "e2e": {"value": B * e2e_steps * world / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": B * WIDTH * 4,
                    "d2h_bytes_per_step": B * WIDTH * 4, "steps": e2e_steps,
                    "calls": ("strata_write (pinned host) + strata_graph_launch of the layer's captured strata_moe_forward + strata_read "
                              "(pinned host, synchronising), host-timed" if e2e_graphs or not args.no_graph else
                              "strata_write (pinned host) + strata_moe_forward + strata_read (pinned host, synchronising), host-timed")},
            "gpu_launches": launches * K,
            "clocks": clocks}
    if cpu:
        line["cpu_baseline"] = cpu
    line.update(blocks)
    if rank == 0:
        print(json.dumps(line), flush=True)
    b.dispose()


EP_N1_CACHE = pathlib.Path("/tmp/strata_bench_ep_n1.json")


def ep_placement(world, layers, zipf, calib_tokens=2048):
    """Owner rank per expert for the expert-parallel runs, balanced by the routed rows of a
    calibration sample (tokens that are not in the timed batches) over the cycled layers, from
    the seeded synthetic router on the host (every rank computes the same placement). None on
    one rank."""
    if world == 1:
        return None
    import numpy as np

    from stratacuda_b200 import synth
    from stratacuda_b200.ep import balanced_placement
    x = synth.activations(7, calib_tokens, WIDTH, start_token=1 << 30).reshape(calib_tokens, WIDTH)
    bias = synth.zipf_bias(1, EXPERTS, zipf) if zipf is not None else np.zeros(EXPERTS, np.float32)
    rows = np.zeros(EXPERTS)
    for layer in range(layers):
        W = synth.router_weights(1, layer, EXPERTS, WIDTH).reshape(EXPERTS, WIDTH)
        top = np.argpartition(-(x @ W.T + bias), TOPK - 1, axis=1)[:, :TOPK]
        rows += np.bincount(top.reshape(-1), minlength=EXPERTS)
    return balanced_placement(rows, world)


def ep_block(args, world, rank, local, b):
    """BASELINE config 4 at this run's N: 16384 tokens split over the ranks, 512 experts sharded
    E/N per GPU, Zipf(1.1) routing; at N >= 2 the library's NCCL dispatch and return run between
    the ranks. Device time of K steps (CUDA events on the library's stream), max over ranks."""
    import torch

    from stratacuda_b200.ep import EpMoeLayer, ep_init, ep_set_placement
    from stratacuda_b200.moe import synth_activations
    total, K, W, NL = args.ep_tokens, min(args.steps, 10), 3, 4
    if total % world:
        return {"skipped": f"{total} tokens must divide over {world} ranks"}
    T = total // world
    zipf = 1.1
    ep_init(b, rank, world)
    owner = ep_placement(world, NL, zipf)
    ep_set_placement(b, owner)
    layers = [EpMoeLayer.synthesize(b, rank, world, seed=1, layer=l, width=WIDTH, ff=FF, experts=EXPERTS, top_k=TOPK, zipf=zipf,
                                    owner=owner) for l in range(NL)]
    n_local = layers[0].local_experts
    n_x = 2
    xs = [synth_activations(b, 2 + s, T, WIDTH, start_token=rank * T) for s in range(n_x)]
    ys = [b.alloc(T * WIDTH, zero=False) for _ in range(n_x)]
    idss = [b.alloc(T * TOPK, "i32") for _ in range(n_x)]
    wss = [b.alloc(T * TOPK, zero=False) for _ in range(n_x)]
    b.idle()
    stream = torch.cuda.ExternalStream(b.stream_handle, device=torch.device("cuda", local))
    step = lambda s: layers[s % NL].forward(xs[s % n_x], T, ys[s % n_x], idss[s % n_x], wss[s % n_x])
    for s in range(W):
        step(s)
    b.idle()
    dist_barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for s in range(W, W + K):
        step(s)
    end.record(stream)
    b.idle()
    torch.cuda.synchronize()
    dist_barrier(world)
    ms_max = dist_max(start.elapsed_time(end), world)
    b.profile(True)
    for s in range(3):
        step(s)
    ph, calls = b.profile_read()
    b.profile(False)
    for L in layers:
        L.free()
    for buf in xs + ys + idss + wss:
        b.free(buf)
    b.idle()
    flops = 2.0 * 3 * WIDTH * FF * (total * TOPK + total)
    peak, kind = peak_tflops()
    per_gpu_tf = flops / (ms_max / 1000.0 / K) / world / 1e12
    tps = total * K / (ms_max / 1000.0)
    out = {"tokens": total, "tokens_per_rank": T, "experts_per_rank": EXPERTS // world, "zipf": zipf, "parallelism": f"ep{world}",
           "placement": "contiguous (one rank)" if owner is None else "balanced by a calibration sample's routed rows",
           "experts_on_rank0": n_local,
           "exchange": "NCCL grouped send/recv inside strata_moe_ep_forward" if world > 1 else "none (one rank)",
           "tokens_per_s": tps, "ms_per_step": ms_max / K, "steps": K, "warmup": W, "layers_cycled": NL,
           "per_gpu_tflops": per_gpu_tf, "per_gpu_frac": per_gpu_tf / peak, "peak_tflops": peak, "peak_kind": kind,
           "phase_ms_per_step_rank0": {k: v / max(1, calls) for k, v in ph.items() if k != "decode_kernel"},
           "timing": "CUDA events around K direct calls (the layer reads the receive counts on the host), max over ranks"}
    key = {"tokens": total, "zipf": zipf, "layers": NL}
    if world == 1 and rank == 0:
        try:
            EP_N1_CACHE.write_text(json.dumps({"key": key, "tokens_per_s": tps}))
        except OSError:
            pass
    elif world > 1:
        try:
            n1 = json.loads(EP_N1_CACHE.read_text())
            if n1["key"] == key:
                out["efficiency_vs_n1"] = tps / (world * n1["tokens_per_s"])
                out["n1_tokens_per_s"] = n1["tokens_per_s"]
        except (OSError, ValueError, KeyError):
            pass
    return out


def run_ep_arm(args, world, rank, local):
    """one expert-parallel layer over the ranks (strata_moe_ep_forward).
    16384 tokens split evenly over the ranks, the 512 experts sharded (E/N per rank), Zipf(1.1)
    router bias, NCCL dispatch and return inside the library; strong scaling; device time of
    the K steps (CUDA events on the library's stream), max over ranks."""
    import torch

    from stratacuda_b200.backend import CudaBackend
    from stratacuda_b200.ep import EpMoeLayer, ep_init, ep_set_placement
    from stratacuda_b200.moe import synth_activations

    torch.cuda.set_device(local)
    b = CudaBackend(local)
    total, K, W, NL = args.ep_tokens, args.steps, args.warmup, args.layers
    if total % world:
        raise SystemExit("--ep-tokens must divide over the ranks")
    T = total // world
    zipf = args.zipf if args.zipf is not None else 1.1
    ep_init(b, rank, world)
    owner = ep_placement(world, NL, zipf)
    ep_set_placement(b, owner)
    layers = [EpMoeLayer.synthesize(b, rank, world, seed=1, layer=l, width=WIDTH, ff=FF, experts=EXPERTS, top_k=TOPK, zipf=zipf,
                                    owner=owner) for l in range(NL)]
    n_x = 4
    xs = [synth_activations(b, 2 + s, T, WIDTH, start_token=rank * T) for s in range(n_x)]
    ys = [b.alloc(T * WIDTH, zero=False) for _ in range(n_x)]
    idss = [b.alloc(T * TOPK, "i32") for _ in range(n_x)]
    wss = [b.alloc(T * TOPK, zero=False) for _ in range(n_x)]
    b.idle()
    stream = torch.cuda.ExternalStream(b.stream_handle, device=torch.device("cuda", local))
    step = lambda s: layers[s % NL].forward(xs[s % n_x], T, ys[s % n_x], idss[s % n_x], wss[s % n_x])
    for s in range(W):
        step(s)
    b.idle()
    dist_barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record(stream)
        for s in range(W, W + K):
            step(s)
        end.record(stream)
        b.idle()
    torch.cuda.synchronize()
    dist_barrier(world)
    ms_max = dist_max(start.elapsed_time(end), world)
    # phase split (second pass, library profile)
    b.profile(True)
    for s in range(3):
        step(s)
    ph, calls = b.profile_read()
    b.profile(False)
    phases = {k: v / max(1, calls) for k, v in ph.items() if k != "decode_kernel"}
    # end to end through the C-ABI: this rank's tokens from pinned host memory, y back
    hx = torch.empty(T * WIDTH, dtype=torch.float32, pin_memory=True)
    hx.copy_(torch.from_numpy(b.read(xs[0])))
    hy = torch.empty(T * WIDTH, dtype=torch.float32, pin_memory=True)
    hx_np, hy_np = hx.numpy(), hy.numpy()
    e2e_steps = min(K, 5)
    dist_barrier(world)
    t0 = time.perf_counter()
    for s in range(e2e_steps):
        b.write(xs[0], hx_np)
        layers[s % NL].forward(xs[0], T, ys[0], idss[0], wss[0])
        b._check(b.lib.strata_read(b.ctx, ys[0].handle, hy_np.ctypes.data, T * WIDTH, 0))
    e2e_s = dist_max(time.perf_counter() - t0, world)
    flops = 2.0 * 3 * WIDTH * FF * (total * TOPK + total)  # whole job per step: routed pairs + shared rows
    step_s = ms_max / 1000.0 / K
    peak, kind = peak_tflops()
    achieved = flops / step_s / world / 1e12
    line = {"metric": METRIC, "value": total * K / (ms_max / 1000.0), "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": ms_max / K, "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded SplitMix64; BASELINE config 4 distributions)",
            "config": {"workload": f"expert-parallel MoE layer, {total} tokens over {world} GPU(s), E512 sharded over the GPUs, "
                                   f"top-10, H2048, F512, Q2 experts + shared expert, Zipf({zipf}) router bias",
                       "tokens": total, "tokens_per_rank": T, "experts_per_rank": EXPERTS // world, "hidden": WIDTH, "ff": FF, "top_k": TOPK,
                       "placement": "contiguous (one rank)" if owner is None else "balanced by a calibration sample's routed rows",
                       "layers_cycled": NL, "zipf": zipf, "l2": "inputs larger than L2: distinct layer replicas cycled",
                       "parallelism": f"ep{world}"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak, "traffic": None,
                         "peak_kind": kind, "kernel": "whole expert-parallel step per GPU (routing, NCCL exchange, tcgen05 GEMMs)",
                         "algorithmic_flops_per_step": flops, "phase_ms_per_step_rank0": phases},
            "e2e": {"value": total * e2e_steps / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": total * WIDTH * 4,
                    "d2h_bytes_per_step": total * WIDTH * 4},
            "gpu_launches": 18 * K,
            "clocks": clocks.summary()}
    if rank == 0:
        print(json.dumps(line), flush=True)
    for L in layers:
        L.free()
    b.dispose()


def prefill_roofline(b, layers, xs, ys, idss, wss, B, NL, n_x, mode, K):
    """Second pass with the library's phase profile: the grouped GEMMs' device time against
    their algorithmic FLOPs, 2 * 3 * H * F * (pairs + tokens) per step (gate/up: 2F x H per
    row, down: H x F per row; every pair and every token's shared-expert row)."""
    steps = max(3, min(K, 20))
    b.profile(True)
    for s in range(steps):
        layers[s % NL].forward(xs[s % n_x], B, ys[s % n_x], idss[s % n_x], wss[s % n_x], mode=mode)
    ph, calls = b.profile_read()
    b.profile(False)
    flops = 2.0 * 3 * WIDTH * FF * (B * TOPK + B)
    gemm_s = (ph["gemm_gate_up"] + ph["gemm_down"]) / 1000.0 / max(1, calls)
    achieved = flops / gemm_s / 1e12
    peak, kind = peak_tflops()
    return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak, "traffic": None,
            "peak_kind": kind, "kernel": "k_pf_gemm gate/up + down (tcgen05, persistent)", "algorithmic_flops_per_step": flops,
            "phase_ms_per_step": {k: v / max(1, calls) for k, v in ph.items()}}


def model_run(b, layers, prompt_len, decode, warmup, mode, graph=True, profile_prefill=False, profile_step=False, batch=64,
              profile_batch_step=False):
    """The full-model workload on backend b: the seeded synthetic model (stratacuda_b200.synthetic)
    resident in HBM, a prompt prefilled in chunks of 64, then greedy decode at batch 1, all through
    StrataEngine (the reference host's call order). Timed by the host clock around each phase,
    which ends in the argmax read: the host dispatch of every entry is inside the numbers.
    With `batch` > 1, greedy decode of `batch` sequences together (SequenceBatch) is timed too:
    every sequence starts from the prefilled prompt's state and takes its own seeded first token,
    then `decode` steps of all sequences (each step reads the batch's tokens back)."""
    from stratacuda_b200.engine import SequenceBatch, StrataEngine
    from stratacuda_b200.synthetic import MODEL_GEOMETRY, MOE_MODES, DeviceStore

    g = dict(MODEL_GEOMETRY, layers=layers)
    t0 = time.perf_counter()
    store = DeviceStore(b, g, seed=1)
    b.idle()
    t_gen = time.perf_counter() - t0
    engine = StrataEngine.create(store, b, MOE_MODES[mode], graph=graph)
    prompt = np.random.default_rng(7).integers(0, g["vocab"], prompt_len).tolist()
    seqs = SequenceBatch(engine, batch, graph=graph) if batch > 1 else None
    for _ in range(max(1, warmup // 3)):  # warm-up: pools, RoPE table, the decode graphs' capture
        engine.prefill(prompt[:64], chunk_size=64)
        if seqs is not None:
            for s in range(batch):
                seqs.admit(s, engine)
            seqs.step(list(range(batch)))
            seqs.step(list(range(batch)))
        engine.step(1)
        engine.step(2)
        engine.reset()
    t0 = time.perf_counter()
    if profile_prefill and prompt_len > 64:  # only the last chunk is inside the capture
        import torch
        engine.prefill(prompt[:-64], chunk_size=64)
        b.idle()
        torch.cuda.cudart().cudaProfilerStart()
        r = engine.prefill(prompt[-64:], chunk_size=64)
        b.idle()
        torch.cuda.cudart().cudaProfilerStop()
    else:
        r = engine.prefill(prompt, chunk_size=64)
    t_prefill = time.perf_counter() - t0
    batch_out = {}
    if seqs is not None:
        for s in range(batch):
            seqs.admit(s, engine)
        step_tokens = np.random.default_rng(8).integers(0, g["vocab"], batch).tolist()
        b.idle()
        t0 = time.perf_counter()
        for k in range(decode):
            last = profile_batch_step and k == decode - 1
            if last:  # only this batch step is inside an `ncu --profile-from-start off` capture
                import torch
                b.idle()
                torch.cuda.cudart().cudaProfilerStart()
            step_tokens = seqs.step(step_tokens)["tokens"]
            if last:
                b.idle()
                torch.cuda.cudart().cudaProfilerStop()
        t_batch = time.perf_counter() - t0
        batch_out = {f"decode_b{batch}_tokens_per_s": batch * decode / t_batch, f"decode_b{batch}_ms_per_step": 1e3 * t_batch / decode,
                     f"decode_b{batch}_last_tokens": step_tokens[:8]}
        seqs.dispose()
    token, tokens = r["token"], []
    t0 = time.perf_counter()
    for k in range(decode):
        last = profile_step and k == decode - 1
        if last:  # only this step is inside an `ncu --profile-from-start off` capture
            import torch
            b.idle()
            torch.cuda.cudart().cudaProfilerStart()
        token = engine.step(token)["token"]
        tokens.append(token)
        if last:
            b.idle()
            torch.cuda.cudart().cudaProfilerStop()
    t_decode = time.perf_counter() - t0
    out = {"decode_tokens_per_s": decode / t_decode, "decode_ms_per_token": 1e3 * t_decode / decode,
           "prefill_tokens_per_s": prompt_len / t_prefill, "prefill_s": t_prefill, "generate_s": t_gen, **batch_out,
           "resident_gb": store.bytes_resident() / 1e9,
           "config": {"workload": f"{g['layers']}-layer synthetic model, hidden {g['width']}, vocab {g['vocab']}, prompt {prompt_len}, "
                                  f"decode {decode}, chunk 64" + (f"; decode batch {batch} from the prompt's state, seeded first tokens"
                                                                  if batch > 1 else ""), "moe_mode": mode, "decode_graph": graph,
                      "timing": "host clock, end to end"},
           "first_tokens": tokens[:8]}
    engine.dispose()
    store.free()
    return out


def model_block(b):
    """BASELINE config 5 at batch 1 (one GPU): the 48-layer synthetic model, prompt 1920, 128
    greedy decode tokens (context 2048)."""
    return model_run(b, 48, 1920, 128, 3, "fast")


def run_model_arm(args):
    """The full-model workload on one GPU (model_run); prints its own JSON line (not the MoE-layer
    metric)."""
    from stratacuda_b200.backend import CudaBackend

    b = CudaBackend(0)
    r = model_run(b, args.model_layers, args.prompt, args.decode, args.warmup, args.mode, graph=not args.no_graph,
                  profile_prefill=args.profile_prefill, profile_step=args.profile_step, batch=args.model_batch,
                  profile_batch_step=args.profile_batch_step)
    line = {"metric": "full-model tokens/s (prefill; greedy decode b=1)", "workload": "model48", "value": r["decode_tokens_per_s"],
            "unit": "tokens/s", "n_gpus": 1, "higher_is_better": True, "dtype": "f32+q2", "data": "synthetic", **r}
    b.dispose()
    print(json.dumps(line), flush=True)


def run_project_shape(args):
    """One exact-order projection (strata_project) of the given shape, timed alone: W warm-up
    launches, then K launches between CUDA events on the library's stream; prints its own line."""
    import torch
    from stratacuda_b200.backend import CudaBackend

    cols, rows, tokens = (int(v) for v in args.project_shape.split(","))
    b = CudaBackend(0)
    rng = np.random.default_rng(1)
    x = b.alloc(rng.normal(0, 1, tokens * cols).astype(np.float32))
    w = b.alloc(rng.normal(0, 0.03, rows * cols).astype(np.float32))
    y = b.alloc(rows * tokens)
    call = dict(X=x, W=w, Y=y, cols=cols, rows=rows, tokens=tokens, outputStride=rows, outputOffset=0)
    for _ in range(args.warmup):
        b.run("strata_project", call, [rows, tokens, 1])
    b.idle()
    stream = torch.cuda.ExternalStream(b.stream_handle, device=torch.device("cuda", 0))
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        b.run("strata_project", call, [rows, tokens, 1])
    t1.record(stream)
    t1.synchronize()
    us = t0.elapsed_time(t1) * 1e3 / args.steps
    print(json.dumps({"metric": "strata_project multiply-adds/s", "shape": {"cols": cols, "rows": rows, "tokens": tokens},
                      "us_per_launch": us, "tmac_per_s": cols * rows * tokens / us / 1e6, "steps": args.steps,
                      "warmup": args.warmup}), flush=True)
    b.dispose()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="strata", choices=["strata", "reference"])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--layers", type=int, default=24)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--mode", default="fast", choices=["fast", "exact"])
    ap.add_argument("--zipf", type=float, default=None, help="router bias skew (default: 1.1 for batches above 64 and --ep)")
    ap.add_argument("--ep", action="store_true", help="expert-parallel layer over the ranks (BASELINE config 4)")
    ap.add_argument("--headline-only", action="store_true",
                    help="skip the nested blocks (decode_b8, decode_b64, prefill_4096, ep, model48) of the default line")
    ap.add_argument("--no-graph", action="store_true", help="time direct launches instead of a CUDA graph replay of the K steps")
    ap.add_argument("--ep-tokens", type=int, default=16384, help="tokens of the expert-parallel job (split over the ranks)")
    ap.add_argument("--model", action="store_true", help="the full-model workload (48-layer synthetic model, 1 GPU)")
    ap.add_argument("--model-layers", type=int, default=48)
    ap.add_argument("--model-batch", type=int, default=64, help="--model: sequences decoded together after the batch-1 decode (1: none)")
    ap.add_argument("--prompt", type=int, default=1920, help="--model: prompt tokens (context 2048 = prompt + decode)")
    ap.add_argument("--decode", type=int, default=128, help="--model: greedy decode tokens")
    ap.add_argument("--profile-prefill", action="store_true",
                    help="--model: bracket the last 64-token prompt chunk with cudaProfilerStart/Stop")
    ap.add_argument("--profile-step", action="store_true",
                    help="--model: bracket the last decode step with cudaProfilerStart/Stop (for ncu --profile-from-start off)")
    ap.add_argument("--profile-batch-step", action="store_true",
                    help="--model: bracket the last batch decode step with cudaProfilerStart/Stop (for ncu --profile-from-start off)")
    ap.add_argument("--project-shape", default=None, metavar="COLS,ROWS,TOKENS",
                    help="time one strata_project shape alone (seeded inputs, CUDA events) and print its own JSON line")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference_arm(args, world, rank)
        return
    if args.model:
        run_model_arm(args)
        return
    if args.project_shape:
        run_project_shape(args)
        return
    world, rank, local = dist_setup(args.gpus)
    try:
        if args.ep:
            run_ep_arm(args, world, rank, local)
        else:
            run_gpu_arm(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
