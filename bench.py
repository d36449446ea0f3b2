#!/usr/bin/env python3
"""Benchmark of the quantized expert hot path (C2: one fused MoE layer, batch-1 decode).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one pass of the hot path over one batch of synthetic input: REPS replays
of a CUDA graph of CALLS fused-MoE-layer calls (1024 layer calls by default), call i
on layer i % LAYERS of a LAYERS-deep expert store
(256 experts x {gate, up Q4_K 512x2048; down Q6_K 2048x512} per layer, 522 MB),
each with its own seeded x (N(0,1), 2048) and router logits (N(0,1), 256).
The store (16 x 522 MB = 8.4 GB) is far larger than the 126 MB L2 and each call
reads 8 random experts of a different layer, so expert bytes come from HBM.

metric = quantised expert bytes read per second (16,318,464 B per call), whole
job; `value` is timed on the device with inputs already in HBM (CUDA graph of
the step's launches, CUDA events); `e2e` is the same metric through the C ABI
with host buffers: upload of the step's inputs from pinned memory, the layer
calls, download of the outputs, each step. N > 1 GPUs run the layer expert-parallel
(experts split over the GPUs, one process per GPU, weak scaling: every GPU brings its
own tokens) and report the max time over ranks; the line then carries a parity check
of every rank's tokens against the single-GPU layer.

The default run also measures the other configurations in the same process and puts
their lines, slimmed, under "secondary": at N = 1 C2 with fp32 activations (the mode
pinned to the reference's CPU kernels), C1 (fp32 and q8_1 activations), C3, C4 (fp32
and q8_1) and C5 (fp32 and q8_1, with the greedy tokens compared against the CPU
composition); at N > 1 C2 as independent replicas, C3 and C5 expert-parallel.
`--no-secondary` skips them; `--config X` measures one configuration alone.
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, F, E, K = 2048, 512, 256, 8
RBG = H // 256 * 144
RBD = F // 256 * 210
EXPERT_BYTES = 2 * F * RBG + H * RBD          # 2,039,808
CALL_BYTES = K * EXPERT_BYTES                  # 16,318,464 quantised expert bytes per call
ACT_BYTES = H * 4 + E * 4 + H * 4              # x, logits in; y out (fp32)
METRIC = "MoE-layer quant-weight GB/s vs HBM peak"
WORKLOAD = ("C2 fused MoE layer, batch-1 decode: hidden 2048, 256 experts, expert FFN 512, "
            "top-8 of softmax(N(0,1) logits), gate/up Q4_K, down Q6_K (N(0,0.02) weights), "
            "x N(0,1) quantised to q8_1 on device")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c2", choices=["c2", "c1", "c3", "c4", "c5"],
                    help="c2: fused MoE layer (headline); c1: dense Q4_K GEMV 6144x2048; c3: ragged "
                         "batch; c4: dense Qwen3-8B decode; c5: hybrid GDN/attention MoE decode")
    ap.add_argument("--dp4a", action="store_true", help="c1: q8_1 activations (KATALI_CUDA_DP4A=1)")
    ap.add_argument("--layers", type=int, default=16)
    ap.add_argument("--dense-layers", type=int, default=36,
                    help="c4: decoder layers; 36 is the configuration (fewer for small profiles)")
    ap.add_argument("--hybrid-layers", type=int, default=40,
                    help="c5: decoder layers (every 4th is gated attention); 40 is the configuration")
    ap.add_argument("--calls", type=int, default=64)
    ap.add_argument("--reps", type=int, default=16,
                    help="c2: replays of the CALLS-call graph per step (a step is CALLS x REPS layer "
                         "calls, so the timed region spans enough clock samples)")
    ap.add_argument("--f32", action="store_true",
                    help="c2: fp32 activations (the mode pinned to the reference's CPU kernels)")
    ap.add_argument("--no-secondary", action="store_true",
                    help="default run: skip the other configurations (C1, C3, C4, C5, C2 fp32)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--hot", type=int, default=0,
                    help="c3: every token routed among experts 0..hot-1 (groups of many tokens)")
    ap.add_argument("--tmin", type=int, default=1, help="c3: smallest batch per call")
    ap.add_argument("--nccl", action="store_true",
                    help="N > 1: exchange with the plugin's NCCL communicator instead of over NVLink "
                         "peer memory inside the kernels (the default)")
    ap.add_argument("--p2p", action="store_true", help=argparse.SUPPRESS)  # the default; kept for old command lines
    ap.add_argument("--replicas", action="store_true",
                    help="N > 1: independent replicas instead of expert parallelism")
    ap.add_argument("--warm", action="store_true",
                    help="diagnostic: every call reuses layer 0 and input 0 (weights stay in L2)")
    ap.add_argument("--trace", action="store_true",
                    help="print the per-phase timeline of the MoE kernel to stderr")
    return ap.parse_args()


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def committed_traffic(name="moe_kernel_traffic.json"):
    """Per-launch DRAM bytes of a kernel from its committed ncu summary (profiles/)."""
    try:
        with open(os.path.join(ROOT, "profiles", name)) as f:
            return json.load(f)
    except Exception:
        return None


REASON_BITS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled during the timed region: NVML
    read every ~2 ms from a thread (read-only queries), or nvidia-smi when NVML is not
    importable. The GPU is looked up by its NVML index (CUDA_VISIBLE_DEVICES aware)."""

    def __init__(self, index: int):
        self.index, self.rows, self.proc, self.nvml = index, [], None, None
        self.stop = threading.Event()
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            try:
                nv = torch.cuda._get_nvml_device_index(index)
            except Exception:
                nv = index
            self.h = pynvml.nvmlDeviceGetHandleByIndex(nv)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.nvml = pynvml
        except Exception:
            self.nvml = None

    def __enter__(self):
        if self.nvml is not None:
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=clocks.sm,clocks.max.sm,"
                 "clocks_event_reasons.active", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _poll(self):
        nv = self.nvml
        while not self.stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.rows.append([str(sm), str(self.max_mhz), hex(rs)])
            except Exception:
                return
            time.sleep(0.002)

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 3:
                self.rows.append(parts)

    def __exit__(self, *a):
        self.stop.set()
        if self.nvml is not None:
            self.t.join(timeout=2)
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        reasons = set()
        for r in self.rows:
            try:
                bits = int(r[2], 16)
            except ValueError:
                continue
            for b, n in REASON_BITS.items():
                if bits & b:
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(self.rows), "source": "nvml" if self.nvml is not None else "nvidia-smi"}


# ---------------------------------------------------------------------------
# CPU legs (the reference's own kernels; test infrastructure under oracle/)
# ---------------------------------------------------------------------------
def cpu_reference_rate(layers_host, seconds: float, seed: int = 7):
    """Time the reference's CPU kernels (composed MoE layer) with all host cores on a
    bounded sample of the workload: as many layer calls as fit in ~`seconds`."""
    from oracle.oracle import Ref
    ref = Ref()
    cores = os.cpu_count() or 1
    rng = np.random.default_rng(seed)
    scratch = ref.moe_scratch(layers_host[0])
    calls, t0 = 0, time.perf_counter()
    while True:
        lw = layers_host[calls % len(layers_host)]
        x = rng.normal(0, 1, H).astype(np.float32)
        lg = rng.normal(0, 1, E).astype(np.float32)
        ref.moe_layer(lw, x, lg, n_threads=cores, scratch=scratch)
        calls += 1
        el = time.perf_counter() - t0
        if (el >= seconds and calls >= 8) or calls >= 100000:
            break
    ref.L.kref_moe_scratch_free(scratch)
    gbs = calls * CALL_BYTES / el / 1e9
    return gbs, cores, calls, el


def host_layer_numpy(seed: int):
    """One layer's experts encoded on the host (oracle C encoder), for the reference arm."""
    from oracle.oracle import Port, make_moe_weights
    return make_moe_weights(Port(), E, H, F, seed=seed, top_k=K)


def run_reference(args, rank):
    if rank != 0:
        return
    layers = [host_layer_numpy(1000 + i) for i in range(2)]
    for _ in range(args.warmup):
        cpu_reference_rate(layers, 0.0)
    rates, total_calls, total_s = [], 0, 0.0
    per_step = max(args.cpu_seconds / max(args.steps, 1), 0.05)
    for s in range(args.steps):
        gbs, cores, calls, el = cpu_reference_rate(layers, per_step, seed=100 + s)
        rates.append(gbs)
        total_calls += calls
        total_s += el
    value = total_calls * CALL_BYTES / total_s / 1e9
    sample = (f"{total_calls} layer calls over {args.steps} steps on 2 host-encoded layers "
              f"(reference kernels: katali_ggml_matvec_fused gate/up, silu_mul_avx2, Q6_K matvec)")
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 * total_s / args.steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "threads": os.cpu_count()},
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": os.cpu_count(),
                             "kind": "reference", "sample": sample},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from katali_lab_b200 import MOE_F32, MOE_Q8_1, MoeLayer, Plugin
    from katali_lab_b200.synth import make_expert_store

    torch.cuda.set_device(local_rank)
    plugin = Plugin()
    if not plugin.probe():
        raise SystemExit(f"no usable B200: {plugin.status()}")
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    plugin.set_stream(stream)

    L, T = args.layers, args.calls
    stores = [make_expert_store(plugin, E, H, F, seed=10_000 * rank + l) for l in range(L)]
    layers = [MoeLayer(plugin, E, H, F, K, st.pointers()) for st in stores]
    g = torch.Generator(device="cuda").manual_seed(77 + rank)
    xs = torch.randn((T, H), generator=g, device="cuda")
    lgs = torch.randn((T, E), generator=g, device="cuda")
    ys = torch.empty((T, H), device="cuda")
    torch.cuda.synchronize()

    plugin.set_async(True)
    mode = MOE_F32 if args.f32 else MOE_Q8_1
    reps = max(args.reps, 1)

    def step():
        for i in range(T):
            j = 0 if args.warm else i
            layers[j % L].forward(xs[j], lgs[j], ys[i], mode)

    # correctness guard: first call equals a synchronous run
    step()
    plugin.sync()

    graph = None
    if not args.no_graph:
        try:
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=stream):
                plugin.set_stream(torch.cuda.current_stream())
                step()
            plugin.set_stream(stream)
            graph = gr
        except Exception as e:  # capture unsupported: time eager launches
            print(f"[bench] graph capture failed ({e}); timing eager launches", file=sys.stderr)
            plugin.set_stream(stream)
            torch.cuda.synchronize()
            graph = None

    one = graph.replay if graph is not None else step

    def run():
        for _ in range(reps):
            one()

    for _ in range(max(args.warmup, 3)):
        run()
    plugin.sync()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with ClockSampler(local_rank) as clk:
        start.record(stream)
        for _ in range(args.steps):
            run()
        end.record(stream)
        end.synchronize()
    barrier()
    plugin.sync()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = world * args.steps * reps * T * CALL_BYTES / (ms / 1e3) / 1e9
    us_per_call = 1e3 * ms / (args.steps * reps * T)

    if args.trace and rank == 0:
        print_trace(plugin, layers, xs, lgs, ys, T, L, args.warm, mode=mode)

    # ---- e2e through the C ABI with host buffers --------------------------
    import ctypes as C
    xh = torch.randn((T, H), generator=torch.Generator().manual_seed(5)).pin_memory()
    lh = torch.randn((T, E), generator=torch.Generator().manual_seed(6)).pin_memory()
    yh = torch.empty((T, H)).pin_memory()
    plugin.set_async(True)
    L_ = plugin.L

    def e2e_step():
        plugin.check(L_.katali_cuda_upload(xs.data_ptr(), xh.data_ptr(), xh.numel() * 4))
        plugin.check(L_.katali_cuda_upload(lgs.data_ptr(), lh.data_ptr(), lh.numel() * 4))
        for i in range(T):
            layers[i % L].forward(xs[i], lgs[i], ys[i], mode)
        plugin.check(L_.katali_cuda_download(yh.data_ptr(), ys.data_ptr(), yh.numel() * 4))

    for _ in range(2):
        e2e_step()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e_start.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e_end.record(stream)
    e_end.synchronize()
    e_ms = e_start.elapsed_time(e_end)
    if world > 1:
        t = torch.tensor([e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
    e2e_value = world * args.steps * T * CALL_BYTES / (e_ms / 1e3) / 1e9

    # ---- CPU baseline (rank 0, N == 1 only) ---------------------------------
    cpu = None
    if rank == 0 and world == 1 and args.cpu_seconds > 0:
        try:
            from oracle.oracle import MoeWeights
            hl = [MoeWeights(st.gate.cpu().numpy(), st.up.cpu().numpy(), st.down.cpu().numpy(),
                             H, F, K) for st in stores[:2]]
            gbs, cores, calls, el = cpu_reference_rate(hl, args.cpu_seconds)
            cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "reference",
                   "sample": f"{calls} layer calls ({el:.1f} s) on 2 of the benchmark's layers, "
                             f"reference CPU kernels composed per call, {cores} threads"}
        except Exception as e:
            cpu = {"value": None, "unit": "GB/s", "cores": os.cpu_count(), "kind": "reference",
                   "sample": f"unavailable: {e}"}

    line = None
    if rank == 0:
        peak, peak_kind = measured_peaks()
        achieved = CALL_BYTES / (us_per_call * 1e-6) / 1e9
        traffic = committed_traffic()
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32" if args.f32 else "int8", "data": "synthetic",
            "config": {"workload": WORKLOAD if not args.f32 else WORKLOAD.replace(
                           "x N(0,1) quantised to q8_1 on device", "fp32 activations (x N(0,1))"),
                       "calls_per_step": T * reps, "graph_calls": T, "layers_in_store": L,
                       "store_bytes_per_gpu": L * E * EXPERT_BYTES,
                       "l2": "inputs larger than L2: 16-layer store (8.4 GB) rotated per call",
                       "graph": graph is not None, "parallelism": f"replicas x{world}",
                       "us_per_layer": round(us_per_call, 3)},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_kind": f"{peak_kind} hbm_gbs",
                         "traffic": traffic.get("dram_bytes_per_launch") if traffic else None,
                         "algorithmic_bytes_per_launch": CALL_BYTES},
            "clocks": clk.summary(),
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": xh.numel() * 4 + lh.numel() * 4,
                    "d2h_bytes_per_step": yh.numel() * 4},
            "e2e_scope": f"{T} layer calls per e2e step through the C ABI (eager), inputs "
                         f"uploaded and outputs downloaded every step",
            "gpu_launches": args.steps * reps * T,
            "cpu_baseline": cpu,
        }
    for l in layers:
        l.close()
    return line


TRACE_SLOTS = 32  # per CTA, as the plugin writes them
TRACE_NAMES = {1: "routed", 2: "x/table staged", 3: "loads issued", 4: "first chunk in",
               5: "gate/up done", 6: "barrier passed", 7: "phase B start", 8: "end",
               9: "route: logits in", 10: "route: sorted", 11: "route: top-k done",
               12: "2nd chunk in", 13: "down rows in", 14: "down rows decoded",
               15: "phase B row0 dots"}


EP_TRACE_NAMES = {**TRACE_NAMES, 1: "slots stored", 11: "pairs received", 18: "rounds done",
                  19: "combine done", 20: "dispatch: routed", 21: "x rows staged",
                  22: "round 0 done", 23: "next round requested", 24: "round 0: first chunk in",
                  25: "round 0: gate/up done", 26: "round 0: barrier passed",
                  27: "round 0: phase B start", 28: "dispatch: ids stored",
                  29: "dispatch: weights formed", 30: "dispatch: weights stored"}


def print_trace(plugin, layers, xs, lgs, ys, T, L, warm=False, call=None, names=TRACE_NAMES,
                tag="[trace]", mode=None):
    """Phase timeline of the fused MoE kernel from its %globaltimer trace (ns). `call(i)`
    runs layer call i (default: the single-GPU layer on token i)."""
    import torch
    from katali_lab_b200 import MOE_Q8_1
    buf = torch.zeros(1024 * TRACE_SLOTS, dtype=torch.int64, device="cuda")
    mhz = []
    rows = []
    slots = sorted(names)
    for n in range(min(T, 32)):
        i = 0 if warm else n
        lay = layers[i % L]
        grid = lay.set_trace(buf)
        if call is None:
            lay.forward(xs[i], lgs[i], ys[i], MOE_Q8_1 if mode is None else mode)
        else:
            call(i)
        plugin.sync()
        lay.set_trace(None)
        t = buf[:grid * TRACE_SLOTS].view(grid, TRACE_SLOTS).cpu().numpy().astype(np.int64)
        t = t[t[:, 0] > 0]  # the CTAs that ran (a launch may use fewer than the grid size)
        buf.zero_()
        mhz.append(np.median((t[:, 17] - t[:, 16]) / np.maximum(t[:, 8] - t[:, 0], 1) * 1e3))
        t0 = t[:, 0].min()
        row = [t[:, 0].max() - t0]
        for s in slots:  # CTAs without phase-A or phase-B rows leave their slot 0
            v = t[:, s][t[:, s] > 0]
            row.append((v.max() - t0) if v.size else 0)
        rows.append(row)
    med = np.median(np.array(rows, dtype=np.float64), axis=0) / 1e3
    print(f"{tag} median over calls, us after the first CTA started (max over CTAs):",
          file=sys.stderr)
    print(f"{tag}   last CTA start {med[0]:.2f}", file=sys.stderr)
    for s, v in sorted(zip(slots, med[1:]), key=lambda sv: sv[1]):
        if v > 0:
            print(f"{tag}   {names[s]:20s} {v:.2f}", file=sys.stderr)
    print(f"{tag}   SM clock inside the kernel: {np.median(mhz):.0f} MHz (cycles / ns)", file=sys.stderr)


C1_ROWS, C1_COLS = 6144, 2048
C1_BYTES = C1_ROWS * (C1_COLS // 256 * 144)  # 7,077,888 B of Q4_K weights per call
C1_WORKLOAD = ("C1 dense Q4_K GEMV, batch 1: W 6144x2048 from N(0,0.02) (seed 0) encoded to Q4_K, "
               "x N(0,1) fp32 len 2048, y fp32 len 6144")


def run_c1(args, rank, world, local_rank):
    """C1: katali_cuda_matvec (the reference's drop-in entry) over 64 distinct weight copies
    (453 MB, far larger than L2), one call per copy per step."""
    from katali_lab_b200 import Q4_K, Plugin
    from katali_lab_b200.synth import make_dense
    old = os.environ.get("KATALI_CUDA_DP4A")
    os.environ["KATALI_CUDA_DP4A"] = "1" if args.dp4a else "0"
    try:
        return _run_c1(args, rank, world, local_rank, Q4_K, Plugin, make_dense)
    finally:
        if old is None:
            os.environ.pop("KATALI_CUDA_DP4A", None)
        else:
            os.environ["KATALI_CUDA_DP4A"] = old


def _run_c1(args, rank, world, local_rank, Q4_K, Plugin, make_dense):
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    plugin = Plugin()
    if not plugin.probe():
        raise SystemExit(f"no usable B200: {plugin.status()}")
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    plugin.set_stream(stream)
    T = args.calls
    ws = [make_dense(plugin, Q4_K, C1_ROWS, C1_COLS, seed=(0 if i == 0 else 1000 + i)) for i in range(T)]
    g = torch.Generator(device="cuda").manual_seed(7 + rank)
    xs = torch.randn((T, C1_COLS), generator=g, device="cuda")
    ys = torch.empty((T, C1_ROWS), device="cuda")
    plugin.set_async(True)

    def step():
        for i in range(T):
            plugin.matvec(Q4_K, ws[i], C1_ROWS, C1_COLS, xs[i], ys[i])

    step()
    plugin.sync()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr, stream=stream):
        plugin.set_stream(torch.cuda.current_stream())
        step()
    plugin.set_stream(stream)
    for _ in range(max(args.warmup, 3)):
        gr.replay()
    plugin.sync()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        s0.record(stream)
        for _ in range(args.steps):
            gr.replay()
        s1.record(stream)
        s1.synchronize()
    plugin.sync()
    ms = s0.elapsed_time(s1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    us_call = 1e3 * ms / (args.steps * T)
    value = world * C1_BYTES / (us_call * 1e-6) / 1e9
    # e2e: the reference's own per-projection sequence (upload x, matvec, download y)
    xh = torch.randn(C1_COLS).pin_memory()
    yh = torch.empty(C1_ROWS).pin_memory()
    plugin.set_async(False)
    L_ = plugin.L
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_e2e = min(T, 64) * args.steps
    e0.record(stream)
    for i in range(n_e2e):
        plugin.check(L_.katali_cuda_upload(xs[i % T].data_ptr(), xh.data_ptr(), C1_COLS * 4))
        plugin.matvec(Q4_K, ws[i % T], C1_ROWS, C1_COLS, xs[i % T], ys[i % T])
        plugin.check(L_.katali_cuda_download(yh.data_ptr(), ys[i % T].data_ptr(), C1_ROWS * 4))
    e1.record(stream)
    e1.synchronize()
    e2e_value = world * C1_BYTES * n_e2e / (e0.elapsed_time(e1) / 1e3) / 1e9
    cpu = None
    if rank == 0 and world == 1 and args.cpu_seconds > 0:
        from oracle.oracle import Ref
        ref = Ref()
        wh = [w.cpu().numpy() for w in ws[:8]]
        xv = xs[0].cpu().numpy()
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < args.cpu_seconds or n < 8:
            ref.matvec(Q4_K, wh[n % 8], C1_ROWS, C1_COLS, xv, n_threads=os.cpu_count() or 1)
            n += 1
        el = time.perf_counter() - t0
        cpu = {"value": round(n * C1_BYTES / el / 1e9, 3), "unit": "GB/s", "cores": os.cpu_count(),
               "kind": "reference", "sample": f"{n} katali_ggml_matvec calls ({el:.1f} s) over 8 weight "
                                               f"copies, {os.cpu_count()} threads"}
    line = None
    if rank == 0:
        peak, peak_kind = measured_peaks()
        achieved = C1_BYTES / (us_call * 1e-6) / 1e9
        line = {
            "metric": "dense Q4_K GEMV quant-weight GB/s vs HBM peak", "value": round(value, 2),
            "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8" if args.dp4a else "f32", "data": "synthetic",
            "config": {"workload": C1_WORKLOAD, "calls_per_step": T, "activations": "q8_1" if args.dp4a else "fp32",
                       "l2": "inputs larger than L2: 64 weight copies (453 MB) rotated per call",
                       "us_per_call": round(us_call, 3)},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": f"{peak_kind} hbm_gbs",
                         "traffic": (committed_traffic("gemv_c1_traffic.json") or {}).get("dram_bytes_per_launch")
                         if not args.dp4a else None,
                         "algorithmic_bytes_per_launch": C1_BYTES},
            "clocks": clk.summary(),
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": C1_COLS * 4,
                    "d2h_bytes_per_step": C1_ROWS * 4},
            "gpu_launches": args.steps * T, "cpu_baseline": cpu}
    return line


C3_WORKLOAD = ("C3 ragged continuous batch of the C2 layer: per call T ~ U{1..64} tokens "
               "(seeded), top-8 of softmax(N(0,1) logits) per token, pairs grouped per expert")


def c3_plan(calls: int, seed: int = 3, tmin: int = 1, tmax: int = 64, hot: int = 0):
    """Token counts per call and the host-side routing of every token (for the distinct-
    expert byte count): T_i ~ U{tmin..tmax}, x and logits N(0,1); hot > 0 adds 8 to the
    logits of experts 0..hot-1 (every token then picks among them: large groups)."""
    rng = np.random.default_rng(seed)
    Ts = rng.integers(tmin, tmax + 1, size=calls)
    X = rng.normal(0, 1, (int(Ts.sum()), H)).astype(np.float32)
    LG = rng.normal(0, 1, (int(Ts.sum()), E)).astype(np.float32)
    if hot:
        LG[:, :hot] += 8.0
    top = np.argsort(-LG, axis=1, kind="stable")[:, :K]
    offs = np.concatenate([[0], np.cumsum(Ts)])
    distinct = [len(np.unique(top[offs[i]:offs[i + 1]])) for i in range(calls)]
    return Ts, offs, X, LG, distinct


def run_c3(args, rank, world, local_rank):
    """C3: katali_cuda_moe_batch over ragged batches; metric = distinct selected expert
    bytes read per second (each selected expert's rows once per call)."""
    import torch
    import torch.distributed as dist

    from katali_lab_b200 import MoeLayer, Plugin
    from katali_lab_b200.synth import make_expert_store
    torch.cuda.set_device(local_rank)
    plugin = Plugin()
    if not plugin.probe():
        raise SystemExit(f"no usable B200: {plugin.status()}")
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    plugin.set_stream(stream)
    L, n = args.layers, args.calls
    stores = [make_expert_store(plugin, E, H, F, seed=10_000 * rank + l) for l in range(L)]
    layers = [MoeLayer(plugin, E, H, F, K, st.pointers()) for st in stores]
    Ts, offs, Xh, LGh, distinct = c3_plan(n, seed=3 + rank, tmin=args.tmin, hot=args.hot)
    ntok = int(Ts.sum())
    xs, lgs = torch.from_numpy(Xh).cuda(), torch.from_numpy(LGh).cuda()
    ys = torch.empty((ntok, H), device="cuda")
    x64 = torch.randn((64, H), device="cuda")
    l64 = torch.randn((64, E), device="cuda")
    y64 = torch.empty((64, H), device="cuda")
    for l in layers:  # grow every layer's batch scratch to 64 tokens before capture
        l.forward_batch(x64, l64, y64)
    plugin.sync()
    plugin.set_async(True)

    def step():
        for i in range(n):
            a, b = int(offs[i]), int(offs[i + 1])
            layers[i % L].forward_batch(xs[a:b], lgs[a:b], ys[a:b])

    step()
    plugin.sync()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr, stream=stream):
        plugin.set_stream(torch.cuda.current_stream())
        step()
    plugin.set_stream(stream)
    for _ in range(max(args.warmup, 3)):
        gr.replay()
    plugin.sync()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        s0.record(stream)
        for _ in range(args.steps):
            gr.replay()
        s1.record(stream)
        s1.synchronize()
    plugin.sync()
    ms = s0.elapsed_time(s1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    step_bytes = sum(distinct) * EXPERT_BYTES
    value = world * args.steps * step_bytes / (ms / 1e3) / 1e9
    tok_s = world * args.steps * ntok / (ms / 1e3)
    # e2e: pinned host inputs uploaded, the calls, outputs downloaded, every step
    xh, lh = torch.from_numpy(Xh).pin_memory(), torch.from_numpy(LGh).pin_memory()
    yh = torch.empty((ntok, H)).pin_memory()
    L_ = plugin.L

    def e2e_step():
        plugin.check(L_.katali_cuda_upload(xs.data_ptr(), xh.data_ptr(), xh.numel() * 4))
        plugin.check(L_.katali_cuda_upload(lgs.data_ptr(), lh.data_ptr(), lh.numel() * 4))
        step()
        plugin.check(L_.katali_cuda_download(yh.data_ptr(), ys.data_ptr(), yh.numel() * 4))

    e2e_step()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    e1.synchronize()
    e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
    e2e_value = world * args.steps * step_bytes / (e_ms / 1e3) / 1e9
    cpu = None
    if rank == 0 and world == 1 and args.cpu_seconds > 0:
        cpu = c3_cpu_rate(stores[:2], Ts, offs, Xh, LGh, distinct, args.cpu_seconds)
    line = None
    if rank == 0:
        peak, peak_kind = measured_peaks()
        us_call = 1e3 * ms / (args.steps * n)
        achieved = step_bytes / n / (us_call * 1e-6) / 1e9
        line = {
            "metric": "MoE-layer distinct-expert quant-weight GB/s vs HBM peak",
            "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic",
            "config": {"workload": C3_WORKLOAD + (f"; hot experts 0..{args.hot - 1} (+8 logits)"
                                                   if args.hot else ""),
                       "tensor_cores": os.environ.get("KATALI_CUDA_NO_TC") != "1",
                       "calls_per_step": n, "tokens_per_step": ntok,
                       "distinct_experts_per_step": int(sum(distinct)),
                       "tokens_per_s": round(tok_s, 1), "us_per_call": round(us_call, 3),
                       "l2": "inputs larger than L2: 16-layer store (8.4 GB) rotated per call",
                       "parallelism": f"replicas x{world}"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_kind": f"{peak_kind} hbm_gbs", "traffic": None,
                         "scope": "whole call (six launches)"},
            "clocks": clk.summary(),
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": xh.numel() * 4 + lh.numel() * 4,
                    "d2h_bytes_per_step": yh.numel() * 4},
            "gpu_launches": args.steps * n * 6, "cpu_baseline": cpu}
    for l in layers:
        l.close()
    return line


def c3_cpu_rate(stores_or_layers, Ts, offs, Xh, LGh, distinct, seconds):
    """The reference CPU composition, one token at a time (its engine's per-token call),
    over the C3 calls in order until ~`seconds`; GB/s of distinct expert bytes."""
    from oracle.oracle import MoeWeights, Ref
    ref = Ref()
    cores = os.cpu_count() or 1
    hl = [s if isinstance(s, MoeWeights) else
          MoeWeights(s.gate.cpu().numpy(), s.up.cpu().numpy(), s.down.cpu().numpy(), H, F, K)
          for s in stores_or_layers]
    scratch = ref.moe_scratch(hl[0])
    calls, toks, nbytes, t0 = 0, 0, 0, time.perf_counter()
    while True:
        i = calls % len(Ts)
        for t in range(int(offs[i]), int(offs[i + 1])):
            ref.moe_layer(hl[i % len(hl)], Xh[t], LGh[t], n_threads=cores, scratch=scratch)
        toks += int(Ts[i])
        nbytes += distinct[i] * EXPERT_BYTES
        calls += 1
        el = time.perf_counter() - t0
        if (el >= seconds and calls >= 2) or calls >= 100000:
            break
    ref.L.kref_moe_scratch_free(scratch)
    return {"value": round(nbytes / el / 1e9, 3), "unit": "GB/s", "cores": cores,
            "kind": "reference",
            "sample": f"{calls} ragged calls ({toks} tokens, {el:.1f} s), reference CPU kernels "
                      f"composed per token, {cores} threads"}


EP_WORKLOAD = ("{cfg} expert-parallel over {n} GPUs: 256 experts split in blocks of {per} per GPU, "
               "every GPU brings its own tokens ({tok}); dispatch/combine {how}")


def ep_parity(plugin, store, world, xs, lgs, ys, offs):
    """Each rank's call-0 tokens (layer 0) of the expert-parallel run against the single-GPU
    fused layer over all experts of layer 0, gathered from every rank's slice (NCCL
    all-gather), at the bar of the expert-parallel GPU tests (rel_L2 <= 1e-5). The single-GPU
    kernel is pinned to the C restatement by the GPU test suite; this check runs no oracle
    code. Returns the max over ranks."""
    import torch
    import torch.distributed as dist

    from katali_lab_b200 import MOE_Q8_1, MoeLayer
    full = []
    for t in (store.gate, store.up, store.down):
        out = torch.empty((world * t.shape[0], t.shape[1]), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(out, t.contiguous())
        full.append(out)
    torch.cuda.synchronize()
    g, u, d = full
    ptrs = [(g.data_ptr() + e * g.shape[1], u.data_ptr() + e * u.shape[1],
             d.data_ptr() + e * d.shape[1]) for e in range(g.shape[0])]
    layer = MoeLayer(plugin, g.shape[0], H, F, K, ptrs)
    y1 = torch.empty(H, device="cuda")
    worst, equal, n = 0.0, 0, 0
    for t in range(int(offs[0]), int(offs[1])):
        layer.forward(xs[t], lgs[t], y1, MOE_Q8_1)
        torch.cuda.synchronize()
        den = float(y1.norm())
        worst = max(worst, float((ys[t] - y1).norm()) / (den if den > 0 else 1.0))
        equal += int((ys[t] == y1).sum())
        n += H
    layer.close()
    v = torch.tensor([worst, float(equal), float(n)], device="cuda", dtype=torch.float64)
    w = v.clone()
    dist.all_reduce(w[:1], op=dist.ReduceOp.MAX)
    dist.all_reduce(w[1:], op=dist.ReduceOp.SUM)
    del full
    return {"ok": bool(w[0].item() <= 1e-5), "max_rel_l2": float(w[0].item()),
            "bit_equal_frac": round(float(w[1].item() / max(w[2].item(), 1.0)), 6),
            "against": "single-GPU fused layer over all experts (gathered), every rank's call-0 tokens",
            "bar": "rel_L2 <= 1e-5"}


def ep_trace(plugin, layers, step, stream, rank, world, L, n):
    """Phase timeline of the single-launch expert-parallel layer as the timed graph runs it
    (calls back to back, ranks in lock step): one trace buffer per layer keeps that layer's
    last call of a replay; rank 0 prints, per rank, the median over layers of each phase's
    end (max over CTAs) after the first CTA of the call started on any rank (%globaltimer;
    the GPUs' timers agree only to within their offset) and the gap from a call's end to the
    next call's first CTA on the same rank."""
    import torch
    import torch.distributed as dist
    bufs = torch.zeros((L, 1024 * TRACE_SLOTS), dtype=torch.int64, device="cuda")
    grids = [layers[l].layer.set_trace(bufs[l]) for l in range(L)]
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2, stream=stream):
        step()
    for _ in range(3):
        g2.replay()
    torch.cuda.synchronize()
    for l in layers:
        l.layer.set_trace(None)
    del g2
    gath = [torch.empty_like(bufs) for _ in range(world)]
    dist.all_gather(gath, bufs)
    torch.cuda.synchronize()
    if rank != 0:
        return
    tr = [g.cpu().numpy() for g in gath]
    last = sorted(range(L), key=lambda l: (n - 1 - l) // L * L + l)  # layers in call order
    names = {0: "CTAs started", **EP_TRACE_NAMES}
    slots = sorted(names)
    rows = {r: [] for r in range(world)}
    gaps = {r: [] for r in range(world)}
    for l in range(L):
        ts = []
        for r in range(world):
            t = tr[r][l][:grids[l] * TRACE_SLOTS].reshape(grids[l], TRACE_SLOTS)
            ts.append(t[t[:, 0] > 0])
        t0 = min(int(t[:, 0].min()) for t in ts)
        for r, t in enumerate(ts):
            row = []
            for s in slots:
                v = t[:, s][t[:, s] > 0]
                row.append((int(v.max()) - t0) if v.size else np.nan)
            rows[r].append(row)
    for i in range(L - 1):  # consecutive calls i, i + 1 of the last stretch of the step
        a, b = last[i], last[i + 1]
        for r in range(world):
            ta = tr[r][a][:grids[a] * TRACE_SLOTS].reshape(grids[a], TRACE_SLOTS)
            tb = tr[r][b][:grids[b] * TRACE_SLOTS].reshape(grids[b], TRACE_SLOTS)
            ta, tb = ta[ta[:, 0] > 0], tb[tb[:, 0] > 0]
            gaps[r].append(int(tb[:, 0].min()) - int(ta[:, 8].max()))
    print("[trace] median over layers, us after the call's first CTA on any rank "
          "(max over a rank's CTAs):", file=sys.stderr)
    for r in range(world):
        med = np.nanmedian(np.array(rows[r], dtype=np.float64), axis=0) / 1e3
        parts = sorted(((v, names[s]) for s, v in zip(slots, med) if v == v and v > 0))
        print(f"[trace r{r}] " + ", ".join(f"{nm} {v:.2f}" for v, nm in parts), file=sys.stderr)
        print(f"[trace r{r}] call end -> next call start: median {np.median(gaps[r]) / 1e3:.2f} us",
              file=sys.stderr)


def run_ep(args, rank, world, local_rank):
    """C2 / C3 with experts split over the GPUs (one process each): every rank holds E/N
    experts of every layer and brings its own tokens (one per call for C2, T ~ U{1..64}
    for C3). metric = distinct selected expert bytes of the whole job per second (every
    selected expert is read once per call by its owner for all tokens routed to it)."""
    import torch
    import torch.distributed as dist

    from katali_lab_b200 import Plugin
    from katali_lab_b200.ep import EpComm, EpMoeLayer, experts_per_rank
    from katali_lab_b200.synth import make_expert_store
    torch.cuda.set_device(local_rank)
    plugin = Plugin()
    if not plugin.probe():
        raise SystemExit(f"no usable B200: {plugin.status()}")
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    plugin.set_stream(stream)
    per = experts_per_rank(E, world)
    L, n = args.layers, args.calls
    ragged = args.config == "c3"
    tmax = 64 if ragged else 1
    stores = [make_expert_store(plugin, per, H, F, seed=10_000 * l + rank) for l in range(L)]
    layers = [EpMoeLayer(plugin, E, H, F, K, st.pointers(), world, rank, tmax) for st in stores]
    comm = EpComm.from_process_group(plugin)
    if not args.nccl:
        comm.use_peer_memory(True)
    # every rank's inputs from its seed, so every rank can count the job's distinct experts
    plans = [c3_plan(n, seed=3 + r, tmin=1 if ragged else 1, tmax=tmax) for r in range(world)]
    Ts, offs, Xh, LGh, _ = plans[rank]
    distinct = []
    for i in range(n):
        sel = set()
        for r in range(world):
            _, o, _, lg, _ = plans[r]
            top = np.argsort(-lg[o[i]:o[i + 1]], axis=1, kind="stable")[:, :K]
            sel.update(int(e) for e in top.ravel())
        distinct.append(len(sel))
    ntok = int(Ts.sum())
    xs, lgs = torch.from_numpy(Xh).cuda(), torch.from_numpy(LGh).cuda()
    ys = torch.empty((ntok, H), device="cuda")
    torch.cuda.synchronize()

    def step():
        for i in range(n):
            a, b = int(offs[i]), int(offs[i + 1])
            layers[i % L].forward(xs[a:b], lgs[a:b], ys[a:b], n_tokens=b - a, comm=comm)

    step()  # sizes every exchange buffer and scratch before capture
    torch.cuda.synchronize()
    parity = None if ragged else ep_parity(plugin, stores[0], world, xs, lgs, ys, offs)
    plugin.set_async(True)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr, stream=stream):
        step()
    for _ in range(max(args.warmup, 3)):
        gr.replay()
    torch.cuda.synchronize()
    dist.barrier()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        s0.record(stream)
        for _ in range(args.steps):
            gr.replay()
        s1.record(stream)
        s1.synchronize()
    plugin.sync()
    ms = s0.elapsed_time(s1)
    t = torch.tensor([ms], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    step_bytes = sum(distinct) * EXPERT_BYTES
    value = args.steps * step_bytes / (ms / 1e3) / 1e9
    tok_all = sum(int(p[0].sum()) for p in plans)
    # e2e: this rank's inputs from pinned host memory, the layer calls, outputs back
    xh, lh = torch.from_numpy(Xh).pin_memory(), torch.from_numpy(LGh).pin_memory()
    yh = torch.empty((ntok, H)).pin_memory()
    L_ = plugin.L

    def e2e_step():
        plugin.check(L_.katali_cuda_upload(xs.data_ptr(), xh.data_ptr(), xh.numel() * 4))
        plugin.check(L_.katali_cuda_upload(lgs.data_ptr(), lh.data_ptr(), lh.numel() * 4))
        step()
        plugin.check(L_.katali_cuda_download(yh.data_ptr(), ys.data_ptr(), yh.numel() * 4))

    e2e_step()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    e1.synchronize()
    t = torch.tensor([e0.elapsed_time(e1)], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_value = args.steps * step_bytes / (float(t.item()) / 1e3) / 1e9
    plugin.sync()
    line = None
    if rank == 0:
        peak, peak_kind = measured_peaks()
        us_call = 1e3 * ms / (args.steps * n)
        line = {
            "metric": METRIC if not ragged else "MoE-layer distinct-expert quant-weight GB/s vs HBM peak",
            "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic",
            "config": {"workload": EP_WORKLOAD.format(cfg="C3 ragged batch" if ragged else
                                                      "C2 batch-1 decode", n=world, per=per,
                                                      tok="T ~ U{1..64} per call" if ragged
                                                      else "one per call",
                                                      how=("over NVLink peer memory inside the kernels"
                                                           + ("" if ragged else "; the whole layer "
                                                              "(dispatch, experts, return, combine) in one "
                                                              "launch per GPU"))
                                                      if not args.nccl else "by the plugin's NCCL communicator "
                                                      "(grouped send/recv of fixed-capacity q8_1 slots)"),
                       "calls_per_step": n, "tokens_per_step_job": tok_all,
                       "distinct_experts_per_step": int(sum(distinct)),
                       "us_per_call": round(us_call, 3), "parallelism": f"ep{world}",
                       "l2": "inputs larger than L2: 16-layer store rotated per call"},
            "roofline": {"bound": "hbm", "achieved": round(value / world, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(value / world / peak, 4),
                         "peak_kind": f"{peak_kind} hbm_gbs, per GPU", "traffic": None,
                         "scope": ("whole call per GPU: one launch doing dispatch, expert "
                                   "decode, return and combine over NVLink peer memory"
                                   if not args.nccl and not ragged else
                                   "whole call per GPU: the layer's launches and the exchanges "
                                   + ("over NVLink peer memory" if not args.nccl
                                      else "by NCCL send/recv"))},
            "collective": ("none on the data path: peer-memory loads and stores inside the "
                           "kernels (NCCL only all-gathers the IPC handles once, at setup)"
                           if not args.nccl else "NCCL grouped send/recv, twice per call"),
            "clocks": clk.summary(),
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": xh.numel() * 4 + lh.numel() * 4,
                    "d2h_bytes_per_step": yh.numel() * 4},
            "parity": parity,
            "gpu_launches": args.steps * n * (1 if not ragged and not args.nccl else 8),
            "cpu_baseline": None}
    del gr
    if args.trace:
        ep_trace(plugin, layers, step, stream, rank, world, L, n)
    comm.close()
    for l in layers:
        l.close()
    return line


C4_WORKLOAD = ("C4 dense Qwen3-8B-shape greedy decode on one GPU: 36 layers, hidden 4096, FFN 12288, "
               "32 q / 8 kv heads of 128, vocab 151936, fp32 KV cache; Q4_K with Q6_K attn_v, "
               "ffn_down and output (N(0,0.02) weights); {n} tokens per step after a 1-token prompt")


def run_c4(args, rank, world, local_rank):
    """C4: katali_cuda_dense_generate; a step = one greedy generation of `calls` tokens from
    an empty cache. metric = quantised weight bytes read per second (every matrix once per
    token); tokens/s in config."""
    import torch

    from katali_lab_b200 import DenseModel, Plugin
    from katali_lab_b200.synth import QWEN3_8B, make_dense_model
    torch.cuda.set_device(local_rank)
    plugin = Plugin()
    if not plugin.probe():
        raise SystemExit(f"no usable B200: {plugin.status()}")
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    cfg = QWEN3_8B if args.dense_layers == QWEN3_8B.n_layers else \
        dataclasses.replace(QWEN3_8B, n_layers=args.dense_layers)
    model = make_dense_model(plugin, cfg, seed=8 + rank)
    plugin.set_stream(stream)
    dm = DenseModel(plugin, model, q8=args.dp4a)
    n = args.calls * 2  # 128 tokens by default
    prompt = [1]
    for _ in range(max(args.warmup, 3)):
        dm.reset()
        dm.generate(prompt, n)
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        s0.record(stream)
        for _ in range(args.steps):
            dm.reset()
            toks = dm.generate(prompt, n)
        s1.record(stream)
        s1.synchronize()
    ms = s0.elapsed_time(s1)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    bpt = model.weight_bytes_per_token
    tok_s = world * args.steps * n / (ms / 1e3)
    value = tok_s * bpt / 1e9
    cpu = None
    if rank == 0 and world == 1 and args.cpu_seconds > 0:
        from oracle.oracle import Ref, RefDense
        ref = RefDense(Ref(), model)
        cores = os.cpu_count() or 1
        t0, k, tok = time.perf_counter(), 0, 1
        while time.perf_counter() - t0 < args.cpu_seconds or k < 2:
            lg = ref.step(tok, k)
            tok = int(np.argmax(lg))
            k += 1
        el = time.perf_counter() - t0
        ref.close()
        cpu = {"value": round(k * bpt / el / 1e9, 3), "unit": "GB/s", "cores": cores,
               "kind": "reference", "tokens_per_s": round(k / el, 3),
               "sample": f"{k} greedy decode steps ({el:.1f} s) of the same model through the "
                         f"reference's CPU kernels (gguf_forward_token composition), {cores} threads"}
    line = None
    if rank == 0:
        peak, peak_kind = measured_peaks()
        achieved = value / world
        line = {
            "metric": "dense decode quant-weight GB/s vs HBM peak", "value": round(value, 2),
            "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8" if args.dp4a else "f32",
            "data": "synthetic",
            "config": {"workload": C4_WORKLOAD.format(n=n), "tokens_per_step": n,
                       "n_layers": cfg.n_layers,
                       "activations": "q8_1 (DP4A)" if args.dp4a else "fp32",
                       "tokens_per_s": round(tok_s, 1), "weight_bytes_per_token": bpt,
                       "us_per_token": round(1e3 * ms / (args.steps * n), 2),
                       "l2": "inputs larger than L2: 4.9 GB of weights read per token",
                       "parallelism": f"replicas x{world}", "last_tokens": [int(t) for t in toks[:8]]},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": f"{peak_kind} hbm_gbs",
                         "traffic": None, "scope": "whole decode step (all kernels)"},
            "clocks": clk.summary(),
            "e2e": {"value": round(value, 2), "unit": "GB/s", "h2d_bytes_per_step": 4 * len(prompt),
                    "d2h_bytes_per_step": 4 * n},
            "gpu_launches": args.steps * n * (1 + 6 * cfg.n_layers + 3), "cpu_baseline": cpu}
    dm.close()
    return line


C5_WORKLOAD = ("C5 35B-A3B-class hybrid greedy decode on one GPU: 40 layers (30 Gated DeltaNet: 16 q/k "
               "and 32 v heads of 128, conv 4; 10 gated attention: 16 q / 2 kv heads of 256, RoPE on 64 "
               "dims, fp32 KV), MoE every layer as C2 (256 experts, FFN 512, top-8, fp32 router), "
               "hidden 2048, vocab 248320; Q4_K with Q6_K attn_v, expert down and output (N(0,0.02) "
               "weights); {n} tokens per step after a 1-token prompt")


def run_c5(args, rank, world, local_rank):
    """C5: katali_cuda_hybrid_generate; a step = one greedy generation of 32 tokens from an
    empty state. metric = decode tokens/s (whole job); roofline = weight + state bytes per
    token x tokens/s against the HBM peak."""
    import torch

    from katali_lab_b200 import HybridModel, Plugin
    from katali_lab_b200.synth import HYBRID_35B, make_hybrid_model
    torch.cuda.set_device(local_rank)
    plugin = Plugin()
    if not plugin.probe():
        raise SystemExit(f"no usable B200: {plugin.status()}")
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    cfg = HYBRID_35B if args.hybrid_layers == HYBRID_35B.n_layers else \
        dataclasses.replace(HYBRID_35B, n_layers=args.hybrid_layers)
    ep = world > 1 and not args.replicas  # experts sharded over the GPUs, one sequence per rank
    q8 = args.dp4a or ep                  # the expert-parallel layer runs q8_1 activations
    model = make_hybrid_model(plugin, cfg, seed=35 if ep else 35 + rank,
                              ep=(world, rank) if ep else None)
    plugin.set_stream(stream)
    hm = HybridModel(plugin, model, q8=q8)
    comm = None
    if ep:
        from katali_lab_b200.ep import EpComm
        comm = EpComm.from_process_group(plugin)
        comm.use_peer_memory(True)
        hm.set_ep(comm)
    n = 32
    prompt = [1 + rank]
    for _ in range(max(args.warmup, 3)):
        hm.reset()
        hm.generate(prompt, n)
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps = args.steps  # each a 32-token generation
    with ClockSampler(local_rank) as clk:
        s0.record(stream)
        for _ in range(steps):
            hm.reset()
            toks = hm.generate(prompt, n)
        s1.record(stream)
        s1.synchronize()
    ms = s0.elapsed_time(s1)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    bpt = model.weight_bytes_per_token + model.state_bytes_per_token
    tok_s = world * steps * n / (ms / 1e3)
    cpu = None
    if rank == 0 and world == 1 and args.cpu_seconds > 0:
        cpu = c5_cpu_leg(model, toks, bpt, args.cpu_seconds, fp32=not q8)
    line = None
    if rank == 0:
        peak, peak_kind = measured_peaks()
        achieved = tok_s / world * bpt / 1e9
        line = {
            "metric": "hybrid MoE decode tok/s", "value": round(tok_s, 2), "unit": "tokens/s",
            "n_gpus": world, "steps": steps, "warmup": args.warmup,
            "ms_per_step": round(ms / steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8" if q8 else "f32",
            "data": "synthetic",
            "config": {"workload": C5_WORKLOAD.format(n=n), "tokens_per_step": n,
                       "n_layers": cfg.n_layers,
                       "activations": "q8_1 (DP4A)" if q8 else "fp32",
                       "bytes_per_token": bpt, "us_per_token": round(1e3 * ms / (steps * n), 2),
                       "l2": "inputs larger than L2: ~1.9 GB of weights and states read per token",
                       "parallelism": (f"ep{world}: experts of every layer split over the GPUs, "
                                       "one sequence per GPU, MoE blocks over NVLink peer memory")
                       if ep else f"replicas x{world}",
                       "last_tokens": [int(t) for t in toks[:8]]},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": f"{peak_kind} hbm_gbs",
                         "traffic": None, "scope": "whole decode step (all kernels), per GPU"},
            "clocks": clk.summary(),
            "e2e": {"value": round(tok_s, 2), "unit": "tokens/s", "h2d_bytes_per_step": 4 * len(prompt),
                    "d2h_bytes_per_step": 4 * n},
            "greedy_match": cpu.get("greedy_tokens_match_gpu") if cpu else None,
            "tokens": n,
            "gpu_launches": steps * n * (1 + (5 if ep else 4) * cfg.n_layers + 3), "cpu_baseline": cpu}
    hm.close()
    if comm is not None:
        comm.close()
    return line


def c5_cpu_leg(model, gpu_tokens, bpt, seconds, fp32=True):
    """The same decode through the CPU composition (reference kernels + the Gated DeltaNet
    restatement) on host copies of the model, for ~`seconds`; its greedy tokens are compared
    with the GPU's (fp32 activations)."""
    try:
        import psutil
        need = sum(w["experts"].gate.numel() * 3 for w in model.layers)
        if psutil.virtual_memory().available < 2 * need:
            return {"value": None, "unit": "tokens/s", "kind": "reference", "cores": 0,
                    "sample": "skipped: not enough host memory for a host copy of the model"}
    except Exception:
        pass
    from oracle.oracle import Ref, RefHybrid
    cores = os.cpu_count() or 1
    rh = RefHybrid(Ref(), model)
    t0, k, tok, toks = time.perf_counter(), 0, 1, []
    while k < len(gpu_tokens) and (time.perf_counter() - t0 < seconds or k < 2):
        lg = rh.step(tok, k)
        tok = int(np.argmax(lg))
        toks.append(tok)
        k += 1
    el = time.perf_counter() - t0
    rh.close()
    match = [int(a) for a in gpu_tokens[:len(toks)]] == toks if fp32 else None
    return {"value": round(k / el, 3), "unit": "tokens/s", "cores": cores, "kind": "reference",
            "gbs": round(k * bpt / el / 1e9, 3), "greedy_tokens_match_gpu": match,
            "tokens_compared": len(toks) if fp32 else 0,
            "sample": f"{k} greedy decode steps ({el:.1f} s) of the same model through the "
                      f"reference's CPU kernels + the Gated DeltaNet restatement, {cores} threads"}


# Keys of a secondary configuration's line kept in the headline's `secondary` object.
SECONDARY_KEYS = ("metric", "value", "unit", "steps", "warmup", "ms_per_step", "dtype", "config",
                  "roofline", "clocks", "e2e", "gpu_launches", "cpu_baseline", "parity",
                  "greedy_match", "tokens")


def run_secondary(args, rank, world, local_rank, headline):
    """The other configurations of the workload, measured in the same process after the
    headline, each under the same rules (>= 3 warm-up steps, CUDA events on the launching
    stream, inputs larger than L2, clocks sampled, e2e through the C ABI, CPU baseline on
    the reference's kernels at N = 1 with a shorter sample). Returns {name: line}."""
    import gc

    import torch

    def sub(**kw):
        a = argparse.Namespace(**vars(args))
        a.__dict__.update(kw)
        return a

    cs = min(args.cpu_seconds, 5.0)
    w = max(args.warmup, 3)
    if world == 1:
        plans = [
            ("c2_f32", run_ours, sub(f32=True, cpu_seconds=0, reps=4)),
            ("c1_f32", run_c1, sub(config="c1", dp4a=False, calls=64, steps=max(args.steps, 200),
                                   cpu_seconds=cs)),
            ("c1_q8_1", run_c1, sub(config="c1", dp4a=True, calls=64, steps=max(args.steps, 200),
                                    cpu_seconds=0)),
            ("c3", run_c3, sub(config="c3", calls=64, cpu_seconds=cs)),
            ("c4_f32", run_c4, sub(config="c4", dp4a=False, calls=64, steps=min(args.steps, 3),
                                   warmup=3, cpu_seconds=2 * cs)),
            ("c4_q8_1", run_c4, sub(config="c4", dp4a=True, calls=64, steps=min(args.steps, 3),
                                    warmup=3, cpu_seconds=0)),
            ("c5_f32", run_c5, sub(config="c5", dp4a=False, steps=min(args.steps, 10), warmup=w,
                                   cpu_seconds=max(cs, 1.0))),
            ("c5_q8_1", run_c5, sub(config="c5", dp4a=True, steps=min(args.steps, 10), warmup=w,
                                    cpu_seconds=0)),
        ]
    else:
        plans = [
            ("c2_replicas", run_ours, sub(replicas=True, cpu_seconds=0)),
            ("c3_ep", run_ep, sub(config="c3", calls=64)),
            ("c5_ep", run_c5, sub(config="c5", steps=min(args.steps, 10), warmup=w, cpu_seconds=0)),
        ]
    out = {}
    for name, fn, a in plans:
        t0 = time.time()
        try:
            line = fn(a, rank, world, local_rank)
        except Exception as e:  # reported, not fatal: the headline stands
            line = {"error": f"{type(e).__name__}: {e}"[:300]}
        gc.collect()
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        if rank == 0 and line is not None:
            kept = {k: line[k] for k in SECONDARY_KEYS if k in line} if "error" not in line else line
            kept["wall_s"] = round(time.time() - t0, 1)
            out[name] = kept
    if rank == 0 and world == 1 and "c2_f32" in out and headline and "cpu_baseline" in out["c2_f32"]:
        # the reference CPU layer runs fp32 activations: the headline's CPU leg is this twin's too
        out["c2_f32"]["cpu_baseline"] = headline.get("cpu_baseline")
    return out


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    out_fd = 1
    if world > 1:
        # Libraries print to file descriptor 1 (NCCL's version banner): for the whole run it
        # points at stderr, and the one JSON line goes to the saved stdout.
        out_fd = os.dup(1)
        os.dup2(2, 1)
        import datetime

        os.environ.setdefault("NCCL_DEBUG", "WARN")
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.config == "c1":
            line = run_c1(args, rank, world, local_rank)
        elif args.config == "c4":
            line = run_c4(args, rank, world, local_rank)
        elif args.config == "c5":
            line = run_c5(args, rank, world, local_rank)
        elif world > 1 and not args.replicas:
            line = run_ep(args, rank, world, local_rank)
        elif args.config == "c3":
            line = run_c3(args, rank, world, local_rank)
        else:
            line = run_ours(args, rank, world, local_rank)
        if args.config == "c2" and not args.no_secondary and not args.f32 and not args.warm \
                and not args.trace:
            sec = run_secondary(args, rank, world, local_rank, line)
            if rank == 0 and line is not None:
                line["secondary"] = sec
        if rank == 0 and line is not None:
            sys.stdout.flush()
            os.write(out_fd, (json.dumps(line) + "\n").encode())
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
