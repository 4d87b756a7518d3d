"""Benchmark: the int4 quantized-weight hot path on B200.

Default line, one GPU: configs[1], one decode token's full weight stream.  For
each of the 48 layers the q, k, v, o, gate, up and down int4 GEMVs, then
lm_head: 337 GEMVs reading 6,617,825,280 bytes of packed weights + f16 scales
(6,250,168,320 with ``--scales fp8``), each with its own f16 N(0, 1)
activation vector and f16 output.  q|k|v and gate|up read the same x in a
decode step and run fused, so a token is 193 GEMV steps; they run as one
persistent chain launch (g4b_gemv_chain) in which each step reads its x only
once the step before it is written.  Weights are N(0, 0.02) quantised exactly
as the engine's quant() does, on the GPU.  The working set (6.6 GB) is ~50x
the 126 MB L2, so every step streams from HBM; no L2 flush is needed.

Several GPUs (torchrun, one rank per GPU): configs[4], the same stream tensor
parallel (g4b.tp: q/k/v/gate/up/lm_head by output columns, o/down by input
rows, two all-reduces per layer, the logits all-gathered); each rank runs its
token as one chain launch with the all-reduces inside it.  "scaling":
"strong": value = the whole model's weight bytes / the token's device time,
max over ranks.

Reported (one JSON line from rank 0):
  value      whole-job GB/s (algorithmic bytes / device time), the step
             replayed as one CUDA graph with its inputs resident in HBM
  e2e        the same metric through the public API with host buffers: every
             step copies its activations in from one pinned host arena and
             its outputs back into another, inside the timed region
  roofline   the dominant kernel's achieved rate (algorithmic bytes or flops
             of its launches / their CUDA-event durations) against the
             measured HBM copy bandwidth or bf16 tensor rate
             (MEASURED_PEAKS.json)
  cpu_baseline  the reference's CPU path on the host cores: the oracle port of
             its shaders (oracle/g4b_oracle.c) on a bounded sample (rank 0,
             N=1); the same sampler as ``--impl reference``
  extras     the other BASELINE.json configs, each with its value and
             roofline: configs[0] (one GEMV), configs[1] with e4m3 scales,
             configs[2] (W4A16, both shapes) and configs[3] (W8A8, W4A8) on one
             GPU; configs[4]'s batched decode (M = 8 and 64 tokens) and its
             M = 8192 prefill split at every N.  --no-extras skips them.

``--impl reference`` times the reference's path for the same workload and
config on the host cores instead, with every host thread: the oracle
restatement of the shaders (the shaders themselves need a Vulkan stack that
these machines do not have).  Under torchrun only rank 0 runs it; the other
ranks exit at once.
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

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "gemma4-12b-snapdragonx2elite_b200"))

HIDDEN, FFN, LAYERS, VOCAB = 3840, 15360, 48, 262144
NQ, NKV = 16 * 256, 8 * 256
LAYER_SHAPES = [("q", NQ, HIDDEN), ("k", NKV, HIDDEN), ("v", NKV, HIDDEN), ("o", HIDDEN, NQ),
                ("gate", FFN, HIDDEN), ("up", FFN, HIDDEN), ("down", HIDDEN, FFN)]
LM_HEAD = ("lm_head", VOCAB, HIDDEN)
STREAM_METRIC = "int4 GEMV HBM GB/s (decode weight stream, 48 layers + lm_head, batch 1)"
# tensor-parallel stream defaults: one chain launch per token with the all-reduces inside it on the worlds whose
# in-chain all-reduce has passed its parity test on B200s (tests/test_gpu_tp.py at 2, 4 and 8 ranks); any other
# world defaults to per-GEMV launches with NCCL's all-reduce (--schedule chain selects the chain there too)
TP_CHAIN_CONFIRMED_WORLDS = (2, 4, 8)
TP_DEFAULT_ALLREDUCE = "nccl"
# prefill GEMMs: name -> (M, N, K, kind, the BASELINE.json config it is quoted on)
GEMM_WORKLOADS = {
    "gemm_i4": (2048, FFN, HIDDEN, "w4a16", "configs[2]: W4A16 prefill GEMM X[2048, 3840] x W[15360, 3840]"),
    "gemm_i4_down": (2048, HIDDEN, FFN, "w4a16", "configs[2]: W4A16 prefill GEMM, down_proj shape K=15360, N=3840"),
    "w8a8": (4096, HIDDEN, FFN, "w8a8", "configs[3]: W8A8 prefill GEMM X[4096, 15360] f16 -> cast_i8 -> int8 GEMM"),
    "w4a8": (4096, HIDDEN, FFN, "w4a8", "configs[3] shape, W4A8: int4 weights requantised in the kernel"),
}
GEMM_NAMES = {"w4a16": "W4A16", "w8a8": "W8A8", "w4a8": "W4A8"}
GEMM_KERNELS = {"w4a16": "gemm_w4a16_kernel", "w8a8": "gemm_s8_kernel<W8A8>", "w4a8": "gemm_s8_kernel<W4A8>"}
PREFILL_M = 8192
DECODE_BATCHES = (8, 64)


def stream_shapes(layers=LAYERS):
    out = []
    for li in range(layers):
        out += [(f"L{li}.{n}", N, K) for (n, N, K) in LAYER_SHAPES]
    out.append(LM_HEAD)
    return out


def weight_bytes(N, K, fp8):
    return N * K // 2 + (K // 32) * N * (1 if fp8 else 2)


def gemv_bytes(N, K, fp8):
    """Algorithmic bytes of one GEMV: packed weights + scales + f16 x + f16 y."""
    return weight_bytes(N, K, fp8) + 2 * K + 2 * N


def layer_flops(M):
    """2*M*N*K over one layer's seven GEMMs."""
    return 2 * M * sum(N * K for _, N, K in LAYER_SHAPES)


# ------------------------------------------------------ per-kernel CUDA events
class GraphEvents:
    """CUDA events recorded as event-record nodes inside a captured graph
    (cudaEventRecordWithFlags(..., cudaEventRecordExternal)), so each kernel's
    duration is measured on its own stream without the host in the loop."""

    def __init__(self, n):
        import ctypes
        self.C = ctypes
        self.rt = ctypes.CDLL("libcudart.so.12")
        self.ev = []
        for _ in range(2 * n):
            e = ctypes.c_void_p()
            assert self.rt.cudaEventCreateWithFlags(ctypes.byref(e), 0) == 0
            self.ev.append(e)

    def record(self, i, stream_handle):
        assert self.rt.cudaEventRecordWithFlags(self.ev[i], self.C.c_void_p(stream_handle), 1) == 0

    def elapsed_ms(self, i, j):
        ms = self.C.c_float()
        assert self.rt.cudaEventElapsedTime(self.C.byref(ms), self.ev[i], self.ev[j]) == 0
        return ms.value

    def close(self):
        for e in self.ev:
            self.rt.cudaEventDestroy(e)


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled during the timed
    region.  NVML is read from a background thread every ~2 ms, so that even a
    timed region of a few milliseconds gets samples; without NVML, nvidia-smi
    polls every 200 ms.  Reading clocks changes no GPU setting."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None
        self.thread = None
        self.rows = []
        self.stop_flag = False

    def start(self):
        import threading
        try:
            import pynvml
            pynvml.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = int(vis.split(",")[self.index]) if vis else self.index
            h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            masks = [(name, getattr(pynvml, attr)) for name, attr in self.REASONS]

            def run():
                while not self.stop_flag:
                    try:
                        sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                        r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.rows.append((sm, mx, [n for n, m in masks if r & m]))
                    except Exception:
                        pass
                    time.sleep(0.002)

            self.thread = threading.Thread(target=run, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.thread = None
        try:
            self.path = f"/tmp/g4b_clocks_{os.getpid()}.csv"
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.thread is not None:
            self.stop_flag = True
            self.thread.join(timeout=5)
            if not self.rows:
                return None
            sm = [r[0] for r in self.rows]
            reasons = sorted({n for r in self.rows for n in r[2]})
            return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(r[1] for r in self.rows),
                    "reasons": reasons, "samples": len(self.rows), "source": "nvml"}
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        try:
            for line in open(self.path):
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
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "source": "nvidia-smi"}


# ------------------------------------------------------------ what a line is
def stream_is_tp(args, world: int) -> bool:
    """The stream runs tensor parallel over several GPUs (or, with --parallel tp, on one)."""
    return args.workload == "stream" and args.parallel != "replicas" and (world > 1 or args.parallel == "tp")


def resolve_defaults(args, world: int) -> None:
    """Fill the schedule and all-reduce the user left unset: the chain on one
    GPU and for tensor parallelism over the confirmed worlds, per-GEMV launches
    with NCCL's all-reduce over the others."""
    tp_run = args.workload == "stream" and world > 1 and args.parallel != "replicas"
    if args.schedule is None:
        args.schedule = "chain" if not tp_run or world in TP_CHAIN_CONFIRMED_WORLDS else "launches"
    if args.allreduce is None:
        args.allreduce = TP_DEFAULT_ALLREDUCE


def describe(args, world: int) -> dict:
    """metric, unit, scaling and config of this run's line.  Both arms print
    these, so that the reference arm's line names the same workload."""
    wl = args.workload
    if wl in GEMM_WORKLOADS:
        M, N, K, kind, text = GEMM_WORKLOADS[wl]
        unit = "TFLOP/s" if kind == "w4a16" else "TOPS"
        return {"metric": f"{GEMM_NAMES[kind]} prefill GEMM {unit} (M={M}, N={N}, K={K})", "unit": unit,
                "scaling": "weak",
                "config": {"workload": text, "M": M, "N": N, "K": K, "parallelism": f"replicas{world}",
                           "l2": "256 MB buffer written between timed iterations (L2 flush, outside the events)"}}
    if wl == "engine":
        return {"metric": "decode tok/s at context 16 (engine harness)", "unit": "tok/s",
                "scaling": "weak",
                "config": {"workload": "benchmarks/bench_engine.py's measurements on the configs[1] stack",
                           "layers": args.layers, "parallelism": f"replicas{world}"}}
    if wl == "prefill":
        return {"metric": f"W4A16 prefill GEMM TFLOP/s (48-layer stack, M={PREFILL_M} split over GPUs)",
                "unit": "TFLOP/s", "scaling": "strong",
                "config": {"workload": f"configs[4] prefill: M={PREFILL_M} rows split over the GPUs, weights "
                                       "replicated", "layers": args.layers, "parallelism": f"m-split{world}",
                           "l2": "working set per GPU > 126 MB L2"}}
    if wl == "gemv":
        if args.shape == "lm_head":
            return {"metric": "int4 GEMV HBM GB/s (W[262144, 3840], batch 1)", "unit": "GB/s", "scaling": "weak",
                    "config": {"workload": "configs[1] lm_head GEMV W[262144, 3840], batch 1, f16 x/y",
                               "scales": args.scales, "parallelism": f"replicas{world}",
                               "l2": "566 MB of weights > 126 MB L2, no flush needed"}}
        return {"metric": "int4 GEMV HBM GB/s (W[15360, 3840], batch 1)", "unit": "GB/s", "scaling": "weak",
                "config": {"workload": "configs[0]: one int4 GEMV W[15360, 3840], batch 1, f16 x/y",
                           "scales": args.scales, "parallelism": f"replicas{world}",
                           "l2": "8 weight copies rotated per launch (266 MB > 126 MB L2)"}}
    if stream_is_tp(args, world):
        return {"metric": STREAM_METRIC, "unit": "GB/s", "scaling": "strong",
                "config": {"workload": "configs[4]: the configs[1] stream tensor-parallel over the GPUs",
                           "scales": args.scales, "layers": args.layers, "parallelism": f"tp{world}",
                           "activations": "f32 hidden state in, f32 logits out (the engine's buffers)",
                           "l2": "working set per GPU > 126 MB L2, no flush needed"}}
    return {"metric": STREAM_METRIC, "unit": "GB/s", "scaling": "weak",
            "config": {"workload": "configs[1]: decode weight stream, 48 layers + lm_head, batch 1",
                       "scales": args.scales, "layers": args.layers, "activations": "f16 N(0,1) per GEMV",
                       "weights": "N(0,0.02) -> int4, 32-blocks",
                       "l2": "working set 6.6 GB > 126 MB L2, no flush needed", "parallelism": f"replicas{world}"}}


def peaks():
    """(HBM GB/s, bf16 TFLOP/s, source) from MEASURED_PEAKS.json, else the pool's fallback figures."""
    try:
        pk = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))
        return float(pk["hbm_gbs"]), float(pk["bf16_tflops"]), "of measured"
    except Exception:
        return 6650.0, 1590.0, "of fallback"


# --------------------------------------------------- the reference's CPU path
def reference_sampler(args) -> dict:
    """The reference's path for this workload on the host cores: the oracle
    restatement of its shaders (oracle/g4b_oracle.c, OpenMP over every host
    thread) on a bounded sample with the workload's shapes.  Returns the
    sample's step function, its algorithmic work per step (bytes or ops), the
    unit and a description.  Both the ``--impl reference`` arm and the
    cpu_baseline key of the main arm use it, so there is one definition."""
    import oracle as O

    fp8 = args.scales == "fp8"
    wl = args.workload
    rng = np.random.default_rng(0)
    if wl in GEMM_WORKLOADS or wl == "prefill":
        rows = 32
        if wl == "prefill":
            shapes = [(N, K, "w4a16") for _, N, K in LAYER_SHAPES]
            unit = "TFLOP/s"
            what = f"{rows} token rows through one layer's seven W4A16 GEMMs (oracle of vk/coopgemm_i4h.comp)"
        else:
            M, N, K, kind, _ = GEMM_WORKLOADS[wl]
            shapes = [(N, K, kind)]
            unit = "TFLOP/s" if kind == "w4a16" else "TOPS"
            what = (f"{rows} token rows x the full [{N}, {K}] weight (oracle of "
                    f"{'vk/coopgemm_i4h.comp' if kind == 'w4a16' else 'vk/cast_i8.comp + vk/coopgemm_' + kind + '.comp'})")
        mats = []
        for N, K, kind in shapes:
            W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
            r = O.pack_reference(W, prefill_i8=kind != "w4a16")
            X = rng.standard_normal((rows, K)).astype(np.float16)
            ratio = O.w4a8_ratio(r["sc_f32"], r["sw_f32"]) if kind == "w4a8" else None
            mats.append((N, K, kind, r, X, ratio))
            del W

        def step():
            for N, K, kind, r, X, ratio in mats:
                if kind == "w4a16":
                    O.gemm_i4(X.view(np.uint16), r["wp"], r["scales16"].view(np.uint16), rows, N, K)
                else:
                    A8, sa = O.cast_i8(X.astype(np.float32))
                    if kind == "w8a8":
                        O.gemm_w8a8(A8, r["w8"], sa, r["sw8"].view(np.uint16))
                    else:
                        O.gemm_w4a8(A8, r["wp"], ratio, sa, r["sw8"].view(np.uint16), N)

        work = sum(2 * rows * N * K for N, K, *_ in mats)
        return {"step": step, "work": work, "unit": unit, "div": 1e12, "sample": what, "cores": O.num_threads()}
    # GEMV workloads: the reference's split (quant()'s heuristic) and reduce
    if wl == "engine":
        # decode tokens/s: one layer's seven GEMVs per step is 1/LAYERS of a token's matmuls
        st = reference_sampler(argparse.Namespace(**{**vars(args), "workload": "stream"}))
        return {"step": st["step"], "work": 1.0 / LAYERS, "unit": "tok/s", "div": 1.0, "cores": st["cores"],
                "sample": st["sample"] + f"; reported as tokens/s of a {LAYERS}-layer token's GEMVs"}
    if wl == "gemv":
        shapes = [("lm_head", VOCAB, HIDDEN)] if args.shape == "lm_head" else [("gate", FFN, HIDDEN)]
        what = f"one GEMV W[{shapes[0][1]}, {shapes[0][2]}] per step"
    else:
        shapes = LAYER_SHAPES
        what = "one layer's seven GEMVs per step (q, k, v, o, gate, up, down)"
    mats = []
    for i, (name, N, K) in enumerate(shapes):
        W = (np.random.default_rng(i).standard_normal((N, K)) * 0.02).astype(np.float32)
        r = O.pack_reference(W, fp8=fp8)
        x = np.random.default_rng(100 + i).standard_normal(K).astype(np.float16).astype(np.float32)
        mats.append((N, K, r["wp"], r["scales"], r["inv"], r["split"], x))
        del W

    def step():
        for N, K, wp, sc, inv, split, x in mats:
            O.gemv(x, wp, sc, 1 if fp8 else 0, inv, N, K, split)

    work = sum(gemv_bytes(N, K, fp8) for N, K, *_ in mats)
    return {"step": step, "work": work, "unit": "GB/s", "div": 1e9, "cores": O.num_threads(),
            "sample": f"{what}, {work / 1e6:.1f} MB, oracle restatement of vk/gemv.comp"
                      f"{' / vk/gemv_fp8.comp' if fp8 else ''} + vk/reduce.comp at the reference's split"}


def cpu_baseline(args, seconds: float) -> dict:
    """The reference sampler repeated for about `seconds` of CPU time."""
    s = reference_sampler(args)
    s["step"]()                                  # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        s["step"]()
        n += 1
        dt = time.perf_counter() - t0
        if dt >= seconds:
            break
    return {"value": round(s["work"] * n / dt / s["div"], 5 if s["div"] > 1e9 else 3), "unit": s["unit"],
            "cores": s["cores"], "kind": "port", "sample": f"{s['sample']}; {n} steps in {dt:.1f} s"}


def run_reference_arm(args) -> None:
    """``--impl reference``: the reference's own path for this workload timed on
    the host cores (rank 0 only; under torchrun the other ranks do no work)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    d = describe(args, world)
    s = reference_sampler(args)
    for _ in range(args.warmup):
        s["step"]()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        s["step"]()
    dt = time.perf_counter() - t0
    val = s["work"] * args.steps / dt / s["div"]
    prec = 5 if s["div"] > 1e9 else 3
    cpu = {"value": round(val, prec), "unit": s["unit"], "cores": s["cores"], "kind": "port",
           "sample": s["sample"]}
    print(json.dumps({"metric": d["metric"], "value": round(val, prec), "unit": d["unit"], "n_gpus": world,
                      "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
                      "higher_is_better": True, "scaling": d["scaling"], "vs_baseline": None,
                      "dtype": "int4 x f32 -> f32 acc" if s["unit"] == "GB/s" else "f32 (oracle)",
                      "data": "synthetic", "config": d["config"], "impl": "reference", "cpu_baseline": cpu,
                      "e2e": {"value": round(val, prec), "unit": s["unit"], "h2d_bytes_per_step": 0,
                              "d2h_bytes_per_step": 0},
                      "note": "the reference's GLSL shaders need a Vulkan stack (unavailable on this box); its "
                              "path is timed through the oracle port of those shaders, on rank 0's host cores"}),
          flush=True)


# ------------------------------------------------------------ GPU context
class Ctx:
    """One rank's device, stream and process group (NCCL when WORLD_SIZE > 1)."""

    def __init__(self):
        import torch
        import torch.distributed as dist
        from datetime import timedelta
        from g4b import _lib as L
        from g4b import comm, ops, tp
        from g4b import quant_gpu as qz

        self.torch, self.dist, self.L, self.ops, self.tp, self.comm, self.qz = torch, dist, L, ops, tp, comm, qz
        self.rank = int(os.environ.get("RANK", "0"))
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.device = torch.device("cuda", self.local)
        if self.world > 1:
            dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=self.device)
        L.load()
        self.stream = torch.cuda.Stream(self.device)
        self.sh = int(self.stream.cuda_stream)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def max(self, *vals):
        """Each value's max over the ranks."""
        if self.world == 1:
            return vals if len(vals) > 1 else vals[0]
        t = self.torch.tensor(list(vals), device=self.device, dtype=self.torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        out = tuple(float(v) for v in t.tolist())
        return out if len(out) > 1 else out[0]

    def gen(self, seed):
        g = self.torch.Generator(device=self.device)
        g.manual_seed(seed)
        return g

    def close(self):
        if self.world > 1:
            self.dist.barrier()
            self.dist.destroy_process_group()


def timed_graph(c, graph, steps):
    """Device ms of `steps` replays of `graph` between CUDA events on the
    launching stream, barrier + synchronize on both sides, max over ranks."""
    torch = c.torch
    c.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(c.stream):
        e0.record(c.stream)
        for _ in range(steps):
            graph.replay()
        e1.record(c.stream)
    c.barrier()
    return c.max(e0.elapsed_time(e1))


def capture(c, fn, warmup, eager=True):
    """Run fn eagerly `warmup` times (eager=False: not at all, e.g. when fn records
    graph-only event nodes), then capture it into a CUDA graph and replay that
    `warmup` times."""
    torch = c.torch
    if eager:
        with torch.cuda.stream(c.stream):
            for _ in range(max(1, warmup)):
                fn()
    c.stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=c.stream):
        fn()
    with torch.cuda.stream(c.stream):
        for _ in range(warmup):
            g.replay()
    c.stream.synchronize()
    return g


def traffic_for(key, algorithmic):
    """roofline.traffic from the committed ncu summaries (profiles/*.json): DRAM
    bytes read + written per launch, either as a measured ratio to the launch's
    algorithmic bytes ("ratios") or as the bytes of one full-size launch ("bytes")."""
    for name in ("gemv_traffic.json", "gemm_traffic.json"):
        p = os.path.join(REPO, "profiles", name)
        if not os.path.exists(p):
            continue
        try:
            t = json.load(open(p))
        except Exception:
            continue
        r = t.get("ratios", {}).get(key)
        if r is not None and algorithmic:
            return int(round(r * algorithmic)), t.get("note")
        b = t.get("bytes", {}).get(key)
        if b is not None:
            return int(b), t.get("note")
    return None, None


# ------------------------------------------------------------ decode stream
def build_stream_model(c, fp8, layers):
    """configs[1]'s 48 layers + lm_head: N(0, 0.02) weights quantised on the GPU into the engine's packed layout."""
    model = []
    gen = c.gen(0)
    for name, N, K in stream_shapes(layers):
        W = c.torch.randn((N, K), generator=gen, device=c.device, dtype=c.torch.float32).mul_(0.02)
        model.append((name, c.qz.quant_device(W, pf=False, fp8=fp8, prefill_i8=False)))
        del W
    c.torch.cuda.empty_cache()
    return model


def stream_groups(layers, unfused, n):
    """Launch groups: GEMVs that read the same x run as one fused launch (the engine's
    q/k/v on the normed hidden state, gate/up on the post-attention one)."""
    if unfused:
        return [[i] for i in range(n)]
    groups = []
    for li in range(layers):
        b = 7 * li
        groups += [[b, b + 1, b + 2], [b + 3], [b + 4, b + 5], [b + 6]]
    groups.append([7 * layers])
    return groups


def measure_stream(c, model, fp8, steps, warmup, schedule="chain", groups=None, e2e=True, seed=1):
    """configs[1] on one GPU: every launch group's x (f16 N(0, 1)) in one device
    arena and every output in another; the token's GEMVs as one chain launch
    (or one launch per group), captured as a CUDA graph and replayed."""
    torch, ops = c.torch, c.ops
    ws_list = [w for _, w in model]
    groups = groups or [[i] for i in range(len(ws_list))]
    kx = [ws_list[g[0]].K for g in groups]
    ny = [w.N for w in ws_list]
    step_bytes = sum(weight_bytes(w.N, w.K, fp8) + 2 * w.N for w in ws_list) + 2 * sum(kx)
    x_arena = torch.randn((sum(kx),), generator=c.gen(seed + c.rank), device=c.device).to(torch.float16)
    y_arena = torch.empty((sum(ny),), device=c.device, dtype=torch.float16)
    xs = list(torch.split(x_arena, kx))
    ys = list(torch.split(y_arena, ny))
    need = 0
    for g in groups:
        ns = [ws_list[i].N for i in g]
        need = max(need, ops.gemv_fused_workspace_bytes(ns, ws_list[g[0]].K) if len(g) > 1
                   else ops.gemv_workspace_bytes(1, ns[0], ws_list[g[0]].K, 0))
    ws = torch.zeros(need + 256, dtype=torch.uint8, device=c.device)
    chain = None
    if schedule == "chain":
        chain = ops.GemvChain([(x, [ws_list[i] for i in g], [ys[i] for i in g]) for g, x in zip(groups, xs)])

    def step(gev=None):
        if chain is not None:
            if gev is not None:
                gev.record(0, c.sh)
            chain.run(c.stream)
            if gev is not None:
                gev.record(1, c.sh)
            return
        for gi, (g, x) in enumerate(zip(groups, xs)):
            if gev is not None:
                gev.record(2 * gi, c.sh)
            if len(g) == 1:
                ops.gemv_i4(x, ws_list[g[0]], out=ys[g[0]], stream=c.stream, workspace=ws, pdl=True)
            else:
                ops.gemv_i4_fused(x, [ws_list[i] for i in g], outs=[ys[i] for i in g], stream=c.stream,
                                  workspace=ws, pdl=True)
            if gev is not None:
                gev.record(2 * gi + 1, c.sh)

    ev_groups = [list(range(len(ws_list)))] if chain is not None else groups
    graph = capture(c, step, warmup)
    gev = GraphEvents(len(ev_groups))
    graph_ev = capture(c, lambda: step(gev), warmup, eager=False)
    clocks = ClockSampler(c.local)
    clocks.start()
    ms = timed_graph(c, graph, steps)
    ms_step = ms / steps
    value = c.world * step_bytes / (ms_step / 1e3) / 1e9
    # roofline: the same step with an event-record node around every launch
    kern_ms, kern_bytes = 0.0, 0
    with torch.cuda.stream(c.stream):
        for _ in range(steps):
            graph_ev.replay()
            c.stream.synchronize()
            for gi, g in enumerate(ev_groups):
                kern_ms += gev.elapsed_ms(2 * gi, 2 * gi + 1)
                if chain is not None:
                    kern_bytes += step_bytes
                else:
                    K = ws_list[g[0]].K
                    kern_bytes += sum(weight_bytes(ws_list[i].N, K, fp8) + 2 * ws_list[i].N for i in g) + 2 * K
    clk = clocks.stop()
    gev.close()
    hbm, _, src = peaks()
    kern_gbs = kern_bytes / (kern_ms / 1e3) / 1e9
    kname = "gemv_i4_chain_kernel" if chain is not None else "gemv_i4_m1_kernel"
    traffic, note = traffic_for("chain" if chain is not None else "stream_launch",
                                step_bytes if chain is not None else kern_bytes // (steps * len(ev_groups)))
    roofline = {"bound": "hbm", "achieved": round(kern_gbs, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(kern_gbs / hbm, 4), "traffic": traffic, "peak_source": src, "kernel": kname,
                "launches_timed": steps * len(ev_groups),
                "avg_launch_us": round(kern_ms * 1e3 / (steps * len(ev_groups)), 3),
                "graph_vs_kernels": round(ms_step / (kern_ms / steps), 4)}
    if note:
        roofline["traffic_note"] = note
    out = {"value": round(value, 1), "ms_per_step": round(ms_step, 4), "roofline": roofline, "clocks": clk,
           "bytes_per_step": step_bytes, "gpu_launches": len(ev_groups) * steps,
           "schedule": (f"one persistent launch per token (g4b_gemv_chain) of {len(groups)} GEMV steps; each step "
                        "reads its x once every tile of the step before it is written" if chain is not None else
                        f"{len(groups)} launches per token, chained by programmatic dependent launch")}
    if e2e:
        # the public API with host buffers: one pinned arena in, one out, every step
        x_h = x_arena.cpu().pin_memory()
        y_h = torch.empty(y_arena.shape, dtype=y_arena.dtype).pin_memory()

        def e2e_step():
            x_arena.copy_(x_h, non_blocking=True)
            step()
            y_h.copy_(y_arena, non_blocking=True)

        with torch.cuda.stream(c.stream):
            for _ in range(2):
                e2e_step()
            c.stream.synchronize()
            c.barrier()
            t0 = time.perf_counter()
            for _ in range(steps):
                e2e_step()
                c.stream.synchronize()          # the caller reads its result every step
            e2e_s = time.perf_counter() - t0
        e2e_s = c.max(e2e_s)
        out["e2e"] = {"value": round(c.world * step_bytes * steps / e2e_s / 1e9, 1), "unit": "GB/s",
                      "h2d_bytes_per_step": x_arena.numel() * 2, "d2h_bytes_per_step": y_arena.numel() * 2}
    del graph, graph_ev
    if chain is not None:
        torch.cuda.synchronize()
        chain.close()
    return out


def measure_gemv(c, fp8, steps, warmup, shape="config0"):
    """one [15360, 3840] GEMV per launch over 8 rotated weight copies
    (266 MB > L2), or the lm_head GEMV [262144, 3840] alone."""
    torch, ops = c.torch, c.ops
    gen = c.gen(0)
    if shape == "lm_head":
        shapes = [(VOCAB, HIDDEN)]
    else:
        shapes = [(FFN, HIDDEN)] * 8
    ws_list = []
    for N, K in shapes:
        W = torch.randn((N, K), generator=gen, device=c.device).mul_(0.02)
        ws_list.append(c.qz.quant_device(W, pf=False, fp8=fp8, prefill_i8=False))
        del W
    torch.cuda.empty_cache()
    x = torch.randn((HIDDEN,), generator=gen, device=c.device).to(torch.float16)
    ys = [torch.empty((w.N,), device=c.device, dtype=torch.float16) for w in ws_list]
    ws = torch.zeros(max(ops.gemv_workspace_bytes(1, w.N, w.K, 0) for w in ws_list) + 256, dtype=torch.uint8,
                     device=c.device)
    per = gemv_bytes(ws_list[0].N, ws_list[0].K, fp8)

    def step(gev=None):
        for i, (w, y) in enumerate(zip(ws_list, ys)):
            if gev is not None:
                gev.record(2 * i, c.sh)
            ops.gemv_i4(x, w, out=y, stream=c.stream, workspace=ws, pdl=gev is None)
            if gev is not None:
                gev.record(2 * i + 1, c.sh)

    graph = capture(c, step, warmup)
    gev = GraphEvents(len(ws_list))
    graph_ev = capture(c, lambda: step(gev), warmup, eager=False)
    ms = timed_graph(c, graph, steps)
    kern_ms = 0.0
    with torch.cuda.stream(c.stream):
        for _ in range(steps):
            graph_ev.replay()
            c.stream.synchronize()
            kern_ms += sum(gev.elapsed_ms(2 * i, 2 * i + 1) for i in range(len(ws_list)))
    gev.close()
    hbm, _, src = peaks()
    n = steps * len(ws_list)
    value = per * n / (ms / 1e3) / 1e9
    achieved = per * n / (kern_ms / 1e3) / 1e9
    traffic, _ = traffic_for("lm_head" if shape == "lm_head" else "gemv", per)
    del graph, graph_ev
    return {"value": round(value, 1), "unit": "GB/s", "ms_per_launch": round(ms / n, 5),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "traffic": traffic, "peak_source": src,
                         "kernel": "gemv_i4_m1_kernel", "avg_launch_us": round(kern_ms * 1e3 / n, 3)}}


# ------------------------------------------------------------ prefill GEMMs
def measure_gemm(c, key, steps, warmup, e2e=False):
    """One prefill GEMM per step; a 256 MB buffer is
    written between timed iterations (L2 flush, outside the events)."""
    torch, ops, L = c.torch, c.ops, c.L
    M, N, K, kind, _ = GEMM_WORKLOADS[key]
    gen = c.gen(0)
    W = torch.randn((N, K), generator=gen, device=c.device).mul_(0.02)
    w = c.qz.quant_device(W, pf=True, fp8=False, prefill_i8=kind != "w4a16", w4a8=kind == "w4a8")
    del W
    X = torch.randn((M, K), generator=gen, device=c.device).to(torch.float16)
    Y = torch.empty((M, N), dtype=torch.float16, device=c.device)
    A8 = torch.empty((M, K), dtype=torch.int8, device=c.device)
    sa = torch.empty((M,), dtype=torch.float32, device=c.device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=c.device)
    lib = L.load()
    flops = 2 * M * N * K

    def step(ev=None):
        if kind != "w4a16":
            L.check("g4b_cast_i8", lib.g4b_cast_i8(X.data_ptr(), L.DT_F16, A8.data_ptr(), sa.data_ptr(), M, K, c.sh))
        if ev is not None:
            ev.record(c.stream)
        if kind == "w4a16":
            ops.gemm_i4(X, w, out=Y, stream=c.stream)
        elif kind == "w8a8":
            ops.gemm_w8a8(A8, sa, w, out=Y, stream=c.stream)
        else:
            ops.gemm_w4a8(A8, sa, w, out=Y, stream=c.stream)

    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    with torch.cuda.stream(c.stream):
        for _ in range(max(3, warmup)):
            step()
    c.barrier()
    with torch.cuda.stream(c.stream):
        for i in range(steps):
            flush.zero_()
            ev[i][0].record(c.stream)
            step(ev[i][1])
            ev[i][2].record(c.stream)
    c.barrier()
    step_ms = sum(e[0].elapsed_time(e[2]) for e in ev)
    kern_ms = sum(e[1].elapsed_time(e[2]) for e in ev)
    step_ms, kern_ms = c.max(step_ms, kern_ms)
    _, bf16, src = peaks()
    peak = bf16 if kind == "w4a16" else 2 * bf16
    if kind != "w4a16":
        src += " bf16 x 2 (the dense int8 rate is twice the f16 rate)"
    achieved = flops * steps / (kern_ms / 1e3) / 1e12
    unit = "TFLOP/s" if kind == "w4a16" else "TOPS"
    traffic, _ = traffic_for(key, None)
    out = {"value": round(c.world * flops * steps / (step_ms / 1e3) / 1e12, 1), "unit": unit,
           "ms_per_step": round(step_ms / steps, 4),
           "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": unit,
                        "frac": round(achieved / peak, 4), "traffic": traffic, "peak_source": src,
                        "kernel": GEMM_KERNELS[kind], "launches_timed": steps,
                        "avg_launch_us": round(kern_ms * 1e3 / steps, 2)},
           "gpu_launches": steps * (1 if kind == "w4a16" else 2)}
    if e2e:
        Xh = X.cpu().pin_memory()
        Yh = torch.empty((M, N), dtype=torch.float16).pin_memory()
        with torch.cuda.stream(c.stream):
            for _ in range(2):
                X.copy_(Xh, non_blocking=True)
                step()
                Yh.copy_(Y, non_blocking=True)
            c.stream.synchronize()
            t0 = time.perf_counter()
            for _ in range(steps):
                X.copy_(Xh, non_blocking=True)
                step()
                Yh.copy_(Y, non_blocking=True)
                c.stream.synchronize()
            e2e_s = time.perf_counter() - t0
        e2e_s = c.max(e2e_s)
        out["e2e"] = {"value": round(c.world * flops * steps / e2e_s / 1e12, 1), "unit": unit,
                      "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 2}
    del flush
    torch.cuda.empty_cache()
    return out


def measure_prefill(c, layer_weights, steps, warmup, e2e=False):
    """configs[4] prefill: M = 8192 f16 N(0, 1) tokens through the 48 layers'
    seven W4A16 GEMMs, the rows split over the ranks with the weights
    replicated (no collective).  value = the total 2*M*N*K / the step's device
    time, max over ranks."""
    torch, ops = c.torch, c.ops
    m0, m1 = c.tp.prefill_rows(PREFILL_M, c.world, c.rank)
    Mr = m1 - m0
    gen = c.gen(7)
    X = {K: torch.randn((PREFILL_M, K), generator=gen, device=c.device).to(torch.float16)[m0:m1].contiguous()
         for K in (HIDDEN, NQ, FFN)}
    Y = {N: torch.empty((Mr, N), dtype=torch.float16, device=c.device) for N in (NQ, NKV, HIDDEN, FFN)}
    flops = layer_flops(PREFILL_M) * len(layer_weights)

    def step():
        for d in layer_weights:
            for w in d:
                ops.gemm_i4(X[w.K], w, out=Y[w.N], stream=c.stream)

    with torch.cuda.stream(c.stream):
        for _ in range(max(1, warmup)):
            step()
    c.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(c.stream):
        e0.record(c.stream)
        for _ in range(steps):
            step()
        e1.record(c.stream)
    c.barrier()
    ms = c.max(e0.elapsed_time(e1)) / steps
    value = flops / (ms / 1e3) / 1e12
    _, bf16, src = peaks()
    out = {"value": round(value, 1), "unit": "TFLOP/s", "ms_per_step": round(ms, 3), "rows_per_gpu": Mr,
           "roofline": {"bound": "tensor", "achieved": round(value / c.world, 1), "peak": bf16, "unit": "TFLOP/s",
                        "frac": round(value / c.world / bf16, 4), "traffic": None, "peak_source": src,
                        "kernel": "gemm_w4a16_kernel (per GPU)"},
           "gpu_launches": 7 * len(layer_weights) * steps}
    if e2e:
        Xh = {K: x.cpu().pin_memory() for K, x in X.items()}
        Yh = torch.empty(Y[HIDDEN].shape, dtype=torch.float16).pin_memory()
        c.barrier()
        with torch.cuda.stream(c.stream):
            t0 = time.perf_counter()
            for _ in range(steps):
                for K, x in X.items():
                    x.copy_(Xh[K], non_blocking=True)
                step()
                Yh.copy_(Y[HIDDEN], non_blocking=True)
                c.stream.synchronize()
            e2e_s = time.perf_counter() - t0
        e2e_s = c.max(e2e_s)
        out["e2e"] = {"value": round(flops * steps / e2e_s / 1e12, 1), "unit": "TFLOP/s",
                      "h2d_bytes_per_step": c.world * sum(x.numel() * 2 for x in X.values()),
                      "d2h_bytes_per_step": c.world * Yh.numel() * 2}
    del X, Y
    torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------ tensor parallel
def build_tp_model(c, fp8, layers):
    """This rank's shards of configs[1]'s stack (world 1: the whole weights):
    q/k/v/gate/up/lm_head by output columns, o/down by input rows.  Every rank
    draws the same full W (seeded) and quantises its own slice."""
    torch, tp = c.torch, c.tp
    kinds = dict(tp.LAYER_KINDS)
    gen = c.gen(0)
    acc = {"full": 0, "mine": 0}

    def shard(N, K, kind):
        W = torch.randn((N, K), generator=gen, device=c.device).mul_(0.02)
        if kind == "col":
            n0, n1 = tp.split_range(N, c.world, c.rank, tp.COL_ALIGN)
            Ws = W[n0:n1].contiguous()
        else:
            k0, k1 = tp.split_range(K, c.world, c.rank, tp.ROW_ALIGN)
            Ws = W[:, k0:k1].contiguous()
        del W
        acc["full"] += weight_bytes(N, K, fp8)
        w = c.qz.quant_device(Ws, pf=False, fp8=fp8, prefill_i8=False)
        acc["mine"] += weight_bytes(w.N, w.K, fp8)
        return w

    tl = [tp.TPLayer(**{n: shard(N, K, kinds[n]) for (n, N, K) in LAYER_SHAPES}) for _ in range(layers)]
    lm = shard(VOCAB, HIDDEN, "col")
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return tl, lm, acc["full"], acc["mine"]


def measure_decode_batch(c, layers, lm, M, steps, warmup, full_bytes):
    """configs[4]'s batched decode: M tokens through the tensor-parallel stack,
    W4A16 tensor-core GEMMs (64-token tiles, K split over the SMs where the
    column tiles cannot fill them; q|k|v and gate|up one launch each,
    g4b_gemm_i4_fused; each launch a programmatic dependent of the kernel
    before it), an NCCL all-reduce after
    o and after down and a logits all-gather, captured as one CUDA graph.  Each
    layer's q/k/v read the same f16 N(0, 1) input block, so the unnormalised
    activations stay in f16 range.  value = the whole model's weight bytes /
    the step's device time."""
    torch, ops = c.torch, c.ops
    f16 = torch.float16
    L0 = layers[0]
    H = L0.q.K
    xin = torch.randn((M, H), generator=c.gen(11), device=c.device).to(f16)
    b = {k: torch.empty((M, getattr(L0, k).N), device=c.device, dtype=f16) for k in ("q", "k", "v", "gate", "up")}
    b["h"] = torch.empty((M, H), device=c.device, dtype=f16)
    b["h2"] = torch.empty((M, H), device=c.device, dtype=f16)
    b["logits_local"] = torch.empty((M, lm.N), device=c.device, dtype=f16)
    b["logits"] = torch.empty((c.world * M, lm.N), device=c.device, dtype=f16)
    need = max(ops.gemm_i4_workspace_bytes(M, w.N, w.K) for Ly in layers for w in vars(Ly).values())
    need = max(need, ops.gemm_i4_workspace_bytes(M, lm.N, lm.K))
    need = max([need] + [ops.gemm_i4_workspace_bytes(M, Ly.q.N + Ly.k.N + Ly.v.N, Ly.q.K) for Ly in layers] +
               [ops.gemm_i4_workspace_bytes(M, Ly.gate.N + Ly.up.N, Ly.gate.K) for Ly in layers])
    ws = torch.zeros(need + 256, dtype=torch.uint8, device=c.device)
    launches = [0]

    def mm(x, w, out):
        # each GEMM a programmatic dependent of the kernel before it (G4B_GEMM_PDL)
        ops.gemm_i4(x, w, out=out, stream=c.stream, workspace=ws, pdl=True)
        launches[0] += 1 + (1 if ops.gemm_i4_workspace_bytes(M, w.N, w.K) else 0)

    def ar(t):
        if c.world > 1:
            c.dist.all_reduce(t)

    def mm3(x, wl, outs):
        # weights that share x (q|k|v, gate|up) as one launch (g4b_gemm_i4_fused)
        ops.gemm_i4_fused(x, wl, outs=outs, stream=c.stream, workspace=ws, pdl=True)
        launches[0] += 1 + (1 if ops.gemm_i4_workspace_bytes(M, sum(w.N for w in wl), wl[0].K) else 0)

    def token():
        for Ly in layers:
            mm3(xin, [Ly.q, Ly.k, Ly.v], [b["q"], b["k"], b["v"]])
            mm(b["q"], Ly.o, b["h"])
            ar(b["h"])
            mm3(b["h"], [Ly.gate, Ly.up], [b["gate"], b["up"]])
            mm(b["gate"], Ly.down, b["h2"])
            ar(b["h2"])
        mm(b["h2"], lm, b["logits_local"])
        if c.world > 1:
            c.dist.all_gather_into_tensor(b["logits"], b["logits_local"])

    graph = capture(c, token, warmup)
    launches[0] = 0
    with torch.cuda.stream(c.stream):
        token()                                   # one eager token: count this repository's launches
    per_step = launches[0]
    ms = timed_graph(c, graph, steps) / steps
    del graph
    hbm, _, src = peaks()
    value = full_bytes / (ms / 1e3) / 1e9
    return {"value": round(value, 1), "unit": "GB/s", "tokens_per_s": round(M / (ms / 1e3), 1),
            "ms_per_step": round(ms, 4), "tokens": M,
            "kernel": "gemm_w4a16_kernel (64-token tiles, split-K where the columns cannot fill the SMs)",
            "roofline": {"bound": "hbm", "achieved": round(value / c.world, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(value / c.world / hbm, 4), "traffic": None, "peak_source": src,
                         "note": "per GPU, collectives included"},
            "gpu_launches": per_step * steps}


def measure_tp_stream(c, layers, lm, full_bytes, my_bytes, steps, warmup, schedule, allreduce):
    """configs[4] at M = 1: the hidden state in, the layers with their
    all-reduces, the logits out.  One CUDA graph per rank; with the chain
    schedule a token is one persistent launch per rank with the all-reduces
    inside it (over NVLink peer stores), then NCCL's logits all-gather."""
    torch, ops, tp, L = c.torch, c.ops, c.tp, c.L
    launches = [0]
    ws = torch.zeros(max(ops.gemv_workspace_bytes(1, w.N, w.K, 0) for Lr in layers for w in vars(Lr).values())
                     + ops.gemv_workspace_bytes(1, lm.N, lm.K, 0) + 256, dtype=torch.uint8, device=c.device)
    L0 = layers[0]
    ws_fused = max(ops.gemv_fused_workspace_bytes([L0.q.N, L0.k.N, L0.v.N], L0.q.K),
                   ops.gemv_fused_workspace_bytes([L0.gate.N, L0.up.N], L0.gate.K))
    if ws.numel() < ws_fused + 256:
        ws = torch.zeros(ws_fused + 256, dtype=torch.uint8, device=c.device)

    def gemv(x, w, out):
        ops.gemv_i4(x, w, out=out, stream=c.stream, workspace=ws, pdl=True)
        launches[0] += 1

    def gemv_fused(x, ws_, outs):
        ops.gemv_i4_fused(x, ws_, outs=outs, stream=c.stream, workspace=ws, pdl=True)
        launches[0] += 1

    peer = c.comm.PeerAllReduce(HIDDEN, c.device) if allreduce == "peer" and c.world > 1 else None

    def all_reduce(t):
        if c.world == 1:
            return
        if peer is not None:
            peer(t, stream=c.stream, pdl=True)
            launches[0] += 1
        else:
            c.dist.all_reduce(t)

    def all_gather(out, t):
        if c.world == 1:
            out.copy_(t)
        else:
            c.dist.all_gather_into_tensor(out, t)

    new_buffer = lambda n: torch.zeros(n, dtype=torch.float32, device=c.device)  # noqa: E731
    dec = tp.TPDecoder(layers=layers, lm_head=lm, gemv=gemv, all_reduce=all_reduce, all_gather=all_gather,
                       new_buffer=new_buffer, hidden=HIDDEN, vocab=VOCAB, world=c.world, gemv_fused=gemv_fused)
    x = torch.randn((HIDDEN,), generator=c.gen(5), device=c.device)
    chain = chain_k = xchg = None
    if schedule == "chain":
        dec.bufs["part"] = torch.zeros(HIDDEN, dtype=torch.float32, device=c.device)
        if c.world > 1:
            steps_ = tp.chain_steps(layers, lm, x, dec.bufs, L.CHAIN_ALLREDUCE)
            xchg = c.comm.PeerBuffers(ops.GemvChain.exchange_bytes(steps_, c.world), c.device)
            chain = ops.GemvChain(steps_, exchange=xchg)
        else:
            chain = ops.GemvChain(tp.chain_steps(layers, lm, x, dec.bufs, 0))

        def token():
            chain.run(c.stream)
            launches[0] += 1
            if c.world > 1:
                c.dist.all_gather_into_tensor(dec.bufs["logits"], dec.bufs["logits_local"])
    else:
        def token():
            dec.step(x)
    graph = capture(c, token, warmup)
    launches[0] = 0
    with torch.cuda.stream(c.stream):
        token()                                   # one eager token: count this repository's launches
    per_step = launches[0]
    clocks = ClockSampler(c.local)
    clocks.start()
    ms_step = timed_graph(c, graph, steps) / steps
    clk = clocks.stop()
    value = full_bytes / (ms_step / 1e3) / 1e9

    # kernels only: the same GEMVs without the collectives, each all-reduced step's local partial as the next x
    dec_k = tp.TPDecoder(layers=layers, lm_head=lm, gemv=gemv, all_reduce=lambda t: None,
                         all_gather=lambda out, t: None, new_buffer=new_buffer, hidden=HIDDEN, vocab=VOCAB,
                         world=c.world, gemv_fused=gemv_fused)
    if chain is not None:
        dec_k.bufs["part"] = torch.zeros(HIDDEN, dtype=torch.float32, device=c.device)
        chain_k = ops.GemvChain(tp.chain_steps(layers, lm, x, dec_k.bufs, 0))
        kstep = lambda: chain_k.run(c.stream)  # noqa: E731
    else:
        kstep = lambda: dec_k.step(x)  # noqa: E731
    graph_k = capture(c, kstep, warmup)
    ms_kern = timed_graph(c, graph_k, steps) / steps
    my_max = c.max(float(my_bytes))
    hbm, _, src = peaks()
    per_gpu = my_max / (ms_kern / 1e3) / 1e9
    roofline = {"bound": "hbm", "achieved": round(per_gpu, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(per_gpu / hbm, 4), "traffic": None, "peak_source": src,
                "kernel": ("gemv_i4_chain_kernel" if chain is not None else "gemv_i4_m1_kernel") +
                          " (per GPU, collectives removed)",
                "kernels_only_aggregate_gbs": round(full_bytes / (ms_kern / 1e3) / 1e9, 1)}
    t, _ = traffic_for("chain" if chain is not None else "stream_launch", my_max)
    roofline["traffic"] = t

    # e2e: the hidden state in from pinned host memory, the gathered logits back, every step
    logits = dec.bufs["logits"] if c.world > 1 or chain is None else dec.bufs["logits_local"]
    xh = x.cpu().pin_memory()
    lh = torch.empty(logits.shape, dtype=torch.float32).pin_memory()
    c.barrier()
    with torch.cuda.stream(c.stream):
        t0 = time.perf_counter()
        for _ in range(steps):
            x.copy_(xh, non_blocking=True)
            token()
            lh.copy_(logits, non_blocking=True)
            c.stream.synchronize()
        e2e_s = time.perf_counter() - t0
    e2e_s = c.max(e2e_s)
    del graph, graph_k
    c.barrier()
    if peer is not None:
        peer.close()
    if chain is not None:
        chain.close()
        chain_k.close()
    if xchg is not None:
        xchg.close()
    return {"value": round(value, 1), "ms_per_step": round(ms_step, 4), "roofline": roofline, "clocks": clk,
            "e2e": {"value": round(full_bytes * steps / e2e_s / 1e9, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": HIDDEN * 4, "d2h_bytes_per_step": VOCAB * 4},
            "gpu_launches": per_step * steps, "bytes_per_step": full_bytes, "bytes_per_gpu_max": int(my_max),
            "ms_per_step_kernels_only": round(ms_kern, 4),
            "schedule": ("one persistent GEMV-chain launch per token and rank, all-reduces inside it "
                         "(g4b_gemv_chain_create_tp)" if chain is not None and c.world > 1 else
                         "one persistent GEMV-chain launch per token" if chain is not None else
                         "one launch per (fused) GEMV"),
            "allreduce": ("none (one GPU)" if c.world == 1 else
                          "in-chain, NVLink peer stores of {value, epoch} words" if chain is not None else
                          "g4b_allreduce_f32 over NVLink peer memory" if peer is not None else "NCCL")}


def tp_extras(c, layers, lm, full_bytes, args):
    """configs[4]'s other workloads on this world: batched decode and the prefill split."""
    ex = {}
    for M in DECODE_BATCHES:
        ex[f"configs[4] decode M={M}"] = measure_decode_batch(c, layers, lm, M, args.steps, args.warmup, full_bytes)
    return ex


def prefill_extra(c, args, layer_weights=None):
    """configs[4] prefill over the full (replicated) 48-layer stack."""
    torch = c.torch
    built = layer_weights is None
    if built:
        gen = c.gen(0)
        layer_weights = []
        for _ in range(args.layers):
            d = []
            for name, N, K in LAYER_SHAPES:
                W = torch.randn((N, K), generator=gen, device=c.device).mul_(0.02)
                d.append(c.qz.quant_device(W, pf=False, fp8=False, prefill_i8=False))
                del W
            layer_weights.append(d)
    out = measure_prefill(c, layer_weights, max(3, min(args.steps, 10)), 1)
    if built:
        del layer_weights
        torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------ runners
def header(args, c, d, value, ms_step, dtype, data):
    return {"metric": d["metric"], "value": value, "unit": d["unit"], "n_gpus": c.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": d["scaling"],
            "vs_baseline": None, "dtype": dtype, "data": data, "config": d["config"]}


def run_stream(args) -> None:
    """configs[1] on one GPU (or independent replicas, one per rank), plus the extras."""
    c = Ctx()
    d = describe(args, c.world)
    fp8 = args.scales == "fp8"
    model = build_stream_model(c, fp8, args.layers)
    groups = stream_groups(args.layers, args.unfused, len(model))
    m = measure_stream(c, model, fp8, args.steps, args.warmup, args.schedule, groups, e2e=True)
    cpu = None
    if c.rank == 0 and c.world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args, args.cpu_seconds)
    extras = {}
    if not args.no_extras and c.world == 1 and args.layers == LAYERS and not fp8:
        extras = one_gpu_extras(c, args, model)
    del model
    if c.rank == 0:
        out = header(args, c, d, m["value"], m["ms_per_step"], "int4 x f16 -> f32 acc",
                     "synthetic (seeded N(0,0.02) weights, N(0,1) activations)")
        out.update({"roofline": m["roofline"], "cpu_baseline": cpu, "e2e": m["e2e"],
                    "gpu_launches": m["gpu_launches"], "clocks": m["clocks"], "bytes_per_step": m["bytes_per_step"],
                    "schedule": m["schedule"]})
        if extras:
            out["extras"] = extras
        print(json.dumps(out), flush=True)
    c.close()


def measure_fused_token(c, layers, lm, steps, warmup, dtype_name="f16"):
    """configs[1]'s weights as a decode token with the engine's element-wise work
    fused in (g4b.decode.FusedDecodeToken: rmsnorm, normadd and gelu*up inside
    the one chain launch, o reading q in place of attention), hidden state in,
    logits out.  value = the token's weight + scale bytes / device time."""
    torch = c.torch
    from g4b import decode

    dt = torch.float16 if dtype_name == "f16" else torch.float32
    gen = c.gen(21)
    H = layers[0].q.K
    nw = lambda: (1.0 + 0.1 * torch.randn((H,), generator=gen, device=c.device))  # noqa: E731
    norms = [decode.LayerNorms(inw=nw(), paw=nw(), pfw=nw(), ofw=nw(), scl=1.0) for _ in layers]
    tok = decode.FusedDecodeToken(layers, norms, lm, nw(), dtype=dt)
    tok.h0.copy_(torch.randn((H,), generator=gen, device=c.device))
    token_bytes = sum(weight_bytes(w.N, w.K, False) for Ly in layers for w in vars(Ly).values()) + \
        weight_bytes(lm.N, lm.K, False)
    graph = capture(c, lambda: tok.run(c.stream), warmup)
    ms = timed_graph(c, graph, steps) / steps
    hbm, _, src = peaks()
    value = token_bytes / (ms / 1e3) / 1e9
    # e2e: the hidden state in from pinned host memory, the logits back, every token
    h_h = tok.h0.cpu().pin_memory()
    l_h = torch.empty(tok.logits.shape, dtype=tok.logits.dtype).pin_memory()
    with torch.cuda.stream(c.stream):
        t0 = time.perf_counter()
        for _ in range(steps):
            tok.h0.copy_(h_h, non_blocking=True)
            tok.run(c.stream)
            l_h.copy_(tok.logits, non_blocking=True)
            c.stream.synchronize()
        e2e_s = time.perf_counter() - t0
    finite = bool(torch.isfinite(tok.logits).all().item())
    del graph
    tok.close()
    return {"value": round(value, 1), "unit": "GB/s", "ms_per_step": round(ms, 4), "steps_per_token": tok.nsteps,
            "activations": dtype_name, "logits_finite": finite,
            "roofline": {"bound": "hbm", "achieved": round(value, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(value / hbm, 4), "traffic": None, "peak_source": src,
                         "kernel": "gemv_i4_chain_kernel (fused rmsnorm / normadd / gelu*up)"},
            "e2e": {"value": round(token_bytes * steps / e2e_s / 1e9, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": H * 4, "d2h_bytes_per_step": tok.logits.numel() * tok.logits.element_size()},
            "gpu_launches": steps}


ENGINE_CTX = (16, 1024, 4096)
PROMPT_LEN = 2048
NH, NKV_HEADS, HEAD_DIM = 16, 8, 256


def measure_engine(c, args):
    """benchmarks/bench_engine.py:14-41 on this stack: decode tok/s at a context
    of 16, 1024 and 4096 tokens, and prefill prompt-tok/s on a 2048-token prompt.

    Decode is all g4b: per layer one fused chain launch (the GEMVs with the
    norms and gelu*up, g4b.decode.SegmentedDecodeToken) and the KV-cache write
    and flash-decode attention in one launch (g4b_attn_decode_prepkv) over a
    synthetic f16 cache (GQA, 16 query and 8 KV heads of 256), timed as K
    graph replays at a fixed context (the reference grows it by 64 tokens).
    Prefill is all g4b too, over the 2048-token prompt in one batch: the row
    norms and gelu*up (g4b_rows_*, g4b_gelumul), the W4A16 GEMMs (or, as
    PREFILL_I8 does, cast_i8 + the W8A8 GEMMs), and the batched KV-cache write
    and causal attention (g4b_attn_prefill_prepkv, g4b_attn_prefill); a third
    key swaps torch's SDPA in for the attention, for comparison.  The logits
    are for the last token."""
    torch = c.torch
    F = torch.nn.functional
    from g4b import decode

    gen = c.gen(31)
    H = HIDDEN
    layers_w, layers_d = [], []
    for _ in range(args.layers):
        dd = {}
        for name, N, K in LAYER_SHAPES:
            W = torch.randn((N, K), generator=gen, device=c.device).mul_(0.02)
            dd[name] = c.qz.quant_device(W, pf=True, fp8=False, prefill_i8=True)
            del W
        layers_w.append(dd)
        layers_d.append(c.tp.TPLayer(**dd))
    W = torch.randn((VOCAB, H), generator=gen, device=c.device).mul_(0.02)
    lm = c.qz.quant_device(W, pf=False, fp8=False, prefill_i8=False)
    del W
    torch.cuda.empty_cache()
    nw = lambda: (1.0 + 0.1 * torch.randn((H,), generator=gen, device=c.device))  # noqa: E731
    norms = [decode.LayerNorms(inw=nw(), paw=nw(), pfw=nw(), ofw=nw(), scl=1.0) for _ in range(args.layers)]
    finw = nw()
    out = {"attention": "decode: g4b_attn_decode_prepkv; prefill: g4b_attn_prefill_prepkv + g4b_attn_prefill "
                        "(GQA 16/8 heads of 256, f16 KV cache)",
           "steps": args.steps}
    # ---- decode
    tok = decode.SegmentedDecodeToken(layers_d, norms, lm, finw, dtype=torch.float16)
    tok.h0.copy_(torch.randn((H,), generator=gen, device=c.device))
    hn = lambda: (1.0 + 0.1 * torch.randn((HEAD_DIM,), generator=gen, device=c.device))  # noqa: E731
    qnw, knw = [hn() for _ in range(args.layers)], [hn() for _ in range(args.layers)]
    for ctx in ENGINE_CTX:
        kc = torch.randn((args.layers, NKV_HEADS, ctx, HEAD_DIM), generator=gen, device=c.device).half()
        vc = torch.randn((args.layers, NKV_HEADS, ctx, HEAD_DIM), generator=gen, device=c.device).half()
        pos = torch.tensor([ctx - 1], dtype=torch.int32, device=c.device)
        ang = (ctx - 1) / 10000.0 ** (torch.arange(0, HEAD_DIM, 2, device=c.device, dtype=torch.float64) / HEAD_DIM)
        cos_t, sin_t = torch.cat([ang, ang]).cos().float(), torch.cat([ang, ang]).sin().float()
        aws = torch.zeros(c.ops.attn_workspace_bytes(NH, NKV_HEADS, HEAD_DIM, ctx) + 256, dtype=torch.uint8,
                          device=c.device)

        def attention(li, stream, kc=kc, vc=vc, pos=pos, cos_t=cos_t, sin_t=sin_t, aws=aws):
            b = tok.bufs
            c.ops.attn_decode_prepkv(b["qkv"], qnw[li], knw[li], cos_t, sin_t, kc[li], vc[li], pos, NH, NKV_HEADS,
                                     HEAD_DIM, NQ, NQ + NKV_HEADS * HEAD_DIM, out=b["attn"], stream=stream,
                                     workspace=aws)

        graph = capture(c, lambda: tok.run(c.stream, attention), args.warmup)
        ms = timed_graph(c, graph, args.steps) / args.steps
        out[f"decode tok/s @ctx {ctx}"] = round(1000.0 / ms, 1)
        out[f"decode ms/token @ctx {ctx}"] = round(ms, 4)
        del graph, kc, vc, aws
        torch.cuda.empty_cache()
    out["decode launches/token"] = f"{len(tok.chains)} chain launches + {args.layers} attention launches"
    tok.close()
    # ---- prefill: one 2048-token prompt
    T = PROMPT_LEN
    X0 = torch.randn((T, H), generator=gen, device=c.device)
    logits = torch.empty((VOCAB,), device=c.device, dtype=torch.float16)
    A8 = torch.empty((T, FFN), dtype=torch.int8, device=c.device)
    sa = torch.empty((T,), dtype=torch.float32, device=c.device)
    lib = c.L.load()

    def mm(x16, w, i8):
        if not i8:
            return c.ops.gemm_i4(x16, w, out_dtype=torch.float16, stream=c.stream)
        M_, K_ = x16.shape
        c.L.check("g4b_cast_i8", lib.g4b_cast_i8(x16.data_ptr(), c.L.DT_F16, A8.data_ptr(), sa.data_ptr(), M_, K_,
                                                 c.sh))
        return c.ops.gemm_w8a8(A8.view(-1)[:M_ * K_].view(M_, K_), sa[:M_], w, stream=c.stream)

    # the prompt's KV caches (one per layer, [KV heads, T, head_dim] f16) and rotation rows
    kcs = [torch.empty((NKV_HEADS, T, HEAD_DIM), dtype=torch.float16, device=c.device) for _ in range(args.layers)]
    vcs = [torch.empty_like(kc) for kc in kcs]
    ang = torch.arange(T, device=c.device, dtype=torch.float64)[:, None] / \
        10000.0 ** (torch.arange(0, HEAD_DIM, 2, device=c.device, dtype=torch.float64) / HEAD_DIM)
    cosM, sinM = torch.cat([ang, ang], 1).cos().float(), torch.cat([ang, ang], 1).sin().float()
    p0 = torch.zeros(1, dtype=torch.int32, device=c.device)
    h = torch.empty((T, H), dtype=torch.float32, device=c.device)
    a16 = torch.empty((T, NQ), dtype=torch.float16, device=c.device)
    x16 = torch.empty((T, H), dtype=torch.float16, device=c.device)
    hl16 = torch.empty((1, H), dtype=torch.float16, device=c.device)
    st = c.stream

    def prefill(i8, torch_attention=False):
        """vk_engine.py's per-layer prefill recording (src/vk_engine.py:413-424) on this stack: pre_norm,
        q / k / v GEMMs, pre_prepkv + pre_attn, o GEMM, pre_na, pre_norm, gate / up GEMMs, gelumul, down
        GEMM, pre_na; then the final norm and lm_head on the prompt's last token."""
        h.copy_(X0)
        for li, (dd, nm) in enumerate(zip(layers_w, norms)):
            c.ops.rows_rmsnorm(h, nm.inw, out=x16, stream=st)
            q, k, v = mm(x16, dd["q"], i8), mm(x16, dd["k"], i8), mm(x16, dd["v"], i8)
            if torch_attention:
                a = F.scaled_dot_product_attention(q.view(T, NH, HEAD_DIM).transpose(0, 1)[None],
                                                   k.view(T, NKV_HEADS, HEAD_DIM).transpose(0, 1)[None],
                                                   v.view(T, NKV_HEADS, HEAD_DIM).transpose(0, 1)[None],
                                                   is_causal=True, enable_gqa=True)
                a16.copy_(a[0].transpose(0, 1).reshape(T, NQ))
            else:
                c.ops.attn_prefill_prepkv(k, v, knw[li], cosM, sinM, kcs[li], vcs[li], p0, NKV_HEADS, HEAD_DIM,
                                          stream=st)
                c.ops.attn_prefill(q, qnw[li], cosM, sinM, kcs[li], vcs[li], p0, NH, NKV_HEADS, HEAD_DIM, out=a16,
                                   stream=st)
            c.ops.rows_normadd(mm(a16, dd["o"], i8), nm.paw, h, 1.0, stream=st)
            c.ops.rows_rmsnorm(h, nm.pfw, out=x16, stream=st)
            act = c.ops.gelumul(mm(x16, dd["gate"], i8), mm(x16, dd["up"], i8), stream=st)
            c.ops.rows_normadd(mm(act, dd["down"], i8), nm.ofw, h, nm.scl, stream=st)
        c.ops.rows_rmsnorm(h[-1:], finw, out=hl16, stream=st)
        c.ops.gemv_i4(hl16.view(-1), lm, out=logits, stream=st)

    runs = (("prefill prompt-tok/s (W4A16)", False, False),
            ("prefill prompt-tok/s (PREFILL_I8: cast_i8 + W8A8)", True, False),
            ("prefill prompt-tok/s (W4A16, torch SDPA in place of g4b_attn_prefill)", False, True))
    for key, i8, ta in runs:
        with torch.cuda.stream(c.stream):
            prefill(i8, ta)                                   # warm-up
            c.stream.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(c.stream)
            prefill(i8, ta)
            e1.record(c.stream)
        c.stream.synchronize()
        ms = c.max(e0.elapsed_time(e1))
        out[key] = round(T / (ms / 1e3), 1)
    del kcs, vcs
    del layers_w, layers_d, X0, A8
    torch.cuda.empty_cache()
    return out


def one_gpu_extras(c, args, model):
    """The other BASELINE.json configs on this GPU, each with its own value and roofline."""
    ex = {}
    ex["configs[0] GEMV W[15360, 3840]"] = measure_gemv(c, False, args.steps, args.warmup)
    # configs[4] on one GPU: batched decode and prefill over the same stack (f16 scales)
    ws = [w for _, w in model]
    layers = [c.tp.TPLayer(**{n: ws[7 * li + i] for i, (n, _, _) in enumerate(LAYER_SHAPES)})
              for li in range(args.layers)]
    full = sum(weight_bytes(w.N, w.K, False) for w in ws)
    ex["configs[1] as decode tokens, element-wise work fused"] = measure_fused_token(c, layers, ws[-1], args.steps,
                                                                                      args.warmup)
    ex.update(tp_extras(c, layers, ws[-1], full, args))
    ex["configs[4] prefill M=8192"] = prefill_extra(c, args, [ws[7 * li:7 * li + 7] for li in range(args.layers)])
    # configs[1] again with e4m3 scales (GEMV_FP8)
    m8 = build_stream_model(c, True, args.layers)
    s8 = measure_stream(c, m8, True, args.steps, args.warmup, args.schedule,
                        stream_groups(args.layers, args.unfused, len(m8)), e2e=False, seed=2)
    ex["configs[1] e4m3 scales (GEMV_FP8)"] = {k: s8[k] for k in ("value", "ms_per_step", "roofline",
                                                                     "bytes_per_step")}
    ex["configs[1] e4m3 scales (GEMV_FP8)"]["unit"] = "GB/s"
    del m8
    c.torch.cuda.empty_cache()
    for key in GEMM_WORKLOADS:
        M, N, K, kind, text = GEMM_WORKLOADS[key]
        r = measure_gemm(c, key, args.steps, args.warmup)
        r["workload"] = text
        ex[f"{'configs[2]' if kind == 'w4a16' else 'configs[3]'} {key}"] = r
    ex["engine harness (benchmarks/bench_engine.py shape)"] = measure_engine(c, args)
    return ex


def run_tp(args) -> None:
    """the stream tensor parallel over the ranks (world 1 with --parallel tp)."""
    c = Ctx()
    why = c.tp.validate_world(HIDDEN, NQ, NKV, FFN, VOCAB, c.world)
    if why:
        raise SystemExit(f"bench: tensor parallel over {c.world} GPUs impossible: {why}")
    d = describe(args, c.world)
    fp8 = args.scales == "fp8"
    layers, lm, full_bytes, my_bytes = build_tp_model(c, fp8, args.layers)
    m = measure_tp_stream(c, layers, lm, full_bytes, my_bytes, args.steps, args.warmup, args.schedule,
                          args.allreduce)
    extras = {}
    if not args.no_extras and args.layers == LAYERS and not fp8:
        extras = tp_extras(c, layers, lm, full_bytes, args)
        del layers, lm
        c.torch.cuda.empty_cache()
        extras["configs[4] prefill M=8192"] = prefill_extra(c, args)
    if c.rank == 0:
        out = header(args, c, d, m["value"], m["ms_per_step"], "int4 x f32 -> f32 acc",
                     "synthetic (seeded N(0,0.02) weights, N(0,1) hidden state)")
        out.update({k: m[k] for k in ("roofline", "e2e", "gpu_launches", "clocks", "bytes_per_step",
                                      "bytes_per_gpu_max", "ms_per_step_kernels_only", "schedule", "allreduce")})
        out["cpu_baseline"] = None
        out["sharding"] = ("q/k/v/gate/up/lm_head by output columns, o/down by input rows (256-aligned shards); "
                           "q|k|v and gate|up fused; 2 all-reduces per layer + logits all-gather")
        if extras:
            out["extras"] = extras
        print(json.dumps(out), flush=True)
    c.close()


def run_gemv(args) -> None:
    """configs[0] (or the lm_head GEMV alone) as the line's workload."""
    c = Ctx()
    d = describe(args, c.world)
    fp8 = args.scales == "fp8"
    r = measure_gemv(c, fp8, args.steps, args.warmup, shape=args.shape)
    cpu = cpu_baseline(args, args.cpu_seconds) if c.rank == 0 and c.world == 1 and not args.no_cpu_baseline else None
    if c.rank == 0:
        out = header(args, c, d, round(r["value"] * c.world, 1), r["ms_per_launch"], "int4 x f16 -> f32 acc",
                     "synthetic (seeded N(0,0.02) weights, N(0,1) activations)")
        out.update({"roofline": r["roofline"], "cpu_baseline": cpu, "e2e": None,
                    "gpu_launches": args.steps * (1 if args.shape == "lm_head" else 8)})
        print(json.dumps(out), flush=True)
    c.close()


def run_gemm(args) -> None:
    """One prefill GEMM per step; value = 2*M*N*K / device time."""
    c = Ctx()
    d = describe(args, c.world)
    M, N, K, kind, _ = GEMM_WORKLOADS[args.workload]
    clocks = ClockSampler(c.local)
    clocks.start()
    r = measure_gemm(c, args.workload, args.steps, args.warmup, e2e=True)
    clk = clocks.stop()
    cpu = cpu_baseline(args, args.cpu_seconds) if c.rank == 0 and c.world == 1 and not args.no_cpu_baseline else None
    if c.rank == 0:
        out = header(args, c, d, r["value"], r["ms_per_step"],
                     "f16 x f16 -> f32 acc" if kind == "w4a16" else "s8 x s8 -> s32 acc",
                     "synthetic (seeded N(0,0.02) weights, N(0,1) f16 activations)")
        out.update({"roofline": r["roofline"], "cpu_baseline": cpu, "e2e": r["e2e"],
                    "gpu_launches": r["gpu_launches"], "clocks": clk})
        print(json.dumps(out), flush=True)
    c.close()


def run_prefill(args) -> None:
    """configs[4] prefill (M = 8192 split over the ranks) as the line's workload."""
    c = Ctx()
    d = describe(args, c.world)
    clocks = ClockSampler(c.local)
    clocks.start()
    gen = c.gen(0)
    layer_weights = []
    for _ in range(args.layers):
        dd = []
        for name, N, K in LAYER_SHAPES:
            W = c.torch.randn((N, K), generator=gen, device=c.device).mul_(0.02)
            dd.append(c.qz.quant_device(W, pf=False, fp8=False, prefill_i8=False))
            del W
        layer_weights.append(dd)
    r = measure_prefill(c, layer_weights, args.steps, args.warmup, e2e=True)
    clk = clocks.stop()
    cpu = cpu_baseline(args, args.cpu_seconds) if c.rank == 0 and c.world == 1 and not args.no_cpu_baseline else None
    if c.rank == 0:
        out = header(args, c, d, r["value"], r["ms_per_step"], "f16 x f16 -> f32 acc",
                     "synthetic (seeded N(0,0.02) weights, N(0,1) f16 activations)")
        out.update({"roofline": r["roofline"], "cpu_baseline": cpu, "e2e": r["e2e"],
                    "gpu_launches": r["gpu_launches"], "clocks": clk, "rows_per_gpu": r["rows_per_gpu"]})
        print(json.dumps(out), flush=True)
    c.close()


def run_engine(args) -> None:
    """The engine harness alone (benchmarks/bench_engine.py's measurements)."""
    c = Ctx()
    d = describe(args, c.world)
    r = measure_engine(c, args)
    if c.rank == 0:
        v = r["decode tok/s @ctx 16"]
        out = header(args, c, d, v, r["decode ms/token @ctx 16"], "int4 x f16 -> f32 acc",
                     "synthetic (seeded N(0,0.02) weights, N(0,1) hidden state and KV cache)")
        out.update({"engine": r, "cpu_baseline": None, "e2e": None, "gpu_launches": None})
        print(json.dumps(out), flush=True)
    c.close()


def select_runner(args, world: int):
    """The function that produces this run's line.  ``--impl reference`` is
    resolved first, whatever the workload and world size, so that the
    reference arm never reaches this repository's GPU code."""
    if args.impl == "reference":
        return run_reference_arm
    if args.workload in GEMM_WORKLOADS:
        return run_gemm
    if args.workload == "prefill":
        return run_prefill
    if args.workload == "gemv":
        return run_gemv
    if args.workload == "engine":
        return run_engine
    if stream_is_tp(args, world):
        return run_tp
    return run_stream


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--scales", default="f16", choices=["f16", "fp8"])
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the extra keys (the other configs measured after the line's own workload)")
    ap.add_argument("--workload", default="stream", choices=["stream", "gemv", "prefill", "engine"] + list(GEMM_WORKLOADS),
                    help="stream: configs[1] decode weight stream (default); gemv: configs[0] single GEMV; "
                         "gemm_i4 / gemm_i4_down: configs[2] W4A16 prefill GEMM; w8a8 / w4a8: configs[3]; "
                         "prefill: configs[4]'s M=8192 prefill split over the GPUs")
    ap.add_argument("--allreduce", default=None, choices=["peer", "nccl"],
                    help="tensor-parallel stream with --schedule launches: the per-layer all-reduce as one kernel "
                         f"over NVLink peer memory (g4b_allreduce_f32) or NCCL's (default: {TP_DEFAULT_ALLREDUCE})")
    ap.add_argument("--shape", default="config0", choices=["config0", "lm_head"],
                    help="gemv workload: config0 = W[15360, 3840] (configs[0]); lm_head = W[262144, 3840]")
    ap.add_argument("--schedule", default=None, choices=["chain", "launches"],
                    help="stream: chain runs the token's GEMVs as one persistent launch (g4b_gemv_chain: each "
                         "step waits for the step before it; tensor parallel: the all-reduces run inside it); "
                         "launches runs one launch per (fused) GEMV, chained by programmatic dependent launch "
                         "(default: chain on one GPU and over the confirmed tensor-parallel worlds)")
    ap.add_argument("--unfused", action="store_true",
                    help="stream: launch all 337 GEMVs separately, each on its own x, instead of fusing "
                         "q|k|v and gate|up (which read the same x in a decode step)")
    ap.add_argument("--parallel", default="auto", choices=["auto", "tp", "replicas"],
                    help="stream: tp shards the output columns / input rows over the GPUs (the default over "
                         "several GPUs; on one GPU it runs the same dependent chain, hidden state in, logits "
                         "out); replicas streams a full copy per GPU")
    return ap.parse_args(argv)


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    resolve_defaults(args, world)
    select_runner(args, world)(args)


if __name__ == "__main__":
    main()
