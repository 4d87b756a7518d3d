"""Benchmark: the int4 decode weight stream on B200.

One step = one decode token's full weight stream: for each of the 48 layers the
q, k, v, o, gate, up and down int4 GEMVs, then lm_head -- 337 GEMVs reading
6,617,825,280 bytes of packed weights + f16 scales (6,250,168,320 with
``--scales fp8``), each with its own f16 N(0, 1) activation vector and f16
output.  Weights are N(0, 0.02) quantised exactly as the engine's quant()
does, on the GPU.  The working set (6.6 GB) is ~50x the 126 MB L2, so every
step streams from HBM; no L2 flush is needed.

Reported (one JSON line from rank 0):
  value      whole-job GB/s (algorithmic bytes / device time), step replayed
             as one CUDA graph with the inputs resident in HBM
  e2e        the same metric through the public API with host buffers: each
             step copies its activations from pinned host memory and the
             outputs back, inside the timed region
  roofline   the GEMV kernel's achieved GB/s (algorithmic bytes of its launches
             / their CUDA-event durations, one eager pass of the timed steps)
             against the measured HBM copy bandwidth
  cpu_baseline  the CPU oracle (oracle/g4b_oracle.c) on the host cores, on a
             bounded sample of the same stream (rank 0, N=1)

``--impl reference`` times the reference's path on the host cores instead (the
oracle restatement of the shaders; the shaders themselves need a Vulkan stack
that these machines do not have).

Multi-GPU (torchrun, one rank per GPU): every rank streams its own copy of the
model for its own token (independent decode streams, no data-path
collective), so the per-GPU work is fixed: "scaling": "weak".
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
# tensor-parallel stream defaults: one chain launch per token with the all-reduces inside it where that has been
# run on a B200 box (2 GPUs: the fastest schedule); wider worlds default to per-GEMV launches with NCCL's
# all-reduce (--schedule chain selects the chain there too)
TP_CHAIN_CONFIRMED_WORLDS = (2,)
TP_DEFAULT_ALLREDUCE = "nccl"


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


# ------------------------------------------------------------- model setup
def build_model(torch, ops, qz, device, fp8, layers):
    """Quantise N(0, 0.02) weights on the GPU into the engine's packed layout."""
    model = []
    gen = torch.Generator(device=device)
    gen.manual_seed(0)
    for name, N, K in stream_shapes(layers):
        W = torch.randn((N, K), generator=gen, device=device, dtype=torch.float32).mul_(0.02)
        model.append((name, qz.quant_device(W, pf=False, fp8=fp8, prefill_i8=False)))
        del W
    return model


def run_cpu_baseline(host_entries, fp8, seconds, oracle):
    """Oracle GEMVs cycling over `host_entries` (the stream's first matrices, in
    order) until `seconds` of CPU time have elapsed."""
    done = 0
    n = 0
    t0 = time.perf_counter()
    while True:
        for name, N, K, wp, sc, inv in host_entries:
            x = np.random.default_rng(n).standard_normal(K).astype(np.float16).astype(np.float32)
            oracle.gemv(x, wp, sc, 1 if fp8 else 0, inv, N, K, 1)
            done += gemv_bytes(N, K, fp8)
            n += 1
            if time.perf_counter() - t0 >= seconds:
                dt = time.perf_counter() - t0
                return done / dt / 1e9, n, done, dt


def resolve_defaults(args, world: int) -> None:
    """Fill the schedule and all-reduce the user left unset: the chain on one
    GPU and for tensor parallelism over the confirmed worlds, per-GEMV launches
    with NCCL's all-reduce over wider ones."""
    tp_run = args.workload == "stream" and world > 1 and args.parallel != "replicas"
    if args.schedule is None:
        args.schedule = "chain" if not tp_run or world in TP_CHAIN_CONFIRMED_WORLDS else "launches"
    if args.allreduce is None:
        args.allreduce = TP_DEFAULT_ALLREDUCE


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--scales", default="f16", choices=["f16", "fp8"])
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="stream", choices=["stream", "gemv", "prefill"] + list(GEMM_WORKLOADS),
                    help="stream: configs[1] decode weight stream (default); gemv: configs[0] single GEMV; "
                         "gemm_i4 / gemm_i4_down: configs[2] W4A16 prefill GEMM; w8a8 / w4a8: configs[3]")
    ap.add_argument("--allreduce", default=None, choices=["peer", "nccl"],
                    help="tensor-parallel stream with --schedule launches: the per-layer all-reduce as one kernel "
                         f"over NVLink peer memory (g4b_allreduce_f32) or NCCL's (default: {TP_DEFAULT_ALLREDUCE})")
    ap.add_argument("--shape", default="config0", choices=["config0", "lm_head"],
                    help="gemv workload: config0 = W[15360, 3840] (configs[0]); lm_head = W[262144, 3840]")
    ap.add_argument("--schedule", default=None, choices=["chain", "launches"],
                    help="stream: chain runs the token's GEMVs as one persistent launch (g4b_gemv_chain: each "
                         "step waits for every tile of the step before it; tensor parallel: the all-reduces run "
                         "inside it); launches runs one launch per (fused) GEMV, chained by programmatic dependent "
                         "launch (default: chain on one GPU and tensor parallel over 2; launches over more)")
    ap.add_argument("--unfused", action="store_true",
                    help="stream: launch all 337 GEMVs separately, each on its own x, instead of fusing "
                         "q|k|v and gate|up (which read the same x in a decode step)")
    ap.add_argument("--parallel", default="auto", choices=["auto", "tp", "replicas"],
                    help="N > 1: tp (default) shards the stream's output columns / input rows over the GPUs "
                         "with NCCL all-reduces per layer; replicas streams a full copy per GPU")
    args = ap.parse_args()
    resolve_defaults(args, int(os.environ.get("WORLD_SIZE", "1")))
    if args.workload in GEMM_WORKLOADS:
        return run_gemm(args)
    if args.workload == "prefill":
        return run_prefill(args)
    if args.workload == "stream" and int(os.environ.get("WORLD_SIZE", "1")) > 1 and args.parallel != "replicas":
        return run_tp(args)
    fp8 = args.scales == "fp8"
    metric = "int4 GEMV HBM GB/s (decode weight stream, 48 layers + lm_head, batch 1)"

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    config = {"workload": "configs[1]: decode weight stream, 48 layers + lm_head, batch 1",
              "scales": args.scales, "layers": args.layers, "activations": "f16 N(0,1) per GEMV",
              "weights": "N(0,0.02) -> int4, 32-blocks", "l2": "working set 6.6 GB > 126 MB L2, no flush needed",
              "parallelism": f"replicas{world}"}

    if args.impl == "reference":
        return run_reference_arm(args, metric, config, rank, world, fp8)

    import torch
    import torch.distributed as dist
    from g4b import _lib as L
    from g4b import ops
    from g4b import quant_gpu as qz

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    L.load()

    if args.workload == "gemv" and args.shape == "lm_head":
        # configs[1]'s largest GEMV on its own: W[262144, 3840] (566 MB > L2)
        gen = torch.Generator(device=device)
        gen.manual_seed(0)
        W = torch.randn((VOCAB, HIDDEN), generator=gen, device=device).mul_(0.02)
        model = [("lm_head", qz.quant_device(W, pf=False, fp8=fp8, prefill_i8=False))]
        del W
        torch.cuda.empty_cache()
        config.update({"workload": "configs[1] lm_head GEMV W[262144, 3840], batch 1, f16 x/y",
                       "l2": "566 MB of weights > 126 MB L2, no flush needed"})
        config.pop("layers", None)
        metric = "int4 GEMV HBM GB/s (W[262144, 3840], batch 1)"
    elif args.workload == "gemv":
        # one [15360, 3840] GEMV; R weight copies rotated so that
        # successive launches read different HBM (R * 33 MB > 126 MB L2)
        R = 8
        gen = torch.Generator(device=device)
        gen.manual_seed(0)
        model = []
        for r in range(R):
            W = torch.randn((FFN, HIDDEN), generator=gen, device=device).mul_(0.02)
            model.append((f"gate.copy{r}", qz.quant_device(W, pf=False, fp8=fp8, prefill_i8=False)))
            del W
        config.update({"workload": "configs[0]: one int4 GEMV W[15360, 3840], batch 1, f16 x/y",
                       "l2": f"{R} weight copies rotated per launch ({R * 33.2:.0f} MB > 126 MB L2)"})
        config.pop("layers", None)
        metric = "int4 GEMV HBM GB/s (W[15360, 3840], batch 1)"
    else:
        model = build_model(torch, ops, qz, device, fp8, args.layers)
    # launch groups: GEMVs that read the same x run as one fused launch (the
    # engine's q/k/v on the normed hidden state, gate/up on the post-attention
    # one); --unfused launches every GEMV on its own x
    groups = []
    if args.workload == "stream" and not args.unfused:
        for li in range(args.layers):
            b = 7 * li
            groups += [[b, b + 1, b + 2], [b + 3], [b + 4, b + 5], [b + 6]]
        groups.append([7 * args.layers])
    else:
        groups = [[i] for i in range(len(model))]
    ws_list = [w for _, w in model]
    if args.workload == "stream":
        config["schedule"] = (f"{len(groups)} launches per token: q|k|v fused, o, gate|up fused, down per layer, "
                              "then lm_head" if not args.unfused else f"{len(groups)} separate GEMVs per token")
    step_bytes = (sum(weight_bytes(w.N, w.K, fp8) + 2 * w.N for w in ws_list)
                  + sum(2 * ws_list[g[0]].K for g in groups))
    # per-group activations (f16 N(0,1)) and per-GEMV outputs, resident in HBM
    gen = torch.Generator(device=device)
    gen.manual_seed(1 + rank)
    xs = [torch.randn((ws_list[g[0]].K,), generator=gen, device=device).to(torch.float16) for g in groups]
    ys = [torch.empty((w.N,), device=device, dtype=torch.float16) for w in ws_list]
    stream = torch.cuda.Stream(device)
    sh = int(stream.cuda_stream)
    need = 0
    for g in groups:
        ns = [ws_list[i].N for i in g]
        need = max(need, ops.gemv_fused_workspace_bytes(ns, ws_list[g[0]].K) if len(g) > 1
                   else ops.gemv_workspace_bytes(1, ns[0], ws_list[g[0]].K, 0))
    ws = torch.zeros(need + 256, dtype=torch.uint8, device=device)

    use_chain = args.workload == "stream" and args.schedule == "chain"
    chain = None
    if use_chain:
        # the token's GEMVs as one persistent launch; step j waits for every
        # tile of step j-1 (the command buffer's barrier) before it reads x
        chain = ops.GemvChain([(x, [ws_list[i] for i in g], [ys[i] for i in g]) for g, x in zip(groups, xs)])
        config["schedule"] = (f"one persistent launch per token (g4b_gemv_chain) of {len(groups)} GEMV steps "
                              f"({'fused q|k|v and gate|up' if not args.unfused else 'unfused'}); each step "
                              "starts reading x once every tile of the step before it is written")
    # event groups: one pair of events per launch
    ev_groups = [list(range(len(ws_list)))] if use_chain else groups

    def step(gev=None):
        if use_chain:
            if gev is not None:
                gev.record(0, sh)
            chain.run(stream)
            if gev is not None:
                gev.record(1, sh)
            return
        for gi, (g, x) in enumerate(zip(groups, xs)):
            if gev is not None:
                gev.record(2 * gi, sh)
            if len(g) == 1:
                ops.gemv_i4(x, ws_list[g[0]], out=ys[g[0]], stream=stream, workspace=ws, pdl=True)
            else:
                ops.gemv_i4_fused(x, [ws_list[i] for i in g], outs=[ys[i] for i in g], stream=stream,
                                  workspace=ws, pdl=True)
            if gev is not None:
                gev.record(2 * gi + 1, sh)

    # warm-up and graph capture (the reference records one command buffer per token)
    with torch.cuda.stream(stream):
        for _ in range(max(1, args.warmup)):
            step()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    gev = GraphEvents(len(ev_groups))
    graph_ev = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_ev, stream=stream):
        step(gev)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()
            graph_ev.replay()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- timed region: K graph replays on the launching stream
    clocks = ClockSampler(local_rank)
    clocks.start()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
    barrier()
    ms = e0.elapsed_time(e1)
    ms = max_over_ranks(ms)
    launches_per_step = len(ev_groups)
    ms_step = ms / args.steps
    value = world * step_bytes / (ms_step / 1e3) / 1e9

    # ---- roofline: the same step with an event-record node around every kernel
    kern_ms = 0.0
    kern_bytes = 0
    per_shape = {}
    with torch.cuda.stream(stream):
        for _ in range(args.steps):
            graph_ev.replay()
            stream.synchronize()
            for gi, g in enumerate(ev_groups):
                d = gev.elapsed_ms(2 * gi, 2 * gi + 1)
                kern_ms += d
                if use_chain:
                    gb = step_bytes
                    key = f"chain of {len(groups)} steps"
                else:
                    K = ws_list[g[0]].K
                    gb = sum(weight_bytes(ws_list[i].N, K, fp8) + 2 * ws_list[i].N for i in g) + 2 * K
                    key = "+".join(str(ws_list[i].N) for i in g) + f"x{K}"
                kern_bytes += gb
                a = per_shape.setdefault(key, [0.0, 0, gb])
                a[0] += d
                a[1] += 1
    clk = clocks.stop()
    gev.close()
    kern_gbs = kern_bytes / (kern_ms / 1e3) / 1e9
    peak = None
    peak_src = "of measured"
    try:
        peak = float(json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))["hbm_gbs"])
    except Exception:
        peak = 6650.0
        peak_src = "of fallback"
    roofline = {"bound": "hbm", "achieved": round(kern_gbs, 1), "peak": peak, "unit": "GB/s",
                "frac": round(kern_gbs / peak, 4), "traffic": None, "peak_source": peak_src,
                "kernel": "gemv_i4_chain_kernel" if use_chain else "gemv_i4_m1_kernel",
                "launches_timed": args.steps * len(ev_groups),
                "avg_launch_us": round(kern_ms * 1e3 / (args.steps * len(ev_groups)), 3),
                "per_shape_gbs": {k: round(v[2] * v[1] / (v[0] / 1e3) / 1e9, 1) for k, v in per_shape.items()},
                "graph_vs_kernels": round(ms_step / (kern_ms / args.steps), 4)}
    tp = os.path.join(REPO, "profiles", "gemv_traffic.json")
    if os.path.exists(tp):
        try:
            t = json.load(open(tp))
            if use_chain:
                roofline["traffic"] = int(round(t.get("chain_traffic_ratio", t["traffic_ratio"]) * step_bytes))
            else:
                key = "lm_head" if args.workload == "gemv" and args.shape == "lm_head" else args.workload
                roofline["traffic"] = t.get("bytes_per_launch_scaled", {}).get(key)
            roofline["traffic_note"] = t.get("note")
        except Exception:
            pass

    # ---- e2e: host buffers through the public API, copies inside the timed region
    xs_h = [x.cpu().pin_memory() for x in xs]
    ys_h = [torch.empty(y.shape, dtype=y.dtype).pin_memory() for y in ys]
    h2d = sum(x.numel() * 2 for x in xs)
    d2h = sum(y.numel() * 2 for y in ys)

    def e2e_step():
        for xh, x in zip(xs_h, xs):
            x.copy_(xh, non_blocking=True)
        step()
        for yh, y in zip(ys_h, ys):
            yh.copy_(y, non_blocking=True)

    with torch.cuda.stream(stream):
        for _ in range(2):
            e2e_step()
        stream.synchronize()
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            e2e_step()
            stream.synchronize()            # the caller reads its result every step
        e2e_s = time.perf_counter() - t0
    e2e_s = max_over_ranks(e2e_s)
    e2e_val = world * step_bytes * args.steps / e2e_s / 1e9

    # ---- CPU baseline: rank 0 at N = 1 only
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle as O

        host_entries = []
        budget = 2 * 10 ** 9                    # host copies of the stream's first ~2 GB of weights
        for name, w in model:
            if budget <= 0:
                break
            wp = w.wp.cpu().numpy().view(np.uint32)
            sc = w.scales.cpu().numpy()
            host_entries.append((name, w.N, w.K, wp, sc.view(np.uint16) if not fp8 else sc, w.inv))
            budget -= weight_bytes(w.N, w.K, fp8)
        gbs, n, done, dt = run_cpu_baseline(host_entries, fp8, args.cpu_seconds, O)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": O.num_threads(), "kind": "port",
               "sample": f"oracle gemv, {n} GEMVs cycling over the workload's first {len(host_entries)} "
                         f"matrices in order ({done / 1e9:.2f} GB in {dt:.1f} s, OpenMP over output columns)"}

    if rank == 0:
        out = {"metric": metric, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
               "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
               "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
               "dtype": "int4 x f16 -> f32 acc", "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
               "config": config, "roofline": roofline, "cpu_baseline": cpu,
               "e2e": {"value": round(e2e_val, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                       "d2h_bytes_per_step": d2h},
               "gpu_launches": launches_per_step * args.steps, "clocks": clk,
               "bytes_per_step": step_bytes}
        print(json.dumps(out), flush=True)
    del graph, graph_ev
    if chain is not None:
        torch.cuda.synchronize()
        chain.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------ prefill GEMMs
# name -> (M, N, K, kind, BASELINE.json config it is quoted on)
GEMM_WORKLOADS = {
    "gemm_i4": (2048, FFN, HIDDEN, "w4a16", "configs[2]: W4A16 prefill GEMM X[2048, 3840] x W[15360, 3840]"),
    "gemm_i4_down": (2048, HIDDEN, FFN, "w4a16", "configs[2]: W4A16 prefill GEMM, down_proj shape K=15360, N=3840"),
    "w8a8": (4096, HIDDEN, FFN, "w8a8", "configs[3]: W8A8 prefill GEMM X[4096, 15360] f16 -> cast_i8 -> int8 GEMM"),
    "w4a8": (4096, HIDDEN, FFN, "w4a8", "configs[3] shape, W4A8: int4 weights requantised in the kernel"),
}


def _gemm_cpu_sample(kind, M, N, K, seconds, O):
    """The oracle GEMM on a bounded sample of the workload: `rows` token rows of
    the same [N, K] weights, repeated until `seconds` have elapsed."""
    rng = np.random.default_rng(0)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    r = O.pack_reference(W, prefill_i8=kind != "w4a16")
    rows = 32
    X = rng.standard_normal((rows, K)).astype(np.float16)
    if kind == "w4a8":
        ratio = O.w4a8_ratio(r["sc_f32"], r["sw_f32"])
    done, n, t0 = 0, 0, time.perf_counter()
    while True:
        if kind == "w4a16":
            O.gemm_i4(X.view(np.uint16), r["wp"], r["scales16"].view(np.uint16), rows, N, K)
        else:
            A8, sa = O.cast_i8(X.astype(np.float32))
            if kind == "w8a8":
                O.gemm_w8a8(A8, r["w8"], sa, r["sw8"].view(np.uint16))
            else:
                O.gemm_w4a8(A8, r["wp"], ratio, sa, r["sw8"].view(np.uint16), N)
        done += 2 * rows * N * K
        n += 1
        dt = time.perf_counter() - t0
        if dt >= seconds:
            return done / dt / 1e12, n, rows, dt


def run_gemm(args):
    """One prefill GEMM per step; value = 2*M*N*K / device time."""
    M, N, K, kind, wl = GEMM_WORKLOADS[args.workload]
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    unit = "TFLOP/s" if kind == "w4a16" else "TOPS"
    metric = f"{'W4A16' if kind == 'w4a16' else kind.upper()} prefill GEMM {unit} (M={M}, N={N}, K={K})"
    config = {"workload": wl, "M": M, "N": N, "K": K, "parallelism": f"replicas{world}",
              "l2": "256 MB buffer written between timed iterations (L2 flush, outside the events)"}
    flops = 2 * M * N * K
    if args.impl == "reference":
        if rank != 0:
            return
        import oracle as O
        val, n, rows, dt = _gemm_cpu_sample(kind, M, N, K, max(2.0, args.cpu_seconds / 2), O)
        cpu = {"value": round(val, 5), "unit": unit, "cores": O.num_threads(), "kind": "port",
               "sample": f"oracle {kind} GEMM on {rows} token rows x the full [{N}, {K}] weight, {n} runs in {dt:.1f} s"}
        print(json.dumps({"metric": metric, "value": cpu["value"], "unit": unit, "n_gpus": world, "steps": n,
                          "warmup": 0, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                          "dtype": "f32" if kind == "w4a16" else "int32", "data": "synthetic", "config": config,
                          "impl": "reference", "cpu_baseline": cpu,
                          "e2e": {"value": cpu["value"], "unit": unit, "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return

    import torch
    import torch.distributed as dist
    from g4b import _lib as L
    from g4b import ops
    from g4b import quant_gpu as qz

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    L.load()
    gen = torch.Generator(device=device)
    gen.manual_seed(0)
    W = torch.randn((N, K), generator=gen, device=device).mul_(0.02)
    w = qz.quant_device(W, pf=True, fp8=False, prefill_i8=kind != "w4a16", w4a8=kind == "w4a8")
    del W
    X = torch.randn((M, K), generator=gen, device=device).to(torch.float16)
    Y = torch.empty((M, N), dtype=torch.float16, device=device)
    A8 = torch.empty((M, K), dtype=torch.int8, device=device)
    sa = torch.empty((M,), dtype=torch.float32, device=device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    stream = torch.cuda.Stream(device)
    sh = int(stream.cuda_stream)
    lib = L.load()

    def gemm():
        if kind == "w4a16":
            ops.gemm_i4(X, w, out=Y, stream=stream)
        elif kind == "w8a8":
            ops.gemm_w8a8(A8, sa, w, out=Y, stream=stream)
        else:
            ops.gemm_w4a8(A8, sa, w, out=Y, stream=stream)

    def step(ev=None, i=0):
        if kind != "w4a16":
            L.check("g4b_cast_i8", lib.g4b_cast_i8(X.data_ptr(), L.DT_F16, A8.data_ptr(), sa.data_ptr(), M, K, sh))
        if ev is not None:
            ev[i][1].record(stream)
        gemm()

    n = args.steps
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(n)]
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            step()
    stream.synchronize()
    clocks = ClockSampler(local_rank)
    clocks.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for i in range(n):
            flush.zero_()
            ev[i][0].record(stream)
            step(ev, i)
            ev[i][2].record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    step_ms = sum(e[0].elapsed_time(e[2]) for e in ev)
    kern_ms = sum(e[1].elapsed_time(e[2]) for e in ev)
    if world > 1:
        t = torch.tensor([step_ms, kern_ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        step_ms, kern_ms = float(t[0]), float(t[1])
    value = world * flops * n / (step_ms / 1e3) / 1e12
    achieved = flops * n / (kern_ms / 1e3) / 1e12
    peak, src = None, "of measured"
    try:
        pk = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))
        peak = float(pk["bf16_tflops"])
    except Exception:
        peak, src = 1590.0, "of fallback"
    if kind != "w4a16":
        peak, src = 2 * peak, src + " bf16 x 2 (dense int8 rate is twice the f16 rate)"
    kname = {"w4a16": "gemm_w4a16_kernel", "w8a8": "gemm_s8_kernel<W8A8>", "w4a8": "gemm_s8_kernel<W4A8>"}[kind]
    roofline = {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": unit,
                "frac": round(achieved / peak, 4), "traffic": None, "peak_source": src, "kernel": kname,
                "launches_timed": n, "avg_launch_us": round(kern_ms * 1e3 / n, 2)}
    tp = os.path.join(REPO, "profiles", "gemm_traffic.json")
    if os.path.exists(tp):
        try:
            roofline["traffic"] = json.load(open(tp)).get(args.workload)
        except Exception:
            pass

    # e2e: f16 activations from pinned host memory, the f16 output back, every step
    Xh = X.cpu().pin_memory()
    Yh = torch.empty((M, N), dtype=torch.float16).pin_memory()
    with torch.cuda.stream(stream):
        for _ in range(2):
            X.copy_(Xh, non_blocking=True)
            step()
            Yh.copy_(Y, non_blocking=True)
        stream.synchronize()
        t0 = time.perf_counter()
        for _ in range(n):
            X.copy_(Xh, non_blocking=True)
            step()
            Yh.copy_(Y, non_blocking=True)
            stream.synchronize()
        e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t[0])
    e2e = world * flops * n / e2e_s / 1e12
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle as O
        val, cn, rows, dt = _gemm_cpu_sample(kind, M, N, K, args.cpu_seconds, O)
        cpu = {"value": round(val, 5), "unit": unit, "cores": O.num_threads(), "kind": "port",
               "sample": f"oracle {kind} GEMM on {rows} token rows x the full [{N}, {K}] weight, {cn} runs in {dt:.1f} s"}
    if rank == 0:
        print(json.dumps({"metric": metric, "value": round(value, 1), "unit": unit, "n_gpus": world, "steps": n,
                          "warmup": args.warmup, "ms_per_step": round(step_ms / n, 4), "higher_is_better": True,
                          "scaling": "weak", "vs_baseline": None,
                          "dtype": "f16 x f16 -> f32 acc" if kind == "w4a16" else "s8 x s8 -> s32 acc",
                          "data": "synthetic (seeded N(0,0.02) weights, N(0,1) f16 activations)", "config": config,
                          "roofline": roofline, "cpu_baseline": cpu,
                          "e2e": {"value": round(e2e, 1), "unit": unit, "h2d_bytes_per_step": M * K * 2,
                                  "d2h_bytes_per_step": M * N * 2},
                          "gpu_launches": n * (1 if kind == "w4a16" else 2), "clocks": clk}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------ prefill over M
PREFILL_M = 8192


def run_prefill(args):
    """configs[4] prefill: M = 8192 f16 N(0, 1) tokens through the 48 layers'
    seven W4A16 GEMMs (the stack of configs[1], f16 scales), the M rows split
    over the ranks with the weights replicated (no collective).  value =
    total 2*M*N*K of the stack / device time of the step (max over ranks)."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from g4b import _lib as L
    from g4b import ops, tp
    from g4b import quant_gpu as qz

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    L.load()
    m0, m1 = tp.prefill_rows(PREFILL_M, world, rank)
    Mr = m1 - m0
    gen = torch.Generator(device=device)
    gen.manual_seed(0)
    layers = []
    for _ in range(args.layers):
        d = []
        for name, N, K in LAYER_SHAPES:
            W = torch.randn((N, K), generator=gen, device=device).mul_(0.02)
            d.append((name, qz.quant_device(W, pf=False, fp8=False, prefill_i8=False)))
            del W
        layers.append(d)
    # the rank's rows of the activations of each input width, and one output per output width
    X = {K: torch.randn((PREFILL_M, K), generator=gen, device=device).to(torch.float16)[m0:m1].contiguous()
         for K in (HIDDEN, NQ, FFN)}
    Y = {N: torch.empty((Mr, N), dtype=torch.float16, device=device) for N in (NQ, NKV, HIDDEN, FFN)}
    flops = 2 * PREFILL_M * sum(N * K for _, N, K in LAYER_SHAPES) * args.layers
    stream = torch.cuda.Stream(device)

    def step():
        for d in layers:
            for name, w in d:
                ops.gemm_i4(X[w.K], w, out=Y[w.N], stream=stream)

    with torch.cuda.stream(stream):
        for _ in range(max(1, args.warmup)):
            step()
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    clocks.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = flops / (ms / 1e3) / 1e12
    peak, src = 1590.0, "of fallback"
    try:
        peak, src = float(json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))["bf16_tflops"]), "of measured"
    except Exception:
        pass
    # e2e: this rank's f16 activations in from pinned host memory, the last output back, every step
    Xh = {K: x.cpu().pin_memory() for K, x in X.items()}
    Yh = torch.empty(Y[HIDDEN].shape, dtype=torch.float16).pin_memory()
    if world > 1:
        dist.barrier()
    with torch.cuda.stream(stream):
        t0 = time.perf_counter()
        for _ in range(args.steps):
            for K, x in X.items():
                x.copy_(Xh[K], non_blocking=True)
            step()
            Yh.copy_(Y[HIDDEN], non_blocking=True)
            stream.synchronize()
        e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    if rank == 0:
        print(json.dumps({
            "metric": f"W4A16 prefill GEMM TFLOP/s (48-layer stack, M={PREFILL_M} split over GPUs)",
            "value": round(value, 1), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16 x f16 -> f32 acc",
            "data": "synthetic (seeded N(0,0.02) weights, N(0,1) f16 activations)",
            "config": {"workload": "configs[4] prefill: M=8192 rows split over the GPUs, weights replicated",
                       "layers": args.layers, "rows_per_gpu": Mr, "parallelism": f"m-split{world}",
                       "l2": "working set per GPU > 126 MB L2"},
            "roofline": {"bound": "tensor", "achieved": round(value / world, 1), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(value / world / peak, 4), "traffic": None, "peak_source": src,
                         "kernel": "gemm_w4a16_kernel (per GPU)"},
            "cpu_baseline": None,
            "e2e": {"value": round(flops * args.steps / e2e_s / 1e12, 1), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": world * sum(x.numel() * 2 for x in X.values()),
                    "d2h_bytes_per_step": world * Yh.numel() * 2},
            "gpu_launches": 7 * args.layers * args.steps, "clocks": clk}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------ tensor parallel
def run_tp(args):
    """the 48-layer stream sharded over the ranks (g4b.tp): q/k/v/
    gate/up/lm_head by output columns, o/down by input rows, two NCCL
    all-reduces per layer and an all-gather of the logits.  One step = one
    token, captured as one CUDA graph per rank (collectives included).
    value = the full model's weight bytes / the step's device time (max over
    ranks): aggregate weight-stream GB/s, strong scaling."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from g4b import _lib as L
    from g4b import comm, ops, tp
    from g4b import quant_gpu as qz

    fp8 = args.scales == "fp8"
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    L.load()
    why = tp.validate_world(HIDDEN, NQ, NKV, FFN, VOCAB, world)
    if why:
        raise SystemExit(f"bench: tensor parallel over {world} GPUs impossible: {why}")
    kinds = dict(tp.LAYER_KINDS)
    gen = torch.Generator(device=device)
    gen.manual_seed(0)
    full_bytes = 0
    my_bytes = 0

    def shard(N, K, kind):
        nonlocal full_bytes, my_bytes
        W = torch.randn((N, K), generator=gen, device=device).mul_(0.02)   # same full W on every rank
        if kind == "col":
            n0, n1 = tp.split_range(N, world, rank, tp.COL_ALIGN)
            Ws = W[n0:n1].contiguous()
        else:
            k0, k1 = tp.split_range(K, world, rank, tp.ROW_ALIGN)
            Ws = W[:, k0:k1].contiguous()
        del W
        full_bytes += weight_bytes(N, K, fp8)
        w = qz.quant_device(Ws, pf=False, fp8=fp8, prefill_i8=False)
        my_bytes += weight_bytes(w.N, w.K, fp8)
        return w

    layers = []
    for _ in range(args.layers):
        d = {n: shard(N, K, kinds[n]) for (n, N, K) in LAYER_SHAPES}
        layers.append(tp.TPLayer(**d))
    lm = shard(VOCAB, HIDDEN, "col")
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device)
    ws = torch.zeros(max(ops.gemv_workspace_bytes(1, w.N, w.K, 0) for Lr in layers for w in vars(Lr).values())
                     + ops.gemv_workspace_bytes(1, lm.N, lm.K, 0) + 256, dtype=torch.uint8, device=device)
    L0 = layers[0]
    ws_fused = max(ops.gemv_fused_workspace_bytes([L0.q.N, L0.k.N, L0.v.N], L0.q.K),
                   ops.gemv_fused_workspace_bytes([L0.gate.N, L0.up.N], L0.gate.K))
    if ws.numel() < ws_fused + 256:
        ws = torch.zeros(ws_fused + 256, dtype=torch.uint8, device=device)
    launches = [0]

    def gemv(x, w, out):
        ops.gemv_i4(x, w, out=out, stream=stream, workspace=ws, pdl=True)
        launches[0] += 1

    def gemv_fused(x, ws_, outs):
        ops.gemv_i4_fused(x, ws_, outs=outs, stream=stream, workspace=ws, pdl=True)
        launches[0] += 1

    peer = comm.PeerAllReduce(HIDDEN, device) if args.allreduce == "peer" else None
    def all_reduce(t):
        if peer is not None:
            peer(t, stream=stream, pdl=True)
            launches[0] += 1          # g4b's own all-reduce kernel
        else:
            dist.all_reduce(t)

    dec = tp.TPDecoder(layers=layers, lm_head=lm, gemv=gemv, all_reduce=all_reduce,
                       all_gather=lambda out, t: dist.all_gather_into_tensor(out, t),
                       new_buffer=lambda n: torch.zeros(n, dtype=torch.float32, device=device),
                       hidden=HIDDEN, vocab=VOCAB, world=world, gemv_fused=gemv_fused)
    x = torch.randn((HIDDEN,), generator=gen, device=device)
    use_chain = args.schedule == "chain"
    chain = chain_k = xchg = None
    if use_chain:
        # one persistent launch per token and rank; the all-reduces run inside it over NVLink
        dec.bufs["part"] = torch.zeros(HIDDEN, dtype=torch.float32, device=device)
        steps = tp.chain_steps(layers, lm, x, dec.bufs, L.CHAIN_ALLREDUCE)
        xchg = comm.PeerBuffers(ops.GemvChain.exchange_bytes(steps, world), device)
        chain = ops.GemvChain(steps, exchange=xchg)

        def token():
            chain.run(stream)
            launches[0] += 1
            dist.all_gather_into_tensor(dec.bufs["logits"], dec.bufs["logits_local"])
    else:
        def token():
            dec.step(x)
    with torch.cuda.stream(stream):
        for _ in range(max(1, args.warmup)):
            token()
    stream.synchronize()
    launches[0] = 0
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        token()
    per_step = launches[0]
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()
    torch.cuda.synchronize()
    dist.barrier()
    clocks = ClockSampler(local_rank)
    clocks.start()
    torch.cuda.synchronize()
    dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    clk = clocks.stop()
    t = torch.tensor([e0.elapsed_time(e1)], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_step = float(t.item()) / args.steps
    value = full_bytes / (ms_step / 1e3) / 1e9

    # kernels only: the same GEMV chain without the collectives, for the roofline
    graph_k = torch.cuda.CUDAGraph()
    dec_k = tp.TPDecoder(layers=layers, lm_head=lm, gemv=gemv, all_reduce=lambda t: None,
                         all_gather=lambda out, t: None,
                         new_buffer=lambda n: torch.zeros(n, dtype=torch.float32, device=device),
                         hidden=HIDDEN, vocab=VOCAB, world=world, gemv_fused=gemv_fused)
    if use_chain:
        # the same chain with each all-reduced step's local partial as the next step's x
        dec_k.bufs["part"] = torch.zeros(HIDDEN, dtype=torch.float32, device=device)
        ksteps = [(st[0] if st[0] is not None else dec_k.bufs["part"], st[1], st[2])
                  for st in tp.chain_steps(layers, lm, x, dec_k.bufs, 0)]
        ksteps[0] = (x, ksteps[0][1], ksteps[0][2])
        chain_k = ops.GemvChain(ksteps)
        kstep = lambda: chain_k.run(stream)  # noqa: E731
    else:
        kstep = lambda: dec_k.step(x)  # noqa: E731
    with torch.cuda.stream(stream):
        kstep()
    with torch.cuda.graph(graph_k, stream=stream):
        kstep()
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph_k.replay()
        e0.record(stream)
        for _ in range(args.steps):
            graph_k.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1)], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_kern = float(t.item()) / args.steps
    mb = torch.tensor([float(my_bytes)], device=device, dtype=torch.float64)
    dist.all_reduce(mb, op=dist.ReduceOp.MAX)
    peak, src = 6650.0, "of fallback"
    try:
        peak, src = float(json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))["hbm_gbs"]), "of measured"
    except Exception:
        pass
    per_gpu_kern = float(mb.item()) / (ms_kern / 1e3) / 1e9
    roofline = {"bound": "hbm", "achieved": round(per_gpu_kern, 1), "peak": peak, "unit": "GB/s",
                "frac": round(per_gpu_kern / peak, 4), "traffic": None, "peak_source": src,
                "kernel": ("gemv_i4_chain_kernel" if use_chain else "gemv_i4_m1_kernel") +
                          " (per GPU, collectives removed)",
                "kernels_only_aggregate_gbs": round(full_bytes / (ms_kern / 1e3) / 1e9, 1)}

    # e2e: hidden state in from pinned host memory, gathered logits back, every step
    xh = x.cpu().pin_memory()
    lh = torch.empty(dec.bufs["logits"].shape, dtype=torch.float32).pin_memory()
    dist.barrier()
    with torch.cuda.stream(stream):
        t0 = time.perf_counter()
        for _ in range(args.steps):
            x.copy_(xh, non_blocking=True)
            graph.replay()
            lh.copy_(dec.bufs["logits"], non_blocking=True)
            stream.synchronize()
        e2e_s = time.perf_counter() - t0
    t = torch.tensor([e2e_s], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e = full_bytes * args.steps / float(t.item()) / 1e9
    if rank == 0:
        print(json.dumps({
            "metric": "int4 GEMV HBM GB/s (decode weight stream, 48 layers + lm_head, batch 1)",
            "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int4 x f32 -> f32 acc", "data": "synthetic (seeded N(0,0.02) weights, N(0,1) hidden state)",
            "config": {"workload": "configs[4]: the configs[1] stream tensor-parallel over the GPUs",
                       "scales": args.scales, "layers": args.layers, "parallelism": f"tp{world}",
                       "sharding": "q/k/v/gate/up/lm_head by output columns, o/down by input rows (256-aligned "
                                   "shards); q|k|v and gate|up fused; 2 all-reduces per layer + "
                                   "logits all-gather (NCCL), inside one CUDA graph",
                       "schedule": ("one persistent GEMV-chain launch per token, all-reduces inside it "
                                    "(g4b_gemv_chain_create_tp)" if use_chain else
                                    "one launch per (fused) GEMV"),
                       "allreduce": ("in-chain, NVLink peer stores of {value, epoch} words" if use_chain else
                                     "g4b_allreduce_f32 over NVLink peer memory" if peer is not None else "NCCL"),
                       "l2": "working set per GPU > 126 MB L2, no flush needed"},
            "roofline": roofline, "cpu_baseline": None,
            "e2e": {"value": round(e2e, 1), "unit": "GB/s", "h2d_bytes_per_step": HIDDEN * 4,
                    "d2h_bytes_per_step": VOCAB * 4},
            "gpu_launches": per_step * args.steps, "clocks": clk, "bytes_per_step": full_bytes,
            "bytes_per_gpu_max": int(mb.item()), "ms_per_step_kernels_only": round(ms_kern, 4)}), flush=True)
    del graph, graph_k
    dist.barrier()
    if peer is not None:
        peer.close()
    if chain is not None:
        chain.close()
        chain_k.close()
        xchg.close()
    dist.destroy_process_group()


def run_reference_arm(args, metric, config, rank, world, fp8):
    """The reference's path on the host cores: the oracle restatement of
    vk/gemv.comp (+ reduce.comp) over one layer's seven GEMVs per step."""
    if rank != 0:
        return
    import oracle as O

    layer = []
    for name, N, K in LAYER_SHAPES:
        W = (np.random.default_rng(len(layer)).standard_normal((N, K)) * 0.02).astype(np.float32)
        r = O.pack_reference(W, fp8=fp8)
        layer.append((name, N, K, r["wp"], r["scales"], r["inv"], r["split"]))
        del W
    xs = [np.random.default_rng(100 + i).standard_normal(K).astype(np.float16).astype(np.float32)
          for i, (_, N, K, *_r) in enumerate(layer)]
    step_bytes = sum(gemv_bytes(N, K, fp8) for _, N, K, *_r in layer)

    def step():
        for (name, N, K, wp, sc, inv, split), x in zip(layer, xs):
            O.gemv(x, wp, sc, 1 if fp8 else 0, inv, N, K, split)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    val = step_bytes * args.steps / dt / 1e9
    out = {"metric": metric, "value": round(val, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "int4 x f32 -> f32 acc", "data": "synthetic",
           "config": config, "impl": "reference",
           "cpu_baseline": {"value": round(val, 3), "unit": "GB/s", "cores": O.num_threads(), "kind": "port",
                            "sample": "one layer's seven GEMVs per step (q,k,v,o,gate,up,down; "
                                      f"{step_bytes / 1e6:.1f} MB), oracle restatement of vk/gemv.comp + "
                                      "vk/reduce.comp with the reference split"},
           "e2e": {"value": round(val, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
           "note": "the reference's GLSL shaders need a Vulkan stack (unavailable on this box); its CPU "
                   "path for this op is timed through the oracle port"}
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
