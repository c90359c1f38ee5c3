#!/usr/bin/env python
"""Benchmark of the nested GDN-2 forward hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config config1] [--path auto|simt|tc]

One "step" is one forward of the op over one batch of synthetic input of the
named configuration (default ``config1``: B=8, T=8192, H=16, K=V=128, L=3
firing every 1/4/16 chunks, m=64, bf16 inputs, fp32 state). Under torchrun
(N > 1) every rank runs the same per-GPU workload on its own seeded batch
(weak scaling; the path shards by (batch, head) and needs no collective);
times are CUDA-event times, max over ranks.

Rank 0 prints one JSON line. ``value`` is whole-job tokens/s (all GPUs)
with inputs resident in HBM, ``value_per_gpu`` the same divided by the GPU
count (the metric's "/GPU" figure); ``e2e`` is the same metric through the public API with
host (pinned) inputs copied in and o / final state copied out every step.
``roofline`` relates the forward to HBM bandwidth (the bound of this path),
``cpu_baseline`` is the CPU oracle (numpy restatement of the reference's
naive.py) timed on a bounded sample on this host.

``--impl reference`` times the reference's CPU algorithm (the oracle port;
the reference itself is Python and cannot travel to the GPU host) on rank 0
only and prints the same metric.
"""

from __future__ import annotations

import argparse
import json
import os
import pathlib
import statistics
import subprocess
import sys
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "nested-GDN layer fwd tokens/s/GPU at 1/2/4/8 B200; % tensor-pipe peak"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--config", default="config1")
    ap.add_argument("--path", choices=("auto", "simt", "tc", "tc_seg"), default="auto")
    ap.add_argument("--gates", choices=("dense", "broadcast"), default="dense",
                    help="b, w, g as materialised tensors (the canonical run) or as the "
                         "stride-0 views of the per-token, per-head scalars the recipe defines "
                         "(the broadcast fast path: the kernels read one scalar, and e2e uploads "
                         "only the scalars)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer e2e leg")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the per-GPU batch (profiling runs on a smaller case)")
    ap.add_argument("--heads", type=int, default=None,
                    help="override the number of heads (profiling runs on a smaller case)")
    ap.add_argument("--seq", type=int, default=None,
                    help="override the sequence length T (profiling runs on a smaller case)")
    ap.add_argument("--model", action="store_true",
                    help="time the full-model forward harness (BASELINE config 4: 12-layer "
                         "NestedGDN-2 LM, B=32 sharded over the GPUs, T=4096); prints its own line")
    ap.add_argument("--backward", action="store_true",
                    help="time the op's forward plus backward (one GPU)")
    ap.add_argument("--decode", action="store_true",
                    help="time the one-token decode step (step_nested_gdn2) on the config's "
                         "B, H, K, V, L instead of the chunked forward; prints its own line")
    return ap.parse_args()


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


# Configurations whose global problem is split by heads across the GPUs
# (strong scaling: 32 / N heads per GPU of one fixed sequence); the others
# give every GPU its own batch (weak scaling).
HEAD_SHARDED = {"config3"}


def workload(cfg_name):
    from nested_recurrent_memory_b200.synthetic import CONFIGS
    B, T, H, K, V, L, m, firing, dtype = CONFIGS[cfg_name]
    return dict(B=B, T=T, H=H, K=K, V=V, L=L, m=m, firing=tuple(firing), dtype=dtype,
                shard="heads" if cfg_name in HEAD_SHARDED else "batch")


def alg_counts(w):
    """Algorithmic flops and bytes per token per head (counting rules: tile
    triangles dense, triangular inverse excluded, intermediate states not
    counted)."""
    C, K, V, L, m = 64, w["K"], w["V"], w["L"], w["m"]
    s = 2 if str(w["dtype"]).endswith(("bfloat16", "float16")) else 4
    flop = (4 * C * C * K + 2 * C * C * (K + V) + 2 * C * C * V + 6 * C * K * V) / C
    for lvl in range(1, L):
        f = w["firing"][lvl]
        flop += 2 * K * V + (8 * m * K * V + 2 * m * V * (2 * K + V)) / (f * C)
    # q (L levels), k, v, g, b, w, mix, o; broadcast gates are one scalar
    # per token and head each.
    gates = 3 if w.get("gates") == "broadcast" else K + K + V
    nbytes = s * (L * K + K + V + gates + L + V)
    nbytes += L * K * V * 4 / w["T"]
    nbytes += (L - 1) * (m * K + 3 * K * V + V * V) * s / w["T"]
    return flop, nbytes


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    """SM clocks and clock-event reasons of one GPU during the timed region.

    NVML is polled every ~2 ms from a background thread; only samples taken
    between ``begin()`` and ``end()`` (which bracket the timed region on the
    host, whose final synchronize waits out the device work) count. Without
    NVML, ``nvidia-smi -lms 20`` is read instead."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
    # NVML clock-event reason bits of the four reasons above.
    BITS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
            "sw_power_cap": 0x4}

    def __init__(self, gpu_index):
        self.gpu_index = gpu_index
        self.proc = None
        self.handle = None
        self.samples = []
        self.window = False

    def start(self):
        import threading
        try:
            import pynvml
            pynvml.nvmlInit()
            gi = str(self.gpu_index)
            self.handle = (pynvml.nvmlDeviceGetHandleByUUID(gi) if gi.startswith(("GPU-", "MIG-"))
                           else pynvml.nvmlDeviceGetHandleByIndex(int(gi)))
            self.nvml = pynvml
            # The first queries can be slow: make them here, before the window.
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            pynvml.nvmlDeviceGetClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            pynvml.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
        except Exception:
            self.handle = None
        if self.handle is None:
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                     "-lms", "20", "-i", str(self.gpu_index)],
                    stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            except OSError:
                self.proc = None
            return
        self.stop_flag = threading.Event()
        self.thread = threading.Thread(target=self._poll, daemon=True)
        self.thread.start()

    def _poll(self):
        nv, h, mx = self.nvml, self.handle, self.max_mhz
        while not self.stop_flag.is_set():
            if self.window:
                try:
                    self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM), mx,
                                         nv.nvmlDeviceGetCurrentClocksEventReasons(h)))
                except Exception:
                    pass
            time.sleep(0.002)

    def begin(self):
        self.window = True

    def end(self):
        self.window = False

    def stop(self):
        if self.handle is not None:
            self.stop_flag.set()
            self.thread.join(timeout=5)
            if not self.samples:
                return None
            reasons = {name for name, bit in self.BITS.items()
                       if any(r & bit for _, _, r in self.samples)}
            return {"sm_mhz": statistics.median(s for s, _, _ in self.samples),
                    "sm_max_mhz": max(m for _, m, _ in self.samples),
                    "samples": len(self.samples), "reasons": sorted(reasons), "source": "nvml"}
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(self.REASONS, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "samples": len(sm), "reasons": sorted(reasons), "source": "nvidia-smi"}


# ---------------------------------------------------------------------------
# CPU baseline: the oracle on a bounded sample
# ---------------------------------------------------------------------------

REF_ROOT = ROOT / "baseline" / "_ref"


def reference_naive():
    """The reference's own CPU implementation of the path,
    ``naive_chunk_nested_gdn2`` (nested_gdn2/ops/naive.py:226-420), from the
    unmodified install in baseline/_ref, or None when it is not installed.
    Its parent packages are stubs: the package ``__init__`` registers the HF
    model, which imports a newer flash-linear-attention than this image
    has; the op modules themselves need torch only."""
    import types
    naive_py = REF_ROOT / "nested_gdn2" / "ops" / "naive.py"
    if not naive_py.exists():
        return None
    sys.dont_write_bytecode = True
    for name, sub in (("nested_gdn2", ""), ("nested_gdn2.ops", "ops")):
        if name not in sys.modules:
            mod = types.ModuleType(name)
            mod.__path__ = [str(REF_ROOT / "nested_gdn2" / sub) if sub else str(REF_ROOT / "nested_gdn2")]
            sys.modules[name] = mod
    try:
        from nested_gdn2.ops.naive import naive_chunk_nested_gdn2
    except Exception:
        return None
    return naive_chunk_nested_gdn2


def cpu_sample_run(w, heads, seed=0, T=None):
    """One bounded sample: one batch row, ``heads`` heads, the first ``T``
    tokens (default the full T), in fp32 on the host cores: the reference's
    own naive_chunk_nested_gdn2 with torch using every host thread when it
    is installed, else the numpy restatement in oracle/. Returns (seconds,
    token-heads processed, kind)."""
    import numpy as np
    import torch

    from nested_recurrent_memory_b200.synthetic import config_inputs

    T = T or w["T"]
    inp = config_inputs(1, T, heads, w["K"], w["V"], w["L"], w["m"], w["firing"],
                        dtype=torch.float32, seed=seed)
    L = inp.pop("L")
    ref = reference_naive()
    if ref is not None:
        torch.set_num_threads(os.cpu_count() or 1)
        t0 = time.perf_counter()
        with torch.no_grad():
            ref(**inp, L=L, output_final_state=True)
        return time.perf_counter() - t0, T * heads, "reference"
    import oracle  # CPU baseline leg only (the reference is not installed)
    a = {k: (v.numpy() if torch.is_tensor(v) else v) for k, v in inp.items()}
    t0 = time.perf_counter()
    oracle.chunk_forward(**a, L=L, output_final_state=True, dtype=np.float32)
    return time.perf_counter() - t0, T * heads, "port"


def cpu_sample_shape(w):
    """Heads and tokens of one CPU sample: about 2-10 s of host work (the
    reference's naive op holds a [heads, T / 64, 64, 64, K] decay tensor,
    so long sequences are sampled by a prefix)."""
    if w["T"] > 16384:
        return 1, 16384
    return 4, w["T"]


def cpu_threads(kind="port"):
    if kind == "reference":
        import torch
        return torch.get_num_threads()
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 0) for i in threadpool_info() if i.get("user_api") == "blas"]
        if n:
            return int(max(n))
    except Exception:
        pass
    return os.cpu_count() or 1


def run_reference(args, w):
    """--impl reference: the CPU algorithm on rank 0; other ranks exit."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    heads, T = cpu_sample_shape(w)
    for _ in range(args.warmup):
        cpu_sample_run(w, heads, T=T)
    secs = []
    kind = "port"
    for i in range(args.steps):
        s, th, kind = cpu_sample_run(w, heads, seed=i, T=T)
        secs.append(s)
    total = sum(secs)
    # token-heads/s divided by H: tokens of the configuration per second
    value = args.steps * T * heads / w["H"] / total
    what = ("the reference's naive_chunk_nested_gdn2 (baseline/_ref, unmodified), torch fp32"
            if kind == "reference" else
            "fp32 numpy oracle (restated reference naive_chunk_nested_gdn2)")
    sample = f"per step: 1 of {w['B']} batch rows, {heads} of {w['H']} heads, T={T}, {what}"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(args, w),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cpu_threads(kind),
                         "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# multi-GPU plumbing (one process per GPU; no data-path collective)
# ---------------------------------------------------------------------------

def shard(world, rank, w):
    """Weak scaling (batch-sharded configurations): every rank runs the
    configuration's per-GPU batch on its own seeded rows of a global batch of
    ``world * B`` sequences. Strong scaling (head-sharded ones): rank r runs
    heads [r H / N, (r + 1) H / N) of the one global sequence batch. (b, h)
    states are independent, so no rank needs another's data."""
    if w["shard"] == "heads":
        if w["H"] % world:
            raise SystemExit(f"{w['H']} heads do not split over {world} GPUs")
        hl = w["H"] // world
        return {"seed": 1000 + rank, "heads": (rank * hl, (rank + 1) * hl), "H_local": hl,
                "global_batch": w["B"]}
    return {"seed": 1000 + rank, "rows": (rank * w["B"], (rank + 1) * w["B"]),
            "global_batch": world * w["B"], "H_local": w["H"]}


def max_over_ranks(value, world, device="cpu"):
    """Max of a per-rank scalar over the process group (any backend)."""
    if world <= 1:
        return float(value)
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_tokens_per_s(w, world, ms_per_step):
    """Whole-job tokens/s: all ranks' tokens over the slowest rank's time
    (head-sharded: the ranks share one batch's tokens, each doing its heads)."""
    rows = w["B"] if w["shard"] == "heads" else world * w["B"]
    return rows * w["T"] / (ms_per_step / 1e3)


def config_dict(args, w):
    if w["shard"] == "heads":
        split = (f"B={w['B']}, H={w['H']} split {w['H'] // args.gpus} heads per GPU")
        par = f"head sharding (strong scaling), {args.gpus} GPU(s), no collective"
        gb = w["B"]
    else:
        split = f"B={w['B']} per GPU, H={w['H']}"
        par = f"(batch, head) sharding (weak scaling), {args.gpus} GPU(s), no collective"
        gb = w["B"] * args.gpus
    return {
        "workload": (f"{args.config}: {split}, T={w['T']}, "
                     f"K=V={w['K']}, L={w['L']} firing {'/'.join(map(str, w['firing']))} chunks, "
                     f"m={w['m']}, C=64, {str(w['dtype']).replace('torch.', '')} inputs, fp32 state"),
        "global_batch": gb, "seq_len": w["T"], "heads": w["H"],
        "parallelism": par,
        "l2": "inputs larger than L2 (no flush needed)",
        "gates": getattr(args, "gates", "dense"),
    }


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def run_ours(args, w):
    import torch
    import torch.distributed as dist

    from nested_recurrent_memory_b200 import FwdCall, chunk_nested_gdn2
    from nested_recurrent_memory_b200.synthetic import config_inputs

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    plan = shard(world, rank, w)
    inp = config_inputs(w["B"], w["T"], plan["H_local"], w["K"], w["V"], w["L"], w["m"],
                        w["firing"], dtype=w["dtype"], seed=plan["seed"], device=dev,
                        gen_device=dev, dense_gates=args.gates == "dense")
    L = inp.pop("L")
    call = FwdCall(**inp, L=L, path=args.path)
    launches_per_step = call.num_launches

    for _ in range(args.warmup):
        call.launch()
    barrier()
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    gpu_index = vis.split(",")[local] if vis else str(local)
    clocks = ClockSampler(gpu_index)
    clocks.start()
    time.sleep(0.3)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    clocks.begin()
    start.record()
    for _ in range(args.steps):
        call.launch()
    end.record()
    barrier()
    clocks.end()
    clk = clocks.stop()
    ms_max = max_over_ranks(start.elapsed_time(end), world, dev)
    ms_step = ms_max / args.steps
    tokens_per_step = w["B"] * w["T"] * world
    value = job_tokens_per_s(w, world, ms_step)

    # Per-stage timing on the launching stream (stage 1 = prep, 2 = scan).
    stage_ms = {1: 0.0, 2: 0.0}
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    for _ in range(args.steps):
        evs[0].record()
        call.launch(1)
        evs[1].record()
        call.launch(2)
        evs[2].record()
        torch.cuda.synchronize()
        stage_ms[1] += evs[0].elapsed_time(evs[1])
        stage_ms[2] += evs[1].elapsed_time(evs[2])
    stage_ms = {k: v / args.steps for k, v in stage_ms.items()}

    # e2e through the public API with pinned host buffers.
    e2e = None
    if not args.no_e2e:
        from nested_recurrent_memory_b200.host import compact_view
        # Pinned host copies; a broadcast (stride-0) input keeps only its
        # distinct elements on the host and is uploaded as such.
        host = {k: (compact_view(v).cpu().pin_memory().expand(v.shape)
                    if torch.is_tensor(v) and v.is_cuda else v)
                for k, v in inp.items()}
        dev_bufs = {k: (torch.empty(compact_view(v).shape, dtype=v.dtype, device=dev)
                        if torch.is_tensor(v) and v.is_pinned() else v)
                    for k, v in host.items()}
        h2d = sum(compact_view(v).numel() * v.element_size() for v in host.values()
                  if torch.is_tensor(v) and v.is_pinned())
        o_host = torch.empty(call.o.shape, dtype=call.o.dtype).pin_memory()
        s_host = torch.empty(call.final.shape, dtype=call.final.dtype).pin_memory()
        d2h = o_host.numel() * o_host.element_size() + s_host.numel() * s_host.element_size()

        def e2e_step():
            args_dev = {}
            for k, v in host.items():
                if torch.is_tensor(v) and v.is_pinned():
                    dev_bufs[k].copy_(compact_view(v), non_blocking=True)
                    args_dev[k] = dev_bufs[k].expand(v.shape)
                else:
                    args_dev[k] = v
            o, s = chunk_nested_gdn2(**args_dev, L=L, output_final_state=True)
            o_host.copy_(o, non_blocking=True)
            s_host.copy_(s, non_blocking=True)

        for _ in range(max(1, args.warmup)):
            e2e_step()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            e2e_step()
        e1.record()
        barrier()
        te = max_over_ranks(e0.elapsed_time(e1), world, dev)
        serial = job_tokens_per_s(w, world, te / args.steps)

        # The same steps through HostPipeline: every step still uploads all
        # of its inputs and downloads o and the final state, but step k + 1
        # uploads while step k runs and downloads.
        from nested_recurrent_memory_b200.host import HostPipeline
        example = {k: v for k, v in host.items() if torch.is_tensor(v) and v.is_pinned()}
        rest = {k: v for k, v in host.items() if k not in example}
        pipe = HostPipeline(example, device=dev, L=L, **rest)
        for _ in range(max(2, args.warmup)):
            pipe.submit(example)
        torch.cuda.synchronize()
        barrier()
        p0 = torch.cuda.Event(enable_timing=True)
        p0.record(pipe.first_stream())
        for _ in range(args.steps):
            handle = pipe.submit(example)
        p1 = torch.cuda.Event(enable_timing=True)
        p1.record(pipe.down)
        pipe.result(handle)
        barrier()
        tp = max_over_ranks(p0.elapsed_time(p1), world, dev)
        e2e = {"value": job_tokens_per_s(w, world, tp / args.steps), "unit": "tokens/s",
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "schedule": "HostPipeline: double-buffered device inputs, upload / compute / "
                           "download streams; step k + 1 uploads while step k runs and downloads",
               "single_stream_value": serial}

    peaks, peak_src = load_peaks()
    flop_th, bytes_th = alg_counts(w)
    token_heads = w["B"] * w["T"] * plan["H_local"]
    alg_bytes = bytes_th * token_heads
    alg_flops = flop_th * token_heads
    # The algorithmic bytes split by the kernel that moves them: prep reads
    # q's level-0 slice, k, v, g, b, w and mix; the scan reads the upper
    # levels' queries and the weights and writes o and the final states.
    s_el = 2 if str(w["dtype"]).endswith(("bfloat16", "float16")) else 4
    gate_el = 3 if w.get("gates") == "broadcast" else 2 * w["K"] + w["V"]
    prep_bytes = s_el * (2 * w["K"] + w["V"] + gate_el + w["L"]) * token_heads
    kernel_bytes = {1: prep_bytes, 2: alg_bytes - prep_bytes}
    traffic = None
    kernel_traffic = {1: None, 2: None}
    tfile = ROOT / "profiles" / "traffic.json"
    # (The committed ncu traffic figures are for the dense-gate runs.)
    if tfile.exists() and w.get("gates", "dense") == "dense":
        tj = json.loads(tfile.read_text())
        key = f"{args.config}:{call.path}"
        if key in tj:
            traffic = tj[key]["dram_bytes_per_token_head"] * token_heads
            per = tj[key].get("per_kernel_dram_bytes_per_token_head", {})
            for st, name in ((1, "prep_tc_kernel"), (2, "scan_tc_kernel")):
                if name in per:
                    kernel_traffic[st] = per[name] * token_heads
    dominant = max(stage_ms, key=stage_ms.get)
    stage_names = {"tc": ("prep_tc_kernel", "scan_tc_kernel"),
                   "tc_seg": ("prep_tc_kernel", "seg levels (seg_scan/combine/probe/read kernels)"),
                   "simt": ("prep_simt_kernel", "scan_simt_kernel")}[call.path]
    dom_name = stage_names[dominant - 1]
    dom_gbs = kernel_bytes[dominant] / (stage_ms[dominant] / 1e3) / 1e9
    whole_gbs = alg_bytes / (ms_step / 1e3) / 1e9
    roofline = {
        "bound": "hbm", "kernel": dom_name, "achieved": dom_gbs, "peak": peaks["hbm_gbs"],
        "unit": "GB/s", "frac": dom_gbs / peaks["hbm_gbs"], "traffic": kernel_traffic[dominant],
        "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured" else peak_src,
        "scope": ("dominant kernel; algorithmic bytes = the op's inputs it reads (prep: q level 0, "
                  "k, v, g, b, w, mix) or the rest of the op's bytes (scan); time = its stage's "
                  "CUDA events on the launching stream (prep's stage includes the two small "
                  "parameter-layout kernels); traffic = its ncu DRAM bytes per launch"),
        "alg_bytes_per_launch": kernel_bytes[dominant],
        "whole_forward": {"achieved": whole_gbs, "frac": whole_gbs / peaks["hbm_gbs"],
                          "traffic": traffic, "alg_bytes_per_launch": alg_bytes,
                          "scope": "prep + scan; algorithmic bytes = inputs + o + final state + weights"},
        "tensor_tflops": alg_flops / (ms_step / 1e3) / 1e12,
        "tensor_frac_of_bf16_peak": alg_flops / (ms_step / 1e3) / 1e12 / peaks["bf16_tflops"],
        "kernels": {"prep_ms": stage_ms[1], "scan_ms": stage_ms[2],
                    "prep_alg_bytes": kernel_bytes[1], "scan_alg_bytes": kernel_bytes[2],
                    "prep_frac": kernel_bytes[1] / (stage_ms[1] / 1e3) / 1e9 / peaks["hbm_gbs"],
                    "scan_frac": kernel_bytes[2] / (stage_ms[2] / 1e3) / 1e9 / peaks["hbm_gbs"],
                    "dominant": "prep" if dominant == 1 else "scan",
                    "dominant_share": stage_ms[dominant] / max(sum(stage_ms.values()), 1e-9)},
    }

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        heads, T = cpu_sample_shape(w)
        secs, th, kind = cpu_sample_run(w, heads, T=T)
        what = ("the reference's naive_chunk_nested_gdn2 (baseline/_ref, unmodified), torch fp32"
                if kind == "reference" else
                "fp32 numpy oracle (restated reference naive_chunk_nested_gdn2)")
        cpu = {"value": th / w["H"] / secs, "unit": "tokens/s", "cores": cpu_threads(kind),
               "kind": kind,
               "sample": (f"1 of {w['B']} batch rows, {heads} of {w['H']} heads, T={T} "
                          f"({secs:.1f} s), {what}")}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s (whole job, all GPUs)",
            "value_per_gpu": value / world, "unit_per_gpu": "tokens/s/GPU", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong" if w["shard"] == "heads" else "weak",
            "vs_baseline": None,
            "dtype": "bf16" if "bfloat16" in str(w["dtype"]) else str(w["dtype"]).replace("torch.", ""),
            "data": "synthetic (seeded; BASELINE config recipe)",
            "config": config_dict(args, w) | {"kernel_path": call.path},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_decode(args, w):
    """One step = one token for every batch row through ``step_nested_gdn2``,
    in place on a resident state, positions advancing from 0 (so the upper
    levels fire on schedule), replayed from a CUDA graph. Single GPU;
    tokens/s = B / step time."""
    import torch

    from nested_recurrent_memory_b200 import step_nested_gdn2
    from nested_recurrent_memory_b200.synthetic import config_inputs

    dev = torch.device("cuda", 0)
    B, H, K, V, L = w["B"], w["H"], w["K"], w["V"], w["L"]
    steps = max(args.steps, 256)
    inp = config_inputs(B, steps, H, K, V, L, w["m"], w["firing"], dtype=w["dtype"],
                        device=dev, gen_device=dev)
    inp.pop("L")
    per_token = ("q", "k", "v", "g", "b", "w", "mix_weights")
    wts = {n: inp[n] for n in inp if n not in per_token}
    state = torch.zeros(B, H, L, K, V, dtype=torch.float32, device=dev)
    ws = torch.empty(64 << 20, dtype=torch.uint8, device=dev)

    def step(t):
        step_nested_gdn2(**{n: inp[n][:, t] for n in per_token}, state=state, position=t,
                         **wts, L=L, out_state=state, workspace=ws)

    for t in range(args.warmup):
        step(t)
    torch.cuda.synchronize()
    # The steps are captured once into a CUDA graph and replayed, so the
    # timing is the GPU's, not the Python launch loop's.
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            for t in range(steps):
                step(t)
    torch.cuda.current_stream(dev).wait_stream(side)
    state.zero_()
    graph.replay()
    torch.cuda.synchronize()
    state.zero_()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    del graph
    peaks, _ = load_peaks()
    nbytes = B * H * (L + 1) * K * V * 4  # state read (all levels) + level-0 write, in place
    print(json.dumps({
        "metric": "nested-GDN decode step tokens/s (one token per row, in-place state)",
        "value": B / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1, "steps": steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "dtype": str(w["dtype"]).replace("torch.", ""), "data": "synthetic",
        "config": {"workload": f"{args.config} decode: B={B}, H={H}, K=V={K}, L={L}, "
                               f"firing {'/'.join(map(str, w['firing']))} chunks, positions 0..{steps - 1}"},
        "roofline": {"bound": "hbm", "achieved": nbytes / (ms / 1e3) / 1e9, "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": nbytes / (ms / 1e3) / 1e9 / peaks["hbm_gbs"],
                     "alg_bytes_per_step": nbytes},
    }), flush=True)


def run_backward(args, w):
    """One step = the op's forward (fast path) plus its backward
    (chunk_nested_gdn2_bwd: checkpointed CUDA-core forward re-run, reverse
    scan, per-chunk gradients) on resident inputs with a resident upstream
    gradient d_o. Single GPU; tokens/s = B * T / step time. The backward's
    share is timed separately with events around the bwd call."""
    import torch

    from nested_recurrent_memory_b200 import FwdCall, chunk_nested_gdn2_bwd
    from nested_recurrent_memory_b200.synthetic import config_inputs

    dev = torch.device("cuda", 0)
    inp = config_inputs(w["B"], w["T"], w["H"], w["K"], w["V"], w["L"], w["m"], w["firing"],
                        dtype=w["dtype"], device=dev, gen_device=dev)
    L = inp.pop("L")
    call = FwdCall(**inp, L=L, path=args.path)
    gen = torch.Generator(device=dev).manual_seed(7)
    d_o = torch.randn(w["B"], w["T"], w["H"], w["V"], generator=gen, device=dev).to(w["dtype"])

    def bwd():
        return chunk_nested_gdn2_bwd(**inp, L=L, do=d_o)

    for _ in range(args.warmup):
        call.launch()
        bwd()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    t_f = t_b = 0.0
    for _ in range(args.steps):
        ev[0].record()
        call.launch()
        ev[1].record()
        bwd()
        ev[2].record()
        torch.cuda.synchronize()
        t_f += ev[0].elapsed_time(ev[1])
        t_b += ev[1].elapsed_time(ev[2])
    ms_f, ms_b = t_f / args.steps, t_b / args.steps
    ms = ms_f + ms_b
    tokens = w["B"] * w["T"]
    print(json.dumps({
        "metric": "nested-GDN layer fwd+bwd tokens/s (the op's training step)",
        "value": tokens / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "dtype": str(w["dtype"]).replace("torch.", ""), "data": "synthetic",
        "config": {"workload": f"{args.config}: B={w['B']}, T={w['T']}, H={w['H']}, "
                               f"K=V={w['K']}, L={w['L']}, firing {'/'.join(map(str, w['firing']))}, "
                               f"m={w['m']}; forward path {call.path}, backward fp32 CUDA cores"},
        "fwd_ms": ms_f, "bwd_ms": ms_b,
    }), flush=True)


def run_model(args):
    """random-init 12-layer NestedGDN-2 LM forward in bf16,
    batch-sharded (32 sequences over the ranks), T=4096, token ids uniform
    over the vocabulary. One step = one forward of the rank's batch plus an
    NCCL all-reduce of the mean logit (the config's data-parallel collective).
    Dense layers run as torch GEMMs, the token mixer as this package's op."""
    import torch
    import torch.distributed as dist

    from nested_recurrent_memory_b200.model import ModelConfig, NestedGDN2ForCausalLM

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    B_total, T = 32, 4096
    B = args.batch or max(1, B_total // world)
    torch.manual_seed(0)
    cfg = ModelConfig()
    model = NestedGDN2ForCausalLM(cfg).to(dev, torch.bfloat16)
    ids = torch.randint(0, cfg.vocab_size, (B, T), device=dev,
                        generator=torch.Generator(device=dev).manual_seed(100 + rank))
    red = torch.zeros(1, device=dev)

    def step():
        with torch.no_grad():
            logits = model(ids)
        red.copy_(logits[:, -1].float().mean().reshape(1))
        if world > 1:
            dist.all_reduce(red)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), world, dev) / args.steps
    if rank == 0:
        print(json.dumps({
            "metric": "nested-GDN LM forward tokens/s (BASELINE config 4)",
            "value": B * T * world / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "dtype": "bf16",
            "data": "synthetic token ids, random-init weights N(0, 0.02)",
            "config": {"workload": f"config4: 12 layers, d 1024, 8x128 heads, L 3 (1/4/16), m 64, "
                                   f"SwiGLU 2816, vocab 32000; B={B} per GPU, T={T}",
                       "parallelism": f"data parallel over {world} GPU(s), NCCL all-reduce per step"},
        }), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse_args()
    if args.model:
        run_model(args)
        return
    w = workload(args.config)
    if args.batch is not None:
        w["B"] = args.batch
    if args.heads is not None:
        w["H"] = args.heads
    if args.seq is not None:
        w["T"] = args.seq
    w["gates"] = args.gates
    if args.decode:
        run_decode(args, w)
    elif args.backward:
        run_backward(args, w)
    elif args.impl == "reference":
        run_reference(args, w)
    else:
        run_ours(args, w)


if __name__ == "__main__":
    main()
