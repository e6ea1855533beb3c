#!/usr/bin/env python
"""Benchmark of rustane's language-model step on B200.

Default workload: the 600M-class decoder (dim 1536, SwiGLU
hidden 4096, 20 layers, 12 heads x 128, seq 512, vocab 8192), per-GPU batch 8 of
uniform-random token ids, weights N(0, 0.02) from seed 1234, fp32 master
weights + AdamW state with bf16 compute.  One step = forward + cross-entropy +
backward + [data-parallel gradient all-reduce] + grad-norm clip + AdamW.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload 600m|5b|7b|30b] [--batch B]

The other BASELINE configs: `5b` trains (per-GPU batch 4, data parallel);
`7b` (batch 1 or 16) and `30b` (batch 8) run forward + loss only, tensor
parallel over the N GPUs.  Under torchrun (N > 1) each rank drives one GPU;
time is the max over ranks.  Prints ONE JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "train-step tok/s & forward ms at 600M/5B/7B; TC util vs B200 bf16 peak"
# Published reference throughput (Apple M4 Max, ANE + CPU), tok/s at batch 1:
PUBLISHED = {
    "600m": (533.0, "600m-A train step 533 tok/s (results/2026-03-18_1830_param-sweep.md:37)"),
    "5b": (74.0, "5b-B train step 74 tok/s (results/2026-03-18_1830_param-sweep.md:78)"),
    "7b": (512 / 3.132, "7B forward 3132 ms for 512 tokens (README.md:70)"),
}
PUBLISHED_TOK_S = PUBLISHED["600m"][0]
SPEC_BF16_TFLOPS = 2250.0
PER_GPU_BATCH = 8
SEED_WEIGHTS = 1234


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16": d["bf16_tflops"], "bf16_sustained": d["bf16_tflops_sustained"],
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


WORKLOADS = {  # name -> (ModelConfig preset, trains?, default batch, label)
    "600m": ("c600m", True, 8, "600M train step"),
    "5b": ("c5b", True, 4, "5B train step"),
    "7b": ("c7b", False, 1, "7B forward + loss"),
    "30b": ("c30b", False, 8, "30B forward + loss"),
}


def workload_cfg(name: str = "600m"):
    from rustane_b200 import ModelConfig
    return getattr(ModelConfig, WORKLOADS[name][0])()


def workload_desc(cfg, name: str = "600m", batch: int = PER_GPU_BATCH) -> str:
    per = "per-GPU batch" if WORKLOADS[name][1] else "batch"
    return (f"{WORKLOADS[name][3]}: dim {cfg.dim}, SwiGLU hidden {cfg.hidden}, {cfg.nlayers} layers, {cfg.heads} "
            f"heads x {cfg.hd}, seq {cfg.seq}, vocab {cfg.vocab}, {per} {batch}")


# --------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks / throttle reasons every 50 ms, kept for the timed region only.

    nvidia-smi is started before the warm-up (its start-up takes a good part of a
    second on an 8-GPU box, longer than some timed regions); a reader thread stamps
    each line on arrival and `summary()` keeps the lines stamped inside `window()`."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        import threading
        self.lines = []
        self.t0 = self.t1 = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(gpu_index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True, bufsize=1)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        import atexit
        atexit.register(self.close)  # no sampler outlives the run, whatever path it ends by

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append((time.monotonic(), ln))

    def window(self):
        sampler = self

        class _Window:
            def __enter__(self):
                sampler.t0 = time.monotonic()

            def __exit__(self, *exc):
                sampler.t1 = time.monotonic()
        return _Window()

    def close(self):
        if self.proc is not None and self.proc.poll() is None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=5)

    def summary(self) -> dict:
        self.close()
        if self.proc is None or self.t0 is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        rows = [ln.split(",") for t, ln in self.lines if self.t0 <= t <= self.t1 and ln.strip()]
        sm, smax, power, reasons = [], None, [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            r = [x.strip() for x in r]
            try:
                sm.append(float(r[1]))
                smax = float(r[2])
                power.append(float(r[3]))
            except (ValueError, IndexError):
                continue
            for name, val in zip(names, r[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        under_load = [s for s, p in zip(sm, power) if p > 200.0] or sm
        return {"sm_mhz": statistics.median(under_load) if under_load else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm), "power_w_max": max(power) if power else None,
                "window_s": round(self.t1 - self.t0, 3)}


# ------------------------------------------------------------ CPU oracle
def oracle_step_seconds(cfg, n_steps: int, budget_s: float = 30.0):
    """The CPU restatement of the reference train step (oracle/, fp32, host BLAS)
    on one 512-token sequence per step.  Returns (seconds per step, threads, blas)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import pyoracle as po
    from rustane_b200.tensors import ModelOptState, ModelTensors
    w = po.reference_init(cfg)
    g, opt = ModelTensors.zeros(cfg), ModelOptState.zeros(cfg)
    o = po.Oracle(cfg, 1)
    rng = np.random.default_rng(1000)
    tc = po.default_train_config()
    times = []
    t_all = time.perf_counter()
    for i in range(n_steps):
        tok = rng.integers(0, cfg.vocab, cfg.seq).astype(np.uint32)
        tgt = rng.integers(0, cfg.vocab, cfg.seq).astype(np.uint32)
        t0 = time.perf_counter()
        o.train_step(w, g, opt, tok, tgt, i, tc)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_all > budget_s:
            break
    return times, po.lib().or_threads(), Path(po.lib().or_blas_name().decode()).name


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg = workload_cfg()
    W, K = args.warmup, args.steps
    # warmup steps (untimed) then K timed steps, each one 512-token sequence
    wt, threads, blas = oracle_step_seconds(cfg, W, budget_s=120.0)
    tt, _, _ = oracle_step_seconds(cfg, K, budget_s=240.0)
    per = statistics.mean(tt)
    value = cfg.seq / per
    sample = f"1 sequence x {cfg.seq} tokens of the 600M train step per step ({len(tt)} timed steps)"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": len(tt), "warmup": len(wt), "ms_per_step": per * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": value / PUBLISHED_TOK_S, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload_desc(cfg) + " (CPU sample: batch 1)", "per_gpu_batch": 1,
                   "seq_len": cfg.seq, "parallelism": "none (host CPU)"},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample,
                         "blas": blas},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": ("the reference (Rust + Apple ANE/Accelerate) cannot run on Linux; its CPU path is timed "
                 "through the fp32 C++ restatement in oracle/ with host OpenBLAS sgemm"),
    }), flush=True)


# ------------------------------------------------------ the other configs
EXTRA = (  # (key, workload, batch, timed steps, warm-up steps): BASELINE configs[2..4]
    ("5b_train_b4", "5b", 4, 5, 3),
    ("7b_fwd_b1", "7b", 1, 10, 3),
    ("7b_fwd_b16", "7b", 16, 5, 3),
    ("30b_fwd_b8", "30b", 8, 3, 3),
)


def measure_workload(wl: str, B: int, K: int, W: int, rank: int, world: int, local: int, dist) -> dict:
    """One context of workload `wl` (data parallel when it trains, tensor parallel
    otherwise), seeded device weights, two staged batches; W warm-up steps, then K
    steps timed by CUDA events on the context stream (max over ranks), then three
    profiled steps for the GEMM roofline.  The context is freed before returning."""
    import torch
    from rustane_b200 import CompiledKernels, TrainConfig, _lib

    train = WORKLOADS[wl][1]
    cfg = workload_cfg(wl)
    L = _lib.lib()
    k = CompiledKernels.compile(cfg, max_batch=B, device=local, forward_only=not train)
    try:
        if world > 1:
            uid = [CompiledKernels.nccl_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(uid, src=0)
            k.dist_init(world, rank, uid[0], _lib.RT_DIST_DATA_PARALLEL if train else _lib.RT_DIST_TENSOR_PARALLEL,
                        timeout_ms=120000)
        k.init_normal(seed=SEED_WEIGHTS, std=0.02)
        rng = np.random.default_rng(1000 + (rank if train else 0))
        for slot in range(2):
            tok = rng.integers(0, cfg.vocab, B * cfg.seq).astype(np.uint32)
            tgt = rng.integers(0, cfg.vocab, B * cfg.seq).astype(np.uint32)
            k._check(L.rt_stage_batch(k.handle, slot, tok.ctypes.data_as(_lib.c_uint32_p),
                                      tgt.ctypes.data_as(_lib.c_uint32_p), B))
        c_tc = TrainConfig().to_c()
        step = 0

        def steps(n):
            nonlocal step
            for _ in range(n):
                if train:
                    k._check(L.rt_train_step_staged(k.handle, step % 2, step, ctypes.byref(c_tc), None))
                else:
                    k._check(L.rt_forward_staged(k.handle, step % 2, ctypes.c_float(0.0)))
                step += 1

        clocks = ClockSampler(local)
        steps(W)
        k._check(L.rt_sync(k.handle, None))
        sp = ctypes.c_void_p()
        k._check(L.rt_ctx_stream(k.handle, ctypes.byref(sp)))
        stream = torch.cuda.ExternalStream(sp.value)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        with clocks.window():
            ev0.record(stream)
            steps(K)
            k._check(L.rt_join(k.handle))
            ev1.record(stream)
            loss = ctypes.c_float()
            k._check(L.rt_sync(k.handle, ctypes.byref(loss)))
            torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1)
        if dist is not None:
            t = torch.tensor([ms], device="cuda", dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        k.profile(True)
        steps(3)
        k._check(L.rt_sync(k.handle, None))
        tm = k.timings()
        k.profile(False)
    finally:
        k.close()
    ms_step = ms / K
    tokens = (world if train else 1) * B * cfg.seq
    flops = (3.0 if train else 1.0) * cfg.flops_per_token_fwd() * B * cfg.seq / (1 if train else world)
    pk = peaks()
    gemm_tf = tm["gemm_flops"] / (tm["gemm_ms"] * 1e-3) / 1e12 if tm["gemm_ms"] > 0 else None
    out = {"workload": workload_desc(cfg, wl, B), "parallelism": (f"dp{world}" if train else f"tp{world}"),
           "ms_per_step": ms_step, "tok_s": tokens / (ms_step * 1e-3),
           "step_tflops_per_gpu": flops / (ms_step * 1e-3) / 1e12,
           "tc_util_vs_spec_2250": flops / (ms_step * 1e-3) / 1e12 / SPEC_BF16_TFLOPS,
           "gemm_roofline": {"achieved": gemm_tf, "peak": pk["bf16_sustained"], "unit": "TFLOP/s",
                             "frac": gemm_tf / pk["bf16_sustained"] if gemm_tf else None,
                             "peak_source": pk["source"] + " sustained bf16"},
           "steps": K, "warmup": W, "loss_last": loss.value, "clocks": clocks.summary()}
    if not train:
        out["fwd_ms"] = ms_step
    if train:
        out["step_breakdown_ms"] = {"fwd": tm["fwd_ms"], "bwd": tm["bwd_ms"], "norm_adam": tm["opt_ms"]}
    if wl in PUBLISHED:
        out["vs_published"] = out["tok_s"] / PUBLISHED[wl][0]
        out["published_basis"] = PUBLISHED[wl][1] + ", Apple M4 Max"
    return out


# ------------------------------------------------------------- our arm
def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="600m", choices=list(WORKLOADS))
    ap.add_argument("--batch", type=int, default=0)
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the 5B / 7B / 30B lines that follow the 600M measurement")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    W = max(args.warmup, 3)
    K = args.steps

    import torch
    from rustane_b200 import CompiledKernels, TrainConfig, _lib

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    wl = args.workload
    train = WORKLOADS[wl][1]
    cfg = workload_cfg(wl)
    B, S = (args.batch or WORKLOADS[wl][2]), cfg.seq
    k = CompiledKernels.compile(cfg, max_batch=B, device=local, forward_only=not train)
    if world > 1:  # tensor-parallel shards must be set before the weights exist
        uid = [CompiledKernels.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        mode = _lib.RT_DIST_DATA_PARALLEL if train else _lib.RT_DIST_TENSOR_PARALLEL
        k.dist_init(world, rank, uid[0], mode, timeout_ms=120000)
    nccl_ranks = k.dist_ranks()
    k.init_normal(seed=SEED_WEIGHTS, std=0.02)

    rng = np.random.default_rng(1000 + (rank if train else 0))  # TP ranks share the batch
    nslots = 4
    batches = []
    for slot in range(nslots):
        tok = rng.integers(0, cfg.vocab, B * S).astype(np.uint32)
        tgt = rng.integers(0, cfg.vocab, B * S).astype(np.uint32)
        batches.append((tok, tgt))
        k._check(_lib.lib().rt_stage_batch(k.handle, slot, tok.ctypes.data_as(_lib.c_uint32_p),
                                           tgt.ctypes.data_as(_lib.c_uint32_p), B))
    tc = TrainConfig()
    c_tc = tc.to_c()
    L = _lib.lib()
    step = 0

    def staged_steps(n):
        nonlocal step
        for _ in range(n):
            if train:
                k._check(L.rt_train_step_staged(k.handle, step % nslots, step, ctypes.byref(c_tc), None))
            else:
                k._check(L.rt_forward_staged(k.handle, step % nslots, ctypes.c_float(0.0)))
            step += 1

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # -------- warm-up (the clock sampler starts here, ready before the timed region)
    clocks = ClockSampler(local)
    staged_steps(W)
    loss_w = ctypes.c_float()
    k._check(L.rt_sync(k.handle, ctypes.byref(loss_w)))

    # -------- timed region: device-resident inputs, CUDA events on the context stream
    sp = ctypes.c_void_p()
    k._check(L.rt_ctx_stream(k.handle, ctypes.byref(sp)))
    stream = torch.cuda.ExternalStream(sp.value)
    launches0 = k.timings()["kernel_launches"]
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with clocks.window():
        ev0.record(stream)
        staged_steps(K)
        k._check(L.rt_join(k.handle))  # the last step's weight all-gathers (sharded data parallel) count too
        ev1.record(stream)
        loss_last = ctypes.c_float()
        k._check(L.rt_sync(k.handle, ctypes.byref(loss_last)))
        torch.cuda.synchronize()
    barrier()
    ms_local = ev0.elapsed_time(ev1)
    ms = max_over_ranks(ms_local)
    launches = k.timings()["kernel_launches"] - launches0
    ms_per_step = ms / K
    tokens = (world if train else 1) * B * S * K  # tensor-parallel ranks share one batch
    value = tokens / (ms / 1e3)

    # -------- the same steps again with a CUDA event pair around every kernel
    # (kernel-class durations for the roofline; kept out of the timed region above)
    KP = max(3, min(K, 10))
    k.profile(True)
    barrier()
    staged_steps(KP)
    k._check(L.rt_sync(k.handle, None))
    tm = k.timings()
    k.profile(False)

    # -------- end to end: host tokens through the public API every step
    host_tok = [np.ascontiguousarray(b[0]) for b in batches]
    host_tgt = [np.ascontiguousarray(b[1]) for b in batches]
    h2d = ctypes.c_int64()
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(K):
        if train:
            k.train_step(host_tok[i % nslots], host_tgt[i % nslots], step, tc)
        else:
            k.forward(host_tok[i % nslots], host_tgt[i % nslots])
        step += 1
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    L.rt_last_h2d_bytes(k.handle, ctypes.byref(h2d))
    e2e_value = tokens / e2e_s

    # -------- roofline of the dominant kernel family (tcgen05 GEMM)
    pk = peaks()
    gemm_tflops = tm["gemm_flops"] / (tm["gemm_ms"] * 1e-3) / 1e12 if tm["gemm_ms"] > 0 else None
    per_launch_flops = tm["gemm_flops"] / max(tm["gemm_launches"], 1)
    # per GPU per step: train = 3 x forward (data parallel); forward shared by the TP ranks
    model_flops = (3.0 * cfg.flops_per_token_fwd() * B * S) if train else cfg.flops_per_token_fwd() * B * S / world
    step_tflops = model_flops / (ms_per_step * 1e-3) / 1e12
    traffic = None
    tfile = ROOT / "profiles" / "gemm_traffic.json"
    if tfile.exists():
        traffic = json.loads(tfile.read_text()).get("dram_bytes_per_launch")

    result = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak" if train else "strong",
        "vs_baseline": (value / PUBLISHED[wl][0]) if wl in PUBLISHED else None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": workload_desc(cfg, wl, B), "per_gpu_batch": B, "seq_len": S,
                   "tokens_per_gpu_step": B * S, "parallelism": (f"dp{world}" if train else f"tp{world}"),
                   "weights": ("N(0,0.02) seed 1234, fp32 master + AdamW state" if train
                               else "N(0,0.02) seed 1234, bf16"),
                   "tokens": "uniform ids, seed 1000+rank" if train else "uniform ids, seed 1000",
                   "nccl_ranks": nccl_ranks,
                   "l2": "not flushed: every step streams > 10 GB of weights/grads/optimizer state (>> 126 MB L2)"},
        "roofline": {"bound": "tensor", "kernel": "tcgen05 GEMM (all projections, FFN, logits, data and weight grads)",
                     "achieved": gemm_tflops, "peak": pk["bf16_sustained"], "unit": "TFLOP/s",
                     "frac": (gemm_tflops / pk["bf16_sustained"]) if gemm_tflops else None,
                     "traffic": traffic, "flops_per_launch": per_launch_flops,
                     "launches": tm["gemm_launches"], "peak_source": pk["source"] + " sustained bf16",
                     "measured": f"CUDA events around every GEMM launch over {KP} profiled steps"},
        "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": int(h2d.value), "d2h_bytes_per_step": 4},
        "gpu_launches": int(launches),
        "clocks": clocks.summary(),
        "step_breakdown_ms": {"fwd": tm["fwd_ms"], "bwd": tm["bwd_ms"], "allreduce": tm["comm_ms"],
                              "norm_adam": tm["opt_ms"]},
        "fwd_ms": tm["fwd_ms"],
        "step_tflops": step_tflops,
        "tc_util": {"vs_measured_peak": step_tflops / pk["bf16"], "vs_spec_2250": step_tflops / SPEC_BF16_TFLOPS},
        "kernel_ms_per_step": {"gemm": tm["gemm_ms"] / KP, "attention": tm["attn_ms"] / KP,
                               "other": tm["other_ms"] / KP, "profiled_steps": KP},
        "loss_last": loss_last.value,
        "vs_baseline_basis": (PUBLISHED[wl][1] + ", Apple M4 Max") if wl in PUBLISHED else None,
    }
    if not train:
        result["fwd_ms"] = ms_per_step
    if rank == 0 and world == 1 and not args.no_cpu_baseline and wl == "600m":
        times, threads, blas = oracle_step_seconds(cfg, 2, budget_s=25.0)
        per = statistics.mean(times)
        result["cpu_baseline"] = {"value": cfg.seq / per, "unit": "tok/s", "cores": threads, "kind": "port",
                                  "sample": f"{len(times)} train step(s) of 1 x {cfg.seq} tokens, 600M config",
                                  "blas": blas}
    k.close()
    if wl == "600m" and not args.no_extra:
        extra = {}
        for key, ewl, eb, ek, ew in EXTRA:
            try:
                extra[key] = measure_workload(ewl, eb, ek, ew, rank, world, local, dist)
            except Exception as e:  # noqa: BLE001 -- reported in the line, the headline stands
                extra[key] = {"error": f"{type(e).__name__}: {e}"}
        result["workloads"] = extra
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
