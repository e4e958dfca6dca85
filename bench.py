"""Benchmark of the decode hot path (driver contract: one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload ("b1"): the 306M decoder (seeded synthetic bf16
weights, N(0,0.02), seed 0), batch 1, the seeded 16-token prompt prefilled,
then greedy decode.  A step = one decode step (one token).  Timed steps run at
positions 16..143 (config 1's 128 greedy positions), wrapping around, with the
device's own argmax fed back as the next token (no host round trip).  With N
GPUs every rank decodes its own replica (weak scaling, no collective on the
data path); `value` is the tokens all ranks produced / max-over-ranks time.

`e2e` runs the same decode through the public call with host buffers: every
step copies the token and position from pinned host memory, launches, and
reads the next token back (as the reference's generate loop does with
``int(tok_out)``, generate.py:115-116), all inside the timed region.

`--impl reference` times the reference algorithm's CPU implementation on the
host cores: the reference needs JAX, which this image lacks, so the oracle's
numpy restatement of model.py (KV-cached, float32) stands in for it.
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
sys.path.insert(0, REPO)

FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1024)
    ap.add_argument("--warmup", type=int, default=64)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["b1"], default="b1")
    ap.add_argument("--cpu-sample-steps", type=int, default=48)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=256)
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def measured_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def profile_traffic():
    """Per-launch DRAM bytes of the decode kernel from the committed ncu summary."""
    p = os.path.join(REPO, "profiles", "decode_b1_cfg1.md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return int(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
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
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_baseline_b1(steps):
    """Oracle (numpy restatement of model.py, KV-cached float32) on host cores."""
    from oracle.ref_forward import CachedDecoder
    from transformer_b200.config import CONFIG_306M
    from transformer_b200.synth import params_f32, prompt_cfg1, synth_params
    P = params_f32(synth_params(CONFIG_306M, 0))
    prompt = prompt_cfg1()
    dec = CachedDecoder(P, CONFIG_306M, 1)
    lg = None
    for p, t in enumerate(prompt):
        lg = dec.step([t], [p])[0]
    tok = int(np.argmax(lg))
    t0 = time.perf_counter()
    for i in range(steps):
        lg = dec.step([tok], [len(prompt) + i])[0]
        tok = int(np.argmax(lg))
    dt = time.perf_counter() - t0
    cores = os.cpu_count()
    return {"value": steps / dt, "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"{steps} greedy decode steps of config 1 (positions 16..{15 + steps}), "
                      f"numpy float32 KV-cached restatement of model.py, BLAS threads={cores}"}


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    cb = cpu_baseline_b1(max(4, min(args.steps, args.cpu_sample_steps)))
    line = {"metric": "decode tok/s (B=1 greedy, 306M, config 1)", "value": cb["value"], "unit": "tok/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000.0 / cb["value"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "b1: 306M, batch 1, 16-token seeded prompt, greedy decode positions 16..143",
                       "global_batch": 1, "seq_len": 512, "parallelism": "cpu"},
            "impl": "reference", "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "reference needs JAX (absent); its numpy restatement (oracle) is timed instead"}
    print(json.dumps(line))
    return 0


def run_ours(args, rank, local_rank, world):
    import torch
    import torch.distributed as dist

    from transformer_b200.config import CONFIG_306M
    from transformer_b200.multi_sm_decode import DecodeEngine
    from transformer_b200.packing import prepare_decode_weights_nlayer
    from transformer_b200.synth import prompt_cfg1, synth_params

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    cfg = CONFIG_306M
    w = prepare_decode_weights_nlayer(synth_params(cfg, 0), cfg, device=dev)
    eng = DecodeEngine(w)
    stream = torch.cuda.current_stream(dev)
    prompt = prompt_cfg1()
    P0, NPOS = len(prompt), 128
    kv = eng.new_kv()
    eng.prefill(prompt, kv)
    tokbuf = torch.zeros(1, dtype=torch.int32, device=dev)
    tokbuf.copy_(torch.argmax(eng.logits[0]).to(torch.int32).reshape(1))
    total = args.warmup + args.steps
    posarr = torch.tensor([P0 + (i % NPOS) for i in range(total)], dtype=torch.int32, device=dev)
    logits = eng.logits

    def run(i0, n):
        for i in range(i0, i0 + n):
            eng.step(tokbuf, posarr[i:i + 1], kv, logits, tokbuf, stream)

    run(0, args.warmup)
    torch.cuda.synchronize(dev)
    eng.check_device()

    # ---- device-timed region ----
    clocks = ClockSampler(local_rank) if rank == 0 else None
    if clocks:
        clocks.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    run(args.warmup, args.steps)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    clk = clocks.stop() if clocks else None
    eng.check_device()
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    value = world * args.steps / (ms / 1000.0)

    # ---- end to end through the public call, host buffers ----
    h_in = torch.zeros(2, dtype=torch.int32, pin_memory=True)
    h_out = torch.zeros(1, dtype=torch.int32, pin_memory=True)
    d_in = torch.zeros(2, dtype=torch.int32, device=dev)
    d_out = torch.zeros(1, dtype=torch.int32, device=dev)
    kv2 = eng.new_kv()
    eng.prefill(prompt, kv2)
    tok = int(torch.argmax(eng.logits[0]).item())
    ne = args.e2e_steps
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(ne):
        h_in[0] = tok
        h_in[1] = P0 + (i % NPOS)
        d_in.copy_(h_in, non_blocking=True)
        eng.step(d_in[0:1], d_in[1:2], kv2, logits, d_out, stream)
        h_out.copy_(d_out, non_blocking=True)
        stream.synchronize()
        tok = int(h_out[0])
    e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_value = world * ne / e2e_s

    # ---- roofline of the decode kernel ----
    positions = [P0 + ((args.warmup + i) % NPOS) for i in range(args.steps)]
    alg_bytes = float(np.mean([cfg.step_bytes([p]) for p in positions]))
    peak, peak_kind = measured_peaks()
    achieved = alg_bytes / (ms_per_step / 1000.0) / 1e9
    traffic = profile_traffic()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_b1(args.cpu_sample_steps)

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": "decode tok/s (B=1 greedy, 306M, config 1)",
        "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_per_step, "us_per_token": ms_per_step * 1000.0,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.02) bf16 weights, seeded prompt; no checkpoint on the box)",
        "config": {"workload": "b1: 306M decoder (d=1024, 16 heads, 4 kv heads, 24 layers, d_ff 2816, "
                               "vocab 32000, ctx 512), batch 1, 16-token seeded prompt, greedy decode at "
                               "positions 16..143, one replica per GPU",
                   "model": "306M", "global_batch": world, "seq_len": 512,
                   "parallelism": f"replicas{world}",
                   "l2": "inputs larger than L2: 607 MB of weights streamed every step"},
        "gpu_launches": args.steps,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_source": f"{peak_kind} hbm_gbs",
                     "traffic": traffic, "algorithmic_bytes_per_launch": alg_bytes},
        "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 4,
                "steps": ne, "note": "host loop: pinned H2D tok+pos, launch, D2H next token, sync per step"},
        "clocks": clk,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line))
    eng.close()
    return 0


def main():
    args = parse()
    rank, local_rank, world = dist_env()
    if args.impl == "reference":
        return run_reference(args, rank, world)
    return run_ours(args, rank, local_rank, world)


if __name__ == "__main__":
    sys.exit(main())
