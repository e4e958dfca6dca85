"""Benchmark of the decode hot path (driver contract: one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload ("serve"): the 306M decoder (seeded
synthetic bf16 weights N(0,0.02), seed 0), 2048 sequences with seeded 64-token
prompts, partitioned evenly over the N ranks (one GPU each, a full weight
replica per GPU, no collective on the data path).  Each rank keeps its
2048/N sequences resident in a paged KV pool and decodes them in waves of at
most 256 (the batched tensor-core step, one CUDA graph per wave).  A step =
one greedy token for every sequence of the job; `value` = 2048 * K tokens /
max-over-ranks device time of the K timed steps (total work fixed as N grows:
"strong" scaling).  Config 5 decodes positions 64..319; the K timed steps are
spread evenly over that range (K >= 256: every position in turn), so the
value represents the whole job rather than its cheapest, shortest-context
steps.  A step's work (weights, KV pages read) depends only on its position,
so each timed step is placed at its position directly.

At N=1, rank 0 also measures the B=1 latency path (configs 1 and 2: the
single-launch decode megakernel, us/token and its HBM roofline), config 3
(B=64 ragged prompts U[32,448], random block table, 64 greedy steps) and
config 4 (B=8, temperature 0.7 / top-p 0.95 / repetition penalty 1.2 with the
seeded uniforms); they appear as sub-objects of the line.

`e2e` runs the serve step through the public call with host buffers: every
step copies each wave's tokens and positions from pinned host memory, runs the
step, and reads the next tokens back, all inside the timed region.

`--impl reference` times the reference algorithm on the host cores: the
reference needs JAX, which this image lacks, so the oracle's numpy
restatement of model.py (KV-cached, float32) stands in for it.  Each of its
K timed steps (after W warm-up steps) is a bounded sample of the workload:
one greedy token for 32 of the 2048 sequences; `ms_per_step` is the measured
time of such a sample step.
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
TOTAL_SEQS = 2048
PROMPT_LEN = 64
DECODE_STEPS = 256  # config 5: positions 64..319
WAVE = 256
REF_SAMPLE_SEQS = 32


def timed_positions(k, first=PROMPT_LEN, n=DECODE_STEPS):
    """Positions of the K timed steps: config 5's decode range first..first+n-1
    spread evenly (every position in turn, wrapping, when k >= n)."""
    if k >= n:
        return [first + (i % n) for i in range(k)]
    if k == 1:
        return [first + n // 2]
    return [first + int(round(i * (n - 1) / (k - 1))) for i in range(k)]


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-sample-steps", type=int, default=16)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the N=1 sub-measurements (configs 1-4)")
    ap.add_argument("--e2e-steps", type=int, default=8)
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


def profile_traffic(name, key="traffic_bytes_per_launch"):
    """DRAM bytes (per launch / per step) from a committed ncu summary."""
    p = os.path.join(REPO, "profiles", name)
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.strip().startswith(key + ":"):
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


_PARAMS = []


def oracle_params():
    if not _PARAMS:
        from transformer_b200.config import CONFIG_306M
        from transformer_b200.synth import params_f32, synth_params
        _PARAMS.append(params_f32(synth_params(CONFIG_306M, 0)))
    return _PARAMS[0]


def cpu_baseline_serve(steps, batch=REF_SAMPLE_SEQS, warmup=1):
    """Oracle (numpy restatement of model.py, KV-cached float32) on the host
    cores: `batch` sequences of the serve workload decoding at positions 64..
    (their caches hold seeded values in place of an ingested prompt: the step's
    work does not depend on them).  `warmup` untimed steps, then `steps` timed
    ones; returns the baseline object with the measured ms per step."""
    from oracle.ref_forward import CachedDecoder
    from transformer_b200.config import CONFIG_306M as cfg
    from transformer_b200.synth import batch_cfg5
    P = oracle_params()
    dec = CachedDecoder(P, cfg, batch)
    rng = np.random.default_rng(0)
    dec.K[:, :, :, :PROMPT_LEN] = rng.standard_normal(dec.K[:, :, :, :PROMPT_LEN].shape, dtype=np.float32)
    dec.V[:, :, :, :PROMPT_LEN] = rng.standard_normal(dec.V[:, :, :, :PROMPT_LEN].shape, dtype=np.float32)
    tok = batch_cfg5(cfg)[:batch, -1]
    for i in range(warmup):
        lg = dec.step(tok, [PROMPT_LEN + i] * batch)
        tok = np.argmax(lg, axis=1)
    p0 = PROMPT_LEN + warmup
    t0 = time.perf_counter()
    for i in range(steps):
        lg = dec.step(tok, [p0 + i] * batch)
        tok = np.argmax(lg, axis=1)
    dt = time.perf_counter() - t0
    cores = os.cpu_count()
    return {"value": steps * batch / dt, "unit": "tok/s", "cores": cores, "kind": "port",
            "ms_per_step": 1000.0 * dt / steps,
            "sample": f"{steps} timed greedy decode steps (after {warmup} untimed) of {batch} of the "
                      f"{TOTAL_SEQS} serve-workload sequences at positions {p0}..{p0 + steps - 1}, numpy "
                      f"float32 KV-cached restatement of model.py, BLAS threads={cores}"}


def cpu_baseline_b1(steps):
    """Oracle on the host cores, config 1 (B=1, 16-token prompt)."""
    from oracle.ref_forward import CachedDecoder
    from transformer_b200.config import CONFIG_306M
    from transformer_b200.synth import prompt_cfg1
    P = oracle_params()
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
    return {"value": steps / dt, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{steps} greedy decode steps of config 1 (positions 16..{15 + steps})"}


METRIC = "batched decode tok/s (config 5: 2048 seqs, 64-token prompts, greedy, replicas over N GPUs)"


def serve_config(world):
    return {"workload": f"serve (config 5): 306M decoder (d=1024, 16 heads, 4 kv heads, 24 layers, d_ff 2816, "
                        f"vocab 32000, ctx 512); {TOTAL_SEQS} sequences, seeded {PROMPT_LEN}-token prompts, "
                        f"{TOTAL_SEQS // world} per GPU decoded in waves of <= {WAVE} on a paged KV pool "
                        f"(16-token blocks, random block tables), greedy",
            "model": "306M", "global_batch": TOTAL_SEQS, "seq_len": 512, "parallelism": f"replicas{world}",
            "positions": f"timed steps spread evenly over config 5's decode positions {PROMPT_LEN}.."
                         f"{PROMPT_LEN + DECODE_STEPS - 1}",
            "l2": "inputs larger than L2: 607 MB of weights per wave-step plus the KV pages"}


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    cb = cpu_baseline_serve(max(1, args.steps), warmup=max(0, args.warmup))
    line = {"metric": METRIC, "value": cb["value"], "unit": "tok/s",
            "n_gpus": args.gpus, "steps": max(1, args.steps), "warmup": max(0, args.warmup),
            "ms_per_step": cb["ms_per_step"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": serve_config(1),
            "impl": "reference", "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": f"reference needs JAX (absent); its numpy restatement (oracle) is timed instead; a step "
                    f"is a bounded sample of the workload, one greedy token for {REF_SAMPLE_SEQS} of the "
                    f"{TOTAL_SEQS} sequences, and ms_per_step is that sample step's measured time"}
    print(json.dumps(line))
    return 0


def events_ms(fn, stream, torch):
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    fn()
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1)


def measure_b1(eng, cfg, dev, stream, torch, prompt, n_steps, label):
    """B=1 megakernel: prefill `prompt`, time n_steps greedy steps (device
    argmax fed back), return us/token and the HBM roofline of the kernel."""
    P0 = len(prompt)
    kv = eng.new_kv()
    eng.prefill(prompt, kv)
    tok = torch.zeros(1, dtype=torch.int32, device=dev)
    tok.copy_(torch.argmax(eng.logits[0]).to(torch.int32).reshape(1))
    span = cfg.context_len - P0
    posarr = torch.tensor([P0 + (i % span) for i in range(n_steps + 3)], dtype=torch.int32, device=dev)
    for i in range(3):
        eng.step(tok, posarr[i:i + 1], kv, eng.logits, tok, stream)
    torch.cuda.synchronize(dev)

    def run():
        for i in range(3, 3 + n_steps):
            eng.step(tok, posarr[i:i + 1], kv, eng.logits, tok, stream)
    ms = events_ms(run, stream, torch)
    eng.check_device()
    us = ms * 1000.0 / n_steps
    # the same tokens from one launch (b2d_decode_steps), when they fit before the context end
    one_launch = None
    if P0 + 3 + n_steps <= cfg.context_len:
        toks = torch.zeros(n_steps, dtype=torch.int32, device=dev)
        ms1 = events_ms(lambda: eng.decode_steps(tok, posarr[3:4], kv, n_steps, tokens=toks, stream=stream),
                        stream, torch)
        eng.check_device()
        one_launch = ms1 * 1000.0 / n_steps
    positions = [P0 + (i % span) for i in range(3, 3 + n_steps)]
    alg = float(np.mean([cfg.step_bytes([p]) for p in positions]))
    peak, kind = measured_peaks()
    ach = alg / (us * 1e-6) / 1e9
    return {"workload": label, "us_per_token": us, "tok_s": 1e6 / us, "steps": n_steps,
            "us_per_token_one_launch": one_launch,
            "roofline": {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                         "peak_source": f"{kind} hbm_gbs", "algorithmic_bytes_per_launch": alg,
                         "traffic": profile_traffic("decode_b1_cfg1.md"),
                         "traffic_note": "ncu capture of the same grid as a plain cluster launch (ncu cannot "
                                         "replay the cooperative one): mean DRAM read + write of three "
                                         "one-token launches, profiles/decode_b1_cfg1.md"},
            "gpu_launches": n_steps}


def measure_b1_e2e(eng, dev, stream, torch, prompt, n_steps):
    """Config 1 through the public host-value call (``decode_token`` /
    ``b2d_decode_token``): each step passes the token and position from the
    host (in the launch's arguments), runs the step with the logits written,
    the kernel writes the next token to mapped pinned host memory, and the
    host synchronises and reads it."""
    P0 = len(prompt)
    kv = eng.new_kv()
    eng.prefill(prompt, kv)
    tok = int(torch.argmax(eng.logits[0]).item())
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    for i in range(n_steps):
        tok = eng.decode_token(tok, P0 + (i % 128), kv, eng.logits, stream)
    dt = time.perf_counter() - t0
    return {"value": n_steps / dt, "unit": "tok/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 4,
            "steps": n_steps}


def measure_one_wave(w, cfg, torch, n_steps=16):
    """Config 5's 2048 sequences on ONE GPU as a single wave of 2048 (the
    weights are read once per step instead of once per 256 sequences): the
    prompts are ingested position by position, the step is captured once, and
    n_steps steps spread over positions 64..319 are timed (CUDA events)."""
    from transformer_b200.batched import BatchedDecoder
    from transformer_b200.multi_sm_decode import DecodeEngine
    from transformer_b200.synth import batch_cfg5
    eng = DecodeEngine(w, max_batch=TOTAL_SEQS)
    dec = BatchedDecoder(eng, TOTAL_SEQS, seed=0)
    dec.ingest(list(batch_cfg5(cfg)))
    dec.capture()
    positions = timed_positions(n_steps)
    for p in positions[:2]:
        dec.pos.fill_(p)
        dec.replay()
    stream = torch.cuda.current_stream()

    def run():
        for p in positions:
            dec.pos.fill_(p)
            dec.replay()
    ms = events_ms(run, stream, torch)
    eng.check_device()
    per_step = eng.lib.b2d_batched_launches(eng.ws)
    alg = float(np.mean([cfg.step_bytes([p] * TOTAL_SEQS) for p in positions]))
    peak, kind = measured_peaks()
    ach = alg / (ms / n_steps * 1e-3) / 1e9
    dec.release()
    del dec
    eng.close()
    return {"workload": f"config 5 on one GPU as a single wave: {TOTAL_SEQS} sequences per step, "
                        f"{n_steps} steps spread over positions {PROMPT_LEN}..{PROMPT_LEN + DECODE_STEPS - 1}",
            "tok_s": TOTAL_SEQS * n_steps / (ms / 1000), "ms_per_step": ms / n_steps,
            "roofline": {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                         "scope": f"whole step ({per_step} kernels)", "peak_source": f"{kind} hbm_gbs"},
            "gpu_launches": per_step * n_steps}


def measure_cfg3(eng, cfg, torch):
    """Config 3: B=64, prompts U[32,448] (seed 2) ingested raggedly into the
    paged pool (random block table), then 64 greedy steps (graph replay)."""
    from transformer_b200.batched import BatchedDecoder
    from transformer_b200.synth import batch_cfg3
    lens, prompts, table = batch_cfg3(cfg)
    dec = BatchedDecoder(eng, len(prompts), table=table, num_blocks=int(table.size))
    dec.ingest(prompts)
    dec.capture()
    per_step = eng.lib.b2d_batched_launches(eng.ws)
    pos0 = dec.pos.cpu().numpy().copy()
    n = 64
    ms = events_ms(lambda: [dec.replay() for _ in range(n)], torch.cuda.current_stream(), torch)
    eng.check_device()
    alg = float(np.mean([cfg.step_bytes(pos0 + i) for i in range(n)]))
    peak, kind = measured_peaks()
    ach = alg / (ms / n * 1e-3) / 1e9
    dec.release()
    return {"workload": "config 3: B=64 paged, prompt lengths U[32,448] seed 2, random block table, "
                        "64 greedy steps", "tok_s": 64 * n / (ms / 1000), "ms_per_step": ms / n,
            "roofline": {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                         "scope": f"whole step ({per_step} kernels)", "peak_source": f"{kind} hbm_gbs"},
            "gpu_launches": per_step * n}


def measure_cfg4(eng, cfg, torch):
    """Config 4: B=8 64-token prompts (seed 3), 128 sampled steps with
    temperature 0.7, top-p 0.95, repetition penalty 1.2 and the seeded
    uniforms [128, 8] (seed 4); one batched step + one sampler launch each."""
    from transformer_b200.batched import BatchedDecoder
    from transformer_b200.generate import Sampler
    from transformer_b200.synth import batch_cfg4
    prompts, u = batch_cfg4(cfg)
    B, steps = prompts.shape[0], u.shape[0]
    dev = eng.device
    dec = BatchedDecoder(eng, B, seed=4)
    last = dec.ingest(list(prompts))
    smp = Sampler(eng, B, steps + 1)
    uni = torch.from_numpy(u.astype(np.float64)).to(dev)
    nxt = torch.zeros(B, dtype=torch.int32, device=dev)
    logits = last.contiguous()
    smp.hist_len.zero_()
    tok = smp.sample(logits, 0.7, 0.95, 1.2, B, uniforms=uni[0]).clone()

    def run():
        nonlocal tok
        for i in range(1, steps):
            smp.history[:, i - 1].copy_(tok)
            smp.hist_len.fill_(i)
            dec.tok.copy_(tok)
            eng.step_paged(dec.tok, dec.pos, dec.pool, dec.table, dec.logits, nxt)
            dec.pos.add_(1)
            tok = smp.sample(dec.logits, 0.7, 0.95, 1.2, B, uniforms=uni[i]).clone()
    ms = events_ms(run, torch.cuda.current_stream(), torch)
    eng.check_device()
    per_step = eng.lib.b2d_batched_launches(eng.ws) + 1  # + the sampler
    return {"workload": "config 4: B=8 sampling (T 0.7, top-p 0.95, rep 1.2, seeded uniforms), 64-token "
                        "prompts, 127 sampled steps after the first", "tok_s": B * (steps - 1) / (ms / 1000),
            "ms_per_step": ms / (steps - 1), "gpu_launches": per_step * (steps - 1)}


def run_ours(args, rank, local_rank, world):
    import torch
    import torch.distributed as dist

    from transformer_b200.batched import BatchedDecoder
    from transformer_b200.config import CONFIG_306M
    from transformer_b200.multi_sm_decode import DecodeEngine
    from transformer_b200.packing import prepare_decode_weights_nlayer
    from transformer_b200.replicas import all_ranks, max_over_ranks, shard
    from transformer_b200.synth import batch_cfg5, prompt_cfg1, prompt_cfg2, synth_params

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    cfg = CONFIG_306M
    w = prepare_decode_weights_nlayer(synth_params(cfg, 0), cfg, device=dev)
    part = shard(TOTAL_SEQS, world, rank, WAVE)
    n_seq, n_waves, wave_b = part.n, part.n_waves, part.wave
    eng = DecodeEngine(w, max_batch=max(2, wave_b))
    stream = torch.cuda.current_stream(dev)
    all_prompts = batch_cfg5(cfg)
    waves = []
    for i in range(n_waves):
        b0, b1 = part.wave_slice(i)
        d = BatchedDecoder(eng, wave_b, seed=1000 * rank + i)
        d.ingest(list(all_prompts[b0:b1]))
        d.capture()
        waves.append(d)
    def one_step(p):
        for d in waves:  # every wave's sequences at position p (the graph advances pos itself)
            d.pos.fill_(p)
            d.replay()

    for i in range(args.warmup):
        one_step(PROMPT_LEN + i % DECODE_STEPS)
    torch.cuda.synchronize(dev)
    eng.check_device()
    positions = timed_positions(args.steps)
    per_wave = eng.lib.b2d_batched_launches(eng.ws)  # kernels of one wave-step (the captured step's)

    # ---- device-timed region ----
    clocks = ClockSampler(local_rank) if rank == 0 else None
    if clocks:
        clocks.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    ms = events_ms(lambda: [one_step(p) for p in positions], stream, torch)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    clk = clocks.stop() if clocks else None
    eng.check_device()
    rank_ms = all_ranks(ms, dev)
    ms = max(rank_ms)
    ms_per_step = ms / args.steps
    value = TOTAL_SEQS * args.steps / (ms / 1000.0)
    alg_step = float(np.mean([n_waves * cfg.step_bytes([p] * wave_b) for p in positions]))
    peak, peak_kind = measured_peaks()
    achieved = alg_step / (ms_per_step / 1000.0) / 1e9
    serve_traffic = profile_traffic("paged_step_b256_pos80.md", "traffic_bytes_per_step") if wave_b == 256 else None

    # ---- end to end through the public call, host buffers ----
    ne = max(1, args.e2e_steps)
    h_in = [torch.zeros(2, wave_b, dtype=torch.int32, pin_memory=True) for _ in waves]
    h_out = [torch.zeros(wave_b, dtype=torch.int32, pin_memory=True) for _ in waves]
    d_in = [torch.zeros(2, wave_b, dtype=torch.int32, device=dev) for _ in waves]
    for i, d in enumerate(waves):
        h_out[i].copy_(d.tok)

    def e2e_step(p):
        for i, d in enumerate(waves):
            h_in[i][0].copy_(h_out[i])
            h_in[i][1].fill_(p)
            d_in[i].copy_(h_in[i], non_blocking=True)
            eng.step_paged(d_in[i][0], d_in[i][1], d.pool, d.table, d.logits, d.tok, stream)
            h_out[i].copy_(d.tok, non_blocking=True)
        stream.synchronize()

    for i in range(2):  # warm-up: the call caches each wave's step graph on its second use
        e2e_step(PROMPT_LEN + i)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for p in timed_positions(ne):
        e2e_step(p)
    e2e_s = max_over_ranks(time.perf_counter() - t0, dev)
    e2e_value = TOTAL_SEQS * ne / e2e_s
    for d in waves:
        d.release()
    del waves, d
    torch.cuda.empty_cache()

    extra = {}
    if rank == 0 and world == 1 and not args.no_configs:
        eng1 = DecodeEngine(w)
        extra["config1_b1"] = measure_b1(eng1, cfg, dev, stream, torch, prompt_cfg1(), 128,
                                         "config 1: B=1, 16-token prompt, greedy positions 16..143")
        extra["config1_b1"]["e2e"] = measure_b1_e2e(eng1, dev, stream, torch, prompt_cfg1(), 128)
        extra["config2_b1_long"] = measure_b1(eng1, cfg, dev, stream, torch, prompt_cfg2(), 128,
                                              "config 2: B=1, 384-token prompt, greedy positions 384..511")
        kvp = eng1.new_kv()
        for _ in range(3):
            eng1.prefill(prompt_cfg2(), kvp)
        pf_ms = events_ms(lambda: [eng1.prefill(prompt_cfg2(), kvp) for _ in range(10)], stream, torch) / 10
        extra["config2_b1_long"]["prefill_384"] = {"ms": pf_ms, "tok_s": 384 / (pf_ms / 1000),
                                                   "how": "b2d_prefill, one 384-row pass, CUDA events"}
        eng1.close()
        eng3 = DecodeEngine(w, max_batch=64)
        extra["config3_paged_b64"] = measure_cfg3(eng3, cfg, torch)
        extra["config4_sampled_b8"] = measure_cfg4(eng3, cfg, torch)
        eng3.close()
        torch.cuda.empty_cache()
        extra["config5_one_wave"] = measure_one_wave(w, cfg, torch)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_serve(args.cpu_sample_steps)
        if "config1_b1" in extra:
            extra["config1_b1"]["cpu_baseline"] = cpu_baseline_b1(16)

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    launches = per_wave * n_waves * args.steps
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.02) bf16 weights, seeded prompts; no checkpoint on the box)",
        "config": serve_config(world),
        "gpu_launches": launches,
        "rank_ms_per_step": [m / args.steps for m in rank_ms],
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": f"{peak_kind} hbm_gbs", "scope": f"whole batched step per GPU ({per_wave} "
                     "kernels per wave: projections on tcgen05 with RMSNorm folded in, paged attention, embedding, argmax)",
                     "traffic": serve_traffic * n_waves if serve_traffic else None,
                     "traffic_source": "profiles/paged_step_b256_pos80.md (one wave-step of 256 at position 80, "
                                       "x waves)",
                     "algorithmic_bytes_per_step": alg_step},
        "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": 8 * n_seq,
                "d2h_bytes_per_step": 4 * n_seq, "steps": ne,
                "note": "per wave: pinned H2D of tokens+positions, b2d_decode_step_paged (replayed from its "
                        "cached step graph after 2 untimed warm-up steps), D2H next tokens; one sync per step; "
                        "positions spread over 64..319 like the device-timed steps"},
        "clocks": clk,
    }
    line.update(extra)
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
