"""Profile the decode kernels (the reference's ``profile_kernels.py`` for this
engine).

    python profile_kernels.py                         # B=1 megakernel, config 1
    python profile_kernels.py --mode paged --batch 256 --pos 64
    python profile_kernels.py --weights weights.pkl   # a trained checkpoint

``measure_decode`` and ``compute_memory_stats`` keep the reference's names,
arguments and results (``profile_kernels.py:44-87``): a host loop of
``multi_sm_decode_nlayer`` calls with an ``int()`` read per token, median of
``n_runs``, and the reference's theoretical memory figures.  The roofline line
uses this engine's algorithmic bytes (weights once, the KV rows actually read,
one row written) and the measured HBM copy bandwidth.

``--mode mixed`` times one fused pass of the batcher (decode rows plus prompt
rows in one ``b2d_prefill_rows`` call), the small case for its ncu captures.

``--mode serve`` runs the continuous batcher (``transformer_b200.serve``) on
a stream of requests and reports generated tokens per second, wall-clock.

``--mode sample`` times B=--batch top-p draws of the device sampler (both
kernels) with their phase stamps.

``--mode paged-att-trace`` times the attention's phases per unit inside the
captured batched step (its global-timer stamps).

``--mode paged`` runs the batched step over a paged KV pool with every
sequence at ``--pos`` (the pool holds zeros: the step's work does not depend
on the cached values), launched eagerly ``--warmup`` + ``--steps`` times; it is
the small, self-contained case the ncu captures use.

Without ``--weights`` the model is the seeded synthetic 306M decoder
(N(0,0.02) bf16 weights, seed 0); with it, a reference checkpoint
(``{"params": ..., "config": ...}`` as written by the reference's trainer,
``generate.py:161-164``) is packed instead.
"""

from __future__ import annotations

import argparse
import json
import os
import pickle
import sys
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)


def load_params(path):
    """``profile_kernels.py:21-25``: a pickled checkpoint's params and config."""
    with open(path, "rb") as f:
        saved = pickle.load(f)
    params = {k: np.asarray(v) for k, v in saved["params"].items()}
    return params, saved["config"]


def measure_prefill(w, config, prompt, n_runs=20):
    """``profile_kernels.py:28-41``: median latency (ms) of a prefill of
    ``prompt`` (the device prefill, ``b2d_prefill``) after 3 warm-ups;
    returns (ms, last-position logits, kv cache)."""
    import torch

    from transformer_b200.multi_sm_decode import engine_for
    eng = engine_for(w)
    kv = eng.new_kv()
    for _ in range(3):
        logits = eng.prefill(prompt, kv)
    torch.cuda.synchronize()
    times = []
    for _ in range(n_runs):
        t0 = time.perf_counter()
        logits = eng.prefill(prompt, kv)
        torch.cuda.synchronize()
        times.append(time.perf_counter() - t0)
    return float(np.median(times)) * 1000, logits, kv


def measure_decode(w, config, tok, start_pos, kv_packed, n_tokens=128, n_runs=10):
    """``profile_kernels.py:44-64``: median wall time (ms) of ``n_tokens``
    greedy steps through ``multi_sm_decode_nlayer`` with a host read of every
    token, after 5 warm-up steps; returns (ms, tokens of the last run)."""
    from transformer_b200.multi_sm_decode import multi_sm_decode_nlayer
    kv_tmp = kv_packed.clone()
    t = tok
    for i in range(5):
        t, _, kv_tmp = multi_sm_decode_nlayer(w, config, t, start_pos + i, kv_tmp)
        _ = int(t)
    times, all_tokens = [], []
    for _ in range(n_runs):
        kv_tmp.copy_(kv_packed)
        t = tok
        tokens = []
        t0 = time.perf_counter()
        for i in range(n_tokens):
            t, _, kv_tmp = multi_sm_decode_nlayer(w, config, t, start_pos + i, kv_tmp)
            tokens.append(int(t))
        times.append(time.perf_counter() - t0)
        all_tokens = tokens
    return float(np.median(times)) * 1000, all_tokens


def compute_memory_stats(config):
    """``profile_kernels.py:67-87``: theoretical weight and KV sizes (MB)."""
    c = config if isinstance(config, dict) else config.as_dict()
    d, n_layers, d_head, ctx = c["d_model"], c["n_layers"], c["d_head"], c["context_len"]
    n_kv_heads = c.get("n_kv_heads", c["n_heads"])
    d_kv = n_kv_heads * d_head
    d_ff = c.get("d_ff", 4 * d)
    per_layer = d + d * d + d * d_kv + d * d_kv + d * d + d + d * d_ff + d * d_ff + d_ff * d
    weight_bytes = (c["vocab_size"] * d + n_layers * per_layer + d) * 2
    kv_total = n_layers * 2 * n_kv_heads * ctx * d_head * 2
    return {"weight_buffer_mb": weight_bytes / 1e6, "kv_cache_mb": kv_total / 1e6,
            "total_inference_mb": (weight_bytes + kv_total) / 1e6}


def hbm_peak():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profile_b1(w, cfg, args, torch):
    from transformer_b200.multi_sm_decode import engine_for
    from transformer_b200.synth import prompt_cfg1, prompt_cfg2
    eng = engine_for(w)
    if args.plain_launch:  # a profiler cannot replay the cooperative launch
        eng.debug_tune(plain_launch=True)
    prefill_ms, _, _ = measure_prefill(w, cfg, prompt_cfg2(cfg)[:min(384, cfg.context_len - 1)], args.n_runs)
    prompt = prompt_cfg1(cfg)
    kv = eng.new_kv()
    first = eng.prefill(prompt, kv)
    tok = int(torch.argmax(first).item())
    ms, tokens = measure_decode(w, cfg, tok, len(prompt), kv, args.gen_len, args.n_runs)
    us = ms * 1000 / args.gen_len
    alg = float(np.mean([cfg.step_bytes([len(prompt) + i]) for i in range(args.gen_len)]))
    peak, kind = hbm_peak()
    return {"mode": "b1", "gen_len": args.gen_len, "prefill_384_ms": prefill_ms, "host_loop_us_per_token": us,
            "tok_s": 1e6 / us, "hbm_frac_host_loop": alg / (us * 1e-6) / 1e9 / peak,
            "peak_gbs": peak, "peak_source": kind, "first_tokens": tokens[:8]}


# Phases of the cluster kernel's per-layer stamps (slot pairs; `head` = only
# the CTAs of head clusters run the phase).  Slot numbers follow the stamps in
# csrc/decode_b1c.cuh.
_B1C_PHASES = [
    ("H gather + RMSNorm1 + q/k/v GEMV + push", 0, 1, True),
    ("q/k/v exchange (cluster)", 1, 2, True),
    ("attention: RoPE", 2, 10, True),
    ("attention: scores + softmax", 10, 11, True),
    ("attention: P.V (+ later passes)", 11, 12, True),
    ("attention: warp merge + K/V append + push", 12, 3, True),
    ("partial exchange + merge (cluster)", 3, 4, True),
    ("Wo GEMV + HM adds", 4, 5, True),
    ("HM gather + RMSNorm2 + gate/up GEMV + SwiGLU", 6, 7, False),
    ("Wd partial + push", 7, 8, False),
    ("cluster reduce + H adds", 8, 9, False),
]


def profile_b1_trace(w, cfg, args, torch):
    """Per-phase timing of the B=1 step from the kernel's global-timer stamps
    (b2d_debug_trace): per layer (layers 2..L-2), per phase, the critical
    increment (latest CTA at the phase end minus latest at its start) and
    the mean per-CTA duration; the stamped kernel is ~8% slower than the
    plain one."""
    from transformer_b200.multi_sm_decode import DecodeEngine, _ptr
    from transformer_b200.synth import prompt_cfg1
    eng = DecodeEngine(w)
    kv = eng.new_kv()
    eng.prefill(prompt_cfg1(cfg), kv)
    tok = torch.tensor([5], dtype=torch.int32, device=eng.device)
    pos = torch.tensor([args.pos], dtype=torch.int32, device=eng.device)
    for _ in range(3):
        eng.step(tok, pos, kv, eng.logits, eng.next_tok)
    per, nl = 13, cfg.n_layers
    stride = eng.trace_slots()
    buf = torch.zeros(eng.grid, stride, dtype=torch.int64, device=eng.device)
    eng.lib.b2d_debug_trace(eng.ws, _ptr(buf), stride)
    eng.step(tok, pos, kv, eng.logits, eng.next_tok)
    torch.cuda.synchronize()
    eng.lib.b2d_debug_trace(eng.ws, None, 0)
    eng.check_device()
    t = buf.cpu().numpy().astype(np.int64)
    nh = 4 * cfg.n_heads
    layers = range(2, nl - 1)
    phases = {}
    for name, a, b, head in _B1C_PHASES:
        rows = slice(0, nh) if head else slice(None)
        crit = np.mean([(t[rows, 1 + l * per + b].max() - t[rows, 1 + l * per + a].max()) / 1e3 for l in layers])
        mean = np.mean([np.mean(t[rows, 1 + l * per + b] - t[rows, 1 + l * per + a]) / 1e3 for l in layers])
        phases[name] = {"crit_us": round(float(crit), 2), "mean_us": round(float(mean), 2)}
    tf = 1 + nl * per
    layer = np.mean([(t[:, 1 + l * per + 9].max() - t[:, 1 + (l - 1) * per + 9].max()) / 1e3 for l in layers])
    return {"mode": "b1-trace", "pos": args.pos, "grid": eng.grid, "layer_us": round(float(layer), 2),
            "phases": phases,
            "final_gather_norm_us": round(float((t[:, tf].max() - t[:, 1 + (nl - 1) * per + 9].max()) / 1e3), 2),
            "logits_argmax_us": round(float((t[:, tf + 1].max() - t[:, tf].max()) / 1e3), 2),
            "step_us_stamped": round(float((t[:, tf + 2].max() - t[:, 0].min()) / 1e3), 1)}


def profile_paged(w, cfg, args, torch):
    from transformer_b200.batched import BatchedDecoder
    from transformer_b200.multi_sm_decode import DecodeEngine
    eng = DecodeEngine(w, max_batch=max(2, args.batch))
    if args.att_splits:
        eng.debug_tune(att_cpc=args.att_splits)  # attention units per (sequence, kv head); 0 = automatic
    dec = BatchedDecoder(eng, args.batch, seed=args.batch)
    dec.pos.fill_(args.pos)
    dec.tok.copy_(torch.randint(0, cfg.vocab_size, (args.batch,), dtype=torch.int32))
    for _ in range(args.warmup):
        dec.step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        dec.step()
    e1.record()
    torch.cuda.synchronize()
    eng.check_device()
    us = e0.elapsed_time(e1) * 1000 / args.steps
    alg = cfg.step_bytes([args.pos] * args.batch)
    peak, kind = hbm_peak()
    return {"mode": "paged", "batch": args.batch, "pos": args.pos, "steps": args.steps, "att_splits": args.att_splits,
            "us_per_step": us, "tok_s": args.batch * 1e6 / us, "algorithmic_bytes_per_step": alg,
            "hbm_frac": alg / (us * 1e-6) / 1e9 / peak, "peak_gbs": peak, "peak_source": kind}


def profile_paged_att_trace(w, cfg, args, torch):
    """Per-unit phase times of the attention inside the captured batched step
    (graph replay, every sequence at --pos): the units' global-timer stamps
    (b2d_debug_tune knob 9), median over units, mean over layers 2..n-2.
    Phases: issue (entry -> first pages requested), pdl_wait (-> the q/k/v
    projection finished), query (-> query fragments and the new K/V row),
    first_pair, rest_pairs, write, merge.  `after_input_us` is a unit's time
    from the projection's end to its result; `kv_bytes` the pages read."""
    import numpy as np
    from transformer_b200.batched import BatchedDecoder
    from transformer_b200.multi_sm_decode import DecodeEngine
    eng = DecodeEngine(w, max_batch=max(2, args.batch))
    if args.att_splits:
        eng.debug_tune(att_cpc=args.att_splits)  # attention units per (sequence, kv head); 0 = automatic
    units = 8192
    dec = BatchedDecoder(eng, args.batch, seed=args.batch)
    dec.pos.fill_(args.pos)
    dec.tok.copy_(torch.randint(0, cfg.vocab_size, (args.batch,), dtype=torch.int32))
    buf = torch.zeros(cfg.n_layers * units * 8, dtype=torch.int64, device="cuda")
    eng.debug_tune(att_trace=buf)
    try:
        dec.capture()
        for _ in range(max(args.warmup, 1)):
            dec.pos.fill_(args.pos)
            dec.replay()
        torch.cuda.synchronize()
        buf.zero_()
        dec.pos.fill_(args.pos)
        dec.replay()
        torch.cuda.synchronize()
        eng.check_device()
        t = buf.view(cfg.n_layers, units, 8).cpu().numpy().astype(np.int64)
    finally:
        eng.debug_tune(att_trace=torch.zeros(0, dtype=torch.int64))
        dec.release()
    names = ["issue", "pdl_wait", "query", "first_pair", "rest_pairs", "write", "merge"]
    ph = {n: [] for n in names}
    after, span, n_units = [], [], 0
    for layer in range(2, cfg.n_layers - 1):
        s = t[layer]
        s = s[s[:, 0] > 0]
        n_units = int(s.shape[0])
        for k, n in enumerate(names):
            ph[n].append(float(np.median(s[:, k + 1] - s[:, k])) / 1e3)
        after.append(float(np.median(s[:, 7] - s[:, 2])) / 1e3)
        span.append(float(s[:, 7].max() - s[:, 2].min()) / 1e3)
    pages = (args.pos // 16 + 1) * 16
    kv_bytes = args.batch * cfg.n_kv_heads * pages * 2 * cfg.d_head * 2
    after_us = float(np.mean(after))
    span_us = float(np.mean(span))
    peak, kind = hbm_peak()
    return {"mode": "paged-att-trace", "batch": args.batch, "pos": args.pos, "att_splits": args.att_splits,
            "units": n_units,
            "median_phase_us": {n: round(float(np.mean(v)), 2) for n, v in ph.items()},
            "after_input_us": round(after_us, 2),
            "first_input_to_last_result_us": round(span_us, 2), "kv_bytes": kv_bytes,
            "hbm_frac_after_input": round(kv_bytes / (span_us * 1e-6) / 1e9 / peak, 3),
            "peak_gbs": peak, "peak_source": kind}


def profile_sample(w, cfg, args, torch):
    """B = --batch top-p draws (T 0.7, top-p 0.95, rep 1.2, 100-token
    histories) on seeded N(0, s^2) logits, s = 0.3 (flat: ~28,400 tokens
    kept), 1.0 and 3.0: microseconds per b2d_sample call (CUDA events, --steps
    calls after --warmup) and the phase stamps (b2d_debug_tune knob 10) of
    one more call, for each kernel choice (knob 13: automatic, clusters of 8,
    one CTA per sequence)."""
    import numpy as np
    from transformer_b200.generate import Sampler
    from transformer_b200.multi_sm_decode import DecodeEngine
    B = args.batch
    eng = DecodeEngine(w, max_batch=max(2, B))
    smp = Sampler(eng, B, 256)
    rng = np.random.default_rng(1)
    hist = torch.from_numpy(rng.integers(0, cfg.vocab_size, (B, 100)).astype(np.int32))
    smp.history[:, :100].copy_(hist)
    smp.hist_len.fill_(100)
    smp.uniforms.copy_(torch.from_numpy(rng.random(B)))
    names = ["exp", "normalise", "sort", "cutoff", "draw"]
    out = []
    labels = {0: "automatic (clusters of 16 where they fit, else 8)", 2: "cluster of 8 CTAs per sequence",
              1: "one CTA per sequence"}
    for mode in (0, 2, 1):
        eng.debug_tune(sample_mode=mode)
        for sigma in (0.3, 1.0, 3.0):
            lg = torch.from_numpy((rng.standard_normal((B, cfg.vocab_size)) * sigma).astype(np.float32)).cuda()
            for _ in range(args.warmup):
                smp.sample(lg, 0.7, 0.95, 1.2, B)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.steps):
                smp.sample(lg, 0.7, 0.95, 1.2, B)
            e1.record()
            torch.cuda.synchronize()
            buf = torch.zeros(B, 8, dtype=torch.int64, device="cuda")
            eng.debug_tune(sample_trace=buf)
            smp.sample(lg, 0.7, 0.95, 1.2, B)
            torch.cuda.synchronize()
            eng.debug_tune(sample_trace=torch.zeros(0, dtype=torch.int64))
            t = buf.cpu().numpy().astype(np.int64)
            out.append({"kernel": labels[mode],
                        "sigma": sigma, "us_per_call": round(e0.elapsed_time(e1) * 1000 / args.steps, 1),
                        "phases_us": {n: round(float(np.mean(t[:, i + 1] - t[:, i])) / 1e3, 1)
                                      for i, n in enumerate(names)},
                        "kept_mean": float(np.mean(t[:, 6] & 0xffffffff))})
    eng.debug_tune(sample_mode=0)
    eng.check_device()
    return {"mode": "sample", "batch": B, "results": out}


def profile_mixed(w, cfg, args, torch):
    """One fused pass of the continuous batcher, timed alone: ``--batch``
    decode rows at position ``--pos`` plus ``--prompts`` prompts of
    ``--prompt-len`` rows, one ``b2d_prefill_rows`` call, eager launches
    (``--warmup`` + ``--steps`` times; each pass rewrites the same cache
    rows, so every pass does the same work)."""
    from transformer_b200.multi_sm_decode import DecodeEngine
    from transformer_b200.serve import PAGE_TOKENS
    eng = DecodeEngine(w, max_batch=max(2, args.batch))
    bps = (cfg.context_len + PAGE_TOKENS - 1) // PAGE_TOKENS
    n_seq = args.batch + args.prompts
    npg = max(args.pos // PAGE_TOKENS + 1, (args.prompt_len + PAGE_TOKENS - 1) // PAGE_TOKENS)
    pool = eng.new_kv_pool(n_seq * npg)  # only the pages the rows reach
    rng = np.random.default_rng(7)
    table = np.zeros((n_seq, bps), np.int32)
    table[:, :npg] = rng.permutation(n_seq * npg).astype(np.int32).reshape(n_seq, npg)
    tok, pos, tab = [], [], []
    for j in range(args.prompts):  # prompt rows but the last (body)
        s_ = args.batch + j
        tok += list(rng.integers(0, cfg.vocab_size, args.prompt_len - 1))
        pos += list(range(args.prompt_len - 1))
        tab += [table[s_]] * (args.prompt_len - 1)
    for b in range(args.batch):  # decode rows (tail)
        tok.append(int(rng.integers(0, cfg.vocab_size)))
        pos.append(args.pos)
        tab.append(table[b])
    for j in range(args.prompts):  # each prompt's last row (tail)
        tok.append(int(rng.integers(0, cfg.vocab_size)))
        pos.append(args.prompt_len - 1)
        tab.append(table[args.batch + j])
    n, n_out = len(tok), args.batch + args.prompts
    d_tok = torch.tensor(tok, dtype=torch.int32, device="cuda")
    d_pos = torch.tensor(pos, dtype=torch.int32, device="cuda")
    d_tab = torch.from_numpy(np.stack(tab)).to("cuda")
    nxt = torch.zeros(n_out, dtype=torch.int32, device="cuda")
    for _ in range(args.warmup):
        eng.prefill_rows(d_tok, d_pos, pool, d_tab, n_out, next_tok=nxt)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        eng.prefill_rows(d_tok, d_pos, pool, d_tab, n_out, next_tok=nxt)
    e1.record()
    torch.cuda.synchronize()
    eng.check_device()
    us = e0.elapsed_time(e1) * 1000 / args.steps
    return {"mode": "mixed", "rows": n, "decode_rows": args.batch, "pos": args.pos, "prompts": args.prompts,
            "prompt_len": args.prompt_len, "us_per_pass": us, "launches": eng.lib.b2d_batched_launches(eng.ws)}


def profile_serve(w, cfg, args, torch):
    """Continuous batching (``transformer_b200.serve``): ``--requests``
    requests (greedy, or a ``--sampled-frac`` share sampled with config 4's
    parameters) with ``--prompt-len``-token prompts and generation lengths
    uniform in [--gen-min, --gen-max] (seeded), ``--batch`` slots over a pool
    of ``--num-blocks`` pages (default: enough for every slot's longest
    sequence).  Wall-clock over the whole run (host scheduling, chunked
    prefills, decode steps, one token read-back per step) after a warm-up run
    of one request per slot."""
    from transformer_b200.multi_sm_decode import DecodeEngine
    from transformer_b200.serve import PAGE_TOKENS, ContinuousBatcher
    eng = DecodeEngine(w, max_batch=max(2, args.batch))
    rng = np.random.default_rng(5)
    longest = args.prompt_len + args.gen_max - 1
    nb = args.num_blocks or args.batch * ((longest + PAGE_TOKENS - 1) // PAGE_TOKENS)
    cb = ContinuousBatcher(eng, args.batch, nb, admission=args.admission, fuse_prefill=not args.no_fuse,
                           pipeline=not args.no_pipeline, admit_batch=args.admit_batch or None)
    for _ in range(args.batch):
        cb.submit(rng.integers(0, cfg.vocab_size, args.prompt_len), 8)
    cb.run()
    cb.stats.clear()
    cb.times.clear()
    gens = rng.integers(args.gen_min, args.gen_max + 1, args.requests)
    sampled = rng.random(args.requests) < args.sampled_frac  # config 4's parameters, a seed per request
    rids = [cb.submit(rng.integers(0, cfg.vocab_size, args.prompt_len), int(g),
                      **(dict(temperature=0.7, top_p=0.95, rep_penalty=1.2, seed=i) if sampled[i] else {}))
            for i, g in enumerate(gens)]
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    out = cb.run()
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    eng.check_device()
    n_tok = sum(len(out[r]) for r in rids)
    assert n_tok == int(gens.sum())
    st = dict(cb.stats)
    return {"mode": "serve", "requests": args.requests, "slots": args.batch, "num_blocks": nb,
            "prompt_len": args.prompt_len, "gen": [args.gen_min, args.gen_max], "seconds": dt,
            "generated_tok_s": n_tok / dt, "generated_tokens": n_tok,
            "prompt_tok_s": args.requests * args.prompt_len / dt, "steps": st.get("steps", 0),
            "mean_rows_per_step": (n_tok - args.requests) / max(1, st.get("steps", 1)),
            "prefill_calls": st.get("prefill_calls", 0), "prefill_rows": st.get("prefill_rows", 0),
            "mixed_steps": st.get("mixed_steps", 0), "pipelined_steps": st.get("pipelined_steps", 0),
            "preemptions": st.get("preemptions", 0), "admission": args.admission,
            "fuse_prefill": not args.no_fuse, "pipeline": not args.no_pipeline, "admit_batch": cb.admit_batch,
            "sampled_requests": int(sampled.sum()),
            "seconds_by_pass": {k: round(v, 4) for k, v in cb.times.items()}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", choices=["b1", "b1-trace", "paged", "paged-att-trace", "sample", "serve", "mixed"],
                    default="b1")
    ap.add_argument("--prompts", type=int, default=4)
    ap.add_argument("--att-splits", type=int, default=0,
                    help="--mode paged / paged-att-trace: force 1, 2 or 4 attention units")
    ap.add_argument("--requests", type=int, default=1024)
    ap.add_argument("--prompt-len", type=int, default=64)
    ap.add_argument("--gen-min", type=int, default=32)
    ap.add_argument("--gen-max", type=int, default=256)
    ap.add_argument("--num-blocks", type=int, default=0)
    ap.add_argument("--admission", choices=["reserve", "optimistic"], default="reserve")
    ap.add_argument("--no-fuse", action="store_true", help="prefill admitted prompts in passes of their own")
    ap.add_argument("--no-pipeline", action="store_true", help="read every decode step's tokens before the next")
    ap.add_argument("--admit-batch", type=int, default=0, help="free slots that trigger an admission (0: default)")
    ap.add_argument("--sampled-frac", type=float, default=0.0,
                    help="--mode serve: fraction of requests sampled (T 0.7, top-p 0.95, rep 1.2)")
    ap.add_argument("--plain-launch", action="store_true",
                    help="--mode b1: launch the B=1 cluster grid without the cooperative attribute (for ncu)")
    ap.add_argument("--gen-len", type=int, default=128)
    ap.add_argument("--n-runs", type=int, default=10)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--pos", type=int, default=64)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--weights", default=None, help="reference checkpoint (pickle with params and config)")
    args = ap.parse_args()

    import torch

    from transformer_b200.config import CONFIG_306M, ModelConfig
    from transformer_b200.packing import prepare_decode_weights_nlayer
    from transformer_b200.synth import synth_params
    if args.weights:
        params, config = load_params(args.weights)
        cfg = ModelConfig.from_dict(config)
    else:
        cfg = CONFIG_306M
        params = synth_params(cfg, 0)
    w = prepare_decode_weights_nlayer(params, cfg, device="cuda")
    out = {"memory": compute_memory_stats(cfg)}
    prof = {"b1": profile_b1, "b1-trace": profile_b1_trace, "paged": profile_paged,
            "paged-att-trace": profile_paged_att_trace, "sample": profile_sample, "serve": profile_serve,
            "mixed": profile_mixed}[args.mode]
    out.update(prof(w, cfg, args, torch))
    print(json.dumps(out))
    return 0


if __name__ == "__main__":
    sys.exit(main())
