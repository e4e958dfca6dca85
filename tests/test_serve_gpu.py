"""GPU: prefill into the paged pool (b2d_prefill_paged) and the continuous
batcher over it.

* The paged prefill runs the same kernels over the same rows as the
  contiguous prefill (only the cache addressing differs), so its logits, its
  argmax and every cache row it writes are bit-identical to b2d_prefill's.
* b2d_prefill_rows (rows of several sequences per call, a long prompt over
  two calls) against the oracle: last-row logits, argmax and cache rows.
* The batcher's greedy streams are checked teacher-forced against the float32
  oracle (argmax equal wherever the oracle's top-2 margin allows), through
  slot refill and preemption; its sampled streams against the CPU sampler on
  the very logits the device sampled from, with each request's uniforms in
  the order its own seeded RandomState draws them."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import MARGIN, assert_logits_close
from oracle import sampler as OS
from oracle.ref_forward import CachedDecoder, top2
from transformer_b200.serve import PAGE_TOKENS, ContinuousBatcher

pytestmark = pytest.mark.gpu


def _paged_vs_contiguous(eng, cfg, chunks, seed):
    """Prefill the prompt pieces `chunks` (start positions follow on) both
    ways; compare logits, argmax and every written cache row bitwise."""
    dev = eng.device
    rng = np.random.default_rng(seed)
    n = sum(chunks)
    bps = (cfg.context_len + PAGE_TOKENS - 1) // PAGE_TOKENS
    nb = bps + 5
    row = rng.permutation(nb)[:bps].astype(np.int32)
    pool = eng.new_kv_pool(nb)
    row_d = torch.from_numpy(row).to(dev)
    kv = eng.new_kv()
    prompt = rng.integers(0, cfg.vocab_size, n).astype(np.int32)
    nt_p = torch.zeros(1, dtype=torch.int32, device=dev)
    start = 0
    for c in chunks:
        lg_c = eng.prefill(prompt[start:start + c], kv, start).clone()
        nt_c = int(eng.next_tok[0].item())
        lg_p = eng.prefill_paged(prompt[start:start + c], pool, row_d, start, next_tok=nt_p).clone()
        assert torch.equal(lg_c, lg_p), f"logits differ after chunk ending at {start + c}"
        assert int(nt_p[0].item()) == nt_c
        start += c
    eng.check_device()
    L, KVH, ctx = cfg.n_layers, cfg.n_kv_heads, cfg.context_len
    cont = kv[:L * 2 * KVH * ctx * cfg.d_head].view(L, 2, KVH, ctx, cfg.d_head)
    pos = np.arange(n)
    blk = torch.from_numpy(row[pos // PAGE_TOKENS].astype(np.int64)).to(dev)
    slot = torch.from_numpy(pos % PAGE_TOKENS).to(dev)
    paged = pool[:, blk, :, :, slot, :]            # [n, L, 2, KVH, dh]
    assert torch.equal(paged.permute(1, 2, 3, 0, 4), cont[:, :, :, :n, :])
    untouched = torch.ones(nb, dtype=torch.bool, device=dev)
    untouched[torch.from_numpy(row[:(n + PAGE_TOKENS - 1) // PAGE_TOKENS].astype(np.int64)).to(dev)] = False
    assert torch.count_nonzero(pool[:, untouched]) == 0
    return prompt, lg_p


@pytest.mark.parametrize("chunks", [[1], [37], [128], [20, 17, 1]])
def test_prefill_paged_tiny_equals_contiguous(engine_tiny, params_tiny, chunks):
    from transformer_b200.config import CONFIG_TINY as cfg
    from transformer_b200.synth import params_f32
    prompt, lg = _paged_vs_contiguous(engine_tiny, cfg, chunks, 700 + sum(chunks))
    dec = CachedDecoder(params_f32(params_tiny), cfg, 1)
    for p, t in enumerate(prompt):
        ref = dec.step([t], [p])[0]
    assert_logits_close(lg.cpu().numpy(), ref, "paged prefill")


def test_prefill_paged_306m_cfg2_equals_contiguous(engine306):
    """Config 2's 384-token prompt (one chunk) and the full 512-position
    context in two calls (500 + 12) on the 306M model."""
    from transformer_b200.config import CONFIG_306M as cfg
    _paged_vs_contiguous(engine306, cfg, [384], 2)
    _paged_vs_contiguous(engine306, cfg, [500, 12], 3)


def test_prefill_rows_several_sequences(engine_tiny_batched, params_tiny):
    """b2d_prefill_rows over rows of several sequences in two calls: call 1
    holds prompts A (37) and C (1) whole and the first 60 positions of B
    (100), call 2 the rest of B and D (128, the full tiny context); each
    call's tail holds the last rows of the prompts it completes.  Their
    logits and argmax, and every cache row, against the oracle."""
    from transformer_b200.config import CONFIG_TINY as cfg
    from transformer_b200.synth import params_f32
    P = params_f32(params_tiny)
    eng = engine_tiny_batched
    dev = eng.device
    rng = np.random.default_rng(808)
    bps = cfg.context_len // PAGE_TOKENS
    lens = {"A": 37, "B": 100, "C": 1, "D": 128}
    nb = sum(bps for _ in lens) + 3
    perm = rng.permutation(nb).astype(np.int32)
    tables = {k: perm[i * bps:(i + 1) * bps] for i, k in enumerate(lens)}
    prompts = {k: rng.integers(0, cfg.vocab_size, n).astype(np.int32) for k, n in lens.items()}
    pool = eng.new_kv_pool(nb)

    def rows_of(k, lo, hi):
        return [(int(prompts[k][p]), p, k) for p in range(lo, hi)]

    calls = [
        (rows_of("A", 0, 36) + rows_of("B", 0, 60), rows_of("A", 36, 37) + rows_of("C", 0, 1)),
        (rows_of("D", 0, 127) + rows_of("B", 60, 99), rows_of("B", 99, 100) + rows_of("D", 127, 128)),
    ]
    got = {}
    for body, tail in calls:
        rows = body + tail
        n, n_out = len(rows), len(tail)
        tok = torch.tensor([r[0] for r in rows], dtype=torch.int32, device=dev)
        pos = torch.tensor([r[1] for r in rows], dtype=torch.int32, device=dev)
        tab = torch.from_numpy(np.stack([tables[r[2]] for r in rows])).to(dev)
        lg = torch.zeros(n_out, cfg.vocab_size, dtype=torch.float32, device=dev)
        nt = torch.zeros(n_out, dtype=torch.int32, device=dev)
        eng.prefill_rows(tok, pos, pool, tab, n_out, lg, nt)
        for j, r in enumerate(tail):
            got[r[2]] = (lg[j].cpu().numpy(), int(nt[j].item()))
    eng.check_device()
    pool_np = pool.float().cpu().numpy()
    for k, pr in prompts.items():
        dec = CachedDecoder(P, cfg, 1)
        for p, t in enumerate(pr):
            ref = dec.step([t], [p])[0]
        assert_logits_close(got[k][0], ref, f"prompt {k}")
        i, _, margin = top2(ref)
        if margin > MARGIN:
            assert got[k][1] == i
        for p in range(len(pr)):
            blk, slot = tables[k][p // PAGE_TOKENS], p % PAGE_TOKENS
            for l in range(cfg.n_layers):
                np.testing.assert_allclose(pool_np[l, blk, 0, :, slot], dec.K[0, l, :, p], atol=2e-2, rtol=1e-2)
                np.testing.assert_allclose(pool_np[l, blk, 1, :, slot], dec.V[0, l, :, p], atol=2e-2, rtol=1e-2)


def test_prefill_paged_rejects_bad_arguments(engine_tiny):
    from transformer_b200.config import CONFIG_TINY as cfg
    dev = engine_tiny.device
    pool = engine_tiny.new_kv_pool(10)
    with pytest.raises(ValueError):  # runs past the table row (2 blocks = 32 positions)
        engine_tiny.prefill_paged(np.zeros(33, np.int32), pool, torch.zeros(2, dtype=torch.int32, device=dev))
    with pytest.raises(ValueError):
        engine_tiny.prefill_paged(np.zeros(4, np.int32), pool,
                                  torch.zeros(cfg.context_len // 16, dtype=torch.int64, device=dev))


def _teacher_forced_greedy(P, cfg, prompt, out):
    dec = CachedDecoder(P, cfg, 1)
    seq = list(prompt) + list(out[:-1])
    checked = 0
    for p, t in enumerate(seq):
        lg = dec.step([t], [p])[0]
        i = p - (len(prompt) - 1)
        if i >= 0:
            am, _, margin = top2(lg)
            if margin > MARGIN:
                assert out[i] == am, f"token {i}: {out[i]} vs oracle {am}"
                checked += 1
    return checked


@pytest.mark.parametrize("fuse,pipe", [(True, True), (False, True), (True, False)])
def test_batcher_greedy_tiny_vs_oracle(engine_tiny_batched, params_tiny, fuse, pipe):
    """12 requests through 4 slots over an 11-block pool (one 128-position
    context is 8 blocks), optimistic admission: slots refill as requests
    finish and requests are preempted and readmitted; prompts prefilled in
    fused passes with the decode rows, or on their own; decode steps
    pipelined (tokens fed back on the device) or not.  Every stream is
    checked against the oracle."""
    from transformer_b200.config import CONFIG_TINY as cfg
    from transformer_b200.synth import params_f32
    P = params_f32(params_tiny)
    rng = np.random.default_rng(21)
    cb = ContinuousBatcher(engine_tiny_batched, 4, 11, admission="optimistic", fuse_prefill=fuse,
                           pipeline=pipe)
    prompts = {}
    for _ in range(12):
        n = int(rng.integers(1, 90))
        g = int(rng.integers(1, cfg.context_len - n + 2))
        pr = rng.integers(0, cfg.vocab_size, n)
        prompts[cb.submit(pr, g)] = (pr, g)
    got = cb.run()
    engine_tiny_batched.check_device()
    assert cb.stats["preemptions"] > 0 and cb.pages.n_free == 11
    assert (cb.stats["pipelined_steps"] > 0) == pipe
    checked = 0
    for rid, (pr, g) in prompts.items():
        assert len(got[rid]) == g
        checked += _teacher_forced_greedy(P, cfg, pr, got[rid])
    assert checked > 200


def test_batcher_sampled_and_greedy_mixed(engine_tiny_batched):
    """Sampled requests (config 4's parameters, own seeds) next to greedy
    ones: each sampled token equals the CPU sampler's choice on the logits the
    device sampled from, with the request's history and its next uniform."""
    from transformer_b200.config import CONFIG_TINY as cfg
    rng = np.random.default_rng(44)
    cb = ContinuousBatcher(engine_tiny_batched, 4, 12)
    seeds = {}
    for k in range(8):
        n = int(rng.integers(1, 60))
        if k % 3 == 2:
            cb.submit(rng.integers(0, cfg.vocab_size, n), 40)
        else:
            rid = cb.submit(rng.integers(0, cfg.vocab_size, n), 40, temperature=0.7, top_p=0.95,
                            rep_penalty=1.2, seed=100 + k)
            seeds[rid] = 100 + k
    drawn = {rid: [] for rid in seeds}
    mismatches = []
    orig = cb._sample_rows

    def recording(logits, rows, greedy_src):
        rows = list(rows)
        lg = logits[:len(rows)].float().cpu().numpy().copy()
        pre = []
        for r in rows:
            if r is not None and not r.greedy:
                st = r.rng.get_state()
                u = np.random.RandomState()
                u.set_state(st)
                pre.append((r, list(r.out), float(u.random_sample())))
            else:
                pre.append(None)
        out = orig(logits, rows, greedy_src)
        for i, item in enumerate(pre):
            if item is None:
                continue
            r, hist, u = item
            drawn[r.rid].append(u)
            want = OS.sample_token(lg[i], r.temperature, r.top_p, r.rep_penalty, hist, u)
            if int(out[i]) != want:
                mismatches.append((r.rid, len(hist), int(out[i]), want))
        return out

    cb._sample_rows = recording
    got = cb.run()
    engine_tiny_batched.check_device()
    assert not mismatches, mismatches
    for rid, seed in seeds.items():
        assert len(got[rid]) == 40
        np.testing.assert_array_equal(drawn[rid], np.random.RandomState(seed).random_sample(40))
