"""GPU: the batched decode step over a paged KV pool (tensor-core projections,
paged attention) against the float32 oracle, teacher-forced.

Sequences are ingested raggedly: at step t sequence b is fed its token t while
t < len(b) and idles (pos = -1) afterwards, so every step mixes active and
idle rows; block tables are random permutations of the pool's blocks."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import MARGIN, assert_logits_close
from oracle.ref_forward import CachedDecoder, top2
from transformer_b200 import _lib
from transformer_b200.multi_sm_decode import PAGE_TOKENS

pytestmark = pytest.mark.gpu


def _table(rng, batch, bps, spare=3):
    nb = batch * bps + spare
    perm = rng.permutation(nb).astype(np.int32)
    return perm[:batch * bps].reshape(batch, bps), nb


def _run_ragged(eng, P, cfg, prompts, rng, check_every=1, check_kv=False):
    """Feed `prompts` (list of int arrays) raggedly; compare every active row
    with its own float32 oracle decoder.  Returns the max abs logit error."""
    dev = eng.device
    B = len(prompts)
    bps = (cfg.context_len + PAGE_TOKENS - 1) // PAGE_TOKENS
    table, nb = _table(rng, B, bps)
    pool = eng.new_kv_pool(nb)
    table_d = torch.from_numpy(table).to(dev)
    decs = [CachedDecoder(P, cfg, 1) for _ in range(B)]
    T = max(len(p) for p in prompts)
    tok = torch.zeros(B, dtype=torch.int32, device=dev)
    pos = torch.zeros(B, dtype=torch.int32, device=dev)
    logits = torch.zeros(B, cfg.vocab_size, dtype=torch.float32, device=dev)
    nxt = torch.zeros(B, dtype=torch.int32, device=dev)
    worst = 0.0
    for t in range(T):
        active = [b for b in range(B) if t < len(prompts[b])]
        tk = np.array([prompts[b][t] if t < len(prompts[b]) else 0 for b in range(B)], np.int32)
        ps = np.array([t if t < len(prompts[b]) else -1 for b in range(B)], np.int32)
        tok.copy_(torch.from_numpy(tk))
        pos.copy_(torch.from_numpy(ps))
        eng.step_paged(tok, pos, pool, table_d, logits, nxt)
        refs = {b: decs[b].step([tk[b]], [t])[0] for b in active}
        if t % check_every and t != T - 1:
            continue
        got = logits.cpu().numpy()
        am = nxt.cpu().numpy()
        for b in active:
            worst = max(worst, assert_logits_close(got[b], refs[b], f"seq {b} pos {t}"))
            i, _, margin = top2(refs[b])
            if margin > MARGIN:
                assert am[b] == i, f"seq {b} pos {t}: argmax {am[b]} vs {i}"
    eng.check_device()
    if check_kv:
        pool_np = pool.float().cpu().numpy()
        for b in range(B):
            for p in range(len(prompts[b])):
                blk, slot = table[b, p // PAGE_TOKENS], p % PAGE_TOKENS
                for l in range(cfg.n_layers):
                    np.testing.assert_allclose(pool_np[l, blk, 0, :, slot], decs[b].K[0, l, :, p],
                                               atol=2e-2, rtol=1e-2)
                    np.testing.assert_allclose(pool_np[l, blk, 1, :, slot], decs[b].V[0, l, :, p],
                                               atol=2e-2, rtol=1e-2)
    return worst


def test_paged_tiny_ragged_all_positions(engine_tiny_batched, params_tiny):
    """Tiny model, 6 ragged sequences up to the full context (128): every
    position of every active row checked, and the paged K/V contents."""
    from transformer_b200.config import CONFIG_TINY
    from transformer_b200.synth import params_f32
    rng = np.random.default_rng(11)
    lens = [128, 3, 40, 17, 77, 1]
    prompts = [rng.integers(0, CONFIG_TINY.vocab_size, n).astype(np.int32) for n in lens]
    _run_ragged(engine_tiny_batched, params_f32(params_tiny), CONFIG_TINY, prompts, rng, check_kv=True)


@pytest.mark.parametrize("cpc,ks", [(1, 1), (3, 2), (32, 8)])
def test_paged_tiny_work_splits(engine_tiny_batched, params_tiny, cpc, ks):
    """Forced attention units per (sequence, kv head) (1; 3 used as 2; 32
    capped at 4: uneven page shares and units without pages included) and K
    splits of the projections give the same parity."""
    from transformer_b200.config import CONFIG_TINY
    from transformer_b200.synth import params_f32
    eng = engine_tiny_batched
    rng = np.random.default_rng(200 + cpc)
    prompts = [rng.integers(0, CONFIG_TINY.vocab_size, n).astype(np.int32) for n in (128, 70, 9)]
    eng.debug_tune(att_cpc=cpc, ksplit=ks)
    try:
        _run_ragged(eng, params_f32(params_tiny), CONFIG_TINY, prompts, rng, check_every=7)
    finally:
        eng.debug_tune(att_cpc=0, ksplit=0)


@pytest.mark.parametrize("B", [2, 17, 33, 64])
def test_paged_tiny_batch_sizes(engine_tiny_batched, params_tiny, B):
    """Each projection tile width (16 / 32 / 64 rows) and a batch spanning
    two tiles."""
    from transformer_b200.config import CONFIG_TINY
    from transformer_b200.synth import params_f32
    rng = np.random.default_rng(100 + B)
    prompts = [rng.integers(0, CONFIG_TINY.vocab_size, int(rng.integers(1, 24))).astype(np.int32)
               for _ in range(B)]
    _run_ragged(engine_tiny_batched, params_f32(params_tiny), CONFIG_TINY, prompts, rng, check_every=5)


def test_paged_306m_ragged(engine306_batched, params306_f32):
    """306M, 4 ragged sequences (lengths 5..40) spanning several KV blocks."""
    from transformer_b200.config import CONFIG_306M
    rng = np.random.default_rng(12)
    prompts = [rng.integers(0, CONFIG_306M.vocab_size, n).astype(np.int32) for n in (40, 5, 23, 33)]
    _run_ragged(engine306_batched, params306_f32, CONFIG_306M, prompts, rng, check_every=4)


@pytest.mark.parametrize("B", [80, 224])
def test_paged_306m_96_row_tiles(engine306_batched, params306_f32, B):
    """96-row batch tiles: at 80 sequences the output projection takes them,
    at 224 the gate/up projection (its 64-row tiles would need a second
    wave).  Three positions; four rows against the oracle, all rows finite."""
    from transformer_b200.config import CONFIG_306M as cfg
    rng = np.random.default_rng(16 + B)
    eng = engine306_batched
    dev = eng.device
    T = 3
    table, nb = _table(rng, B, cfg.context_len // PAGE_TOKENS)
    pool = eng.new_kv_pool(nb)
    table_d = torch.from_numpy(table).to(dev)
    toks = rng.integers(0, cfg.vocab_size, (T, B)).astype(np.int32)
    checked = [0, 31, B // 2 + 7, B - 1]
    decs = {b: CachedDecoder(params306_f32, cfg, 1) for b in checked}
    tok = torch.zeros(B, dtype=torch.int32, device=dev)
    pos = torch.zeros(B, dtype=torch.int32, device=dev)
    logits = torch.zeros(B, cfg.vocab_size, dtype=torch.float32, device=dev)
    nxt = torch.zeros(B, dtype=torch.int32, device=dev)
    for t in range(T):
        tok.copy_(torch.from_numpy(toks[t].copy()))
        pos.fill_(t)
        eng.step_paged(tok, pos, pool, table_d, logits, nxt)
        got, am = logits.cpu().numpy(), nxt.cpu().numpy()
        assert np.isfinite(got).all()
        for b in checked:
            ref = decs[b].step([toks[t, b]], [t])[0]
            assert_logits_close(got[b], ref, f"row {b} pos {t}")
            i, _, margin = top2(ref)
            if margin > MARGIN:
                assert am[b] == i
    eng.check_device()


def test_paged_306m_640_rows_shallow_rings(engine306, params306_f32):
    """640 sequences (2560 attention units, far more than the warps that fit
    at once): the attention runs with shallower page rings.  Three positions;
    four rows against the oracle, all rows finite.  Each row owns one block
    (positions < 16 read only page 0)."""
    from transformer_b200.config import CONFIG_306M as cfg
    from transformer_b200.multi_sm_decode import DecodeEngine
    B, T = 640, 3
    eng = DecodeEngine(engine306.w, max_batch=B)
    try:
        dev = eng.device
        rng = np.random.default_rng(640)
        table = np.zeros((B, cfg.context_len // PAGE_TOKENS), np.int32)
        table[:, 0] = rng.permutation(B).astype(np.int32)
        pool = eng.new_kv_pool(B)
        table_d = torch.from_numpy(table).to(dev)
        toks = rng.integers(0, cfg.vocab_size, (T, B)).astype(np.int32)
        checked = [0, 97, 333, B - 1]
        decs = {b: CachedDecoder(params306_f32, cfg, 1) for b in checked}
        tok = torch.zeros(B, dtype=torch.int32, device=dev)
        pos = torch.zeros(B, dtype=torch.int32, device=dev)
        logits = torch.zeros(B, cfg.vocab_size, dtype=torch.float32, device=dev)
        nxt = torch.zeros(B, dtype=torch.int32, device=dev)
        for t in range(T):
            tok.copy_(torch.from_numpy(toks[t].copy()))
            pos.fill_(t)
            eng.step_paged(tok, pos, pool, table_d, logits, nxt)
            got, am = logits.cpu().numpy(), nxt.cpu().numpy()
            assert np.isfinite(got).all()
            for b in checked:
                ref = decs[b].step([toks[t, b]], [t])[0]
                assert_logits_close(got[b], ref, f"row {b} pos {t}")
                i, _, margin = top2(ref)
                if margin > MARGIN:
                    assert am[b] == i
        eng.check_device()
    finally:
        eng.close()


def test_paged_306m_long_context(engine306_batched, params306_f32):
    """306M, positions near the end of the 512 context (config 2's length):
    ingested without checks, then the last 8 positions compared."""
    from transformer_b200.config import CONFIG_306M
    cfg = CONFIG_306M
    rng = np.random.default_rng(13)
    eng = engine306_batched
    dev = eng.device
    B, n = 2, cfg.context_len
    bps = cfg.context_len // PAGE_TOKENS
    table, nb = _table(rng, B, bps)
    pool = eng.new_kv_pool(nb)
    table_d = torch.from_numpy(table).to(dev)
    prompts = rng.integers(0, cfg.vocab_size, (B, n)).astype(np.int32)
    dec = CachedDecoder(params306_f32, cfg, B)
    tok = torch.zeros(B, dtype=torch.int32, device=dev)
    pos = torch.zeros(B, dtype=torch.int32, device=dev)
    logits = torch.zeros(B, cfg.vocab_size, dtype=torch.float32, device=dev)
    for t in range(n):
        tok.copy_(torch.from_numpy(prompts[:, t].copy()))
        pos.fill_(t)
        eng.step_paged(tok, pos, pool, table_d, logits)
        ref = dec.step(prompts[:, t], [t] * B)
        if t >= n - 8:
            got = logits.cpu().numpy()
            for b in range(B):
                assert_logits_close(got[b], ref[b], f"seq {b} pos {t}")
    eng.check_device()


def test_paged_306m_attention_splits(engine306_batched, params306_f32):
    """Rows at ragged long positions (mid page, a page's last slot, the
    context end) with every attention split count forced in turn: the last
    step's logits match the float32 oracle (argmax where the margin allows)
    for each count, and re-running a step at the same position is harmless
    (the owner unit rewrites the same K/V)."""
    from transformer_b200.config import CONFIG_306M
    cfg = CONFIG_306M
    rng = np.random.default_rng(15)
    eng = engine306_batched
    dev = eng.device
    lens = [203, 336, cfg.context_len]  # last positions 202 (mid page), 335 (page end), 511
    B = len(lens)
    bps = cfg.context_len // PAGE_TOKENS
    table, nb = _table(rng, B, bps)
    pool = eng.new_kv_pool(nb)
    table_d = torch.from_numpy(table).to(dev)
    prompts = [rng.integers(0, cfg.vocab_size, n).astype(np.int32) for n in lens]
    tok = torch.zeros(B, dtype=torch.int32, device=dev)
    pos = torch.zeros(B, dtype=torch.int32, device=dev)
    logits = torch.zeros(B, cfg.vocab_size, dtype=torch.float32, device=dev)
    for t in range(max(lens) - 1):  # ragged ingestion up to each row's last position
        tok.copy_(torch.from_numpy(np.array([p[t] if t < len(p) - 1 else 0 for p in prompts], np.int32)))
        pos.copy_(torch.from_numpy(np.array([t if t < len(p) - 1 else -1 for p in prompts], np.int32)))
        eng.step_paged(tok, pos, pool, table_d, logits)
    refs = []
    for p in prompts:
        dec = CachedDecoder(params306_f32, cfg, 1)
        for t, tk in enumerate(p):
            r = dec.step([tk], [t])[0]
        refs.append(r)
    tok.copy_(torch.from_numpy(np.array([p[-1] for p in prompts], np.int32)))
    pos.copy_(torch.from_numpy(np.array([n - 1 for n in lens], np.int32)))
    nxt = torch.zeros(B, dtype=torch.int32, device=dev)
    try:
        for splits in (0, 1, 2, 4):
            eng.debug_tune(att_cpc=splits)
            eng.step_paged(tok, pos, pool, table_d, logits, nxt)
            got, am = logits.cpu().numpy(), nxt.cpu().numpy()
            for b in range(B):
                assert_logits_close(got[b], refs[b], f"splits {splits} row {b}")
                i, _, margin = top2(refs[b])
                if margin > MARGIN:
                    assert am[b] == i, f"splits {splits} row {b}: argmax {am[b]} vs {i}"
    finally:
        eng.debug_tune(att_cpc=0)
    eng.check_device()


def test_paged_matches_single_sequence_kernel(engine306_batched, engine306):
    """The batched path and the B=1 megakernel agree on the same sequence
    (both bf16 weights; activation rounding differs, so within tolerance)."""
    from transformer_b200.config import CONFIG_306M
    cfg = CONFIG_306M
    rng = np.random.default_rng(14)
    prompt = rng.integers(0, cfg.vocab_size, 24).astype(np.int32)
    kv = engine306.new_kv()
    ref = engine306.prefill(prompt, kv).cpu().numpy()
    eng = engine306_batched
    dev = eng.device
    table, nb = _table(rng, 1, cfg.context_len // PAGE_TOKENS)
    pool = eng.new_kv_pool(nb)
    table_d = torch.from_numpy(table).to(dev)
    logits = torch.zeros(2, cfg.vocab_size, dtype=torch.float32, device=dev)
    tok = torch.zeros(2, dtype=torch.int32, device=dev)
    pos = torch.full((2,), -1, dtype=torch.int32, device=dev)
    table2 = torch.cat([table_d, table_d])  # row 1 idles and never writes
    for t in range(len(prompt)):
        tok[0] = int(prompt[t])
        pos[0] = t
        eng.step_paged(tok, pos, pool, table2, logits)
    assert_logits_close(logits[0].cpu().numpy(), ref, "batched vs B=1 kernel")


def test_paged_step_bitwise_reproducible(engine306_batched):
    """Every reduction of the batched step has a fixed order (cluster split-K
    partials in rank order, attention partials in CTA order): the same step
    repeated gives bit-identical logits and cache rows."""
    from transformer_b200.config import CONFIG_306M as cfg
    eng = engine306_batched
    dev = eng.device
    rng = np.random.default_rng(21)
    B = 64
    table, nb = _table(rng, B, cfg.context_len // PAGE_TOKENS)
    table_d = torch.from_numpy(table).to(dev)
    pool = eng.new_kv_pool(nb)
    pool.copy_((torch.randn(pool.shape, generator=torch.Generator().manual_seed(3)) * 0.5).to(torch.bfloat16))
    tok = torch.from_numpy(rng.integers(0, cfg.vocab_size, B).astype(np.int32)).to(dev)
    pos = torch.from_numpy(rng.integers(0, 400, B).astype(np.int32)).to(dev)
    outs = []
    for _ in range(3):
        logits = torch.zeros(B, cfg.vocab_size, dtype=torch.float32, device=dev)
        nxt = torch.zeros(B, dtype=torch.int32, device=dev)
        eng.step_paged(tok, pos, pool, table_d, logits, nxt)
        outs.append((logits.clone(), nxt.clone(), pool.clone()))
    eng.check_device()
    for lg, nx, pl in outs[1:]:
        assert torch.equal(lg, outs[0][0]) and torch.equal(nx, outs[0][1]) and torch.equal(pl, outs[0][2])


def test_paged_step_graph_replay_matches_direct(engine306_batched):
    """b2d_decode_step_paged replays a cached CUDA graph from the second call
    with the same arguments: a greedy run through the cache (positions
    advanced in the same device buffer) equals a run with direct launches
    bit for bit, logits, tokens and cache rows."""
    from transformer_b200.config import CONFIG_306M as cfg
    eng = engine306_batched
    dev = eng.device
    rng = np.random.default_rng(22)
    B, steps = 16, 6
    table, nb = _table(rng, B, cfg.context_len // PAGE_TOKENS)
    table_d = torch.from_numpy(table).to(dev)
    shape = tuple(eng.new_kv_pool(nb).shape)
    base = (torch.randn(shape, generator=torch.Generator().manual_seed(5)) * 0.5).to(torch.bfloat16)
    tok0 = rng.integers(0, cfg.vocab_size, B).astype(np.int32)
    pos0 = rng.integers(0, 300, B).astype(np.int32)
    runs = []
    try:
        for graphs in (0, 1):
            eng.debug_tune(graphs=bool(graphs))
            pool = eng.new_kv_pool(nb)
            pool.copy_(base.to(dev))
            tok = torch.from_numpy(tok0).to(dev)
            pos = torch.from_numpy(pos0).to(dev)
            logits = torch.zeros(B, cfg.vocab_size, dtype=torch.float32, device=dev)
            out = []
            for _ in range(steps):
                eng.step_paged(tok, pos, pool, table_d, logits, tok)
                pos.add_(1)
                out.append((logits.clone(), tok.clone()))
            runs.append((out, pool.clone()))
    finally:
        eng.debug_tune(graphs=True)
    eng.check_device()
    (a, pa), (b, pb) = runs
    for i, ((la, ta), (lb, tb)) in enumerate(zip(a, b)):
        assert torch.equal(la, lb) and torch.equal(ta, tb), f"step {i}"
    assert torch.equal(pa, pb)


def test_paged_bad_inputs_set_status(engine_tiny_batched):
    """An out-of-range token or block-table entry is reported through the
    workspace status word (B2D_ERR_DEVICE_INPUT), not a fault."""
    eng = engine_tiny_batched
    cfg = eng.cfg
    dev = eng.device
    bps = cfg.context_len // PAGE_TOKENS
    pool = eng.new_kv_pool(2 * bps)
    table = torch.arange(2 * bps, dtype=torch.int32, device=dev).reshape(2, bps)
    tok = torch.tensor([1, 2], dtype=torch.int32, device=dev)
    pos = torch.tensor([0, 0], dtype=torch.int32, device=dev)
    eng.reset()
    eng.step_paged(tok, pos, pool, table)
    assert eng.last_error()[0] == _lib.B2D_OK
    bad_tok = torch.tensor([1, cfg.vocab_size], dtype=torch.int32, device=dev)
    eng.step_paged(bad_tok, pos, pool, table)
    st, word = eng.last_error()
    assert st == _lib.B2D_ERR_DEVICE_INPUT and word == 0x201
    eng.reset()
    bad_table = table.clone()
    bad_table[1, 0] = 2 * bps  # one past the pool
    eng.step_paged(tok, pos, pool, bad_table)
    st, word = eng.last_error()
    assert st == _lib.B2D_ERR_DEVICE_INPUT and word == 0x203
    eng.reset()
    assert eng.last_error()[0] == _lib.B2D_OK


def test_paged_host_validation(engine_tiny_batched, engine_tiny):
    eng = engine_tiny_batched
    dev = eng.device
    pool = eng.new_kv_pool(8)
    table = torch.zeros(1, 8, dtype=torch.int32, device=dev)
    t = torch.zeros(1, dtype=torch.int32, device=dev)
    with pytest.raises(ValueError):
        eng.step_paged(t, t, pool.float(), table)
    with pytest.raises(ValueError):
        eng.step_paged(t, t, pool, table.long())
    with pytest.raises(ValueError):
        engine_tiny.step_paged(t, t, pool, table)  # max_batch 1
    z65 = torch.zeros(65, dtype=torch.int32, device=dev)
    with pytest.raises(_lib.B2DError):  # batch above the workspace's max_batch: rejected by the C ABI
        eng.step_paged(z65, z65, pool, torch.zeros(65, 8, dtype=torch.int32, device=dev), next_tok=z65.clone())
