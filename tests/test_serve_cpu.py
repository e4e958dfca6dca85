"""CPU: the continuous batcher's scheduling over the paged pool (page
allocation, slot refill, preemption and readmission), driven through a fake
engine.  The fake stores each fed token in its page and derives the next token
from a hash of the whole sequence read back through the block table, so a page
shared between live sequences, freed early, or addressed at a wrong position
changes the output; it also checks that live sequences never share a block."""

from __future__ import annotations

import types

import numpy as np
import pytest
import torch

from transformer_b200.serve import PAGE_TOKENS, ContinuousBatcher, PagePool, PoolExhausted


def _hash_next(seq, vocab):
    h = 7
    for t in seq:
        h = (h * 1000003 + int(t) + 1) % ((1 << 61) - 1)
    return h % vocab


def _expected(prompt, n, vocab, eos=None):
    seq = list(prompt)
    out = [_hash_next(seq, vocab)]
    while len(out) < n and out[-1] != eos:
        seq.append(out[-1])
        out.append(_hash_next(seq, vocab))
    return out


class FakeEngine:
    def __init__(self, ctx=64, vocab=97, max_batch=4, rows_max=24):
        self.cfg = types.SimpleNamespace(context_len=ctx, vocab_size=vocab)
        self.device = torch.device("cpu")
        self.max_batch = max_batch
        self.prefill_rows_max = rows_max
        self.prefill_calls = []
        self.logits = torch.zeros(max_batch, vocab)
        self.next_tok = torch.zeros(max_batch, dtype=torch.int32)
        self.steps = []

    def new_kv_pool(self, num_blocks):
        return torch.full((num_blocks, PAGE_TOKENS), -1, dtype=torch.int64)

    def _next(self, pool, row, last):
        seq = [int(pool[row[p // PAGE_TOKENS], p % PAGE_TOKENS]) for p in range(last + 1)]
        assert min(seq) >= 0, "read an unwritten position"
        return _hash_next(seq, self.cfg.vocab_size)

    def prefill_paged(self, prompt, pool, table_row, start=0, stream=None, next_tok=None):
        row = table_row.tolist()
        for i, t in enumerate(prompt):
            p = start + i
            pool[row[p // PAGE_TOKENS], p % PAGE_TOKENS] = int(t)
        n = self._next(pool, row, start + len(prompt) - 1)
        (self.next_tok if next_tok is None else next_tok)[0] = n
        self.logits[0].zero_()
        self.logits[0, n] = 1.0
        return self.logits[0]

    def prefill_rows(self, tok, pos, pool, table, n_out, logits=None, next_tok=None, n_rows=None, stream=None):
        assert logits is None  # greedy only in these tests
        assert 1 <= n_rows <= self.prefill_rows_max and 0 <= n_out <= n_rows
        assert (next_tok is not None) == (n_out > 0)
        self.prefill_calls.append((n_rows, n_out))
        rows = [(int(tok[i]), int(pos[i]), table[i].tolist()) for i in range(n_rows)]
        for t, p, row in rows:  # every row's K/V first ...
            pool[row[p // PAGE_TOKENS], p % PAGE_TOKENS] = t
        for i, (t, p, row) in enumerate(rows):  # ... then each row sees positions <= its own
            nxt = self._next(pool, row, p)
            if i >= n_rows - n_out:
                next_tok[i - (n_rows - n_out)] = nxt

    def step_paged(self, tok, pos, pool, block_table, logits=None, next_tok=None, stream=None, batch=None):
        assert logits is None  # greedy only in these tests
        owner = {}
        for b in range(batch):
            p = int(pos[b])
            if p < 0:
                continue
            for blk in block_table[b, :p // PAGE_TOKENS + 1].tolist():
                assert owner.setdefault(blk, b) == b, f"block {blk} shared by rows {owner[blk]} and {b}"
        self.steps.append(int(sum(int(pos[b]) >= 0 for b in range(batch))))
        for b in range(batch):
            p = int(pos[b])
            if p >= 0:
                pool[int(block_table[b, p // PAGE_TOKENS]), p % PAGE_TOKENS] = int(tok[b])
        for b in range(batch):
            p = int(pos[b])
            if p >= 0:
                next_tok[b] = self._next(pool, block_table[b].tolist(), p)
            else:  # the device argmax also writes idle rows: a wrong token there
                next_tok[b] = (7 * b + 3) % self.cfg.vocab_size


def test_page_pool():
    pp = PagePool(5)
    a = pp.alloc(3)
    assert sorted(a) == [0, 1, 2] and pp.n_free == 2
    with pytest.raises(PoolExhausted):
        pp.alloc(3)
    pp.free([1])
    assert pp.n_free == 3
    with pytest.raises(ValueError):
        pp.free([1])
    with pytest.raises(ValueError):
        pp.free([7])
    b = pp.alloc(3)
    assert sorted(b) == [1, 3, 4] and pp.n_free == 0


@pytest.mark.parametrize("pipe", [True, False])
@pytest.mark.parametrize("fuse", [True, False])
@pytest.mark.parametrize("seed,num_blocks,admission", [(0, 4, "optimistic"), (1, 6, "optimistic"),
                                                       (2, 9, "optimistic"), (3, 40, "optimistic"),
                                                       (4, 6, "reserve"), (5, 9, "reserve")])
def test_batcher_matches_sequential(seed, num_blocks, admission, fuse, pipe):
    """Requests of random lengths through 4 slots: every token stream equals
    the one-at-a-time generation, prompts prefilled in fused passes or on
    their own, decode steps pipelined (tokens fed back on the device) or not;
    small pools force preemptions under optimistic admission and none under
    reserving admission."""
    rng = np.random.default_rng(seed)
    eng = FakeEngine(ctx=64, vocab=97, max_batch=4, rows_max=64)
    cb = ContinuousBatcher(eng, 4, num_blocks, admission=admission, fuse_prefill=fuse, pipeline=pipe)
    want = {}
    for _ in range(14):
        n_prompt = int(rng.integers(1, 48))
        n_gen = int(rng.integers(1, 64 - n_prompt + 2))
        prompt = rng.integers(0, 97, n_prompt)
        rid = cb.submit(prompt, n_gen)
        want[rid] = _expected(prompt, n_gen, 97)
    got = cb.run()
    assert got == want
    assert cb.pages.n_free == num_blocks
    assert cb.idle()
    assert cb.stats["tokens"] >= sum(len(v) for v in want.values())
    if admission == "reserve":
        assert cb.stats["preemptions"] == 0
    elif num_blocks <= 6:
        assert cb.stats["preemptions"] > 0
    if num_blocks == 40:  # room for every slot: several rows per pass on average
        assert cb.stats["preemptions"] == 0 and cb.stats["tokens"] > 2 * cb.stats["steps"]
    assert (cb.stats["mixed_steps"] > 0) == fuse
    assert (cb.stats["pipelined_steps"] > 0) == pipe


def test_batcher_events_and_eos():
    """step() reports each token as produced; an end-of-sequence id ends a
    request early and frees its slot for the next one."""
    rng = np.random.default_rng(5)
    eng = FakeEngine(ctx=64, vocab=11, max_batch=2)
    cb = ContinuousBatcher(eng, 2, 8, eos_id=3)
    want, seen = {}, {}
    for _ in range(6):
        prompt = rng.integers(0, 11, int(rng.integers(1, 20)))
        rid = cb.submit(prompt, 30)
        want[rid] = _expected(prompt, 30, 11, eos=3)
    while not cb.idle():
        for rid, t in cb.step():
            seen.setdefault(rid, []).append(t)
    assert seen == want == cb.finished
    assert any(v[-1] == 3 and len(v) < 30 for v in want.values())


def test_batcher_prefill_chunks():
    """Admission packs prompts into prefill calls of at most prefill_rows_max
    rows: a prompt longer than one call spans several (earlier positions
    first), short prompts share a call, and only first-token rows are
    outputs."""
    rng = np.random.default_rng(9)
    eng = FakeEngine(ctx=64, vocab=97, max_batch=4, rows_max=24)
    cb = ContinuousBatcher(eng, 4, 16, fuse_prefill=False)
    want = {}
    for n in (50, 3, 4, 30):
        pr = rng.integers(0, 97, n)
        want[cb.submit(pr, 5)] = _expected(pr, 5, 97)
    cb.step()  # admits all four: 87 rows in 4 calls
    assert sum(r for r, _ in eng.prefill_calls) == 87
    assert max(r for r, _ in eng.prefill_calls) == 24 and len(eng.prefill_calls) == 4
    assert sum(o for _, o in eng.prefill_calls) == 4
    assert cb.run() == want


def test_batcher_long_prompts_prefilled_on_their_own():
    """With fused passes on, a prefix longer than one pass (here 24 rows) is
    prefilled on its own in chunks while short prompts join the fused pass."""
    rng = np.random.default_rng(10)
    eng = FakeEngine(ctx=64, vocab=97, max_batch=4, rows_max=24)
    cb = ContinuousBatcher(eng, 4, 16)
    want = {}
    for n in (50, 3, 4, 30, 2):
        pr = rng.integers(0, 97, n)
        want[cb.submit(pr, 6)] = _expected(pr, 6, 97)
    assert cb.run() == want
    assert cb.stats["mixed_steps"] > 0 and cb.stats["prefill_calls"] == 4  # 50 + 30 rows in 24-row chunks


def test_batcher_single_token_and_full_context():
    eng = FakeEngine(ctx=32, vocab=50, max_batch=2)
    cb = ContinuousBatcher(eng, 2, 2)
    r1 = cb.submit([5], 1)                      # first token from the prefill only
    r2 = cb.submit(np.arange(20) % 50, 13)      # positions up to the last one (31)
    got = cb.run()
    assert got[r1] == _expected([5], 1, 50)
    assert got[r2] == _expected(np.arange(20) % 50, 13, 50)
    assert cb.pages.n_free == 2


def test_batcher_validation():
    eng = FakeEngine(ctx=32, vocab=50, max_batch=4)
    with pytest.raises(ValueError):
        ContinuousBatcher(eng, 8, 4)            # more slots than the engine's workspace
    with pytest.raises(ValueError):
        ContinuousBatcher(eng, 4, 1)            # pool smaller than one full context
    cb = ContinuousBatcher(eng, 4, 4)
    for bad in (dict(prompt=[], max_tokens=1), dict(prompt=[1], max_tokens=0),
                dict(prompt=[1] * 20, max_tokens=14), dict(prompt=[50], max_tokens=1),
                dict(prompt=[1], max_tokens=1, top_p=0.0)):
        with pytest.raises(ValueError):
            cb.submit(**bad)
    cb.submit([1] * 20, 13)
    assert len(cb.waiting) == 1
