"""Continuous batching over the paged KV pool.

The reference's batched server and paged KV cache (``serve.py``,
``kernels/paged_kv.py``) were deleted upstream; ``knowledge/program.md:213-216,
257`` describes them: per-sequence position tracking, a ``PagePool`` of
fixed-size KV pages, and batch slots refilled as sequences complete.  Here:

* ``PagePool`` hands out the physical blocks of one paged pool (16 positions
  each, the layout of ``b2d_decode_step_paged``) from a free list.
* ``ContinuousBatcher`` keeps up to ``max_batch`` requests in slots.  Waiting
  requests are admitted into free slots while the pool has the pages for
  their prompts; their prompts go through ``b2d_prefill_rows`` together, up to
  512 positions of any number of prompts per pass over the weights, writing
  K/V through each slot's block-table row, and each prompt's last logits give
  its first token (as ``generate.py:68-89``).  Each ``step()`` runs one
  batched decode step over every slot (idle slots as ``pos = -1`` rows),
  feeding each request its previous token at ``pos = prompt_len + i``
  (``generate.py:92-123``).  A page
  is taken when a request's next position starts one; when none is free the
  most recently admitted request is preempted: its pages return to the pool
  and it waits at the head of the queue, to be prefilled again over its prompt
  and the tokens it has generated (its tokens so far are kept).

Greedy requests (temperature 0, no repetition penalty, ``generate.py:102,
115``) take the step's argmax; the others go through the device sampler with
their generated tokens as history and one uniform per token from their own
``numpy.random.RandomState(seed)``, the draw ``np.random.choice`` makes after
``np.random.seed(seed)`` in the reference.
"""

from __future__ import annotations

import collections
import dataclasses
import time

import numpy as np
import torch

PAGE_TOKENS = 16  # positions per block (b2d_decode_step_paged's page)


class PoolExhausted(RuntimeError):
    pass


class PagePool:
    """Free list over the blocks 0..num_blocks-1 of one paged KV pool."""

    def __init__(self, num_blocks: int):
        if num_blocks < 1:
            raise ValueError("num_blocks must be positive")
        self.num_blocks = num_blocks
        self._free = list(range(num_blocks - 1, -1, -1))  # pop() hands out low ids first
        self._used = np.zeros(num_blocks, dtype=bool)

    @property
    def n_free(self) -> int:
        return len(self._free)

    def alloc(self, n: int) -> list[int]:
        if n < 0:
            raise ValueError("negative page count")
        if n > len(self._free):
            raise PoolExhausted(f"{n} pages wanted, {len(self._free)} free")
        out = [self._free.pop() for _ in range(n)]
        self._used[out] = True
        return out

    def free(self, blocks) -> None:
        for b in blocks:
            if not (0 <= b < self.num_blocks) or not self._used[b]:
                raise ValueError(f"block {b} is not allocated")
            self._used[b] = False
            self._free.append(b)


@dataclasses.dataclass
class Request:
    rid: int
    prompt: np.ndarray
    max_tokens: int
    temperature: float = 0.0
    top_p: float = 1.0
    rep_penalty: float = 1.0
    seed: int | None = None
    out: list = dataclasses.field(default_factory=list)
    blocks: list = dataclasses.field(default_factory=list)
    slot: int = -1
    admitted: int = -1       # admission order (the preemption victim is the latest)
    preemptions: int = 0
    fed: int = 0             # decode rows issued (the first token comes from the prompt's last row)
    rng: object = None

    @property
    def greedy(self) -> bool:
        return self.temperature == 0.0 and self.rep_penalty == 1.0

    def next_pos(self) -> int:
        """Position of the token fed at this request's next decode row."""
        return len(self.prompt) + self.fed


class ContinuousBatcher:
    """Requests in ``max_batch`` slots over one paged pool of ``num_blocks``
    blocks.  ``submit`` queues a request; ``step`` admits what fits and runs
    one pass, returning the ``(rid, token)`` pairs it produced (admitted
    requests' first tokens included); ``run`` steps until every request has
    finished and returns ``{rid: tokens}``.

    ``fuse_prefill``: a step that admits requests runs their prompt rows and
    the running requests' decode rows in one ``b2d_prefill_rows`` pass (up to
    512 rows; admission stops at that budget), instead of a prefill pass
    followed by a decode step.  ``admission``: "reserve" admits a request only
    while the pool can hold every admitted request at its longest (no
    preemption); "optimistic" only needs the prompt's pages and one spare page
    per running request, and preempts when the pool runs dry."""

    def __init__(self, engine, max_batch: int, num_blocks: int, eos_id: int | None = None,
                 hist_cap: int | None = None, admission: str = "reserve", fuse_prefill: bool = True,
                 pipeline: bool = True, admit_batch: int | None = None):
        cfg = engine.cfg
        self.eng = engine
        self.ctx = cfg.context_len
        self.vocab = cfg.vocab_size
        self.bps = (self.ctx + PAGE_TOKENS - 1) // PAGE_TOKENS
        if max_batch < 2 or max_batch > engine.max_batch:
            raise ValueError(f"max_batch must be in [2, {engine.max_batch}] (the engine's workspace)")
        if num_blocks < self.bps:
            raise ValueError(f"num_blocks must hold one full-context sequence ({self.bps} blocks)")
        if admission not in ("reserve", "optimistic"):
            raise ValueError("admission must be 'reserve' or 'optimistic'")
        self.max_batch, self.eos_id = max_batch, eos_id
        self.admission, self.fuse_prefill, self.pipeline = admission, fuse_prefill, pipeline
        self.admit_batch = admit_batch or max(1, max_batch // 32)
        self.pages = PagePool(num_blocks)
        self.pool = engine.new_kv_pool(num_blocks)
        dev = engine.device
        self._cuda = dev.type == "cuda"
        pin = self._cuda
        # tok | pos | table rows, one host->device copy per step
        n_stage = 2 * max_batch + max_batch * self.bps
        self._h_stage = torch.zeros(n_stage, dtype=torch.int32, pin_memory=pin)
        self._d_stage = torch.zeros(n_stage, dtype=torch.int32, device=dev)
        self._h_tok = self._h_stage[:max_batch].numpy()
        self._h_pos = self._h_stage[max_batch:2 * max_batch].numpy()
        self._h_table = self._h_stage[2 * max_batch:].numpy().reshape(max_batch, self.bps)
        self._d_tok = self._d_stage[:max_batch]
        self._d_pos = self._d_stage[max_batch:2 * max_batch]
        self._d_table = self._d_stage[2 * max_batch:].view(max_batch, self.bps)
        self._d_next = torch.zeros(max_batch, dtype=torch.int32, device=dev)
        # prefill chunks: tok | pos | table rows
        self._rows_max = int(engine.prefill_rows_max)
        cap = self._rows_max
        self._hp_stage = torch.zeros(2 * cap + cap * self.bps, dtype=torch.int32, pin_memory=pin)
        self._dp_stage = torch.zeros(2 * cap + cap * self.bps, dtype=torch.int32, device=dev)
        self._hp_tok = self._hp_stage[:cap].numpy()
        self._hp_pos = self._hp_stage[cap:2 * cap].numpy()
        self._hp_table = self._hp_stage[2 * cap:].numpy().reshape(cap, self.bps)
        self._dp_tok = self._dp_stage[:cap]
        self._dp_pos = self._dp_stage[cap:2 * cap]
        self._dp_table = self._dp_stage[2 * cap:].view(cap, self.bps)
        self._dp_next = torch.zeros(cap, dtype=torch.int32, device=dev)
        self._logits_rows = max(max_batch, cap)
        self._h_next = torch.zeros(self._logits_rows, dtype=torch.int32, pin_memory=pin)
        self._h_table[:] = 0
        self._h_pos[:] = -1
        # pipelined decode steps: each slot's latest token stays on the device (the
        # step reads and overwrites it); positions and table rows go through two
        # pinned staging buffers, the tokens come back through two more
        self._d_slot_tok = torch.zeros(max_batch, dtype=torch.int32, device=dev)
        self._dq_stage = torch.zeros(max_batch + max_batch * self.bps, dtype=torch.int32, device=dev)
        self._dq_pos = self._dq_stage[:max_batch]
        self._dq_table = self._dq_stage[max_batch:].view(max_batch, self.bps)
        self._hq_stage = [torch.zeros(max_batch + max_batch * self.bps, dtype=torch.int32, pin_memory=pin)
                          for _ in range(2)]
        self._hq_out = [torch.zeros(max_batch, dtype=torch.int32, pin_memory=pin) for _ in range(2)]
        self._hq_event = [torch.cuda.Event() for _ in range(2)] if self._cuda else [None, None]
        self._ring = 0
        self._inflight = None      # (ring index, [(slot, request)]) of the step whose tokens are unread
        self._tok_dirty = True     # slots' latest tokens known only on the host
        self.slots: list[Request | None] = [None] * max_batch
        self.waiting: collections.deque[Request] = collections.deque()
        self.finished: dict[int, list] = {}
        self._next_rid = 0
        self._admit_tick = 0
        self._hist_cap = hist_cap or self.ctx
        self._sampler = None
        self._logits = None
        self._logits_c = None      # sampled rows gathered for the sampler
        self._d_idx = None
        self.stats = collections.Counter()
        self.times = collections.Counter()  # wall seconds per pass kind (each pass ends with a token read-back)

    # ---- requests --------------------------------------------------------
    def submit(self, prompt, max_tokens: int, temperature: float = 0.0, top_p: float = 1.0,
               rep_penalty: float = 1.0, seed: int | None = None) -> int:
        prompt = np.asarray(prompt, dtype=np.int32).reshape(-1)
        if prompt.size == 0:
            raise ValueError("empty prompt")
        if max_tokens < 1:
            raise ValueError("max_tokens must be >= 1")
        if prompt.size + max_tokens - 1 > self.ctx:
            raise ValueError(f"prompt ({prompt.size}) + max_tokens - 1 ({max_tokens - 1}) exceeds the context "
                             f"({self.ctx})")
        if prompt.min() < 0 or prompt.max() >= self.vocab:
            raise ValueError("token id out of range")
        if not (temperature >= 0.0 and top_p > 0.0 and rep_penalty > 0.0):
            raise ValueError("bad sampling parameters")
        if max_tokens > self._hist_cap:
            raise ValueError("max_tokens exceeds the sampler history capacity")
        rid = self._next_rid
        self._next_rid += 1
        r = Request(rid, prompt, int(max_tokens), float(temperature), float(top_p), float(rep_penalty), seed)
        if not r.greedy:
            r.rng = np.random.RandomState(seed)
        self.waiting.append(r)
        return rid

    @property
    def running(self) -> list[Request]:
        return [r for r in self.slots if r is not None]

    def idle(self) -> bool:
        return not self.waiting and self._inflight is None and all(r is None for r in self.slots)

    def run(self) -> dict[int, list]:
        while not self.idle():
            self.step()
        return dict(self.finished)

    # ---- one scheduling step --------------------------------------------
    def step(self) -> list[tuple[int, int]]:
        """Admit what fits, then one pass over the weights for every running
        request (and, with ``fuse_prefill``, the admitted prompts' rows).

        With ``pipeline``, a decode step of greedy requests is issued without
        waiting for its tokens: the next call issues the following step (the
        tokens feed back on the device) before reading them, so the host's
        scheduling overlaps the GPU.  Admissions, sampling, preemption and a
        pool without a free page for every next position drain the pipeline
        first."""
        events: list[tuple[int, int]] = []
        if self._inflight is not None:
            t0 = time.perf_counter()
            if self._can_continue():
                prev = self._inflight
                self._issue_decode()
                self._consume(prev, events)
                self.times["decode"] += time.perf_counter() - t0
                return events
            prev, self._inflight = self._inflight, None
            self._consume(prev, events)
            self.times["decode"] += time.perf_counter() - t0
        n_run = sum(r is not None for r in self.slots)
        budget = self._rows_max - n_run if self.fuse_prefill else None
        fused, dedicated = self._admit(budget)
        if dedicated:
            t0 = time.perf_counter()
            self._prefill(dedicated, events)
            self.times["prefill"] += time.perf_counter() - t0
        self._reserve_pages()
        fused = [(r, p) for r, p in fused if r.slot >= 0]  # not preempted since
        t0 = time.perf_counter()
        if fused:
            self._mixed_step(fused, events)
            self.times["mixed"] += time.perf_counter() - t0
        elif any(r is not None for r in self.slots):
            if self._pipelinable():
                self._issue_decode()
            else:
                self._decode_step(events)
            self.times["decode"] += time.perf_counter() - t0
        return events

    # ---- pipelined decode steps -----------------------------------------
    def _pipelinable(self) -> bool:
        return self.pipeline and all(r is None or r.greedy for r in self.slots)

    def _admit_threshold(self) -> int:
        """Free slots that trigger an admission: a few at a time while requests
        run (each admission is a pass of its own and drains the pipeline)."""
        if all(r is None for r in self.slots):
            return 1
        return max(1, min(self.admit_batch, len(self.waiting)))

    def _can_continue(self) -> bool:
        """Another decode step can be issued before the in-flight one's tokens
        are read: every request is greedy, one has rows left, no admission is
        due once the in-flight step's last tokens finish their requests, and a
        free page exists for every next position that starts one."""
        if not self._pipelinable():
            return False
        running = [r for r in self.slots if r is not None]
        issuing = [r for r in running if r.fed < r.max_tokens - 1]
        if not issuing:
            return False
        if self.waiting:
            free_after = self.slots.count(None) + (len(running) - len(issuing))
            if free_after >= self._admit_threshold():
                head = self.waiting[0]  # drain only for an admission the pool can take
                rows = self._prefix(head).size + (1 if head.out else 0)
                if self._pages_allow(head, (rows + PAGE_TOKENS - 1) // PAGE_TOKENS):
                    return False
        need = sum(1 for r in issuing if r.next_pos() // PAGE_TOKENS >= len(r.blocks))
        return need <= self.pages.n_free

    def _issue_decode(self) -> None:
        """Launch one decode step over the slots whose requests have rows left
        (tokens: each slot's latest, on the device), its tokens copied back
        asynchronously."""
        if self._tok_dirty:
            h = np.zeros(self.max_batch, np.int32)
            for i, r in enumerate(self.slots):
                if r is not None and r.out:
                    h[i] = r.out[-1]
            self._d_slot_tok.copy_(torch.from_numpy(h))
            self._tok_dirty = False
        k = self._ring
        self._ring ^= 1
        hq = self._hq_stage[k].numpy()
        pos = hq[:self.max_batch]
        table = hq[self.max_batch:].reshape(self.max_batch, self.bps)
        rows, batch = [], 2
        for i, r in enumerate(self.slots):
            if r is None or r.fed >= r.max_tokens - 1:
                pos[i] = -1
                continue
            p = r.next_pos()
            if p // PAGE_TOKENS >= len(r.blocks):  # free pages were checked by the caller
                b = self.pages.alloc(1)[0]
                self._h_table[i, len(r.blocks)] = b
                r.blocks.append(b)
            pos[i] = p
            r.fed += 1
            rows.append((i, r))
            batch = max(batch, i + 1)
        table[:batch] = self._h_table[:batch]
        n = self.max_batch + batch * self.bps
        self._dq_stage[:n].copy_(self._hq_stage[k][:n], non_blocking=self._cuda)
        self.eng.step_paged(self._d_slot_tok, self._dq_pos, self.pool, self._dq_table, None, self._d_slot_tok,
                            batch=batch)
        self._hq_out[k][:batch].copy_(self._d_slot_tok[:batch], non_blocking=self._cuda)
        if self._cuda:
            self._hq_event[k].record()
        self._inflight = (k, rows)
        self.stats["steps"] += 1
        self.stats["pipelined_steps"] += 1

    def _consume(self, inflight, events) -> None:
        """Read an issued step's tokens (waiting for that step only)."""
        k, rows = inflight
        if self._cuda:
            t0 = time.perf_counter()
            self._hq_event[k].synchronize()
            self.times["gpu_wait"] += time.perf_counter() - t0
        toks = self._hq_out[k].numpy()
        for i, r in rows:
            if r.slot != i:  # finished (end of sequence) while this step was in flight
                continue
            t = int(toks[i])
            r.out.append(t)
            events.append((r.rid, t))
            self.stats["tokens"] += 1
            self._maybe_finish(r)

    def _decode_step(self, events) -> None:
        """b2d_decode_step_paged over slots 0..batch-1 (idle slots as pos = -1
        rows; the step replays a CUDA graph while its arguments repeat)."""
        batch = max(2, 1 + max(i for i, r in enumerate(self.slots) if r is not None))
        for i in range(batch):
            r = self.slots[i]
            if r is None:
                self._h_tok[i], self._h_pos[i] = 0, -1
            else:
                self._h_tok[i], self._h_pos[i] = r.out[-1], r.next_pos()
                r.fed += 1
        self._d_stage.copy_(self._h_stage, non_blocking=self._cuda)
        need_logits = any(r is not None and not r.greedy for r in self.slots[:batch])
        logits = self._logits_buf() if need_logits else None
        self.eng.step_paged(self._d_tok, self._d_pos, self.pool, self._d_table, logits, self._d_next,
                            batch=batch)
        if need_logits:
            toks = self._sample_rows(logits, self.slots[:batch], self._d_next)
        else:
            toks = self._fetch(self._d_next, batch)
        self.stats["steps"] += 1
        self._emit([(i, r) for i, r in enumerate(self.slots[:batch]) if r is not None], toks, events)

    def _mixed_step(self, fused, events) -> None:
        """One b2d_prefill_rows pass: the admitted prefixes (body) plus, in the
        tail, a decode row for every request that has tokens (running and
        readmitted ones) and the last prompt row of every new request."""
        toks, poss, slots = [], [], []
        tail: list[Request] = []
        t_tok, t_pos, t_slot = [], [], []
        for r, prefix in fused:
            n = prefix.size if r.out else prefix.size - 1  # a new request's last row is a tail row
            toks.append(prefix[:n])
            poss.append(np.arange(n, dtype=np.int32))
            slots.append(np.full(n, r.slot, np.int32))
            if not r.out:
                tail.append(r)
                t_tok.append(int(prefix[-1]))
                t_pos.append(prefix.size - 1)
                t_slot.append(r.slot)
        for r in self.slots:
            if r is not None and r.out:
                tail.append(r)
                t_tok.append(r.out[-1])
                t_pos.append(r.next_pos())
                t_slot.append(r.slot)
                r.fed += 1
        tok = np.concatenate(toks + [np.asarray(t_tok, np.int32)])
        pos = np.concatenate(poss + [np.asarray(t_pos, np.int32)])
        slot = np.concatenate(slots + [np.asarray(t_slot, np.int32)])
        n, n_out = tok.size, len(tail)
        assert n <= self._rows_max
        self._hp_tok[:n] = tok
        self._hp_pos[:n] = pos
        self._hp_table[:n] = self._h_table[slot]
        self._dp_stage.copy_(self._hp_stage, non_blocking=self._cuda)
        sampled = any(not q.greedy for q in tail)
        logits = self._logits_buf() if sampled else None
        self.eng.prefill_rows(self._dp_tok, self._dp_pos, self.pool, self._dp_table, n_out,
                              logits=logits, next_tok=self._dp_next, n_rows=n)
        out = self._sample_rows(logits, tail, self._dp_next) if sampled else self._fetch(self._dp_next, n_out)
        self.stats["steps"] += 1
        self.stats["mixed_steps"] += 1
        self.stats["prefill_rows"] += n - n_out + sum(1 for r, _ in fused if not r.out)
        self._emit(list(enumerate(tail)), out, events)

    def _emit(self, rows, toks, events) -> None:
        self._tok_dirty = True
        for i, r in rows:
            t = int(toks[i])
            r.out.append(t)
            events.append((r.rid, t))
            self.stats["tokens"] += 1
            self._maybe_finish(r)

    def _admit(self, budget):
        """Admit waiting requests in order while a slot and the pages for their
        prefix (plus, for a readmitted request, its next position) are free,
        and, when ``budget`` (rows of this step's fused pass) is not None,
        while their rows fit it.  Returns (fused, dedicated): the admissions
        for the fused pass, and those prefilled on their own (a prefix longer
        than one pass, or fusing off)."""
        fused, dedicated = [], []
        if self.slots.count(None) < self._admit_threshold():
            return fused, dedicated
        while self.waiting and None in self.slots:
            r = self.waiting[0]
            prefix = self._prefix(r)
            rows = prefix.size + (1 if r.out else 0)  # a readmitted request's decode row joins the pass
            need = (rows + PAGE_TOKENS - 1) // PAGE_TOKENS
            if not self._pages_allow(r, need):
                break
            own = budget is None or rows > self._rows_max
            cost = 1 if own else rows  # rows it adds to this step's fused pass (own prefill: its decode row)
            if budget is not None and cost > budget:
                break
            self.waiting.popleft()
            slot = self.slots.index(None)
            r.blocks = self.pages.alloc(need)
            r.slot = slot
            r.admitted = self._admit_tick
            self._admit_tick += 1
            self.slots[slot] = r
            self._tok_dirty = True  # the slot's device token belongs to its previous request
            self._h_table[slot, :] = 0
            self._h_table[slot, :need] = r.blocks
            (dedicated if own else fused).append((r, prefix))
            if budget is not None:
                budget -= cost
        return fused, dedicated

    def _max_pages(self, r: Request) -> int:
        return (len(r.prompt) + r.max_tokens - 1 + PAGE_TOKENS - 1) // PAGE_TOKENS

    def _pages_allow(self, r: Request, need: int) -> bool:
        """admission = "reserve": the pool must hold every running request and
        this one at their longest (prompt + max_tokens - 1 positions), so no
        request is ever preempted.  "optimistic": the prefix's pages plus one
        free page per running request; the pool may run dry later, and then the
        latest admissions are preempted."""
        running = [q for q in self.slots if q is not None]
        if self.admission == "reserve":
            owed = sum(self._max_pages(q) - len(q.blocks) for q in running)
            return self._max_pages(r) + owed <= self.pages.n_free
        return need + len(running) <= self.pages.n_free or (not running and need <= self.pages.n_free)

    @staticmethod
    def _prefix(r: Request) -> np.ndarray:
        """Tokens whose K/V a (re)admitted request needs: its prompt, plus, after
        a preemption, every generated token but the last (fed at the next step)."""
        if not r.out:
            return r.prompt
        return np.concatenate([r.prompt, np.asarray(r.out[:-1], np.int32)])

    def _prefill(self, admitted, events) -> None:
        """The admitted prefixes in chunks of up to ``prefill_rows_max`` rows
        (one pass over the weights each).  A new request's last row goes to its
        chunk's tail, whose outputs give the first tokens; a readmitted
        request's next token is already chosen."""
        cap = self._rows_max
        body: list[tuple[int, int, int]] = []       # (token, position, slot)
        tail: list[tuple[int, int, int, Request]] = []

        def flush():
            rows = body + [t[:3] for t in tail]
            n, n_out = len(rows), len(tail)
            arr = np.asarray(rows, dtype=np.int64)
            self._hp_tok[:n] = arr[:, 0]
            self._hp_pos[:n] = arr[:, 1]
            self._hp_table[:n] = self._h_table[arr[:, 2]]
            self._dp_stage.copy_(self._hp_stage, non_blocking=self._cuda)
            reqs = [t[3] for t in tail]
            sampled = any(not q.greedy for q in reqs)
            logits = self._logits_buf() if sampled else None
            self.eng.prefill_rows(self._dp_tok, self._dp_pos, self.pool, self._dp_table, n_out,
                                  logits=logits, next_tok=self._dp_next if n_out else None, n_rows=n)
            self.stats["prefill_rows"] += n
            self.stats["prefill_calls"] += 1
            if n_out:
                toks = (self._sample_rows(logits, reqs, self._dp_next) if sampled
                        else self._fetch(self._dp_next, n_out))
                for q, t in zip(reqs, toks):
                    q.out.append(int(t))
                    events.append((q.rid, int(t)))
                    self.stats["tokens"] += 1
                    self._maybe_finish(q)
            elif self._cuda:  # the pinned staging is rewritten by the next chunk
                torch.cuda.current_stream(self.eng.device).synchronize()
            body.clear()
            tail.clear()

        for r, prefix in admitted:
            n, wants_out = prefix.size, not r.out
            for k in range(n):
                if len(body) + len(tail) == cap:
                    flush()
                row = (int(prefix[k]), k, r.slot)
                if k == n - 1 and wants_out:
                    tail.append(row + (r,))
                else:
                    body.append(row)
        if body or tail:
            flush()

    def _reserve_pages(self) -> None:
        """Every running request gets the page its next position lands in,
        preempting the most recently admitted requests while none is free."""
        for r in sorted(self.running, key=lambda q: q.admitted):
            if r.slot < 0:  # preempted below while serving an earlier request
                continue
            while r.next_pos() // PAGE_TOKENS >= len(r.blocks):
                if self.pages.n_free == 0:
                    victim = max(self.running, key=lambda q: q.admitted)
                    self._preempt(victim)
                    if victim is r:
                        break
                    continue
                b = self.pages.alloc(1)[0]
                self._h_table[r.slot, len(r.blocks)] = b
                r.blocks.append(b)

    def _preempt(self, r: Request) -> None:
        self.pages.free(r.blocks)
        r.blocks = []
        self.slots[r.slot] = None
        self._h_table[r.slot, :] = 0
        r.slot = -1
        r.fed = len(r.out) - 1  # no step is in flight here: every issued row has its token
        r.preemptions += 1
        self.stats["preemptions"] += 1
        self.waiting.appendleft(r)

    def _maybe_finish(self, r: Request) -> None:
        if len(r.out) < r.max_tokens and (self.eos_id is None or r.out[-1] != self.eos_id):
            return
        self.pages.free(r.blocks)
        r.blocks = []
        self.slots[r.slot] = None
        self._h_table[r.slot, :] = 0
        r.slot = -1
        self.finished[r.rid] = list(r.out)

    # ---- device helpers --------------------------------------------------
    def _fetch(self, d: torch.Tensor, n: int) -> np.ndarray:
        h = self._h_next[:n]
        h.copy_(d[:n], non_blocking=self._cuda)
        if self._cuda:
            t0 = time.perf_counter()
            torch.cuda.current_stream(self.eng.device).synchronize()
            self.times["gpu_wait"] += time.perf_counter() - t0
        return h.numpy().copy()

    def _logits_buf(self) -> torch.Tensor:
        if self._logits is None:
            self._logits = torch.empty(self._logits_rows, self.vocab, dtype=torch.float32, device=self.eng.device)
        return self._logits

    def _sample_rows(self, logits: torch.Tensor, rows, greedy_src: torch.Tensor) -> np.ndarray:
        """Tokens for the requests ``rows`` (row i of ``logits``; None = idle):
        sampled for non-greedy requests, with their generated tokens as history
        and their next uniform; for greedy ones the argmax the step or the
        prefill left in ``greedy_src``."""
        from .generate import Sampler
        if self._sampler is None:
            self._sampler = Sampler(self.eng, self._logits_rows, self._hist_cap)
        smp = self._sampler
        batch = len(rows)
        out = np.zeros(batch, np.int32)
        groups: dict = {}
        for i, r in enumerate(rows):
            if r is not None and not r.greedy:
                groups.setdefault((r.temperature, r.top_p, r.rep_penalty), []).append(i)
        greedy_rows = [i for i, r in enumerate(rows) if r is not None and r.greedy]
        if greedy_rows:
            out[greedy_rows] = self._fetch(greedy_src, batch)[greedy_rows]
        for (temp, top_p, rp), idx in groups.items():
            # one sampler launch per parameter set, over that set's rows only
            # (gathered into a preallocated buffer when they are not all rows)
            m = len(idx)
            hist = np.zeros((m, self._hist_cap), np.int32)
            hlen = np.zeros(m, np.int32)
            u = np.zeros(m, np.float64)
            for k, i in enumerate(idx):
                r = rows[i]
                hist[k, :len(r.out)] = r.out
                hlen[k] = len(r.out)
                if r.temperature > 0.0:
                    u[k] = r.rng.random_sample()
            smp.history[:m].copy_(torch.from_numpy(hist))
            smp.hist_len[:m].copy_(torch.from_numpy(hlen))
            smp.uniforms[:m].copy_(torch.from_numpy(u))
            if m == batch:
                lg = logits[:batch]
            else:
                if self._logits_c is None:
                    self._logits_c = torch.empty_like(self._logits_buf())
                    self._d_idx = torch.zeros(self._logits_rows, dtype=torch.int64, device=self.eng.device)
                self._d_idx[:m].copy_(torch.as_tensor(idx, dtype=torch.int64))
                lg = self._logits_c[:m]
                torch.index_select(logits, 0, self._d_idx[:m], out=lg)
            out[idx] = smp.sample(lg, temp, top_p, rp, m).cpu().numpy()[:m]
        return out
