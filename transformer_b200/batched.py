"""Batched decode over a paged KV pool.

``BatchedDecoder`` owns one group ("wave") of up to ``max_batch`` sequences:
their slice of a paged KV pool, block table, token / position buffers and the
step's logits.  It ingests ragged prompts (a sequence idles with ``pos = -1``
once its prompt is in), then decodes greedily with the device argmax fed back
as the next token, optionally through a captured CUDA graph of one step (the
step is ~120 dependent kernel launches; the graph replays them without host
launch overhead, and the kernels' programmatic-launch edges are kept).

The reference has no batched decode kernel (its batched variants were removed:
``kernels/`` holds only the B=1 path); the step's math is the B=1 step's
(``kernels/multi_sm_decode.py``), one row per sequence.
"""

from __future__ import annotations

import numpy as np
import torch

from .multi_sm_decode import PAGE_TOKENS, DecodeEngine


class BatchedDecoder:
    """One wave of sequences on a batched engine (``max_batch >= batch``)."""

    def __init__(self, engine: DecodeEngine, batch: int, table: np.ndarray | None = None,
                 num_blocks: int | None = None, seed: int = 0):
        if engine.max_batch < max(2, batch):
            raise ValueError("engine max_batch is smaller than the batch")
        self.eng = engine
        cfg = engine.cfg
        self.cfg = cfg
        self.B = batch
        dev = engine.device
        self.bps = (cfg.context_len + PAGE_TOKENS - 1) // PAGE_TOKENS
        if table is None:  # a random permutation of the pool's blocks
            nb = num_blocks or batch * self.bps
            table = np.random.default_rng(seed).permutation(nb)[:batch * self.bps].reshape(batch, self.bps)
        else:
            nb = num_blocks or int(table.max()) + 1
        self.num_blocks = nb
        self.table = torch.from_numpy(np.ascontiguousarray(table, dtype=np.int32)).to(dev)
        self.pool = engine.new_kv_pool(nb)
        self.tok = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.logits = torch.zeros(batch, cfg.vocab_size, dtype=torch.float32, device=dev)
        self.graph = None

    # ---- one step -----------------------------------------------------------
    def step(self, stream=None):
        """Decode step at (tok, pos) -> logits; argmax written back to tok."""
        self.eng.step_paged(self.tok, self.pos, self.pool, self.table, self.logits, self.tok, stream)

    def ingest(self, prompts, stream=None) -> torch.Tensor:
        """Feed ragged prompts position by position; returns each sequence's
        last-prompt-position logits (device [B, vocab]) and leaves ``tok`` =
        argmax of those, ``pos`` = prompt lengths."""
        lens = np.array([len(p) for p in prompts], np.int64)
        if len(prompts) != self.B or lens.min() < 1 or lens.max() > self.cfg.context_len:
            raise ValueError("one non-empty prompt per sequence, no longer than the context")
        T = int(lens.max())
        toks = np.zeros((T, self.B), np.int32)
        poss = np.full((T, self.B), -1, np.int32)
        for b, p in enumerate(prompts):
            toks[:len(p), b] = p
            poss[:len(p), b] = np.arange(len(p))
        toks_d = torch.from_numpy(toks).to(self.eng.device)
        poss_d = torch.from_numpy(poss).to(self.eng.device)
        last = torch.zeros_like(self.logits)
        nxt = torch.zeros_like(self.tok)
        lens_d = torch.from_numpy(lens).to(self.eng.device)
        for t in range(T):
            self.eng.step_paged(toks_d[t], poss_d[t], self.pool, self.table, self.logits, nxt, stream)
            done = lens_d == t + 1  # sequences whose prompt ends here
            if bool((lens == t + 1).any()):
                last[done] = self.logits[done]
                self.tok[done] = nxt[done]
        self.pos.copy_(torch.from_numpy(lens.astype(np.int32)))
        return last

    # ---- graph-captured greedy decode ----------------------------------------
    def capture(self):
        """Capture one greedy step (+ pos += 1) as a CUDA graph."""
        s = torch.cuda.Stream(self.eng.device)
        s.wait_stream(torch.cuda.current_stream(self.eng.device))
        save_tok, save_pos = self.tok.clone(), self.pos.clone()
        with torch.cuda.stream(s):  # warm-up outside capture (tensor maps, attributes)
            self.step(s)
            self.pos.add_(1)
        torch.cuda.current_stream(self.eng.device).wait_stream(s)
        torch.cuda.synchronize(self.eng.device)
        self.tok.copy_(save_tok)
        self.pos.copy_(save_pos)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.step()
            self.pos.add_(1)
        self.graph = g
        return g

    def replay(self):
        self.graph.replay()

    def greedy(self, n_steps: int, use_graph: bool = True) -> torch.Tensor:
        """Run n_steps greedy steps; returns device int32 [n_steps, B] where
        row i is the argmax of the logits at position pos0 + i (the token the
        step after ``ingest``'s first token produces, and so on)."""
        out = torch.zeros(n_steps, self.B, dtype=torch.int32, device=self.eng.device)
        if use_graph and self.graph is None:
            self.capture()
        for i in range(n_steps):
            if use_graph:
                self.replay()
            else:
                self.step()
                self.pos.add_(1)
            out[i].copy_(self.tok)
        return out

    def release(self):
        self.graph = None
