"""Decode entry points over the C ABI.

``multi_sm_decode_nlayer`` keeps the reference's call shape
(``kernels/multi_sm_decode.py:369-432``): ``(w, config, token_id, pos,
kv_packed, kv_splits=1) -> (next_token, logits, kv)``.  Differences, by design:
the KV cache is updated in place (the returned ``kv`` is the same tensor; the
reference returns a fresh copy, :198-208), the workspace is allocated once per
model instead of zeroed per call (:390-400), and ``token_id`` / ``pos`` may be
device int32 tensors so a loop can feed the previous step's output without a
host round trip.

``DecodeEngine`` is the lower-level handle the host loop, tests and bench use:
one bound model, one workspace, preallocated step buffers.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from .config import ModelConfig
from .packing import kv_elems, new_kv_cache

PAGE_TOKENS = 16  # positions per KV block of the paged pool


def _ptr(t: torch.Tensor | None):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _stream_ptr(stream) -> ctypes.c_void_p:
    if stream is None:
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


class DecodeEngine:
    """A packed model bound to the C ABI plus one workspace."""

    def __init__(self, w: dict, max_batch: int = 1):
        self.lib = _lib.load()
        self.w = w
        self.cfg: ModelConfig = w["config"]
        buf = w["packed_w"]
        self.device = buf.device
        self._cfg_c = _lib.make_config(self.cfg)
        if not self.lib.b2d_config_supported(ctypes.byref(self._cfg_c)):
            raise _lib.B2DError(_lib.B2D_ERR_UNSUPPORTED, "b2d_config_supported", str(self.cfg))
        model = ctypes.c_void_p()
        _lib.check(self.lib.b2d_model_create(ctypes.byref(self._cfg_c), _ptr(buf), buf.numel(),
                                             self.device.index or 0, ctypes.byref(model)),
                   "b2d_model_create")
        self.model = model
        ws = ctypes.c_void_p()
        try:
            _lib.check(self.lib.b2d_workspace_create(self.model, max_batch, ctypes.byref(ws)),
                       "b2d_workspace_create")
        except Exception:
            self.lib.b2d_model_destroy(self.model)
            raise
        self.ws = ws
        self.max_batch = max_batch
        self.grid = self.lib.b2d_model_grid(self.model)
        dev = self.device
        self.tok = torch.zeros(max_batch, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(max_batch, dtype=torch.int32, device=dev)
        self.next_tok = torch.zeros(max_batch, dtype=torch.int32, device=dev)
        self.logits = torch.zeros(max_batch, self.cfg.vocab_size, dtype=torch.float32, device=dev)

    def close(self):
        if getattr(self, "ws", None):
            self.lib.b2d_workspace_destroy(self.ws)
            self.ws = None
        if getattr(self, "model", None):
            self.lib.b2d_model_destroy(self.model)
            self.model = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- buffers -------------------------------------------------------
    def new_kv(self, batch: int = 1) -> torch.Tensor:
        return new_kv_cache(self.cfg, batch, self.device)

    @property
    def kv_elems(self) -> int:
        return kv_elems(self.cfg)

    # ---- one step ------------------------------------------------------
    def step(self, tok: torch.Tensor, pos: torch.Tensor, kv: torch.Tensor,
             logits: torch.Tensor | None = None, next_tok: torch.Tensor | None = None,
             stream=None, batch: int = 1) -> None:
        """Launch one decode step (async, stream-ordered).  All device tensors."""
        if next_tok is None:
            next_tok = self.next_tok
        for t, name in ((tok, "tok"), (pos, "pos"), (next_tok, "next_tok")):
            if t.dtype != torch.int32 or t.device != self.device or t.numel() < batch:
                raise ValueError(f"{name} must be an int32 tensor on {self.device} with >= {batch} items")
        if kv.dtype != torch.bfloat16 or kv.device != self.device or kv.numel() < batch * self.kv_elems:
            raise ValueError("kv must be a bf16 cache on the model device (see new_kv)")
        if logits is not None and (logits.dtype != torch.float32 or logits.numel() < batch * self.cfg.vocab_size):
            raise ValueError("logits must be float32 [batch, vocab]")
        st = self.lib.b2d_decode_step(self.model, self.ws, _ptr(tok), _ptr(pos), batch, _ptr(kv),
                                      _ptr(logits), _ptr(next_tok), _stream_ptr(stream))
        _lib.check(st, "b2d_decode_step")

    def decode_token(self, tok: int, pos: int, kv: torch.Tensor, logits: torch.Tensor | None = None,
                     stream=None) -> int:
        """One greedy step with host values (``b2d_decode_token``): the token
        and position go in the launch's arguments, the kernel writes the
        argmax to mapped pinned memory; returns it as a Python int (the stream
        is synchronised)."""
        if kv.dtype != torch.bfloat16 or kv.device != self.device or kv.numel() < self.kv_elems:
            raise ValueError("kv must be a bf16 cache on the model device (see new_kv)")
        if logits is not None and (logits.dtype != torch.float32 or logits.device != self.device or
                                   logits.numel() < self.cfg.vocab_size):
            raise ValueError("logits must be float32 [vocab] on the model device")
        nt = ctypes.c_int32()
        st = self.lib.b2d_decode_token(self.model, self.ws, int(tok), int(pos), _ptr(kv),
                                       _ptr(logits) if logits is not None else None, ctypes.byref(nt),
                                       _stream_ptr(stream))
        _lib.check(st, "b2d_decode_token")
        return int(nt.value)

    def decode_steps(self, tok: torch.Tensor, pos: torch.Tensor, kv: torch.Tensor, n_steps: int,
                     tokens: torch.Tensor | None = None, logits: torch.Tensor | None = None,
                     stream=None) -> torch.Tensor:
        """``n_steps`` greedy decode steps of one sequence in one launch
        (``b2d_decode_steps``): step s feeds step s-1's argmax back at position
        ``pos + s``.  Returns the device int32 [n_steps] tokens (async)."""
        if n_steps < 1:
            raise ValueError("n_steps must be >= 1")
        for t, name in ((tok, "tok"), (pos, "pos")):
            if t.dtype != torch.int32 or t.device != self.device or t.numel() < 1:
                raise ValueError(f"{name} must be an int32 tensor on {self.device}")
        if tokens is None:
            tokens = torch.zeros(n_steps, dtype=torch.int32, device=self.device)
        if tokens.dtype != torch.int32 or tokens.device != self.device or tokens.numel() < n_steps:
            raise ValueError(f"tokens must be an int32 tensor on {self.device} with >= {n_steps} items")
        if kv.dtype != torch.bfloat16 or kv.device != self.device or kv.numel() < self.kv_elems:
            raise ValueError("kv must be a bf16 cache on the model device (see new_kv)")
        if logits is not None and (logits.dtype != torch.float32 or logits.numel() < self.cfg.vocab_size):
            raise ValueError("logits must be float32 [vocab]")
        st = self.lib.b2d_decode_steps(self.model, self.ws, _ptr(tok), _ptr(pos), int(n_steps), _ptr(kv),
                                       _ptr(tokens), _ptr(logits), _stream_ptr(stream))
        _lib.check(st, "b2d_decode_steps")
        return tokens[:n_steps]

    def new_kv_pool(self, num_blocks: int) -> torch.Tensor:
        """Zeroed paged KV pool: bf16 [n_layers, num_blocks, 2 (K|V), kv_heads,
        16, d_head]; block i of a sequence holds its positions 16i..16i+15."""
        c = self.cfg
        return torch.zeros(c.n_layers, num_blocks, 2, c.n_kv_heads, PAGE_TOKENS, c.d_head,
                           dtype=torch.bfloat16, device=self.device)

    def _check_pool(self, pool: torch.Tensor) -> None:
        c = self.cfg
        if (pool.dtype != torch.bfloat16 or pool.device != self.device or not pool.is_contiguous() or pool.dim() != 6
                or tuple(pool.shape[i] for i in (0, 2, 3, 4, 5)) != (c.n_layers, 2, c.n_kv_heads, PAGE_TOKENS,
                                                                     c.d_head)):
            raise ValueError("pool must be a paged KV pool of this model (see new_kv_pool)")

    def step_paged(self, tok: torch.Tensor, pos: torch.Tensor, pool: torch.Tensor,
                   block_table: torch.Tensor, logits: torch.Tensor | None = None,
                   next_tok: torch.Tensor | None = None, stream=None, batch: int | None = None) -> None:
        """One batched decode step over a paged KV pool (async, stream-ordered).

        ``tok`` / ``pos``: int32 [batch] (``pos < 0``: sequence idle this step);
        ``block_table``: int32 [batch, blocks_per_seq]; ``logits``: float32
        [batch, vocab] or None; ``next_tok``: int32 [batch] (argmax)."""
        if self.max_batch < 2:
            raise ValueError("step_paged needs an engine created with max_batch >= 2")
        batch = batch or tok.numel()
        if next_tok is None:
            next_tok = self.next_tok
        for t, name in ((tok, "tok"), (pos, "pos"), (next_tok, "next_tok")):
            if t.dtype != torch.int32 or t.device != self.device or t.numel() < batch or not t.is_contiguous():
                raise ValueError(f"{name} must be a contiguous int32 tensor on {self.device} with >= {batch} items")
        c = self.cfg
        self._check_pool(pool)
        if (block_table.dtype != torch.int32 or block_table.device != self.device or block_table.dim() != 2
                or block_table.shape[0] < batch or not block_table.is_contiguous()):
            raise ValueError("block_table must be a contiguous int32 [batch, blocks_per_seq] device tensor")
        if logits is not None and (logits.dtype != torch.float32 or logits.numel() < batch * c.vocab_size
                                   or not logits.is_contiguous()):
            raise ValueError("logits must be contiguous float32 [batch, vocab]")
        st = self.lib.b2d_decode_step_paged(self.model, self.ws, _ptr(tok), _ptr(pos), batch, _ptr(pool),
                                            _ptr(block_table), block_table.shape[1], pool.shape[1],
                                            _ptr(logits), _ptr(next_tok), _stream_ptr(stream))
        _lib.check(st, "b2d_decode_step_paged")

    def last_error(self, stream=None):
        """(status, raw device word); synchronises the stream."""
        detail = ctypes.c_uint32(0)
        st = self.lib.b2d_last_error(self.ws, _stream_ptr(stream), ctypes.byref(detail))
        return st, detail.value

    def check_device(self, stream=None):
        st, detail = self.last_error(stream)
        if st != _lib.B2D_OK:
            raise _lib.B2DError(st, "device status", f"word 0x{detail:x}")

    def reset(self, stream=None):
        _lib.check(self.lib.b2d_workspace_reset(self.ws, _stream_ptr(stream)), "b2d_workspace_reset")

    def debug_set(self, wait_ns: int, extra_ctas: int = 0):
        _lib.check(self.lib.b2d_debug_set(self.ws, int(wait_ns), int(extra_ctas)), "b2d_debug_set")

    def trace_slots(self) -> int:
        return 1 + 13 * self.cfg.n_layers + 3

    def debug_trace(self, enable: bool = True) -> torch.Tensor | None:
        """Turn per-CTA phase stamps on (returns the int64 [grid, slots]
        device buffer the kernel fills) or off (returns None)."""
        if enable:
            self._trace = torch.zeros(self.grid, self.trace_slots(), dtype=torch.int64, device=self.device)
            _lib.check(self.lib.b2d_debug_trace(self.ws, _ptr(self._trace), self.trace_slots()), "b2d_debug_trace")
            return self._trace
        _lib.check(self.lib.b2d_debug_trace(self.ws, None, 0), "b2d_debug_trace")
        self._trace = None
        return None

    def debug_tune(self, poll_ns: int | None = None, max_inflight: int | None = None,
                   pdl: bool | None = None, ksplit: int | None = None, att_cpc: int | None = None,
                   gemm_trace: torch.Tensor | None = None, att_trace: torch.Tensor | None = None,
                   sample_trace: torch.Tensor | None = None, graphs: bool | None = None,
                   flat: bool | None = None, sample_mode: int | None = None, plain_launch: bool | None = None):
        """Diagnostic knobs: back-off between failed polls (ns), weight copies
        in flight per CTA; batched step: programmatic dependent launch on/off,
        forced K split, forced attention units per (sequence, kv head) (0 =
        automatic); device stamp buffers for the projections, the attention
        and the sampler (empty tensor = off); graph replay of repeated
        batched steps on / off; B=1 step on the flat one-CTA-per-SM kernel
        (True) or on the cluster kernel where it fits (False, default); the
        top-p sampler's kernel (0, default: a cluster of 16 CTAs per sequence
        where the batch's clusters fit one wave, else of 8; 1: one CTA per
        sequence; 2: clusters of 8 where they fit); the B=1
        cluster grid without the cooperative launch attribute (True: for
        profilers) or with it (False, default)."""
        if plain_launch is not None:
            _lib.check(self.lib.b2d_debug_tune(self.ws, 14, int(bool(plain_launch))), "b2d_debug_tune")
        if sample_mode is not None:
            _lib.check(self.lib.b2d_debug_tune(self.ws, 13, int(sample_mode)), "b2d_debug_tune")
        if flat is not None:
            _lib.check(self.lib.b2d_debug_tune(self.ws, 12, int(bool(flat))), "b2d_debug_tune")
        if graphs is not None:
            _lib.check(self.lib.b2d_debug_tune(self.ws, 11, int(bool(graphs))), "b2d_debug_tune")
        if sample_trace is not None:
            _lib.check(self.lib.b2d_debug_tune(self.ws, 10, sample_trace.data_ptr() if sample_trace.numel() else 0),
                       "b2d_debug_tune")
        if att_trace is not None:
            _lib.check(self.lib.b2d_debug_tune(self.ws, 9, att_trace.data_ptr() if att_trace.numel() else 0),
                       "b2d_debug_tune")
        if gemm_trace is not None:
            _lib.check(self.lib.b2d_debug_tune(self.ws, 6, gemm_trace.data_ptr() if gemm_trace.numel() else 0),
                       "b2d_debug_tune")
        if att_cpc is not None:
            _lib.check(self.lib.b2d_debug_tune(self.ws, 5, int(att_cpc)), "b2d_debug_tune")
        if pdl is not None:
            _lib.check(self.lib.b2d_debug_tune(self.ws, 3, int(bool(pdl))), "b2d_debug_tune")
        if ksplit is not None:
            _lib.check(self.lib.b2d_debug_tune(self.ws, 4, int(ksplit)), "b2d_debug_tune")
        if poll_ns is not None:
            _lib.check(self.lib.b2d_debug_tune(self.ws, 1, int(poll_ns)), "b2d_debug_tune")
        if max_inflight is not None:
            _lib.check(self.lib.b2d_debug_tune(self.ws, 2, int(max_inflight)), "b2d_debug_tune")

    # ---- prompt ingestion ----------------------------------------------
    def prefill(self, prompt, kv: torch.Tensor, start: int = 0, stream=None) -> torch.Tensor:
        """Device prefill (``b2d_prefill``): the prompt's positions run through
        the batched tensor-core step, writing the KV cache ``kv`` (one
        sequence, reference layout); returns the logits of the last prompt
        position (device [vocab]) and leaves its argmax in ``next_tok[0]``."""
        prompt = np.asarray(prompt, dtype=np.int32).reshape(-1)
        if prompt.size == 0:
            raise ValueError("empty prompt")
        if start + prompt.size > self.cfg.context_len:
            raise ValueError("prompt longer than the context")
        if kv.dtype != torch.bfloat16 or kv.device != self.device or kv.numel() < self.kv_elems:
            raise ValueError("kv must be a bf16 cache on the model device (see new_kv)")
        toks = torch.from_numpy(prompt).to(self.device)
        st = self.lib.b2d_prefill(self.model, self.ws, _ptr(toks), int(prompt.size), int(start), _ptr(kv),
                                  _ptr(self.logits), _ptr(self.next_tok), _stream_ptr(stream))
        _lib.check(st, "b2d_prefill")
        return self.logits[0]

    def prefill_paged(self, prompt, pool: torch.Tensor, table_row: torch.Tensor, start: int = 0,
                      stream=None, next_tok: torch.Tensor | None = None) -> torch.Tensor:
        """``b2d_prefill_paged``: as ``prefill``, into the paged pool ``pool``
        (see ``new_kv_pool``) through one sequence's block-table row
        ``table_row`` (device int32 [blocks_per_seq]).  Returns the last
        position's logits (device [vocab]); the argmax goes to ``next_tok[0]``
        (default: this engine's ``next_tok``)."""
        prompt = np.asarray(prompt, dtype=np.int32).reshape(-1)
        if prompt.size == 0:
            raise ValueError("empty prompt")
        self._check_pool(pool)
        if (table_row.dtype != torch.int32 or table_row.device != self.device or table_row.dim() != 1
                or not table_row.is_contiguous()):
            raise ValueError("table_row must be a contiguous int32 [blocks_per_seq] device tensor")
        if start < 0 or start + prompt.size > min(self.cfg.context_len, PAGE_TOKENS * table_row.numel()):
            raise ValueError("prompt runs past the context or the table row")
        nt = self.next_tok if next_tok is None else next_tok
        if nt.dtype != torch.int32 or nt.device != self.device:
            raise ValueError("next_tok must be an int32 device tensor")
        toks = torch.from_numpy(prompt).to(self.device)
        st = self.lib.b2d_prefill_paged(self.model, self.ws, _ptr(toks), int(prompt.size), int(start), _ptr(pool),
                                        _ptr(table_row), table_row.numel(), pool.shape[1], _ptr(self.logits),
                                        _ptr(nt), _stream_ptr(stream))
        _lib.check(st, "b2d_prefill_paged")
        return self.logits[0]

    @property
    def prefill_rows_max(self) -> int:
        """Rows one ``prefill_rows`` call takes (one prefill chunk)."""
        return int(self.lib.b2d_prefill_rows_max())

    def prefill_rows(self, tok: torch.Tensor, pos: torch.Tensor, pool: torch.Tensor, table: torch.Tensor,
                     n_out: int, logits: torch.Tensor | None = None, next_tok: torch.Tensor | None = None,
                     n_rows: int | None = None, stream=None) -> None:
        """``b2d_prefill_rows``: ``n_rows`` (<= 512) rows of tokens ``tok`` at
        positions ``pos`` of the sequences whose block-table rows are
        ``table`` [n_rows, blocks_per_seq] (device int32) through one pass
        over the weights, writing their K/V into ``pool``; the last ``n_out``
        rows get logits (float32 [n_out, vocab]) and / or argmax (int32
        [n_out]) when those buffers are given (async, stream-ordered)."""
        n_rows = n_rows or tok.numel()
        if not 1 <= n_rows <= self.lib.b2d_prefill_rows_max():
            raise ValueError(f"n_rows must be in [1, {self.lib.b2d_prefill_rows_max()}]")
        if not 0 <= n_out <= n_rows:
            raise ValueError("n_out must be in [0, n_rows]")
        for t, name in ((tok, "tok"), (pos, "pos")):
            if t.dtype != torch.int32 or t.device != self.device or t.numel() < n_rows or not t.is_contiguous():
                raise ValueError(f"{name} must be a contiguous int32 tensor on {self.device} with >= {n_rows} items")
        self._check_pool(pool)
        if (table.dtype != torch.int32 or table.device != self.device or table.dim() != 2
                or table.shape[0] < n_rows or not table.is_contiguous()):
            raise ValueError("table must be a contiguous int32 [n_rows, blocks_per_seq] device tensor")
        if logits is not None and (logits.dtype != torch.float32 or logits.device != self.device
                                   or logits.numel() < n_out * self.cfg.vocab_size or not logits.is_contiguous()):
            raise ValueError("logits must be contiguous float32 [n_out, vocab] on the model device")
        if next_tok is not None and (next_tok.dtype != torch.int32 or next_tok.device != self.device
                                     or next_tok.numel() < n_out):
            raise ValueError("next_tok must be int32 [n_out] on the model device")
        if n_out == 0 and (logits is not None or next_tok is not None):
            raise ValueError("outputs given with n_out = 0")
        st = self.lib.b2d_prefill_rows(self.model, self.ws, _ptr(tok), _ptr(pos), int(n_rows), _ptr(pool),
                                       _ptr(table), table.shape[1], pool.shape[1], int(n_out), _ptr(logits),
                                       _ptr(next_tok), _stream_ptr(stream))
        _lib.check(st, "b2d_prefill_rows")

    def prefill_stepwise(self, prompt, kv: torch.Tensor, start: int = 0, stream=None) -> torch.Tensor:
        """Feed prompt tokens one decode step at a time (teacher forcing),
        writing the KV cache; returns the logits of the last prompt position."""
        prompt = np.asarray(prompt, dtype=np.int32).reshape(-1)
        if prompt.size == 0:
            raise ValueError("empty prompt")
        if start + prompt.size > self.cfg.context_len:
            raise ValueError("prompt longer than the context")
        toks = torch.from_numpy(prompt).to(self.device)
        poss = torch.arange(start, start + prompt.size, dtype=torch.int32, device=self.device)
        for i in range(prompt.size):
            self.step(toks[i:i + 1], poss[i:i + 1], kv, self.logits, self.next_tok, stream)
        return self.logits[0]


_ENGINES: dict = {}


def engine_for(w: dict) -> DecodeEngine:
    """One engine per packed weight buffer (the workspace is reused)."""
    key = w["packed_w"].data_ptr()
    eng = _ENGINES.get(key)
    if eng is None or eng.w is not w:
        eng = DecodeEngine(w)
        _ENGINES[key] = eng
    return eng


def multi_sm_decode_nlayer(w, config, token_id, pos, kv_packed, kv_splits=1):
    """Reference-compatible single decode step (``multi_sm_decode.py:369-432``).

    Returns ``(next_token, logits, kv_packed)``: a 0-d int32 device tensor, the
    float32 logits ``[vocab]`` (device) and the KV cache, updated in place.
    ``token_id`` / ``pos``: Python ints (range-checked here) or int32 device
    tensors (range-checked by the kernel, which then sets the device status).
    """
    eng = engine_for(w)
    cfg = eng.cfg
    if isinstance(token_id, torch.Tensor):
        tok = token_id.reshape(-1)[:1].to(device=eng.device, dtype=torch.int32)
    else:
        token_id = int(token_id)
        if not 0 <= token_id < cfg.vocab_size:
            raise _lib.B2DError(_lib.B2D_ERR_INVALID_ARG, "multi_sm_decode_nlayer", f"token_id {token_id}")
        tok = torch.tensor([token_id], dtype=torch.int32).to(eng.device, non_blocking=True)
    if isinstance(pos, torch.Tensor):
        p = pos.reshape(-1)[:1].to(device=eng.device, dtype=torch.int32)
    else:
        pos = int(pos)
        if not 0 <= pos < cfg.context_len:
            raise _lib.B2DError(_lib.B2D_ERR_INVALID_ARG, "multi_sm_decode_nlayer", f"pos {pos}")
        p = torch.tensor([pos], dtype=torch.int32).to(eng.device, non_blocking=True)
    logits = torch.empty(cfg.vocab_size, dtype=torch.float32, device=eng.device)
    nxt = torch.empty(1, dtype=torch.int32, device=eng.device)
    eng.step(tok, p, kv_packed, logits, nxt)
    return nxt[0], logits, kv_packed
