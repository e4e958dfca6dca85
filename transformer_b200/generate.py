"""Host generation loop over the device decode step and the device sampler.

Mirrors the reference's ``generate.py``:

* ``sample_token`` (ref :28-65) — same arguments; the draw runs on the device
  (``b2d_sample``).  The uniform that numpy's ``np.random.choice`` would draw is
  taken from ``u`` or, when omitted, from numpy's global legacy RNG exactly as
  the reference consumes it, so a seeded run draws the same uniforms.
* ``stream_tokens`` / ``generate_tokens`` (ref :92-130) — prefill, first token
  from the prompt's last logits, then ``max_tokens - 1`` decode steps at
  ``pos = prompt_len + i``; greedy (temperature 0 and no penalty) uses the
  kernel's argmax, everything else the sampler with the generated history.

The prompt goes through the device prefill (``b2d_prefill``: every prompt
position in one pass of the batched tensor-core step, K/V written into the
reference-layout cache), where the reference prefills with JAX
(``model.py:194-231``).  For many concurrent requests see
``transformer_b200.serve``.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from .multi_sm_decode import DecodeEngine, _ptr, _stream_ptr
from .packing import prepare_decode_weights_nlayer


class Sampler:
    """Device buffers for ``b2d_sample`` over up to ``max_batch`` sequences."""

    def __init__(self, engine: DecodeEngine, max_batch: int = 1, hist_cap: int = 512):
        self.eng = engine
        self.lib = engine.lib
        dev = engine.device
        self.max_batch, self.hist_cap = max_batch, hist_cap
        self.history = torch.zeros(max_batch, hist_cap, dtype=torch.int32, device=dev)
        self.hist_len = torch.zeros(max_batch, dtype=torch.int32, device=dev)
        self.uniforms = torch.zeros(max_batch, dtype=torch.float64, device=dev)
        self.out = torch.zeros(max_batch, dtype=torch.int32, device=dev)

    def sample(self, logits: torch.Tensor, temperature: float, top_p: float, rep_penalty: float,
               batch: int | None = None, uniforms: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """Sample one token per row of ``logits`` [batch, vocab] (device, f32).
        ``self.history[:batch]`` / ``self.hist_len`` hold each row's generated
        tokens; ``uniforms`` (device f64 [batch]) defaults to ``self.uniforms``."""
        batch = batch or logits.shape[0]
        if logits.dtype != torch.float32 or not logits.is_contiguous() or logits.device != self.eng.device:
            raise ValueError("logits must be contiguous float32 on the model device")
        if batch > self.max_batch:
            raise ValueError("batch exceeds the sampler's max_batch")
        u = self.uniforms if uniforms is None else uniforms
        params = _lib.Sampling(float(temperature), float(top_p), float(rep_penalty))
        st = self.lib.b2d_sample(self.eng.ws, _ptr(logits), batch, logits.shape[-1], _ptr(self.history),
                                 self.hist_cap, _ptr(self.hist_len), _ptr(u), ctypes.byref(params),
                                 _ptr(self.out), _stream_ptr(stream))
        _lib.check(st, "b2d_sample")
        return self.out[:batch]


_SAMPLERS: dict = {}


def _sampler_for(engine: DecodeEngine, hist_cap: int) -> Sampler:
    key = (id(engine), hist_cap)
    s = _SAMPLERS.get(key)
    if s is None:
        s = Sampler(engine, 1, hist_cap)
        _SAMPLERS[key] = s
    return s


def sample_token(logits, temperature, top_p, rep_penalty, generated_ids, u=None, engine=None):
    """``generate.py:28-65`` on the device.  ``logits``: float32 [vocab] device
    tensor; ``generated_ids``: tokens generated so far; ``u``: the uniform
    (default: one draw from numpy's global legacy RNG, as np.random.choice
    would make).  Returns the token id (int)."""
    if engine is None:
        from .multi_sm_decode import _ENGINES
        if not _ENGINES:
            raise RuntimeError("sample_token needs a DecodeEngine (pass engine=)")
        engine = next(iter(_ENGINES.values()))
    gen = list(generated_ids)
    smp = _sampler_for(engine, max(512, len(gen)))
    if temperature == 0.0:
        u = 0.0
    elif u is None:
        u = np.random.random_sample()
    n = len(gen)
    if n:
        smp.history[0, :n].copy_(torch.tensor(gen, dtype=torch.int32))
    smp.hist_len[0] = n
    smp.uniforms[0] = float(u)
    lg = logits.reshape(1, -1).to(device=engine.device, dtype=torch.float32).contiguous()
    return int(smp.sample(lg, temperature, top_p, rep_penalty, 1).item())


def _prefill(w, config, prompt_ids):
    """``generate.py:68-89``: returns (engine, first_logits, start_pos, kv)."""
    eng = w if isinstance(w, DecodeEngine) else DecodeEngine(w)
    kv = eng.new_kv()
    first = eng.prefill(np.asarray(prompt_ids, dtype=np.int32), kv).clone()
    return eng, first, len(prompt_ids), kv


def stream_tokens(params, config, prompt_ids, max_tokens=128, temperature=0.0, top_p=1.0,
                  rep_penalty=1.0, seed=None, uniforms=None):
    """``generate.py:92-123``.  ``params``: the reference parameter dict, a
    ``prepare_decode_weights_nlayer`` result, or a ``DecodeEngine``.
    ``uniforms``: optional per-step uniforms (else numpy's seeded legacy RNG)."""
    if seed is not None:
        np.random.seed(seed)
    if isinstance(params, DecodeEngine) or (isinstance(params, dict) and "packed_w" in params):
        w = params
    else:
        w = prepare_decode_weights_nlayer(params, config)
    eng, first_logits, start_pos, kv = _prefill(w, config, prompt_ids)
    greedy = temperature == 0.0 and rep_penalty == 1.0
    cap = max(start_pos + max_tokens, 1)
    smp = Sampler(eng, 1, cap)
    dev = eng.device
    tok_buf = torch.zeros(1, dtype=torch.int32, device=dev)
    pos_buf = torch.zeros(1, dtype=torch.int32, device=dev)
    logits = eng.logits
    step = 0

    def draw():
        if temperature == 0.0:
            return 0.0
        if uniforms is not None:
            return float(uniforms[step])
        return np.random.random_sample()

    def choose(lg_row):
        if greedy:
            return int(torch.argmax(lg_row).item())
        smp.uniforms[0] = draw()
        return int(smp.sample(lg_row.reshape(1, -1), temperature, top_p, rep_penalty, 1).item())

    tok = choose(first_logits)
    smp.history[0, 0] = tok
    smp.hist_len[0] = 1
    yield tok
    for i in range(max_tokens - 1):
        step = i + 1
        tok_buf[0] = tok
        pos_buf[0] = start_pos + i
        eng.step(tok_buf, pos_buf, kv, logits, eng.next_tok)
        if greedy:
            tok = int(eng.next_tok[0].item())
        else:
            tok = choose(logits[0])
        smp.history[0, step] = tok
        smp.hist_len[0] = step + 1
        yield tok


def generate_tokens(params, config, prompt_ids, n_tokens=128, temperature=0.0, top_p=1.0,
                    rep_penalty=1.0, seed=None, uniforms=None):
    """``generate.py:126-130``."""
    return list(stream_tokens(params, config, prompt_ids, n_tokens, temperature, top_p, rep_penalty,
                              seed, uniforms))
