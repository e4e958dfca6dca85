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
* ``main`` (ref :133-236) — the command line: a reference ``weights.pkl``, the
  BPE tokenizer the reference's ``data.py:55-70`` locates, the same flags
  (``--prompt --max-tokens --weights --no-stream --temp --top-p
  --rep-penalty --seed``) and the same output (prompt, then the generated
  text, streamed token by token; timing on stderr).

The prompt goes through the device prefill (``b2d_prefill``: every prompt
position in one pass of the batched tensor-core step, K/V written into the
reference-layout cache), where the reference prefills with JAX
(``model.py:194-231``).  For many concurrent requests see
``transformer_b200.serve``.
"""

from __future__ import annotations

import argparse
import ctypes
import os
import pickle
import sys
import time

import numpy as np
import torch

from . import _lib
from .config import ModelConfig
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


# ---- command line (generate.py:133-236) -----------------------------------

def load_checkpoint(path):
    """``generate.py:158-164``: a pickled ``{"params": {name: array}, "config":
    dict}`` checkpoint -> (params as numpy arrays, ModelConfig)."""
    with open(path, "rb") as f:
        saved = pickle.load(f)
    params = {k: np.asarray(v) for k, v in saved["params"].items()}
    return params, ModelConfig.from_dict(saved["config"])


def _tokenizer_file(tokenizer=None, weights=None):
    """The tokenizer JSON to load.  ``tokenizer`` may name the JSON itself or
    a ``bpe_vocab.pkl`` pointer file (``{"tokenizer_path", "vocab_size"}``,
    written by the reference's ``data.py:44-47``); by default the reference's
    own pointer, ``data/bpe_vocab.pkl`` beside the weights file, whose relative
    ``tokenizer_path`` is resolved against that directory (``data.py:59-63``)."""
    if tokenizer is None:
        root = os.path.dirname(os.path.abspath(weights or "."))
        tokenizer = os.path.join(root, "data", "bpe_vocab.pkl")
    if tokenizer.endswith(".pkl"):
        with open(tokenizer, "rb") as f:
            saved = pickle.load(f)
        path = saved["tokenizer_path"]
        if not os.path.isabs(path):
            path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(tokenizer))), path)
        return path
    return tokenizer


def load_tokenizer(tokenizer=None, weights=None):
    """``data.py:55-70`` ``load_bpe_vocab`` + ``generate.py:176-179``:
    returns (encode_fn(text) -> ids, decode_fn(ids) -> text)."""
    from tokenizers import Tokenizer
    tok = Tokenizer.from_file(_tokenizer_file(tokenizer, weights))
    return (lambda text: tok.encode(text).ids), (lambda ids: tok.decode([int(i) for i in ids]))


def fit_prompt(prompt_ids, context_len, max_tokens):
    """``generate.py:190-193``: keep at most ``context_len - 1`` prompt tokens
    and generate at most up to the context end -> (ids int32, max_gen)."""
    ids = list(prompt_ids)
    if len(ids) >= context_len:
        ids = ids[:context_len - 1]
    return np.asarray(ids, np.int32), min(max_tokens, context_len - len(ids))


def parse_args(argv=None):
    """The reference's flags (``generate.py:142-157``) plus ``--tokenizer``."""
    ap = argparse.ArgumentParser(description="Generate text with the B200 decode engine")
    ap.add_argument("--prompt", type=str, default="Once upon a time", help="Text prompt to continue")
    ap.add_argument("--max-tokens", type=int, default=256, help="Maximum tokens to generate")
    ap.add_argument("--weights", type=str, default="weights.pkl", help="Path to weights file")
    ap.add_argument("--tokenizer", type=str, default=None,
                    help="tokenizers JSON (or bpe_vocab.pkl); default: data/bpe_vocab.pkl beside the weights")
    ap.add_argument("--no-stream", action="store_true", help="Generate all tokens at once (no streaming)")
    ap.add_argument("--temp", type=float, default=0.0, help="Sampling temperature (0 = greedy)")
    ap.add_argument("--top-p", type=float, default=1.0, help="Nucleus sampling threshold")
    ap.add_argument("--rep-penalty", type=float, default=1.0, help="Repetition penalty (1.0 = off)")
    ap.add_argument("--seed", type=int, default=None, help="Random seed for reproducible sampling")
    return ap.parse_args(argv)


def main(argv=None, out=None, err=None):
    """``generate.py:133-236``: prompt text in, generated text out."""
    args = parse_args(argv)
    out = out or sys.stdout
    err = err or sys.stderr
    params, cfg = load_checkpoint(args.weights)
    encode_fn, decode_fn = load_tokenizer(args.tokenizer, args.weights)
    print(f"Model: d={cfg.d_model} h={cfg.n_heads} l={cfg.n_layers} ctx={cfg.context_len}", file=err)
    print(f"Params: {sum(p.size for p in params.values()):,}", file=err)
    if args.temp > 0:
        print(f"Sampling: temp={args.temp} top_p={args.top_p} rep_penalty={args.rep_penalty}", file=err)
    else:
        print("Decoding: greedy (argmax)", file=err)
    print(file=err)
    prompt_ids, max_gen = fit_prompt(encode_fn(args.prompt), cfg.context_len, args.max_tokens)
    print(f"Prompt ({len(prompt_ids)} tokens): {args.prompt}", file=err)
    print(f"Generating {max_gen} tokens...", file=err)
    print(file=err)
    eng = DecodeEngine(prepare_decode_weights_nlayer(params, cfg))
    out.write(args.prompt)
    out.flush()
    tokens = []
    t0 = time.perf_counter()
    if args.no_stream:
        tokens = generate_tokens(eng, cfg, prompt_ids, max_gen, args.temp, args.top_p, args.rep_penalty,
                                 args.seed)
        elapsed = time.perf_counter() - t0
        out.write(decode_fn(tokens))
        out.write("\n")
        out.flush()
        print(f"\n[{max_gen} tokens in {elapsed * 1000:.0f}ms = {max_gen / elapsed:.0f} tok/s]", file=err)
    else:
        t_first = None
        for token_id in stream_tokens(eng, cfg, prompt_ids, max_gen, args.temp, args.top_p, args.rep_penalty,
                                      args.seed):
            if t_first is None:
                t_first = time.perf_counter()
            tokens.append(token_id)
            piece = decode_fn([token_id])
            if piece:
                out.write(piece)
                out.flush()
        elapsed = time.perf_counter() - t0
        out.write("\n")
        out.flush()
        ttft = (t_first - t0) * 1000 if t_first else 0.0
        decode_time = elapsed - (t_first - t0) if t_first else elapsed
        rate = (max_gen - 1) / decode_time if decode_time > 0 else 0.0
        print(f"\n[{max_gen} tokens, TTFT={ttft:.0f}ms, decode={rate:.0f} tok/s]", file=err)
    eng.close()
    return tokens


if __name__ == "__main__":
    main()
