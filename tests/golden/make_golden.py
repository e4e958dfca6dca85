"""Generate the golden fixtures under tests/golden/ from the reference's own code.

Run in the build container, where the reference checkout is readable:

    python tests/golden/make_golden.py --ref <path to zahlmann/transformer> [--only NAME]

The reference imports ``jax``, ``jax.numpy`` and ``jax_triton``, none of which
are installed.  This script registers a small numpy-backed stand-in for the
handful of jax calls the reference's forward, prefill, packing and sampling
code makes (array creation, elementwise math, ``.at[].set``, ``jax.checkpoint``,
``jax.nn.silu``, ``jax.nn.dot_product_attention``), then imports the
reference's unmodified ``model.py``, ``generate.py`` and
``kernels/fused_decode_nlayer.py`` and records what they compute.  The
attention primitive is restated from jax 0.9.2's XLA implementation
(``jax._src.nn.functions._dot_product_attention_xla``): grouped heads
(query head n reads kv head n // G), ``einsum * scale``, causal ``tril`` mask
filled with ``-0.7 * finfo.max``, float32 softmax, ``einsum`` with values.

Fixtures (all small):
  tiny.npz          tiny model: forward logits, prefill logits + bf16 KV caches,
                    reference rms_norm / rope outputs, packed-format digests
  cfg1_greedy.npz   306M config 1: reference greedy stream (full-prefix
                    recompute, f32), per-step top-1 / margin, full logits at
                    18 steps (0, 1, every 8th, the last)
  cfg2_long.npz     306M config 2: same over a 384-token prompt to ctx 512
  sampling.npz      reference sample_token vs supplied-uniform restatement
  cfg4_sampled.npz  306M config 4: sampled token streams from the oracle
"""

from __future__ import annotations

import argparse
import hashlib
import math
import os
import sys
import time
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

import ml_dtypes  # noqa: E402

from transformer_b200.config import CONFIG_306M, CONFIG_TINY  # noqa: E402
from transformer_b200 import synth  # noqa: E402


# --------------------------------------------------------------------------
# numpy-backed stand-in for the jax surface the reference touches
# --------------------------------------------------------------------------

class Arr(np.ndarray):
    """ndarray with jax's functional ``.at[idx].set(v)``."""

    @property
    def at(self):
        arr = self

        class _At:
            def __getitem__(self, idx):
                class _Upd:
                    def set(self, v):
                        out = np.array(arr, copy=True).view(Arr)
                        out[idx] = v
                        return out
                return _Upd()
        return _At()

    def block_until_ready(self):
        return self


def _wrap(x):
    return np.asarray(x).view(Arr)


def _make_jax():
    jnp = types.ModuleType("jax.numpy")
    jnp.float32 = np.float32
    jnp.bfloat16 = ml_dtypes.bfloat16
    jnp.int32 = np.int32
    for name in ("sqrt", "mean", "cos", "sin", "exp", "log", "sum", "max", "argmax",
                 "maximum", "where", "tril", "einsum", "take_along_axis", "pad"):
        fn = getattr(np, name)
        setattr(jnp, name, (lambda f: lambda *a, **k: _wrap(f(*a, **k)))(fn))
    jnp.arange = lambda *a, **k: _wrap(np.arange(*a, **k))
    jnp.zeros = lambda *a, **k: _wrap(np.zeros(*a, **k))
    jnp.ones = lambda *a, **k: _wrap(np.ones(*a, **k))
    jnp.full = lambda *a, **k: _wrap(np.full(*a, **k))
    jnp.array = lambda a, dtype=None: _wrap(np.array(a, dtype=dtype))
    jnp.asarray = jnp.array
    jnp.concatenate = lambda xs, axis=0: _wrap(np.concatenate([np.asarray(x) for x in xs], axis=axis))
    jnp.promote_types = np.promote_types

    nn = types.ModuleType("jax.nn")

    def silu(x):
        x = np.asarray(x)
        return _wrap(x * (x.dtype.type(1) / (x.dtype.type(1) + np.exp(-x))))

    def softmax(x, axis=-1):
        m = np.max(x, axis=axis, keepdims=True)
        e = np.exp(x - m)
        return e / np.sum(e, axis=axis, keepdims=True)

    def dot_product_attention(query, key, value, bias=None, mask=None, *, scale=None,
                              is_causal=False, implementation=None, **kw):
        if implementation not in (None, "xla"):
            raise RuntimeError(f"implementation={implementation!r} needs a GPU")
        q, k, v = (np.asarray(t) for t in (query, key, value))
        squeeze = q.ndim == 3
        if squeeze:
            q, k, v = q[None], k[None], v[None]
        B, T, N, H = q.shape
        _, S, K, _ = k.shape
        G = N // K
        sc = np.float32(1.0 / math.sqrt(H) if scale is None else scale)
        qg = q.reshape(B, T, K, G, H)
        logits = np.einsum("btkgh,bskh->bkgts", qg, k).astype(np.float32) * sc
        if is_causal:
            cm = np.tril(np.ones((T, S), dtype=bool))
            logits = np.where(cm, logits, np.float32(-0.7 * np.finfo(np.float32).max))
        probs = softmax(logits.astype(np.float32), axis=-1).astype(k.dtype)
        enc = np.einsum("bkgts,bskh->btkgh", probs, v).reshape(B, T, N, H)
        return _wrap(enc[0] if squeeze else enc)

    nn.silu = silu
    nn.softmax = softmax
    nn.log_softmax = lambda x, axis=-1: _wrap(x - np.log(np.sum(np.exp(x - x.max(axis, keepdims=True)),
                                                                axis, keepdims=True)) - x.max(axis, keepdims=True))
    nn.dot_product_attention = dot_product_attention

    jax = types.ModuleType("jax")
    jax.numpy = jnp
    jax.nn = nn
    jax.checkpoint = lambda f, **kw: f
    jax.vmap = lambda f, *a, **k: (lambda xs: _wrap(np.stack([f(x) for x in xs])))

    class _CustomVJP:
        def __init__(self, fun, nondiff_argnums=()):
            self.fun = fun

        def defvjp(self, fwd, bwd):
            pass

        def __call__(self, *a, **k):
            return self.fun(*a, **k)

    jax.custom_vjp = _CustomVJP
    jax.random = types.ModuleType("jax.random")
    jax.tree = types.SimpleNamespace(leaves=lambda t: list(t.values()) if isinstance(t, dict) else [t])
    jax.devices = lambda: [types.SimpleNamespace(device_kind="cpu")]
    jax.ShapeDtypeStruct = lambda shape, dtype: (shape, dtype)

    jt = types.ModuleType("jax_triton")

    def _no_triton_call(*a, **k):
        raise RuntimeError("the reference Triton kernel needs a GPU")
    jt.triton_call = _no_triton_call
    return jax, jnp, nn, jt


def import_reference(ref_dir):
    jax, jnp, nn, jt = _make_jax()
    sys.modules.update({"jax": jax, "jax.numpy": jnp, "jax.nn": nn, "jax_triton": jt,
                        "jax.random": jax.random})
    sys.path.insert(0, ref_dir)
    import model as ref_model  # noqa: E402
    import generate as ref_generate  # noqa: E402
    from kernels import fused_decode_nlayer as ref_fdn  # noqa: E402
    return ref_model, ref_generate, ref_fdn


def ref_params(cfg, seed=0):
    """Seeded synthetic params as the reference consumes them: float32 arrays
    holding bf16 values (generate.py:163 loads float32 params)."""
    p = synth.params_f32(synth.synth_params(cfg, seed))
    return {k: _wrap(v) for k, v in p.items()}, p


def ref_config(cfg):
    return {"vocab_size": cfg.vocab_size, "d_model": cfg.d_model, "n_heads": cfg.n_heads,
            "n_kv_heads": cfg.n_kv_heads, "n_layers": cfg.n_layers, "d_head": cfg.d_head,
            "d_ff": cfg.d_ff, "context_len": cfg.context_len, "n_mtp_heads": 0,
            "gradient_checkpoint": False}


def top2(lg):
    lg = np.asarray(lg, dtype=np.float32)
    i = int(np.argmax(lg))
    part = np.partition(lg, -2)
    return i, float(part[-1]), float(part[-1] - part[-2])


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# --------------------------------------------------------------------------
# fixtures
# --------------------------------------------------------------------------

def make_tiny(ref):
    ref_model, ref_generate, ref_fdn = ref
    cfg = CONFIG_TINY
    P, _ = ref_params(cfg)
    conf = ref_config(cfg)
    prompt = np.random.default_rng(1).integers(0, cfg.vocab_size, 24).astype(np.int32)
    logits_fwd = np.asarray(ref_model.transformer_forward(P, conf, prompt), np.float32)
    lg_pre, kc, vc = ref_model.prefill_with_kv(P, conf, prompt)
    kv_ref = np.asarray(ref_fdn.pack_kv_caches(kc, vc)).view(np.uint16)
    # the reference packs weights in its own (in,out) flat layout; record digests
    packed = np.asarray(ref_fdn.pack_weights(P, conf)).view(np.uint16)
    w = ref_fdn.prepare_decode_weights_nlayer(P, conf)
    x = np.random.default_rng(7).standard_normal((5, cfg.d_model)).astype(np.float32)
    scale = np.random.default_rng(8).standard_normal(cfg.d_model).astype(np.float32)
    rms = np.asarray(ref_model.rms_norm(_wrap(x), _wrap(scale)), np.float32)
    cos, sin = ref_model.precompute_rope_table(cfg.context_len, cfg.d_head)
    xr = np.random.default_rng(9).standard_normal((3, 6, cfg.d_head)).astype(np.float32)
    roped = np.asarray(ref_model.apply_rope(_wrap(xr), np.asarray(cos)[:6], np.asarray(sin)[:6]), np.float32)
    np.savez_compressed(
        os.path.join(HERE, "tiny.npz"), prompt=prompt, logits_forward=logits_fwd,
        logits_prefill=np.asarray(lg_pre, np.float32), kv_packed_bits=kv_ref,
        packed_w_sha=sha(packed), packed_w_len=packed.size, vocab_pad=int(w["vocab_pad"]),
        out_proj_shape=np.array(np.asarray(w["output_proj_padded"]).shape),
        rms_x=x, rms_scale=scale, rms_out=rms, rope_cos=np.asarray(cos, np.float32),
        rope_sin=np.asarray(sin, np.float32), rope_x=xr, rope_out=roped)
    print("tiny.npz written")


def greedy_full_recompute(ref_model, P, conf, prompt, n_tokens, keep_steps):
    """generate.py:92-123 greedy semantics with the reference forward as the
    per-step oracle (F6: decode step p == transformer_forward(prefix)[-1])."""
    seq = list(int(t) for t in prompt)
    toks, top1, margin, kept = [], [], [], {}
    t0 = time.time()
    for i in range(n_tokens):
        lg = np.asarray(ref_model.transformer_forward(P, conf, np.array(seq, np.int32))[-1], np.float32)
        a, v, m = top2(lg)
        toks.append(a)
        top1.append(v)
        margin.append(m)
        if i in keep_steps:
            kept[i] = lg
        seq.append(a)
        if i % 16 == 0:
            print(f"  step {i} tok {a} margin {m:.4f} ({time.time() - t0:.0f}s)", flush=True)
    return np.array(toks, np.int32), np.array(top1, np.float32), np.array(margin, np.float32), kept


def make_cfg_greedy(ref, name, prompt, n_tokens):
    ref_model = ref[0]
    cfg = CONFIG_306M
    P, _ = ref_params(cfg)
    conf = ref_config(cfg)
    # full logits at 18 steps spread over the stream (0, 1, every 8th, the last)
    keep = tuple(sorted({0, 1, n_tokens - 1, *range(8, n_tokens - 1, 8)}))
    toks, top1, margin, kept = greedy_full_recompute(ref_model, P, conf, prompt, n_tokens, keep)
    np.savez_compressed(os.path.join(HERE, name), prompt=prompt.astype(np.int32), tokens=toks,
                        top1=top1, margin=margin, logits_steps=np.array(keep, np.int32),
                        logits=np.stack([kept[k] for k in keep]))
    print(name, "written; tokens[:8] =", toks[:8])


def make_sampling(ref):
    """Reference sample_token (np.random.seed) vs the supplied-uniform oracle."""
    ref_generate = ref[1]
    sys.path.insert(0, REPO)
    from oracle.sampler import sample_token as oracle_sample
    rng = np.random.default_rng(11)
    cases = []
    n_exact = n_total = n_agree_unpatched = 0
    real_np = ref_generate.np

    class PatchedNp:
        """numpy with the host-independent exp and tie order the oracle defines."""
        def __getattr__(self, k):
            return getattr(real_np, k)

        @staticmethod
        def exp(x):
            return np.exp(np.asarray(x, np.float64)).astype(np.asarray(x).dtype)

        @staticmethod
        def argsort(a):
            a = np.asarray(a)
            return np.lexsort((np.arange(a.size), a))
    for case in range(48):
        vocab = 32000
        logits = (rng.standard_normal(vocab) * 0.64 * (1 + case % 3)).astype(np.float32)
        temp = [0.7, 1.0, 0.3, 0.0][case % 4]
        top_p = [0.95, 1.0, 0.5][case % 3]
        rp = [1.2, 1.0][case % 2]
        hist = rng.integers(0, vocab, case % 40).astype(np.int32)
        seed = 1000 + case
        u = np.random.RandomState(seed).random_sample()
        ours = oracle_sample(logits, temp, top_p, rp, list(hist), u)
        np.random.seed(seed)
        ref_generate.np = PatchedNp()
        try:
            ref_tok = ref_generate.sample_token(logits, temp, top_p, rp, list(hist))
        finally:
            ref_generate.np = real_np
        np.random.seed(seed)
        ref_unpatched = ref_generate.sample_token(logits, temp, top_p, rp, list(hist))
        n_total += 1
        n_exact += int(ours == ref_tok)
        n_agree_unpatched += int(ours == ref_unpatched)
        cases.append((case, temp, top_p, rp, seed, u, ref_tok, ref_unpatched, len(hist)))
    arr = np.array(cases, dtype=np.float64)
    np.savez_compressed(os.path.join(HERE, "sampling.npz"), cases=arr,
                        columns=np.array(["case", "temp", "top_p", "rp", "seed", "u", "ref_tok",
                                          "ref_tok_host_exp", "hist_len"]),
                        logits_seed=11)
    print(f"sampling.npz: oracle == reference(host-independent exp) {n_exact}/{n_total}; "
          f"== reference(host np.exp) {n_agree_unpatched}/{n_total}")
    assert n_exact == n_total


def make_cfg4(ref):
    """Config 4 sampled streams on the oracle (B=8, T=0.7, top-p 0.95, rp 1.2)."""
    sys.path.insert(0, REPO)
    from oracle.ref_forward import CachedDecoder
    from oracle.sampler import sample_token
    cfg = CONFIG_306M
    _, P = ref_params(cfg)
    prompts, u = synth.batch_cfg4(cfg, steps=128)
    B, L = prompts.shape
    dec = CachedDecoder(P, cfg, B)
    lg = None
    for p in range(L):
        lg = dec.step(prompts[:, p], np.full(B, p))
    gen = [[] for _ in range(B)]
    margins = np.zeros((128, B), np.float32)
    t0 = time.time()
    for i in range(128):
        toks = []
        for b in range(B):
            t = sample_token(lg[b], 0.7, 0.95, 1.2, gen[b], u[i, b])
            gen[b].append(t)
            toks.append(t)
        if i + 1 < 128:
            lg = dec.step(np.array(toks), np.full(B, L + i))
        if i % 16 == 0:
            print(f"  cfg4 step {i} ({time.time() - t0:.0f}s)", flush=True)
    np.savez_compressed(os.path.join(HERE, "cfg4_sampled.npz"), prompts=prompts, uniforms=u,
                        tokens=np.array(gen, np.int32), temperature=0.7, top_p=0.95, rep_penalty=1.2)
    print("cfg4_sampled.npz written")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the reference checkout")
    ap.add_argument("--only", default=None)
    a = ap.parse_args()
    ref = import_reference(os.path.abspath(a.ref))
    todo = {
        "tiny": lambda: make_tiny(ref),
        "sampling": lambda: make_sampling(ref),
        "cfg1": lambda: make_cfg_greedy(ref, "cfg1_greedy.npz", synth.prompt_cfg1(), 128),
        "cfg2": lambda: make_cfg_greedy(ref, "cfg2_long.npz", synth.prompt_cfg2(), 128),
        "cfg4": lambda: make_cfg4(ref),
    }
    for k, fn in todo.items():
        if a.only is None or k in a.only.split(","):
            fn()


if __name__ == "__main__":
    main()
