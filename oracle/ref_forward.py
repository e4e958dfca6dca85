"""Float32 numpy restatement of the reference model forward (TEST ORACLE).

Test infrastructure only; see ``oracle/__init__.py``.  Every function cites
the reference line it restates (paths inside zahlmann/transformer).  The
reference runs these in float32 on CPU (its bf16 attention branch needs cuDNN,
``model.py:136-143``), over float32 parameters holding bf16-representable
values; so does this oracle.
"""

from __future__ import annotations

import math

import numpy as np

f32 = np.float32


def round_bf16(x):
    """float32 -> nearest bf16 value (ties to even), returned as float32."""
    u = np.ascontiguousarray(x, dtype=f32).view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return u.astype(np.uint32).view(f32)


def rms_norm(x, scale, eps=1e-5):
    """``model.py:94-98``: ``scale * (x / sqrt(mean(x^2) + eps))`` in f32."""
    x32 = x.astype(f32)
    rms = np.sqrt(np.mean(x32 ** 2, axis=-1, keepdims=True) + f32(eps)).astype(x.dtype)
    return scale * (x / rms)


def precompute_rope_table(context_len, d_head, base=10000.0):
    """``model.py:101-107``: f32 cos/sin tables of shape (ctx, d_head//2)."""
    half = d_head // 2
    freqs = base ** (-np.arange(0, half, dtype=f32) * 2.0 / d_head)
    positions = np.arange(context_len, dtype=f32)
    angles = positions[:, None] * freqs[None, :]
    return np.cos(angles).astype(f32), np.sin(angles).astype(f32)


def apply_rope(x, cos, sin):
    """``model.py:110-117``: rotate-half RoPE on the last dim."""
    half = x.shape[-1] // 2
    x_even, x_odd = x[..., :half], x[..., half:]
    return np.concatenate([x_even * cos - x_odd * sin,
                           x_even * sin + x_odd * cos], axis=-1)


def softmax(x, axis=-1):
    """``jax.nn.softmax`` (jax 0.9.2): exp(x - max) / sum, in f32."""
    m = np.max(x, axis=axis, keepdims=True)
    e = np.exp(x - m)
    return e / np.sum(e, axis=axis, keepdims=True)


def dot_product_attention_causal(q, k, v):
    """Restatement of ``jax.nn.dot_product_attention(q, k, v, is_causal=True)``
    on its XLA path (jax 0.9.2), as called at ``model.py:143``.

    q: (T, N, H), k/v: (S, K, H) with N a multiple of K; query head n reads kv
    head n // (N // K).  logits = einsum(q, k) * (1/sqrt(H)), masked with a
    large negative number above the diagonal, f32 softmax, einsum with v.
    """
    T, N, H = q.shape
    S, K, _ = k.shape
    G = N // K
    scale = f32(1.0 / math.sqrt(H))
    kk = np.repeat(k, G, axis=1)  # (S, N, H): head n -> kv head n // G
    vv = np.repeat(v, G, axis=1)
    logits = np.einsum("tnh,snh->nts", q, kk).astype(f32) * scale
    mask = np.tril(np.ones((T, S), dtype=bool))
    big_neg = f32(-0.7 * np.finfo(f32).max)
    logits = np.where(mask[None], logits, big_neg)
    probs = softmax(logits, axis=-1).astype(f32)
    return np.einsum("nts,snh->tnh", probs, vv).astype(f32)


def silu(x):
    """``jax.nn.silu`` = x * sigmoid(x)."""
    return x * (f32(1) / (f32(1) + np.exp(-x)))


def causal_attention(x, wq, wk, wv, wo, n_heads, n_kv_heads, cos, sin):
    """``model.py:122-145`` (f32 branch)."""
    T, d = x.shape
    dh = d // n_heads
    q = (x @ wq).reshape(T, n_heads, dh)
    k = (x @ wk).reshape(T, n_kv_heads, dh)
    v = (x @ wv).reshape(T, n_kv_heads, dh)
    c, s = cos[:T], sin[:T]
    q = apply_rope(q.transpose(1, 0, 2), c[None], s[None]).transpose(1, 0, 2)
    k = apply_rope(k.transpose(1, 0, 2), c[None], s[None]).transpose(1, 0, 2)
    out = dot_product_attention_causal(q, k, v.astype(q.dtype))
    return out.reshape(T, d) @ wo


def layer_forward(h, P, l, cfg, cos, sin):
    """``model.py:150-160`` ``_attn_layer``: pre-norm attention + SwiGLU."""
    p = f"layer{l}"
    hn = rms_norm(h, P[f"{p}.ln1.scale"], cfg.rms_eps)
    h = h + causal_attention(hn, P[f"{p}.attn.q"], P[f"{p}.attn.k"], P[f"{p}.attn.v"],
                             P[f"{p}.attn.o"], cfg.n_heads, cfg.n_kv_heads, cos, sin)
    hn2 = rms_norm(h, P[f"{p}.ln2.scale"], cfg.rms_eps)
    ff = (silu(hn2 @ P[f"{p}.ffn.gate"]) * (hn2 @ P[f"{p}.ffn.up"])) @ P[f"{p}.ffn.down"]
    return h + ff


def transformer_forward(P, cfg, x):
    """``model.py:163-191``: logits (T, vocab) for tokens x (T,)."""
    cos, sin = precompute_rope_table(cfg.context_len, cfg.d_head, cfg.rope_base)
    h = P["token_emb"][np.asarray(x)]
    for l in range(cfg.n_layers):
        h = layer_forward(h, P, l, cfg, cos, sin)
    h = rms_norm(h, P["ln_final.scale"], cfg.rms_eps)
    return h @ P["token_emb"].T


def prefill_with_kv(P, cfg, x):
    """``model.py:194-231``: logits plus bf16 K (post-RoPE) / V caches.

    Caches are returned as float32 arrays holding bf16-rounded values, shape
    (n_kv_heads, context_len, d_head) per layer.
    """
    x = np.asarray(x)
    T = x.shape[0]
    cos, sin = precompute_rope_table(cfg.context_len, cfg.d_head, cfg.rope_base)
    h = P["token_emb"][x]
    kc, vc = [], []
    for l in range(cfg.n_layers):
        p = f"layer{l}"
        hn = rms_norm(h, P[f"{p}.ln1.scale"], cfg.rms_eps)
        k = (hn @ P[f"{p}.attn.k"]).reshape(T, cfg.n_kv_heads, cfg.d_head)
        v = (hn @ P[f"{p}.attn.v"]).reshape(T, cfg.n_kv_heads, cfg.d_head)
        k = apply_rope(k, cos[:T, None, :], sin[:T, None, :])
        K = np.zeros((cfg.n_kv_heads, cfg.context_len, cfg.d_head), f32)
        V = np.zeros_like(K)
        K[:, :T] = round_bf16(k.transpose(1, 0, 2))
        V[:, :T] = round_bf16(v.transpose(1, 0, 2))
        kc.append(K)
        vc.append(V)
        h = h + causal_attention(hn, P[f"{p}.attn.q"], P[f"{p}.attn.k"], P[f"{p}.attn.v"],
                                 P[f"{p}.attn.o"], cfg.n_heads, cfg.n_kv_heads, cos, sin)
        hn2 = rms_norm(h, P[f"{p}.ln2.scale"], cfg.rms_eps)
        h = h + (silu(hn2 @ P[f"{p}.ffn.gate"]) * (hn2 @ P[f"{p}.ffn.up"])) @ P[f"{p}.ffn.down"]
    logits = rms_norm(h, P["ln_final.scale"], cfg.rms_eps) @ P["token_emb"].T
    return logits, kc, vc


class CachedDecoder:
    """KV-cached decode with the reference forward's float32 numerics.

    Step p of ``step`` returns ``transformer_forward(prefix[:p+1])[-1]`` (the
    oracle for decode step p, since the reference has no cached decode of its
    own): keys/values of every earlier position are kept in float32, exactly
    as the full-prefix forward recomputes them, and the new position attends
    over positions 0..p.  Works on a batch of independent sequences.
    """

    def __init__(self, P, cfg, batch=1):
        self.P, self.cfg, self.B = P, cfg, batch
        self.cos, self.sin = precompute_rope_table(cfg.context_len, cfg.d_head, cfg.rope_base)
        shape = (batch, cfg.n_layers, cfg.n_kv_heads, cfg.context_len, cfg.d_head)
        self.K = np.zeros(shape, f32)
        self.V = np.zeros(shape, f32)
        self.layers = [tuple(P[f"layer{l}.{n}"] for n in
                             ("ln1.scale", "attn.q", "attn.k", "attn.v", "attn.o",
                              "ln2.scale", "ffn.gate", "ffn.up", "ffn.down"))
                       for l in range(cfg.n_layers)]

    def step(self, tokens, positions):
        """tokens, positions: int arrays (B,). Returns logits (B, vocab) f32."""
        cfg, P = self.cfg, self.P
        tokens = np.asarray(tokens).reshape(-1)
        positions = np.asarray(positions).reshape(-1)
        B, H, KVH, dh = len(tokens), cfg.n_heads, cfg.n_kv_heads, cfg.d_head
        G = H // KVH
        scale = f32(1.0 / math.sqrt(dh))
        h = P["token_emb"][tokens].astype(f32)  # (B, d)
        for l, (ln1, wq, wk, wv, wo, ln2, wg, wu, wd) in enumerate(self.layers):
            hn = rms_norm(h, ln1, cfg.rms_eps)
            q = (hn @ wq).reshape(B, H, dh)
            k = (hn @ wk).reshape(B, KVH, dh)
            v = (hn @ wv).reshape(B, KVH, dh)
            att = np.empty((B, H, dh), f32)
            for b in range(B):
                p = int(positions[b])
                c, s = self.cos[p], self.sin[p]
                qb = apply_rope(q[b], c, s)
                self.K[b, l, :, p] = apply_rope(k[b], c, s)
                self.V[b, l, :, p] = v[b]
                Kb = self.K[b, l, :, :p + 1]  # (KVH, p+1, dh)
                Vb = self.V[b, l, :, :p + 1]
                for n in range(H):
                    lg = (Kb[n // G] @ qb[n]).astype(f32) * scale
                    pr = softmax(lg).astype(f32)
                    att[b, n] = pr @ Vb[n // G]
            h = h + att.reshape(B, H * dh) @ wo
            hn2 = rms_norm(h, ln2, cfg.rms_eps)
            h = h + (silu(hn2 @ wg) * (hn2 @ wu)) @ wd
        h = rms_norm(h, P["ln_final.scale"], cfg.rms_eps)
        return h @ P["token_emb"].T


def top2(logits):
    """(argmax, top1 value, top1 - top2 margin) of a 1-D logits vector."""
    i = int(np.argmax(logits))
    part = np.partition(logits, -2)
    return i, float(part[-1]), float(part[-1] - part[-2])


def greedy_stream(P, cfg, prompt, n_tokens, batch_decoder=None):
    """``generate.py:92-123`` greedy path (temp 0, rp 1) on the oracle.

    First token from the prompt's last logits, then ``n_tokens - 1`` decode
    steps at ``pos = prompt_len + i``.  Returns (tokens, per-step logits list
    used for each token) — step 0's logits are the prompt's last position.
    """
    dec = batch_decoder or CachedDecoder(P, cfg, 1)
    prompt = np.asarray(prompt)
    lg = None
    for p, t in enumerate(prompt):
        lg = dec.step([t], [p])[0]
    toks, all_logits = [], []
    for i in range(n_tokens):
        all_logits.append(lg)
        t = int(np.argmax(lg))
        toks.append(t)
        if i + 1 < n_tokens:
            lg = dec.step([t], [len(prompt) + i])[0]
    return toks, all_logits
