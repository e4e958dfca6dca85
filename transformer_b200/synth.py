"""Seeded synthetic weights and prompts for the benchmark configurations.

There is no checkpoint or dataset on the GPU box, so every configuration runs
on seeded synthetic inputs of the reference model's shape:

* weights: each matrix N(0, 0.02) drawn as float32 from
  ``numpy.random.default_rng(seed)`` in the reference's parameter order
  (``model.py:49-83``: ``token_emb``, then per layer ``attn.q, attn.k, attn.v,
  attn.o, ffn.gate, ffn.up, ffn.down``), rounded to bf16 (round-to-nearest-even).
  Norm gains are 1.  Shapes follow the reference ``(in, out)`` convention.
* prompts / lengths / uniforms: the per-configuration seeds below.

Parameter names are the reference's, so the dict can be fed to the packer
exactly like ``weights.pkl["params"]`` (``generate.py:161-164``).
"""

from __future__ import annotations

import numpy as np

try:
    import ml_dtypes
    BF16 = ml_dtypes.bfloat16
except ImportError:  # pragma: no cover - ml_dtypes ships with the image
    BF16 = None

from .config import ModelConfig


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns (uint16), round-to-nearest-even."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if BF16 is not None:
        return x.astype(BF16).view(np.uint16)
    u = x.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def param_shapes(cfg: ModelConfig):
    """(name, shape) in the reference's init order (model.py:49-89)."""
    d, kv, f = cfg.d_model, cfg.d_kv, cfg.d_ff
    out = [("token_emb", (cfg.vocab_size, d))]
    for l in range(cfg.n_layers):
        p = f"layer{l}"
        out += [(f"{p}.ln1.scale", (d,)),
                (f"{p}.attn.q", (d, d)), (f"{p}.attn.k", (d, kv)),
                (f"{p}.attn.v", (d, kv)), (f"{p}.attn.o", (d, d)),
                (f"{p}.ln2.scale", (d,)),
                (f"{p}.ffn.gate", (d, f)), (f"{p}.ffn.up", (d, f)),
                (f"{p}.ffn.down", (f, d))]
    out.append(("ln_final.scale", (d,)))
    return out


def synth_params(cfg: ModelConfig, seed: int = 0, std: float = 0.02):
    """Seeded bf16 weights as a dict name -> uint16 bf16-bit array.

    Norm scales are float32 ones.  Matrices are drawn in the reference order
    and rounded to bf16 once; every consumer (oracle, packer) reads these bits.
    """
    rng = np.random.default_rng(seed)
    params = {}
    for name, shape in param_shapes(cfg):
        if name.endswith(".scale"):
            params[name] = np.ones(shape, dtype=np.float32)
        else:
            a = rng.standard_normal(shape, dtype=np.float32)
            a *= np.float32(std)
            params[name] = to_bf16_bits(a)
    return params


def params_f32(params: dict) -> dict:
    """bf16-bit dict -> float32 dict (the values the f32 oracle computes on)."""
    out = {}
    for k, v in params.items():
        out[k] = bf16_bits_to_f32(v) if v.dtype == np.uint16 else np.asarray(v, np.float32)
    return out


# ---- per-configuration inputs -----------------------

def prompt_cfg1(cfg: ModelConfig = None, n: int = 16):
    """Config 1: 16-token prompt uniform in [0, vocab) from seed 1."""
    vocab = (cfg or ModelConfig()).vocab_size
    return np.random.default_rng(1).integers(0, vocab, n).astype(np.int32)


def prompt_cfg2(cfg: ModelConfig = None, n: int = 384):
    """Config 2: 384-token prompt from seed 1 (prefilled, then decode to 512)."""
    vocab = (cfg or ModelConfig()).vocab_size
    return np.random.default_rng(1).integers(0, vocab, n).astype(np.int32)


def batch_cfg3(cfg: ModelConfig = None, batch: int = 64, lo: int = 32, hi: int = 448,
               block: int = 16):
    """Config 3: B=64 prompts with lengths U[32,448] from seed 2, token ids from
    the same generator, and a random block table (a permutation of physical
    16-token blocks, each sequence owning ctx/16 of them)."""
    cfg = cfg or ModelConfig()
    rng = np.random.default_rng(2)
    lens = rng.integers(lo, hi + 1, batch).astype(np.int32)
    prompts = [rng.integers(0, cfg.vocab_size, int(L)).astype(np.int32) for L in lens]
    per_seq = cfg.context_len // block
    table = rng.permutation(batch * per_seq).astype(np.int32).reshape(batch, per_seq)
    return lens, prompts, table


def batch_cfg4(cfg: ModelConfig = None, batch: int = 8, prompt_len: int = 64, steps: int = 128):
    """Config 4: B=8 64-token prompts (seed 3) and per-step uniforms f32
    [steps, B] from seed 4 for the sampler."""
    cfg = cfg or ModelConfig()
    prompts = np.random.default_rng(3).integers(0, cfg.vocab_size, (batch, prompt_len)).astype(np.int32)
    u = np.random.default_rng(4).random((steps, batch), dtype=np.float32)
    return prompts, u


def batch_cfg5(cfg: ModelConfig = None, total: int = 2048, prompt_len: int = 64):
    """Config 5: 2048 64-token prompts (seed 5), partitioned across GPUs."""
    cfg = cfg or ModelConfig()
    return np.random.default_rng(5).integers(0, cfg.vocab_size, (total, prompt_len)).astype(np.int32)
