"""Weight and KV-cache packing (device side, PyTorch owns the buffers).

Mirrors the reference packing helpers in ``kernels/fused_decode_nlayer.py``:

* ``pack_weights`` (ref :250-270) — the reference concatenates each layer's
  ``[ln1, q, k, v, o, ln2, gate, up, down]`` in their ``(in, out)`` layout.
  Here every matrix is stored output-row-major (row r = the weights producing
  output r, contiguous along the reduction dimension), q/k/v rows are stacked
  into one ``qkv`` block, gate and up rows are interleaved per hidden unit, and
  norm gains stay float32.  The tied embedding is used in place as the output
  projection, so the reference's transposed, padded copy
  (``prepare_decode_weights_nlayer`` :312-319) is not made.  Byte offsets come
  from ``b2d_weights_layout`` so Python and the kernels agree.
* ``pack_kv_caches`` / ``unpack_kv_caches`` (ref :273-296) — unchanged format:
  ``[layer][K|V][kv_head][context_len][d_head]`` bf16, K post-RoPE.
* ``prepare_decode_weights_nlayer`` (ref :299-321) — returns the dict ``w`` the
  decode entry point takes.
"""

from __future__ import annotations

import numpy as np
import torch

from . import _lib
from .config import ModelConfig


def rope_tables(cfg: ModelConfig):
    """float32 cos/sin tables (context_len, d_head//2), ``model.py:101-107``."""
    half = cfg.d_head // 2
    freqs = cfg.rope_base ** (-np.arange(0, half, dtype=np.float32) * 2.0 / cfg.d_head)
    positions = np.arange(cfg.context_len, dtype=np.float32)
    angles = positions[:, None] * freqs[None, :]
    return np.cos(angles).astype(np.float32), np.sin(angles).astype(np.float32)


def _as_config(config) -> ModelConfig:
    return config if isinstance(config, ModelConfig) else ModelConfig.from_dict(config)


def _bf16(a, device) -> torch.Tensor:
    """Parameter -> bf16 device tensor.  numpy uint16 arrays are bf16 bit
    patterns (``synth``); float arrays are rounded to nearest-even."""
    if isinstance(a, torch.Tensor):
        return a.to(device=device, dtype=torch.bfloat16)
    a = np.asarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(device).view(torch.bfloat16)
    if a.dtype.name == "bfloat16":
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(device).view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(device).to(torch.bfloat16)


def _f32(a, device) -> torch.Tensor:
    if isinstance(a, torch.Tensor):
        return a.to(device=device, dtype=torch.float32)
    a = np.asarray(a)
    if a.dtype == np.uint16:
        a = (a.astype(np.uint32) << 16).view(np.float32)
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(device)


def _section(buf: torch.Tensor, off: int, shape, dtype) -> torch.Tensor:
    n = int(np.prod(shape))
    nbytes = n * torch.empty((), dtype=dtype).element_size()
    return buf[off:off + nbytes].view(dtype).view(*shape)


def pack_weights(params: dict, config, device=None) -> torch.Tensor:
    """Pack reference-named params into one device buffer (uint8 tensor)."""
    cfg = _as_config(config)
    device = torch.device(device or "cuda")
    lay = _lib.weights_layout(cfg)
    buf = torch.zeros(int(lay.total_bytes), dtype=torch.uint8, device=device)
    d, f, H, KVH, dh, L = cfg.d_model, cfg.d_ff, cfg.n_heads, cfg.n_kv_heads, cfg.d_head, cfg.n_layers
    qkv_rows = (H + 2 * KVH) * dh
    ln1 = _section(buf, lay.off_ln1, (L, d), torch.float32)
    ln2 = _section(buf, lay.off_ln2, (L, d), torch.float32)
    for l in range(L):
        p = f"layer{l}"
        base = l * lay.layer_stride
        qkv = _section(buf, base + lay.off_qkv, (qkv_rows, d), torch.bfloat16)
        qkv[:H * dh].copy_(_bf16(params[f"{p}.attn.q"], device).T)
        qkv[H * dh:(H + KVH) * dh].copy_(_bf16(params[f"{p}.attn.k"], device).T)
        qkv[(H + KVH) * dh:].copy_(_bf16(params[f"{p}.attn.v"], device).T)
        _section(buf, base + lay.off_o, (d, d), torch.bfloat16).copy_(_bf16(params[f"{p}.attn.o"], device).T)
        gu = _section(buf, base + lay.off_gu, (f, 2, d), torch.bfloat16)
        gu[:, 0].copy_(_bf16(params[f"{p}.ffn.gate"], device).T)
        gu[:, 1].copy_(_bf16(params[f"{p}.ffn.up"], device).T)
        _section(buf, base + lay.off_down, (d, f), torch.bfloat16).copy_(
            _bf16(params[f"{p}.ffn.down"], device).T)
        ln1[l].copy_(_f32(params[f"{p}.ln1.scale"], device))
        ln2[l].copy_(_f32(params[f"{p}.ln2.scale"], device))
    _section(buf, lay.off_emb, (cfg.vocab_size, d), torch.bfloat16).copy_(_bf16(params["token_emb"], device))
    _section(buf, lay.off_lnf, (d,), torch.float32).copy_(_f32(params["ln_final.scale"], device))
    cos, sin = rope_tables(cfg)
    _section(buf, lay.off_cos, cos.shape, torch.float32).copy_(torch.from_numpy(cos))
    _section(buf, lay.off_sin, sin.shape, torch.float32).copy_(torch.from_numpy(sin))
    return buf


def kv_elems(config) -> int:
    cfg = _as_config(config)
    return int(_lib.kv_layout(cfg).elems_per_seq)


def new_kv_cache(config, batch: int = 1, device=None) -> torch.Tensor:
    """Zeroed KV caches for ``batch`` sequences, reference layout, batch-major."""
    return torch.zeros(batch * kv_elems(config), dtype=torch.bfloat16, device=device or "cuda")


def pack_kv_caches(k_caches, v_caches, device=None) -> torch.Tensor:
    """``fused_decode_nlayer.py:273-283``: [layer0_k, layer0_v, layer1_k, ...]."""
    parts = []
    for k, v in zip(k_caches, v_caches):
        parts.append(_bf16(k, device or "cuda").reshape(-1))
        parts.append(_bf16(v, device or "cuda").reshape(-1))
    return torch.cat(parts)


def unpack_kv_caches(packed, n_layers, n_kv_heads, max_seq, d_head):
    """``fused_decode_nlayer.py:286-296``: flat buffer -> per-layer (K, V) views."""
    layer = 2 * n_kv_heads * max_seq * d_head
    half = n_kv_heads * max_seq * d_head
    ks, vs = [], []
    for i in range(n_layers):
        b = i * layer
        ks.append(packed[b:b + half].reshape(n_kv_heads, max_seq, d_head))
        vs.append(packed[b + half:b + layer].reshape(n_kv_heads, max_seq, d_head))
    return ks, vs


def prepare_decode_weights_nlayer(params: dict, config, kv_splits: int = 1, device=None) -> dict:
    """``fused_decode_nlayer.py:299-321``: everything the decode step reads.

    ``kv_splits`` is accepted for signature compatibility; the engine chooses
    its attention split by the current position.  ``vocab_pad`` equals the
    vocabulary: no padded output projection exists.
    """
    cfg = _as_config(config)
    buf = pack_weights(params, cfg, device)
    lay = _lib.weights_layout(cfg)
    return {
        "packed_w": buf,
        "token_emb": _section(buf, lay.off_emb, (cfg.vocab_size, cfg.d_model), torch.bfloat16),
        "lnf_s": _section(buf, lay.off_lnf, (cfg.d_model,), torch.float32),
        "vocab_pad": cfg.vocab_size,
        "config": cfg,
        "layout": lay,
        "device": buf.device,
    }
