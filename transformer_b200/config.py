"""Model configuration, same keys as the reference config dict.

The reference builds its config in ``model.py:37-47`` (``init_transformer``):
``vocab_size, d_model, n_heads, n_kv_heads, n_layers, d_head, d_ff,
context_len, n_mtp_heads``.  The decode path reads exactly those keys
(``kernels/multi_sm_decode.py:371-382``).  RMSNorm eps (``model.py:94``) and the
RoPE base (``model.py:101``) are fixed constants there and fields here.
"""

from __future__ import annotations

import dataclasses


def swiglu_d_ff(d_model: int) -> int:
    """SwiGLU hidden width, ``model.py:13-20``: 8d/3 rounded up to 128."""
    return ((8 * d_model // 3 + 127) // 128) * 128


@dataclasses.dataclass(frozen=True)
class ModelConfig:
    vocab_size: int = 32000
    d_model: int = 1024
    n_heads: int = 16
    n_kv_heads: int = 4
    n_layers: int = 24
    d_head: int = 64
    d_ff: int = 2816
    context_len: int = 512
    n_mtp_heads: int = 0
    rms_eps: float = 1e-5
    rope_base: float = 10000.0

    @classmethod
    def from_dict(cls, d: dict) -> "ModelConfig":
        keys = {f.name for f in dataclasses.fields(cls)}
        kw = {k: v for k, v in d.items() if k in keys}
        if "d_head" not in kw and "d_model" in kw and "n_heads" in kw:
            kw["d_head"] = kw["d_model"] // kw["n_heads"]
        if "d_ff" not in kw and "d_model" in kw:
            kw["d_ff"] = swiglu_d_ff(kw["d_model"])
        kw.setdefault("n_kv_heads", kw.get("n_heads", cls.n_heads))
        return cls(**kw)

    def as_dict(self) -> dict:
        return dataclasses.asdict(self)

    # ---- byte accounting used by the roofline ---------------------------
    @property
    def d_kv(self) -> int:
        return self.n_kv_heads * self.d_head

    @property
    def layer_matrix_elems(self) -> int:
        d, kv, f = self.d_model, self.d_kv, self.d_ff
        return d * d + 2 * d * kv + d * d + 3 * d * f

    @property
    def weight_bytes_per_step(self) -> int:
        """Algorithmic weight bytes streamed by one decode step.

        24 layers of bf16 matrices plus two bf16-sized norm vectors per layer
        (the reference packs them as bf16, ``fused_decode_nlayer.py:250-270``),
        the tied embedding read once as the output projection, one embedding
        row and the final norm: 606,703,616 B for the 306M model.
        """
        d = self.d_model
        per_layer = 2 * (self.layer_matrix_elems + 2 * d)
        return self.n_layers * per_layer + 2 * self.vocab_size * d + 2 * d + 2 * d

    @property
    def kv_bytes_per_position(self) -> int:
        """K+V bytes of one cached position over all layers (bf16)."""
        return 2 * 2 * self.n_layers * self.d_kv

    def step_bytes(self, positions) -> int:
        """Algorithmic HBM bytes of one step over sequences at ``positions``.

        ``W + sum_b [2*d*(b>0) + kv_bytes_per_position*(p_b+1)]``: each extra
        sequence reads its own embedding row; each reads p_b cached positions
        of K+V and writes one.
        """
        positions = list(positions)
        extra = sum(2 * self.d_model * (i > 0) + self.kv_bytes_per_position * (p + 1)
                    for i, p in enumerate(positions))
        return self.weight_bytes_per_step + extra

    @property
    def kv_elems_per_seq(self) -> int:
        return self.n_layers * 2 * self.n_kv_heads * self.context_len * self.d_head


#: The 306M model every BASELINE config uses.
CONFIG_306M = ModelConfig()

#: A small model with the same structure, used by fast parity tests.
CONFIG_TINY = ModelConfig(vocab_size=512, d_model=256, n_heads=4, n_kv_heads=2,
                          n_layers=2, d_head=64, d_ff=swiglu_d_ff(256),
                          context_len=128)
