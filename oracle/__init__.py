"""CPU oracle for the decode hot path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may import this package, and only as the checker (or as the
timed stand-in for the reference's own CPU implementation).  The product path
(``transformer_b200``) never imports it and has no CPU fallback.

Contents
--------
``ref_forward``  numpy float32 restatement of the reference model numerics
                 (``model.py:94-231``): RMSNorm, RoPE, GQA causal attention,
                 SwiGLU, tied logits, ``prefill_with_kv``, plus a KV-cached
                 decode step with the same math.
``sampler``      restatement of ``generate.py:28-65`` ``sample_token`` with
                 ``np.random.choice`` replaced by its inverse-CDF on a
                 supplied uniform.

Pinning
-------
The reference needs JAX, which is absent from this image.  Its own Python
code (``model.py``, ``generate.py``, ``kernels/fused_decode_nlayer.py``) is
imported in the build container through a numpy-backed stand-in for the few
``jax`` calls it makes (``tests/golden/make_golden.py``), and its outputs are
committed as fixtures under ``tests/golden/``.  The CPU tests check this
oracle against those fixtures, so the oracle is pinned to the reference's own
code.  The two third-party primitives the reference calls,
``jax.nn.dot_product_attention`` and ``jax.nn.silu`` (jax 0.9.2 per the
reference ``uv.lock``), are restated from their published definitions; that
restatement is the one piece not pinned by running the reference.
"""
