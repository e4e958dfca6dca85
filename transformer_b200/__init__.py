"""B200-native decode engine for the zahlmann/transformer 306M decoder.

The hot path is one persistent sm_100a CUDA kernel per decode step (all layers,
logits and argmax), reached through the C ABI in ``include/b2d.h``
(``libb2d.so``) via ``ctypes``.  Submodules mirror the reference's host API:

* ``multi_sm_decode``  ``multi_sm_decode_nlayer`` (kernels/multi_sm_decode.py)
* ``packing``          ``pack_weights`` / ``pack_kv_caches`` / ``unpack_kv_caches`` /
                       ``prepare_decode_weights_nlayer`` (kernels/fused_decode_nlayer.py)
* ``generate``         ``sample_token`` / ``stream_tokens`` / ``generate_tokens``
                       (generate.py)

The reference's measurement functions (``measure_decode`` /
``compute_memory_stats``, profile_kernels.py) live in the top-level
``profile_kernels.py`` beside ``bench.py``, not in this package.

Heavy imports (torch, the shared library) happen in those submodules, so
``config`` and ``synth`` stay importable on a CPU-only host.
"""

from .config import ModelConfig, CONFIG_306M, CONFIG_TINY  # noqa: F401
