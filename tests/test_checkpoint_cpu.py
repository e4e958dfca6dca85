"""CPU: loading a reference-format checkpoint (``weights.pkl``:
``{"params": {name: array}, "config": dict}``, generate.py:161-164)."""

from __future__ import annotations

import pickle

import numpy as np

from transformer_b200.config import CONFIG_TINY, ModelConfig
from transformer_b200.synth import params_f32, synth_params


def test_load_reference_checkpoint(tmp_path):
    import profile_kernels as pk
    params = params_f32(synth_params(CONFIG_TINY, 0))
    cfg = {k: v for k, v in CONFIG_TINY.as_dict().items()}
    cfg["n_mtp_heads"] = 0  # keys the decoder does not use are ignored
    path = tmp_path / "weights.pkl"
    with open(path, "wb") as f:
        pickle.dump({"params": params, "config": cfg}, f)
    got, config = pk.load_params(str(path))
    assert set(got) == set(params)
    for k in params:
        np.testing.assert_array_equal(got[k], params[k])
    assert ModelConfig.from_dict(config) == CONFIG_TINY
