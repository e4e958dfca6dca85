"""The decode step that allocates nothing (b2d_decode_step_static).

Some users of this library cannot let it allocate device memory: a serving
process or plugin host that owns every device buffer through its own memory
pool, or code running where calling cudaMalloc is not allowed.  For them the
library offers a decode step whose scratch lives in a fixed 4 MiB array of
device memory inside the library instead of a workspace from
b2d_workspace_create.  These tests call it through the C ABI and check that it
computes what the regular entry point computes.

This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import assert_logits_close
from transformer_b200 import _lib
from transformer_b200.config import CONFIG_306M, CONFIG_TINY, ModelConfig


def _p(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def test_static_step_rejects_models_beyond_its_fixed_scratch():
    """A model whose exchange area exceeds the fixed array is refused with
    B2D_ERR_SCRATCH_LIMIT before any device work (no GPU needed)."""
    from transformer_b200 import build
    build.build()
    lib = _lib.load()
    big = _lib.make_config(ModelConfig(n_layers=64))  # ~5.4 MB of exchange words
    fake = ctypes.c_void_p(0x100000)  # never dereferenced: rejected first
    st = lib.b2d_decode_step_static(ctypes.byref(big), fake, ctypes.c_uint64(1 << 40), fake, fake, fake, None,
                                    fake, None)
    assert st == _lib.B2D_ERR_SCRATCH_LIMIT
    assert "4 MiB" in lib.b2d_status_str(st).decode()


@pytest.mark.gpu
@pytest.mark.parametrize("which", ["tiny", "306m"])
def test_static_step_matches_workspace_step(which, request):
    """Two calls in a row of the no-allocation step produce the logits, next
    tokens and KV-cache writes of the regular step (same tolerance as the
    parity tests), the second call starting from the first call's outputs."""
    eng = request.getfixturevalue("engine_tiny" if which == "tiny" else "engine306")
    cfg = CONFIG_TINY if which == "tiny" else CONFIG_306M
    lib = _lib.load()
    dev = eng.device
    buf = eng.w["packed_w"]
    ccfg = _lib.make_config(cfg)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    kv_ref, kv_sta = eng.new_kv(), eng.new_kv()
    lg_ref = torch.zeros(cfg.vocab_size, dtype=torch.float32, device=dev)
    lg_sta = torch.zeros_like(lg_ref)
    nx_ref = torch.zeros(1, dtype=torch.int32, device=dev)
    nx_sta = torch.zeros_like(nx_ref)
    tok = torch.tensor([7], dtype=torch.int32, device=dev)
    for call in range(2):
        pos = torch.tensor([call], dtype=torch.int32, device=dev)
        eng.step(tok, pos, kv_ref, lg_ref, nx_ref)
        st = lib.b2d_decode_step_static(ctypes.byref(ccfg), _p(buf), ctypes.c_uint64(buf.numel()), _p(tok),
                                        _p(pos), _p(kv_sta), _p(lg_sta), _p(nx_sta), stream)
        assert st == _lib.B2D_OK, lib.b2d_status_str(st).decode()
        torch.cuda.synchronize(dev)
        assert_logits_close(lg_sta.cpu().numpy(), lg_ref.cpu().numpy(), f"{which} call {call}")
        assert int(nx_sta.item()) == int(nx_ref.item())
        assert int(nx_sta.item()) == int(np.argmax(lg_sta.cpu().numpy()))
        tok = nx_ref.clone()
    np.testing.assert_allclose(kv_sta.float().cpu().numpy(), kv_ref.float().cpu().numpy(), atol=3e-2, rtol=2e-2)
    eng.check_device()
