"""The decode step that allocates nothing (b2d_decode_step_static).

Some users of this library cannot let it allocate device memory: a serving
process or plugin host that owns every device buffer through its own memory
pool, or code running where calling cudaMalloc is not allowed.  For them the
library offers a decode step whose scratch lives in a fixed 4 MiB array of
device memory inside the library instead of a workspace from
b2d_workspace_create.  These tests call it through the C ABI and check that it
computes exactly what the regular entry point computes, and that its device
status word can be read back without a workspace.

This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from transformer_b200 import _lib
from transformer_b200.config import CONFIG_306M, CONFIG_TINY, ModelConfig


def _p(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def test_static_step_rejects_models_beyond_its_fixed_scratch():
    """A model whose scratch exceeds the fixed array for either B=1 kernel
    (the flat kernel's exchange words, the cluster kernel's residual
    accumulators) is refused with B2D_ERR_SCRATCH_LIMIT before any device
    work (no GPU needed)."""
    from transformer_b200 import build
    build.build()
    lib = _lib.load()
    big = _lib.make_config(ModelConfig(n_layers=160))  # ~13.6 MB of exchange words, 5.2 MB of accumulators
    fake = ctypes.c_void_p(0x100000)  # never dereferenced: rejected first
    st = lib.b2d_decode_step_static(ctypes.byref(big), fake, ctypes.c_uint64(1 << 40), fake, fake, fake, None,
                                    fake, None)
    assert st == _lib.B2D_ERR_SCRATCH_LIMIT
    assert "4 MiB" in lib.b2d_status_str(st).decode()


def _static_status(lib, stream):
    detail = ctypes.c_uint32(0)
    st = lib.b2d_static_last_error(stream, ctypes.byref(detail))
    return st, detail.value


@pytest.mark.gpu
@pytest.mark.parametrize("which", ["tiny", "306m"])
def test_static_step_matches_workspace_step(which, request):
    """Two calls in a row of the no-allocation step produce exactly the
    logits, next tokens and KV-cache writes of the regular step: it is the
    same kernel on the same inputs, only its scratch lives elsewhere, so the
    results must be bit-identical (not merely within the parity tolerance).
    The second call starts from the first call's outputs, and the status word
    of each call is read back through b2d_static_last_error."""
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
        assert _static_status(lib, stream) == (_lib.B2D_OK, 0)
        torch.cuda.synchronize(dev)
        assert torch.equal(lg_sta, lg_ref), f"{which} call {call}: logits differ from the workspace step"
        assert int(nx_sta.item()) == int(nx_ref.item())
        assert int(nx_sta.item()) == int(np.argmax(lg_sta.cpu().numpy()))
        tok = nx_ref.clone()
    assert torch.equal(kv_sta, kv_ref), f"{which}: KV cache differs from the workspace step"
    eng.check_device()


@pytest.mark.gpu
def test_static_step_reports_device_errors(engine_tiny):
    """A position past the context, read on the device, is reported by
    b2d_static_last_error as B2D_ERR_DEVICE_INPUT (raw word 0x202: bad
    position) and writes no output; the next valid call clears the word and
    computes normally.  A host pointer for the cache is refused on the host
    before any launch."""
    eng, cfg = engine_tiny, CONFIG_TINY
    lib = _lib.load()
    dev = eng.device
    buf = eng.w["packed_w"]
    ccfg = _lib.make_config(cfg)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    kv = eng.new_kv()
    lg = torch.full((cfg.vocab_size,), 7.0, dtype=torch.float32, device=dev)
    nx = torch.full((1,), -5, dtype=torch.int32, device=dev)
    tok = torch.tensor([3], dtype=torch.int32, device=dev)
    bad_pos = torch.tensor([cfg.context_len], dtype=torch.int32, device=dev)

    def call(pos_t, kv_t=kv):
        return lib.b2d_decode_step_static(ctypes.byref(ccfg), _p(buf), ctypes.c_uint64(buf.numel()), _p(tok),
                                          _p(pos_t), kv_t, _p(lg), _p(nx), stream)

    assert call(bad_pos, _p(kv)) == _lib.B2D_OK  # accepted on the host: the position is read on the device
    assert _static_status(lib, stream) == (_lib.B2D_ERR_DEVICE_INPUT, 0x202)
    torch.cuda.synchronize(dev)
    assert int(nx.item()) == -5 and bool((lg == 7.0).all()), "a rejected step wrote outputs"
    assert not bool(kv.any()), "a rejected step wrote the cache"

    host_kv = np.zeros(16, np.uint16)  # not device memory
    assert call(bad_pos, ctypes.c_void_p(host_kv.ctypes.data)) == _lib.B2D_ERR_INVALID_ARG

    assert call(torch.tensor([0], dtype=torch.int32, device=dev), _p(kv)) == _lib.B2D_OK
    assert _static_status(lib, stream) == (_lib.B2D_OK, 0)
    torch.cuda.synchronize(dev)
    assert int(nx.item()) == int(np.argmax(lg.cpu().numpy()))
