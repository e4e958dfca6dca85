"""CPU: the C-ABI library loads and exports every symbol include/b2d.h
declares; host-side layout queries and argument validation (no GPU work)."""

from __future__ import annotations

import ctypes
import os
import re

import pytest

from conftest import REPO
from transformer_b200 import _lib
from transformer_b200.config import CONFIG_306M, CONFIG_TINY, ModelConfig


def header_symbols():
    src = open(os.path.join(REPO, "include", "b2d.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(b2d_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from transformer_b200 import build
    build.build()
    return _lib.load()


def test_every_declared_symbol_is_exported(lib):
    syms = header_symbols()
    assert len(syms) >= 14
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(_lib._SIGS), "ctypes signatures must cover the header exactly"


def test_status_strings(lib):
    for s in range(0, 9):
        assert lib.b2d_status_str(s).decode()
    assert _lib.status_str(_lib.B2D_ERR_DEVICE_TIMEOUT) == "device wait timed out"


def test_weights_layout_306m(lib):
    lay = _lib.weights_layout(CONFIG_306M)
    # per layer: qkv 1536x1024, o 1024x1024, gu 2816x2x1024, down 1024x2816 (bf16)
    assert lay.layer_stride == 2 * (1536 * 1024 + 1024 * 1024 + 2816 * 2048 + 1024 * 2816)
    assert lay.off_emb == 24 * lay.layer_stride
    for f in ("off_qkv", "off_o", "off_gu", "off_down", "off_emb", "off_ln1", "off_ln2", "off_lnf",
              "off_cos", "off_sin", "total_bytes"):
        assert getattr(lay, f) % 256 == 0, f
    assert lay.total_bytes >= 2 * 303_000_000


def test_kv_layout_matches_reference_pack(lib):
    kv = _lib.kv_layout(CONFIG_306M)
    assert kv.kv_half_elems == 4 * 512 * 64
    assert kv.layer_elems == 2 * kv.kv_half_elems
    assert kv.elems_per_seq == 24 * kv.layer_elems  # reference total_kv_size (multi_sm_decode.py:382)


def test_supported_shapes(lib):
    for cfg in (CONFIG_306M, CONFIG_TINY):
        c = _lib.make_config(cfg)
        assert lib.b2d_config_supported(ctypes.byref(c)) == 1
    odd = _lib.make_config(ModelConfig(d_model=768, n_heads=12, n_kv_heads=4, d_ff=2048))
    assert lib.b2d_config_supported(ctypes.byref(odd)) == 0


def test_host_argument_validation(lib):
    out = ctypes.c_void_p()
    c = _lib.make_config(CONFIG_306M)
    # null weights / misaligned pointer / bad config are rejected before any CUDA call
    assert lib.b2d_model_create(ctypes.byref(c), None, 0, 0, ctypes.byref(out)) == _lib.B2D_ERR_INVALID_ARG
    assert lib.b2d_model_create(ctypes.byref(c), ctypes.c_void_p(0x1001), 1 << 40, 0,
                                ctypes.byref(out)) == _lib.B2D_ERR_INVALID_ARG
    bad = _lib.make_config(ModelConfig(d_head=32))
    assert lib.b2d_model_create(ctypes.byref(bad), ctypes.c_void_p(0x1000), 1 << 40, 0,
                                ctypes.byref(out)) == _lib.B2D_ERR_INVALID_ARG
    assert lib.b2d_decode_step(None, None, None, None, 1, None, None, None, None) == _lib.B2D_ERR_INVALID_ARG
    assert lib.b2d_workspace_create(None, 1, ctypes.byref(out)) == _lib.B2D_ERR_INVALID_ARG
    assert lib.b2d_last_error(None, None, None) == _lib.B2D_ERR_INVALID_ARG
    sp = _lib.Sampling(0.7, 0.95, 1.2)
    assert lib.b2d_sample(None, None, 1, 32000, None, 0, None, None, ctypes.byref(sp), None,
                          None) == _lib.B2D_ERR_INVALID_ARG
    assert lib.b2d_debug_set(None, 1, 0) == _lib.B2D_ERR_INVALID_ARG
    assert lib.b2d_debug_tune(None, 1, 0) == _lib.B2D_ERR_INVALID_ARG
    assert lib.b2d_debug_trace(None, None, 0) == _lib.B2D_ERR_INVALID_ARG
    # prefill entry points: null handles and buffers are rejected before any CUDA call
    assert lib.b2d_prefill(None, None, None, 4, 0, None, None, None, None) == _lib.B2D_ERR_INVALID_ARG
    assert lib.b2d_prefill_paged(None, None, None, 4, 0, None, None, 32, 64, None, None,
                                 None) == _lib.B2D_ERR_INVALID_ARG
    assert lib.b2d_prefill_rows(None, None, None, None, 8, None, None, 32, 64, 2, None, None,
                                None) == _lib.B2D_ERR_INVALID_ARG
    assert lib.b2d_prefill_rows_max() == 512
    assert lib.b2d_decode_step_paged(None, None, None, None, 2, None, None, 32, 64, None, None,
                                     None) == _lib.B2D_ERR_INVALID_ARG


def test_product_path_has_no_oracle_import():
    """The shipped package never imports the test oracle."""
    pkg = os.path.join(REPO, "transformer_b200")
    for root, _, files in os.walk(pkg):
        for f in files:
            if f.endswith(".py"):
                src = open(os.path.join(root, f)).read()
                assert "import oracle" not in src and "from oracle" not in src, f
