"""GPU: the device prefill (b2d_prefill) — prompt positions through the
batched tensor-core step, K/V written into the reference-layout cache —
against the float32 oracle and the step-by-step decode ingestion."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import MARGIN, assert_logits_close
from oracle.ref_forward import CachedDecoder, top2

pytestmark = pytest.mark.gpu


def _oracle_prefix(P, cfg, prompt):
    dec = CachedDecoder(P, cfg, 1)
    lg = None
    for p, t in enumerate(prompt):
        lg = dec.step([t], [p])[0]
    return dec, lg


@pytest.mark.parametrize("n", [1, 5, 127, 128, 129])
def test_prefill_tiny_chunk_boundaries(engine_tiny, params_tiny, n):
    """Prompt lengths around 128 rows (a projection tile width) and a single
    position: last logits (the output projection runs on the last row only)
    and every written cache row against the oracle; argmax where the margin
    allows."""
    from transformer_b200.config import CONFIG_TINY as cfg
    from transformer_b200.packing import unpack_kv_caches
    from transformer_b200.synth import params_f32
    if n > cfg.context_len:
        pytest.skip("longer than the tiny context")
    P = params_f32(params_tiny)
    rng = np.random.default_rng(300 + n)
    prompt = rng.integers(0, cfg.vocab_size, n).astype(np.int32)
    eng = engine_tiny
    kv = eng.new_kv()
    lg = eng.prefill(prompt, kv).cpu().numpy()
    dec, ref = _oracle_prefix(P, cfg, prompt)
    assert_logits_close(lg, ref, f"prefill n={n}")
    i, _, margin = top2(ref)
    if margin > MARGIN:
        assert int(eng.next_tok[0].item()) == i
    ks, vs = unpack_kv_caches(kv.float().cpu(), cfg.n_layers, cfg.n_kv_heads, cfg.context_len, cfg.d_head)
    for l in range(cfg.n_layers):
        np.testing.assert_allclose(ks[l][:, :n].numpy(), dec.K[0, l, :, :n], atol=2e-2, rtol=1e-2)
        np.testing.assert_allclose(vs[l][:, :n].numpy(), dec.V[0, l, :, :n], atol=2e-2, rtol=1e-2)
        assert torch.count_nonzero(ks[l][:, n:]) == 0 and torch.count_nonzero(vs[l][:, n:]) == 0
    eng.check_device()


def test_prefill_continuation_then_decode(engine_tiny, params_tiny):
    """Prefill in two pieces (start > 0) and then decode steps: every output
    matches the oracle fed the same tokens."""
    from transformer_b200.config import CONFIG_TINY as cfg
    from transformer_b200.synth import params_f32
    P = params_f32(params_tiny)
    rng = np.random.default_rng(7)
    prompt = rng.integers(0, cfg.vocab_size, 90).astype(np.int32)
    eng = engine_tiny
    kv = eng.new_kv()
    eng.prefill(prompt[:37], kv)
    lg = eng.prefill(prompt[37:], kv, start=37).cpu().numpy()
    dec, ref = _oracle_prefix(P, cfg, prompt)
    assert_logits_close(lg, ref, "two-piece prefill")
    dev = eng.device
    tok = torch.zeros(1, dtype=torch.int32, device=dev)
    pos = torch.zeros(1, dtype=torch.int32, device=dev)
    for i in range(8):
        t = int(rng.integers(0, cfg.vocab_size))
        tok[0] = t
        pos[0] = 90 + i
        eng.step(tok, pos, kv, eng.logits, eng.next_tok)
        ref = dec.step([t], [90 + i])[0]
        assert_logits_close(eng.logits[0].cpu().numpy(), ref, f"decode after prefill, step {i}")
    eng.check_device()


def test_prefill_equals_stepwise_306m(engine306):
    """Config 2's 384-token prompt (one 512-row chunk): device prefill against the
    one-position-per-step ingestion (both bf16 caches): last logits within the
    parity tolerance of each other, caches within bf16 rounding."""
    from transformer_b200.synth import prompt_cfg2
    eng = engine306
    prompt = prompt_cfg2()
    kv_a, kv_b = eng.new_kv(), eng.new_kv()
    la = eng.prefill(prompt, kv_a).cpu().numpy().copy()
    lb = eng.prefill_stepwise(prompt, kv_b).cpu().numpy().copy()
    assert_logits_close(la, lb, "prefill vs stepwise")
    torch.testing.assert_close(kv_a.float(), kv_b.float(), atol=3e-2, rtol=2e-2)
    eng.check_device()


def test_prefill_host_validation(engine_tiny):
    eng = engine_tiny
    kv = eng.new_kv()
    with pytest.raises(ValueError):
        eng.prefill(np.zeros(0, np.int32), kv)
    with pytest.raises(ValueError):
        eng.prefill(np.zeros(eng.cfg.context_len + 1, np.int32), kv)
    with pytest.raises(ValueError):
        eng.prefill(np.zeros(4, np.int32), kv.float())
