"""CPU: the oracle against fixtures produced by the reference's own code
(tests/golden/make_golden.py imports the reference model.py / generate.py)."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden
from oracle import ref_forward as R
from oracle import sampler as OS
from transformer_b200.config import CONFIG_306M, CONFIG_TINY
from transformer_b200.synth import params_f32


def test_rms_norm_and_rope_match_reference():
    g = golden("tiny.npz")
    np.testing.assert_allclose(R.rms_norm(g["rms_x"], g["rms_scale"]), g["rms_out"], rtol=1e-6, atol=1e-6)
    cos, sin = R.precompute_rope_table(CONFIG_TINY.context_len, CONFIG_TINY.d_head)
    np.testing.assert_array_equal(cos, g["rope_cos"])
    np.testing.assert_array_equal(sin, g["rope_sin"])
    np.testing.assert_allclose(R.apply_rope(g["rope_x"], cos[:6], sin[:6]), g["rope_out"], rtol=1e-6, atol=1e-6)


def test_forward_and_prefill_match_reference(params_tiny):
    g = golden("tiny.npz")
    P = params_f32(params_tiny)
    lg = R.transformer_forward(P, CONFIG_TINY, g["prompt"])
    np.testing.assert_allclose(lg, g["logits_forward"], rtol=1e-4, atol=1e-5)
    lg2, kc, vc = R.prefill_with_kv(P, CONFIG_TINY, g["prompt"])
    np.testing.assert_allclose(lg2, g["logits_prefill"], rtol=1e-4, atol=1e-5)
    # KV caches in the reference's packed layout, bf16 bits
    from transformer_b200.synth import to_bf16_bits
    packed = np.concatenate([np.concatenate([k.reshape(-1), v.reshape(-1)]) for k, v in zip(kc, vc)])
    bits = to_bf16_bits(packed)
    ref_bits = g["kv_packed_bits"]
    # allow a 1-ulp bf16 difference from float32 summation-order noise
    diff = np.abs(bits.astype(np.int32) - ref_bits.astype(np.int32))
    assert diff.max() <= 1 and (diff > 0).mean() < 0.01


def test_cached_decoder_equals_full_forward(params_tiny):
    g = golden("tiny.npz")
    P = params_f32(params_tiny)
    dec = R.CachedDecoder(P, CONFIG_TINY, 1)
    out = np.stack([dec.step([t], [p])[0] for p, t in enumerate(g["prompt"])])
    np.testing.assert_allclose(out, g["logits_forward"], rtol=1e-4, atol=1e-5)


def test_batched_cached_decoder_matches_single(params_tiny):
    P = params_f32(params_tiny)
    rng = np.random.default_rng(3)
    prompts = rng.integers(0, CONFIG_TINY.vocab_size, (3, 9))
    multi = R.CachedDecoder(P, CONFIG_TINY, 3)
    outs = [multi.step(prompts[:, p], np.full(3, p)) for p in range(9)]
    for b in range(3):
        one = R.CachedDecoder(P, CONFIG_TINY, 1)
        for p in range(9):
            np.testing.assert_allclose(outs[p][b], one.step([prompts[b, p]], [p])[0], rtol=1e-5, atol=1e-6)


def test_oracle_greedy_stream_matches_reference_cfg1(params306_f32):
    """Config 1: the cached oracle reproduces the reference's full-recompute
    greedy stream (teacher forced) and its logits at the recorded steps."""
    g = golden("cfg1_greedy.npz")
    dec = R.CachedDecoder(params306_f32, CONFIG_306M, 1)
    prompt, toks = g["prompt"], g["tokens"]
    lg = None
    for p, t in enumerate(prompt):
        lg = dec.step([t], [p])[0]
    kept = dict(zip(g["logits_steps"].tolist(), g["logits"]))
    for i in range(len(toks)):
        if i in kept:
            np.testing.assert_allclose(lg, kept[i], rtol=1e-4, atol=2e-5)
        a, v, m = R.top2(lg)
        if g["margin"][i] > 1e-3:
            assert a == toks[i], f"step {i}"
        assert abs(v - g["top1"][i]) < 1e-4
        if i + 1 < len(toks):
            lg = dec.step([toks[i]], [len(prompt) + i])[0]


def test_sampler_matches_reference_sample_token():
    """Reference generate.sample_token (with np.random seeded) == the oracle's
    supplied-uniform restatement, on recorded cases."""
    g = golden("sampling.npz")
    cols = list(g["columns"])
    rng = np.random.default_rng(int(g["logits_seed"]))
    for row in g["cases"]:
        r = dict(zip(cols, row))
        case = int(r["case"])
        logits = (rng.standard_normal(32000) * 0.64 * (1 + case % 3)).astype(np.float32)
        hist = rng.integers(0, 32000, case % 40).astype(np.int32)
        tok = OS.sample_token(logits, r["temp"], r["top_p"], r["rp"], list(hist), r["u"])
        assert tok == int(r["ref_tok"]), f"case {case}"


def test_pairwise_sum_is_numpy_sum():
    rng = np.random.default_rng(5)
    for n in (1, 7, 8, 127, 128, 129, 1000, 32000):
        a = rng.random(n, dtype=np.float32)
        assert OS.pairwise_sum_f32(a) == np.float32(np.sum(a))


def test_choice_inverse_cdf_matches_numpy_choice():
    rng = np.random.default_rng(6)
    for s in range(200):
        p = rng.random(50).astype(np.float32)
        p /= p.sum()
        a = np.arange(50) * 3
        np.random.seed(s)
        want = int(np.random.choice(a, p=p))
        u = np.random.RandomState(s).random_sample()
        assert OS.choice_inverse_cdf(a, p, u) == want


@pytest.mark.parametrize("temp,top_p,rp", [(0.0, 1.0, 1.2), (0.7, 0.95, 1.2), (1.0, 1.0, 1.0)])
def test_sampler_edge_cases(temp, top_p, rp):
    logits = np.zeros(100, np.float32)
    logits[7] = 5.0
    logits[9] = 5.0  # tie: first index wins for greedy
    t = OS.sample_token(logits, temp, top_p, rp, [], 0.0)
    if temp == 0.0 or top_p < 1.0:
        # greedy: first index of the max; top-p: sorted order, ties by id
        assert t == 7
    else:
        # no top-p: numpy's choice walks the CDF in token-id order
        assert t == 0
    # repetition penalty lowers a seen positive logit
    t2 = OS.sample_token(logits, 0.0, 1.0, 2.0, [7], 0.5)
    assert t2 == 9
