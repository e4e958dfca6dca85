"""Restatement of the reference host sampler (TEST ORACLE).

Test infrastructure only; see ``oracle/__init__.py``.

``generate.py:28-65`` ``sample_token`` applies, in float32 numpy: repetition
penalty over ``set(generated_ids)`` (``l > 0 ? l / rp : l * rp``), then
temperature (``l / T``), softmax (``l -= max; p = exp(l); p /= p.sum()``),
top-p (``argsort(-p)``, ``cumsum``, ``cutoff = searchsorted(cumsum, top_p) + 1``,
renormalise the kept probabilities) and ``np.random.choice``.

Three points are pinned down here so that the result is a function of
(logits, uniform) alone:

* ``np.random.choice(a, p=p)`` (numpy legacy ``RandomState``) draws one
  uniform ``u`` and returns ``a[searchsorted(cumsum(float64(p)) / last, u,
  side='right')]``.  This module takes ``u`` as an argument instead.
  ``tests/golden/make_golden.py`` checks the equivalence against the
  reference's own ``sample_token`` under ``np.random.seed``.
* ``np.exp`` on float32 is not correctly rounded on AVX-512 hosts (up to 2 ulp,
  host dependent).  The oracle rounds the float64 exponential to float32
  instead (``exp_f32``), a host-independent definition the device sampler
  reproduces exactly.
* ``np.argsort`` is not stable, so the order among equal probabilities is
  host dependent.  The oracle breaks ties by ascending token id.

Everything else follows numpy's own arithmetic: float32 division by the
float32-rounded temperature / penalty, numpy's pairwise float32 sum
(``np.sum``) for the normalisers, a sequential float32 ``cumsum`` for the
top-p cutoff, and a float64 comparison against ``top_p``
(``np.searchsorted`` promotes the Python float).
"""

from __future__ import annotations

import numpy as np

f32 = np.float32


def exp_f32(x):
    """float32 exp, correctly rounded via float64."""
    return np.exp(np.asarray(x, dtype=np.float64)).astype(f32)


def pairwise_sum_f32(a):
    """numpy's float32 pairwise summation (``np.sum`` of a contiguous 1-D
    float32 array): blocks of <=128 with 8 accumulators, recursive halving
    at multiples of 8 above that.  Equal to ``np.sum(a)`` bit for bit."""
    return f32(f32(0) + np.sum(np.ascontiguousarray(a, dtype=f32)))


def apply_rep_penalty(logits, rep_penalty, generated_ids):
    """``generate.py:32-39``."""
    logits = np.array(logits, dtype=f32)
    if rep_penalty != 1.0 and len(generated_ids):
        for tid in set(int(t) for t in generated_ids):
            if logits[tid] > 0:
                logits[tid] /= rep_penalty
            else:
                logits[tid] *= rep_penalty
    return logits


def choice_inverse_cdf(a, p, u):
    """numpy legacy ``RandomState.choice(a, p=p)`` given its uniform ``u``."""
    cdf = np.asarray(p, dtype=np.float64).cumsum()
    cdf /= cdf[-1]
    return int(np.asarray(a)[int(cdf.searchsorted(np.float64(u), side="right"))])


def sample_token(logits, temperature, top_p, rep_penalty, generated_ids, u):
    """``generate.py:28-65`` with a supplied uniform ``u``."""
    logits = apply_rep_penalty(logits, rep_penalty, generated_ids)
    if temperature == 0.0:
        return int(np.argmax(logits))
    if temperature != 1.0:
        logits = logits / temperature
    logits -= logits.max()
    probs = exp_f32(logits)
    probs /= pairwise_sum_f32(probs)
    if top_p < 1.0:
        idx = np.arange(probs.size)
        sorted_idx = np.lexsort((idx, -probs))  # descending p, ties by id
        sorted_probs = probs[sorted_idx]
        cumsum = np.cumsum(sorted_probs)  # sequential float32
        cutoff = int(np.searchsorted(cumsum, top_p)) + 1
        keep_idx = sorted_idx[:cutoff]
        filtered = probs[keep_idx]
        filtered /= pairwise_sum_f32(filtered)
        return choice_inverse_cdf(keep_idx, filtered, u)
    return choice_inverse_cdf(np.arange(probs.size), probs, u)
