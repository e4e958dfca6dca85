"""GPU: the host generation loop (``stream_tokens`` / ``generate_tokens``,
the reference's ``generate.py:92-130``) and its command line
(``generate.py:133-236``), driven end to end on the device.

* greedy: the 306M config-1 stream equals the reference's recorded stream
  (``tests/golden/cfg1_greedy.npz``) up to the first step whose reference
  top-2 margin is at most 0.05, and every token is the argmax of the logits
  the loop produced for it;
* sampled with supplied uniforms (config 4's parameters): every token equals
  the oracle's ``sample_token`` (``oracle/sampler.py``, a restatement of
  ``generate.py:28-65``) on the same logits, history and uniform, which checks
  the loop's history and uniform bookkeeping;
* seeded: without supplied uniforms the loop draws from numpy's legacy global
  RNG once per sampled token, as ``np.random.choice`` does in the reference;
* a repetition penalty at temperature 0 goes through the sampler (greedy on
  the penalised logits), not the kernel's argmax (``generate.py:102, 115``);
* the CLI prints the prompt followed by the decoded generated tokens.
"""

from __future__ import annotations

import io
import pickle

import numpy as np
import pytest

from conftest import MARGIN, golden
from oracle.sampler import sample_token as oracle_sample
from transformer_b200.config import CONFIG_306M, CONFIG_TINY
from transformer_b200.generate import generate_tokens, main, stream_tokens
from transformer_b200.synth import batch_cfg4

pytestmark = pytest.mark.gpu


def _run(eng, cfg, prompt, n, **kw):
    """Tokens of stream_tokens and, for each, the logits it was chosen from
    (the engine's logits buffer holds them when the token is yielded)."""
    toks, lgs = [], []
    for t in stream_tokens(eng, cfg, prompt, n, **kw):
        toks.append(int(t))
        lgs.append(eng.logits[0].cpu().numpy().copy())
    return toks, lgs


def test_stream_tokens_greedy_matches_reference_stream(engine306):
    g = golden("cfg1_greedy.npz")
    toks, lgs = _run(engine306, CONFIG_306M, g["prompt"], 128)
    assert len(toks) == 128
    for i, (t, lg) in enumerate(zip(toks, lgs)):
        assert t == int(np.argmax(lg)), f"token {i} is not the argmax of its logits"
    n = 0
    for i in range(128):
        if toks[i] != int(g["tokens"][i]):
            assert g["margin"][i] <= MARGIN, f"token {i} differs at a reference margin of {g['margin'][i]:.3f}"
            break
        n += 1
    print(f"greedy stream_tokens: {n} of 128 tokens equal the reference before the first near-tie fork")
    engine306.check_device()


def test_stream_tokens_sampled_supplied_uniforms(engine306):
    prompts, u = batch_cfg4(CONFIG_306M)
    prompt, uu = prompts[0], u[:, 0].astype(np.float64)
    toks, lgs = _run(engine306, CONFIG_306M, prompt, 48, temperature=0.7, top_p=0.95, rep_penalty=1.2,
                     uniforms=uu)
    hist = []
    for i, (t, lg) in enumerate(zip(toks, lgs)):
        want = oracle_sample(lg, 0.7, 0.95, 1.2, hist, float(uu[i]))
        assert t == want, f"token {i}: {t} vs oracle {want}"
        hist.append(t)
    assert len(set(toks)) > 1
    engine306.check_device()


def test_stream_tokens_seeded_legacy_rng(engine306):
    prompt = np.arange(5, 37, dtype=np.int32)
    toks, lgs = _run(engine306, CONFIG_306M, prompt, 24, temperature=1.0, top_p=0.9, rep_penalty=1.0, seed=7)
    np.random.seed(7)
    hist = []
    for i, (t, lg) in enumerate(zip(toks, lgs)):
        want = oracle_sample(lg, 1.0, 0.9, 1.0, hist, np.random.random_sample())
        assert t == want, f"token {i}"
        hist.append(t)
    # generate_tokens is the same loop collected into a list
    assert generate_tokens(engine306, CONFIG_306M, prompt, 24, 1.0, 0.9, 1.0, seed=7) == toks


def test_stream_tokens_penalty_at_temperature_zero(engine306):
    prompt = np.arange(100, 120, dtype=np.int32)
    toks, lgs = _run(engine306, CONFIG_306M, prompt, 32, temperature=0.0, rep_penalty=1.5)
    hist = []
    for i, (t, lg) in enumerate(zip(toks, lgs)):
        assert t == oracle_sample(lg, 0.0, 1.0, 1.5, hist, 0.0), f"token {i}"
        hist.append(t)


def _tiny_tokenizer(path):
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers, trainers
    tok = Tokenizer(models.BPE(unk_token="[UNK]"))
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    tok.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=300, special_tokens=["[UNK]"],
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet())
    text = ["Once upon a time there was a small model.", "It decoded one token at a time, greedily.",
            "The quick brown fox jumps over the lazy dog."] * 20
    tok.train_from_iterator(text, trainer)
    assert tok.get_vocab_size() <= CONFIG_TINY.vocab_size
    tok.save(str(path))
    return tok


@pytest.mark.parametrize("stream", [True, False])
def test_cli_end_to_end_tiny(tmp_path, params_tiny, stream):
    """The command line on a reference-format checkpoint of the tiny model
    and a BPE tokenizer found through the reference's data/bpe_vocab.pkl."""
    from transformer_b200.synth import params_f32
    (tmp_path / "data").mkdir()
    tok = _tiny_tokenizer(tmp_path / "data" / "tok.json")
    with open(tmp_path / "data" / "bpe_vocab.pkl", "wb") as f:
        pickle.dump({"tokenizer_path": "data/tok.json", "vocab_size": tok.get_vocab_size()}, f)
    weights = tmp_path / "weights.pkl"
    with open(weights, "wb") as f:
        pickle.dump({"params": params_f32(params_tiny), "config": CONFIG_TINY.as_dict()}, f)
    out, err = io.StringIO(), io.StringIO()
    argv = ["--weights", str(weights), "--prompt", "Once upon a time", "--max-tokens", "40"]
    if not stream:
        argv.append("--no-stream")
    ids = main(argv, out=out, err=err)
    assert len(ids) == 40
    if stream:
        want = "Once upon a time" + "".join(tok.decode([i]) for i in ids) + "\n"
    else:
        want = "Once upon a time" + tok.decode(ids) + "\n"
    assert out.getvalue() == want
    assert "Decoding: greedy" in err.getvalue() and "Generating 40 tokens" in err.getvalue()
    # the same tokens as the oracle's greedy stream wherever its margin allows
    from oracle.ref_forward import greedy_stream
    prompt = tok.encode("Once upon a time").ids
    ref, ref_lg = greedy_stream(params_f32(params_tiny), CONFIG_TINY, prompt, 40)
    for i in range(40):
        if ids[i] != ref[i]:
            part = np.partition(ref_lg[i], -2)
            assert part[-1] - part[-2] <= MARGIN, f"token {i}"
            break
