"""CPU: the parts of the generation command line that need no GPU
(``generate.py:133-236`` and the tokenizer lookup of ``data.py:55-70``):
flags and their defaults, the reference checkpoint format, the tokenizer
found through ``data/bpe_vocab.pkl`` beside the weights, and the prompt
truncation to the context."""

from __future__ import annotations

import pickle

import numpy as np
import pytest

from transformer_b200.config import CONFIG_TINY


@pytest.fixture(scope="module")
def tiny_tok_dir(tmp_path_factory):
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers, trainers
    root = tmp_path_factory.mktemp("ckpt")
    (root / "data").mkdir()
    tok = Tokenizer(models.BPE(unk_token="[UNK]"))
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    tok.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=300, special_tokens=["[UNK]"],
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet())
    tok.train_from_iterator(["Once upon a time there was a small model."] * 20, trainer)
    tok.save(str(root / "data" / "tok.json"))
    with open(root / "data" / "bpe_vocab.pkl", "wb") as f:
        pickle.dump({"tokenizer_path": "data/tok.json", "vocab_size": tok.get_vocab_size()}, f)
    return root, tok


def test_flags_and_defaults_match_the_reference():
    from transformer_b200.generate import parse_args
    a = parse_args([])
    assert (a.prompt, a.max_tokens, a.weights, a.no_stream, a.temp, a.top_p, a.rep_penalty, a.seed) == \
        ("Once upon a time", 256, "weights.pkl", False, 0.0, 1.0, 1.0, None)
    a = parse_args(["--temp", "0.7", "--top-p", "0.95", "--rep-penalty", "1.2", "--seed", "3", "--no-stream",
                    "--max-tokens", "9", "--prompt", "hi", "--weights", "w.pkl", "--tokenizer", "t.json"])
    assert (a.temp, a.top_p, a.rep_penalty, a.seed, a.no_stream, a.max_tokens, a.prompt, a.weights,
            a.tokenizer) == (0.7, 0.95, 1.2, 3, True, 9, "hi", "w.pkl", "t.json")


def test_tokenizer_lookup(tiny_tok_dir):
    from transformer_b200.generate import load_tokenizer
    root, tok = tiny_tok_dir
    text = "Once upon a time"
    want = tok.encode(text).ids
    for kw in ({"weights": str(root / "weights.pkl")},                      # data/bpe_vocab.pkl beside it
               {"tokenizer": str(root / "data" / "bpe_vocab.pkl")},          # the pointer file itself
               {"tokenizer": str(root / "data" / "tok.json")}):              # the JSON directly
        enc, dec = load_tokenizer(**kw)
        assert enc(text) == want
        assert dec(want) == text


def test_checkpoint_and_prompt_fit(tmp_path):
    from transformer_b200.generate import fit_prompt, load_checkpoint
    from transformer_b200.synth import params_f32, synth_params
    params = params_f32(synth_params(CONFIG_TINY, 0))
    path = tmp_path / "weights.pkl"
    with open(path, "wb") as f:
        pickle.dump({"params": params, "config": CONFIG_TINY.as_dict()}, f)
    got, cfg = load_checkpoint(str(path))
    assert cfg == CONFIG_TINY and set(got) == set(params)
    ids, n = fit_prompt(range(10), 128, 256)
    assert ids.dtype == np.int32 and len(ids) == 10 and n == 118
    ids, n = fit_prompt(range(200), 128, 5)  # longer than the context: ctx - 1 tokens kept
    assert len(ids) == 127 and n == 1
