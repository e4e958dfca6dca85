"""GPU: the batched step at BASELINE config 3's and config 5's own shapes,
against the reference forward run in float32 on the host.

Config 3: B=64 sequences, prompt lengths U[32,448] (seed 2), the seeded random
block table, ragged ingestion, then 64 greedy steps by CUDA-graph replay.
Config 5: one wave of 256 sequences as ``bench.py`` builds it (the first 256
seeded 64-token prompts, a random block table), ingested, captured, and
replayed for all 256 decode steps, positions 64..319.

The oracle follows each checked row's own greedy stream: after the GPU run,
``transformer_forward`` (``model.py:163-191``, restated in ``oracle/``) runs
once over the row's prompt plus the tokens the GPU chose, and its row t is
the reference's logits for the step at position t (a decode step at position
p equals ``transformer_forward(prefix)[-1]``).  Every compared step must match
within the north-star tolerance, and the GPU's token must equal the oracle's
argmax wherever the oracle's top-2 margin exceeds 0.05.  The per-row
semantics are those of ``kernels/multi_sm_decode.py:369-432`` applied to each
sequence of the batch.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import MARGIN, assert_logits_close
from oracle.ref_forward import top2, transformer_forward

pytestmark = pytest.mark.gpu


def _check_rows(P, cfg, rows, prompts, gen, got):
    """rows: checked row ids; prompts[b]: its prompt; gen[b]: int list of the
    GPU's tokens (gen[b][0] = argmax of the ingest logits, gen[b][i + 1] =
    argmax of step i); got[b]: dict position -> GPU logits (f32 [vocab]).
    Returns (rows x positions compared, worst abs error)."""
    n, worst = 0, 0.0
    for b in rows:
        seq = np.concatenate([np.asarray(prompts[b], np.int64), np.asarray(gen[b][:-1], np.int64)])
        want = sorted(got[b])
        ref_all = transformer_forward(P, cfg, seq[:max(want) + 1])
        for p in want:
            ref = ref_all[p]
            worst = max(worst, assert_logits_close(got[b][p], ref, f"row {b} position {p}"))
            i, _, margin = top2(ref)
            chosen = gen[b][p - len(prompts[b]) + 1]  # the token the GPU picked from these logits
            if margin > MARGIN:
                assert chosen == i, f"row {b} position {p}: token {chosen} vs reference argmax {i}"
            n += 1
    return n, worst


def test_cfg3_shape_parity(engine306_batched, params306_f32):
    """Config 3 exactly: 64 ragged sequences, random block table, 64 greedy
    steps by graph replay.  Eight rows spread over the length range are
    compared at the last prompt position and at every decode step."""
    from transformer_b200.batched import BatchedDecoder
    from transformer_b200.config import CONFIG_306M as cfg
    from transformer_b200.synth import batch_cfg3
    eng = engine306_batched
    lens, prompts, table = batch_cfg3(cfg)
    B, steps = len(prompts), 64
    order = np.argsort(lens, kind="stable")
    rows = sorted({int(order[int(round(k * (B - 1) / 7))]) for k in range(8)})
    assert len(rows) == 8 and lens[rows].min() == lens.min() and lens[rows].max() == lens.max()

    dec = BatchedDecoder(eng, B, table=table, num_blocks=int(table.size))
    last = dec.ingest(prompts)
    got = {b: {int(lens[b]) - 1: last[b].cpu().numpy()} for b in rows}
    gen = {b: [int(dec.tok[b].item())] for b in rows}
    dec.capture()
    sel = torch.tensor(rows, device=eng.device)
    for i in range(steps):
        dec.replay()
        lg = dec.logits[sel].cpu().numpy()
        tk = dec.tok[sel].cpu().numpy()
        for j, b in enumerate(rows):
            got[b][int(lens[b]) + i] = lg[j]
            gen[b].append(int(tk[j]))
    dec.release()
    eng.check_device()
    n, worst = _check_rows(params306_f32, cfg, rows, prompts, gen, got)
    assert n == 8 * (steps + 1)
    print(f"config 3: {n} (row, position) pairs within tolerance, max abs err {worst:.3g}")


def test_cfg5_wave_parity(engine306_batched, params306_f32):
    """Config 5's B=256 wave as bench.py runs it: 64-token prompts ingested,
    the step captured once, then all 256 decode steps (positions 64..319) by
    graph replay.  Six rows across the batch are compared at the prompt's
    last position and at decode positions 64, 190 and 319."""
    from transformer_b200.batched import BatchedDecoder
    from transformer_b200.config import CONFIG_306M as cfg
    from transformer_b200.synth import batch_cfg5
    eng = engine306_batched
    B, L, steps = 256, 64, 256
    prompts = list(batch_cfg5(cfg)[:B])
    rows = [0, 37, 101, 128, 200, 255]
    check_pos = (L, 190, L + steps - 1)

    dec = BatchedDecoder(eng, B, seed=0)  # bench.py's wave 0 on rank 0
    last = dec.ingest(prompts)
    got = {b: {L - 1: last[b].cpu().numpy()} for b in rows}
    gen = {b: [int(dec.tok[b].item())] for b in rows}
    dec.capture()
    sel = torch.tensor(rows, device=eng.device)
    toks = torch.zeros(steps, len(rows), dtype=torch.int32, device=eng.device)
    for i in range(steps):
        dec.replay()
        toks[i].copy_(dec.tok[sel])
        if L + i in check_pos:
            lg = dec.logits[sel].cpu().numpy()
            for j, b in enumerate(rows):
                got[b][L + i] = lg[j]
    assert int(dec.pos[0].item()) == L + steps
    tk = toks.cpu().numpy()
    for j, b in enumerate(rows):
        gen[b].extend(int(t) for t in tk[:, j])
    dec.release()
    eng.check_device()
    n, worst = _check_rows(params306_f32, cfg, rows, prompts, gen, got)
    assert n == len(rows) * (1 + len(check_pos))
    print(f"config 5 wave: {n} (row, position) pairs within tolerance, max abs err {worst:.3g}")
