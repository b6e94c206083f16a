"""Generate ``tests/golden/ctc_beam_golden.npz`` with the reference's own CTC prefix
beam search (src/asr/decode/csrc/ctc.cpp), compiled from its source into
oracle/_ref/ by ``make -C oracle ref REF=/path/to/samgd-asr``:

    make -C oracle ref REF=/path/to/samgd-asr
    python tests/golden/make_ctc_beam_golden.py

Log-probs are seeded draws: log_softmax of N(0, s^2) logits (s sets how peaked the
frames are; trained models are peaked), some with blank-dominated frames or a
token held over several frames (the repeat / merge paths of the search). Cases
cover beam widths 1..32, a beam wider than the vocabulary, empty and short
utterances and a BPE-size vocabulary.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from oracle import ctc_beam  # noqa: E402


def cases():
    # (name, B, T, V, beam, scale, in_lens, kind)
    yield "tiny_w1", 2, 8, 5, 1, 2.0, [8, 5], "plain"
    yield "tiny_w2", 2, 10, 5, 2, 2.0, [10, 7], "plain"
    yield "char_w8", 3, 40, 29, 8, 3.0, [40, 31, 12], "plain"
    yield "char_w32_wider_than_vocab", 2, 50, 29, 32, 3.0, [50, 44], "plain"
    yield "blank_heavy", 3, 60, 29, 8, 3.0, [60, 50, 20], "blank"
    yield "held_tokens", 2, 60, 20, 8, 2.0, [60, 47], "held"
    yield "empty_and_one_frame", 3, 12, 10, 4, 2.0, [0, 1, 12], "plain"
    yield "flat", 2, 30, 16, 8, 0.3, [30, 25], "plain"
    yield "bpe_w16", 2, 60, 300, 16, 4.0, [60, 41], "plain"
    yield "bpe1024_w32", 2, 80, 1024, 32, 5.0, [80, 66], "blank"


def draw(rng, B, T, V, scale, kind):
    logits = rng.standard_normal((B, T, V)) * scale
    if kind == "blank":
        logits[..., 0] += scale * 1.5
    if kind == "held":
        for b in range(B):
            for t0 in range(0, T, 6):
                v = rng.integers(1, V)
                logits[b, t0: t0 + 4, v] += scale * 3
    return torch.log_softmax(torch.tensor(logits, dtype=torch.float32), -1).numpy()


def main():
    if not ctc_beam.reference_available():
        raise SystemExit("build the reference op first: make -C oracle ref REF=/path/to/samgd-asr")
    out: dict[str, np.ndarray] = {}
    for i, (name, B, T, V, W, scale, il, kind) in enumerate(cases()):
        rng = np.random.default_rng(5000 + i)
        lp = draw(rng, B, T, V, scale, kind)
        il = np.asarray(il, np.int32)
        hyps = ctc_beam.reference_beam_decode(lp, il, W)
        p = f"ctc_beam/{name}/"
        out[p + "log_probs"], out[p + "in_lens"], out[p + "beam"] = lp, il, np.array(W, np.int32)
        out[p + "hyp_lens"] = np.array([len(h) for h in hyps], np.int32)
        out[p + "hyp_flat"] = np.array([x for h in hyps for x in h], np.int32)
        print(name, [len(h) for h in hyps])
    np.savez_compressed(HERE / "ctc_beam_golden.npz", **out)
    print("ctc_beam", len(out), "arrays")


if __name__ == "__main__":
    main()
