"""TEST INFRASTRUCTURE ONLY: restatement of the reference's CTC prefix beam search
(src/asr/decode/csrc/ctc.cpp:46-137), the checker for asr_b200.decode.ctc; and a
loader for the reference op itself compiled into oracle/_ref/ (``make -C oracle
ref``). Nothing in the product imports this module.

Algorithm (per utterance, log domain, float32 arithmetic as the reference):
  beam = [root] with p_blank = 0, p_nonblank = -inf
  for t < in_len: for each beam entry, for each token v:
    v = 0 (blank)              -> same prefix,   p_blank    ⊕= total + lp[v]
    v = last token of prefix   -> same prefix,   p_nonblank ⊕= p_nonblank + lp[v]
                                  prefix + v,    p_nonblank ⊕= p_blank + lp[v]
    otherwise                  -> prefix + v,    p_nonblank ⊕= total + lp[v]
  keep the beam_width candidates of highest total = p_blank ⊕ p_nonblank.
The result is the prefix of the best surviving entry. ⊕ is logaddexp.
"""

from __future__ import annotations

import math
from pathlib import Path

import numpy as np

NEG = -math.inf
_REF = Path(__file__).resolve().parent / "_ref" / "libref_ctc_beam.so"


def _lae(a, b):
    a, b = np.float32(a), np.float32(b)
    if a == NEG:
        return b
    if b == NEG:
        return a
    hi, lo = max(a, b), min(a, b)
    return np.float32(hi + np.float32(math.log1p(math.exp(float(lo - hi)))))


def beam_decode_one(lp, beam_width):
    """lp: (T_b, V) float32 log-probs of one utterance; returns the token list."""
    lp = np.asarray(lp, np.float32)
    beam = {(): (np.float32(0.0), np.float32(NEG))}  # prefix -> (p_blank, p_nonblank)
    for t in range(lp.shape[0]):
        row = lp[t]
        nxt: dict[tuple, list] = {}

        def slot(p):
            if p not in nxt:
                nxt[p] = [np.float32(NEG), np.float32(NEG)]
            return nxt[p]

        for prefix, (pb, pnb) in beam.items():
            total = _lae(pb, pnb)
            last = prefix[-1] if prefix else -1
            for v in range(row.shape[0]):
                x = row[v]
                if v == 0:
                    s = slot(prefix)
                    s[0] = _lae(s[0], total + x)
                elif v == last:
                    s = slot(prefix)
                    s[1] = _lae(s[1], pnb + x)
                    s = slot(prefix + (v,))
                    s[1] = _lae(s[1], pb + x)
                else:
                    s = slot(prefix + (v,))
                    s[1] = _lae(s[1], total + x)
        ranked = sorted(nxt.items(), key=lambda kv: -float(_lae(*kv[1])))
        beam = {p: (s[0], s[1]) for p, s in ranked[:beam_width]}
    best = max(beam.items(), key=lambda kv: float(_lae(*kv[1])))
    return list(best[0])


def beam_decode(log_probs, in_lens, beam_width=32):
    return [beam_decode_one(log_probs[b, : int(in_lens[b])], beam_width) for b in range(log_probs.shape[0])]


def greedy_decode(log_probs, in_lens):
    """src/asr/decode/ctc.py:10-31: argmax per frame, collapse repeats, drop blanks."""
    out = []
    for b in range(log_probs.shape[0]):
        tok = np.argmax(log_probs[b, : int(in_lens[b])], axis=-1)
        keep = np.ones_like(tok, dtype=bool)
        keep[1:] = tok[1:] != tok[:-1]
        c = tok[keep]
        out.append(c[c != 0].tolist())
    return out


def reference_available() -> bool:
    return _REF.exists()


def reference_beam_decode(log_probs, in_lens, beam_width=32):
    """The reference op itself (oracle/_ref), on CPU tensors."""
    import torch

    if not getattr(reference_beam_decode, "_loaded", False):
        torch.ops.load_library(str(_REF))
        reference_beam_decode._loaded = True
    lp = torch.as_tensor(np.ascontiguousarray(log_probs, np.float32))
    il = torch.as_tensor(np.asarray(in_lens, np.int64))
    return [o.tolist() for o in torch.ops.asr.beam_decode(lp, il, int(beam_width))]
