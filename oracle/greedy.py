"""TEST INFRASTRUCTURE ONLY: a numpy restatement of the reference's greedy
transducer decoders, the checker for asr_b200.decode. Nothing in the product
imports this module.

Reference semantics:
  * RNN-T: src/asr/decode/rnnt.py:12-37. Per utterance, start from the <sos>
    prefix; for every frame t < in_len emit argmax tokens of joint(enc[t], pred)
    until a blank or max_symbols_per_frame tokens, re-running the predictor on
    the whole prefix after every emitted token.
  * TDT: src/asr/decode/tdt.py:14-62. Same, with a duration argmax d per step
    (recorded for every step, blanks included): a token is emitted when not
    blank; d > 0 advances t by d; otherwise a blank advances t by 1; a frame that
    reaches max_symbols_per_frame advances t by 1.

`joint` is tanh(enc_t + pred) @ W.T and `joint_dur` tanh(enc_t + pred) @ W_dur.T,
computed in float32 like the systems' nn.Linear joints (system/tdt.py:31-43);
argmax takes the first maximal index (torch.argmax semantics). `predict(prefix)`
returns the predictor output for the last position of the (L,) int prefix.
`margins`, when a list, receives the relative top-2 gap of every argmax taken:
tests use it to show that no decision was a float32 near-tie.
"""

from __future__ import annotations

import numpy as np


def _argmax_joint(e, p, W, margins=None):
    h = np.tanh((e + p).astype(np.float32))
    z = W.astype(np.float32) @ h
    i = int(np.argmax(z))
    if margins is not None and z.size > 1:
        top = np.partition(z, -2)[-2:]
        margins.append(float((top[1] - top[0]) / max(1.0, abs(float(top[1])))))
    return i


def greedy_rnnt(enc, in_lens, predict, W, blank_id=0, sos_id=1, max_symbols_per_frame=10, margins=None):
    hyps = []
    for b in range(enc.shape[0]):
        prefix = [sos_id]
        pred = predict(np.array(prefix))
        hyp = []
        for t in range(int(in_lens[b])):
            for _ in range(max_symbols_per_frame):
                token = _argmax_joint(enc[b, t], pred, W, margins)
                if token == blank_id:
                    break
                hyp.append(token)
                prefix.append(token)
                pred = predict(np.array(prefix))
        hyps.append(hyp)
    return hyps


def greedy_tdt(enc, in_lens, predict, W, W_dur, max_duration, blank_id=0, sos_id=1, max_symbols_per_frame=10,
               margins=None):
    durations = list(range(max_duration + 1))
    hyps, chosen = [], []
    for b in range(enc.shape[0]):
        prefix = [sos_id]
        pred = predict(np.array(prefix))
        hyp, durs = [], []
        t, T_b = 0, int(in_lens[b])
        while t < T_b:
            advanced = False
            for _ in range(max_symbols_per_frame):
                token = _argmax_joint(enc[b, t], pred, W, margins)
                dv = durations[_argmax_joint(enc[b, t], pred, W_dur, margins)]
                durs.append(dv)
                if token != blank_id:
                    hyp.append(token)
                    prefix.append(token)
                    pred = predict(np.array(prefix))
                if dv > 0:
                    t += dv
                    advanced = True
                    break
                if token == blank_id:
                    t += 1
                    advanced = True
                    break
            if not advanced:
                t += 1
        hyps.append(hyp)
        chosen.append(durs)
    return hyps, chosen


def table_predictor(P, Q):
    """Position-wise (causal) predictor used by the decode tests:
    out[..., i, :] = P[tokens[..., i]] + Q[(i + 1) % len(Q)], so the last output of
    an (L,) prefix is P[prefix[-1]] + Q[L % len(Q)] exactly, in any framework."""

    def predict(prefix):
        prefix = np.asarray(prefix)
        return (P[prefix[-1]] + Q[len(prefix) % len(Q)]).astype(np.float32)

    return predict
