"""Batched greedy TDT decoding (interface of reference src/asr/decode/tdt.py:14-62)."""

from __future__ import annotations

import torch

from asr_b200.decode._greedy import decode, joint_weight


@torch.no_grad()
def greedy_decode(encoder_out, in_lens, predict, joint, joint_dur, max_duration: int, blank_id: int = 0,
                  sos_id: int = 1, max_symbols_per_frame: int = 10, *,
                  batch_predict=False) -> tuple[list[list[int]], list[list[int]]]:
    """Greedy TDT decode of a batch; same results as the reference decoder.

    Arguments as ``asr_b200.decode.rnnt.greedy_decode``, plus ``joint_dur``
    (the system's bias-free duration ``nn.Linear`` or its (n_dur, d) weight) and
    ``max_duration``: durations are ``range(max_duration + 1)``, indexed by the
    duration argmax. Per step: a non-blank token is emitted (predictor re-run);
    a duration d > 0 advances d frames; a blank with d = 0 advances one frame; a
    frame that reaches ``max_symbols_per_frame`` steps advances one frame.

    Returns the hypotheses and, per utterance, the duration chosen at every
    step, blanks included.
    """
    hyps, durs = decode(encoder_out, in_lens, predict, joint_weight(joint, "joint"),
                        joint_weight(joint_dur, "joint_dur"), int(max_duration), blank_id, sos_id,
                        max_symbols_per_frame, batch_predict)
    return hyps, durs
