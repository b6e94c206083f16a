"""Batched greedy RNN-T decoding (interface of reference src/asr/decode/rnnt.py:12-37)."""

from __future__ import annotations

import torch

from asr_b200.decode._greedy import decode, joint_weight


@torch.no_grad()
def greedy_decode(encoder_out, in_lens, predict, joint, blank_id: int = 0, sos_id: int = 1,
                  max_symbols_per_frame: int = 10, *, batch_predict=False) -> list[list[int]]:
    """Greedy RNN-T decode of a batch; same results as the reference decoder.

    encoder_out (B, T, d) on the GPU (decoded in float32, as the systems pass
    ``enc.float()``); in_lens (B,); predict maps a (1, L) int64 prefix
    ``[<sos>, tokens...]`` to (1, L, d) predictor outputs. ``joint`` is the
    joint projection applied to tanh(enc_t + pred_u): the system's bias-free
    ``nn.Linear`` (``system.joint``) or its (V, d) weight, where the reference
    takes the closure ``system._joint`` around it. Every step computes
    argmax over V of joint(tanh(enc[b, t] + pred)); a blank moves to the next
    frame, a token is appended and the predictor re-run; at most
    ``max_symbols_per_frame`` tokens per frame. ``batch_predict``: see
    ``asr_b200.decode._greedy``.
    """
    hyps, _ = decode(encoder_out, in_lens, predict, joint_weight(joint, "joint"), None, 0, blank_id, sos_id,
                     max_symbols_per_frame, batch_predict)
    return hyps
