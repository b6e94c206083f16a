"""Greedy transducer decoders with the interface of the reference's
``asr.decode.rnnt`` / ``asr.decode.tdt`` modules, run as one batched GPU scan
over all utterances (``asr_b200.decode.rnnt.greedy_decode``,
``asr_b200.decode.tdt.greedy_decode``).

``last_token_predictor`` wraps the reference system's LSTM predictor into an
exact batched form for ``batch_predict``."""

from asr_b200.decode._greedy import last_token_predictor

__all__ = ["last_token_predictor"]
