"""Greedy transducer decoders with the interface of the reference's
``asr.decode.rnnt`` / ``asr.decode.tdt`` modules, run as one batched GPU scan
over all utterances (``asr_b200.decode.rnnt.greedy_decode``,
``asr_b200.decode.tdt.greedy_decode``)."""
