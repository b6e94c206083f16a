"""B200-native fused sequence losses (CTC, RNN-T, TDT) with their joint network.

Drop-in for the loss path of samgd/asr: ``asr_b200.loss`` mirrors
``asr.loss`` (same classes, functions, argument order and config dataclasses)
and the native library registers the same ``torch.ops.asr.*`` op schemas.
"""

__version__ = "0.1.0"
