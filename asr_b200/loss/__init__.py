"""Loss modules with the interface of the reference's ``asr.loss`` package."""

from asr_b200.loss.ctc import CTCLoss
from asr_b200.loss.rnnt import RNNTLoss
from asr_b200.loss.tdt import TDTLoss

__all__ = ["CTCLoss", "RNNTLoss", "TDTLoss"]
