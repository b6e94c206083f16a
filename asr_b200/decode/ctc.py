"""CTC decoding (interface of reference src/asr/decode/ctc.py:10-40): greedy and
prefix beam search, both on the GPU. The beam search runs the kernel of
``asr_b200/csrc/ctc_beam.cu`` (the reference runs its C++ op on the CPU)."""

from __future__ import annotations

import ctypes

import torch

from asr_b200 import _lib

_P = ctypes.c_void_p
_I = ctypes.c_int
_bound = False


def _capi() -> ctypes.CDLL:
    global _bound
    lib = _lib.capi()
    if not _bound:
        lib.asr_ctc_beam_workspace_bytes.restype = ctypes.c_size_t
        lib.asr_ctc_beam_workspace_bytes.argtypes = [_I, _I, _I]
        lib.asr_ctc_beam_decode.argtypes = [_P, _P, _I, _I, _I, _I, _P, _P, _P, ctypes.c_size_t, _P]
        lib.asr_status_string.restype = ctypes.c_char_p
        _bound = True
    return lib


def _on_gpu(x: torch.Tensor) -> torch.Tensor:
    # The reference accepts log-probs on any device; decoding here runs on the GPU.
    if x.is_cuda:
        return x
    if not torch.cuda.is_available():
        raise RuntimeError("asr_b200 CTC decoding runs on the GPU (no CUDA device is available)")
    return x.cuda()


@torch.no_grad()
def greedy_decode(log_probs, in_lens) -> list[list[int]]:
    """Per frame argmax, repeats collapsed, blanks (0) removed (reference
    decode/ctc.py:10-31)."""
    lp = _on_gpu(log_probs)
    B, T, _ = lp.shape
    tok = lp.argmax(-1)
    keep = torch.ones_like(tok, dtype=torch.bool)
    keep[:, 1:] = tok[:, 1:] != tok[:, :-1]
    lens = torch.as_tensor(in_lens, device=lp.device).reshape(-1, 1)
    keep &= (tok != 0) & (torch.arange(T, device=lp.device) < lens)
    tok, keep = tok.cpu(), keep.cpu()
    return [tok[b][keep[b]].tolist() for b in range(B)]


@torch.no_grad()
def beam_decode(log_probs, in_lens, beam_width: int = 32) -> list[list[int]]:
    """CTC prefix beam search (reference decode/ctc.py:34-40 over the C++ op
    decode/csrc/ctc.cpp), blank = 0, float32; beam_width <= 64."""
    lp = _on_gpu(log_probs).float().contiguous()
    B, T, V = lp.shape
    lens = torch.as_tensor(in_lens).to(lp.device, torch.int32).reshape(-1)
    if lens.numel() != B:
        raise ValueError(f"in_lens has {lens.numel()} entries for a batch of {B}")
    if B == 0:
        return []
    lib = _capi()
    nbytes = lib.asr_ctc_beam_workspace_bytes(B, T, int(beam_width))
    if nbytes == 0:
        raise ValueError(f"beam_width must be in [1, 64], got {beam_width}")
    ws = torch.empty(nbytes, dtype=torch.uint8, device=lp.device)
    tokens = torch.empty(B, max(T, 1), dtype=torch.int32, device=lp.device)
    lengths = torch.empty(B, dtype=torch.int32, device=lp.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(lp.device).cuda_stream)
    rc = lib.asr_ctc_beam_decode(lp.data_ptr(), lens.data_ptr(), B, T, V, int(beam_width), tokens.data_ptr(),
                                 lengths.data_ptr(), ws.data_ptr(), nbytes, stream)
    if rc != 0:
        raise RuntimeError(f"asr_ctc_beam_decode failed: {lib.asr_status_string(rc).decode()} (status {rc})")
    tok, ln = tokens.cpu(), lengths.cpu().tolist()
    return [tok[b, : ln[b]].tolist() for b in range(B)]
