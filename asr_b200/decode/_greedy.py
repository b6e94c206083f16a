"""Host loop shared by the batched greedy RNN-T and TDT decoders.

The reference decoders (src/asr/decode/rnnt.py:12-37, src/asr/decode/tdt.py:14-62)
walk one utterance at a time and make one joint call per step. Here every
utterance advances at once: each ``asr_greedy_scan`` launch moves all unfinished
utterances to their next emitted token (or their end) on the GPU, the host reads
one (B,) report, runs the predictor for the utterances that emitted, and
launches again. The loop ends when no utterance emitted; the number of launches
is the longest hypothesis plus one.

The predictor is called exactly as the reference calls it: on the (1, L) int64
prefix ``[<sos>, tokens...]`` of one utterance, taking the output at the last
position (``batch_predict=False``). Two batched forms make one call per launch
for all utterances that emitted:
  * ``batch_predict=True``: ``predict`` on the right-padded (n, L_max) prefixes,
    row i read at position L_i - 1. Equivalent only for predictors whose rows
    are independent and causal along the sequence (a batch_first LSTM, a causal
    transformer). The reference's own LSTM predictor (model/lstm.py:8-15) is
    built with batch_first=False and mixes rows under this form.
  * ``batch_predict=f``, a callable ``f(tokens, lengths) -> (n, d)`` given the
    right-padded (n, L_max) int64 prefixes and their (n,) int64 lengths, whose
    row i must equal ``predict(tokens[i:i+1, :lengths[i]])[0, -1]``. For the
    reference's LSTM predictor that output depends only on the last token (its
    (1, L) input is read as L independent one-step sequences), so
    ``last_token_predictor(predict)`` is an exact batched form of it.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from asr_b200 import _lib

_P = ctypes.c_void_p
_I = ctypes.c_int
_bound = False

# Windows of 8 frames one utterance scans per launch before it pauses (see
# asr_greedy_scan): bounds each launch by a short chain instead of the longest
# run of blanks in the batch.
MAX_WINDOWS = 1


def _capi() -> ctypes.CDLL:
    global _bound
    lib = _lib.capi()
    if not _bound:
        lib.asr_greedy_pack_weights.argtypes = [_P, _I, _I, _P, _I, _P]
        lib.asr_greedy_init.argtypes = [_P, _P, _I, _I, _I, _P]
        lib.asr_greedy_scan.argtypes = [_P] * 3 + [_I] + [_P] * 3 + [_I] + [_P] * 4 + [_I] * 10 + [_P]
        lib.asr_status_string.restype = ctypes.c_char_p
        _bound = True
    return lib


def _check(lib, rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed: {lib.asr_status_string(rc).decode()} (status {rc})")


def last_token_predictor(predict):
    """Batched form of a predictor whose output at the last prefix position depends
    only on the last token, as the reference's LSTM(batch_first=False) predictor
    behaves on a (1, L) prefix: the last tokens of all n prefixes are passed as one
    (1, n) call, i.e. n independent one-step sequences."""

    def f(tokens, lengths):
        last = tokens.gather(1, (lengths - 1).unsqueeze(1))  # (n, 1)
        return predict(last.reshape(1, -1))[0]

    return f


def joint_weight(joint, name: str) -> torch.Tensor:
    """The (V, d) projection of a joint Linear(tanh(enc + pred)) without bias: the
    nn.Linear itself (the systems' ``self.joint`` / ``self.joint_dur``) or its weight."""
    if isinstance(joint, torch.nn.Module):
        if getattr(joint, "bias", None) is not None:
            raise ValueError(f"{name}: the joint projection must have no bias (the systems use bias=False)")
        joint = getattr(joint, "weight", None)
    if not isinstance(joint, torch.Tensor) or joint.dim() != 2:
        raise TypeError(f"{name} must be the joint nn.Linear (bias=False) or its (V, d) weight tensor; the fused "
                        "kernel evaluates Linear(tanh(enc_t + pred_u)) itself")
    return joint.detach()


@torch.no_grad()
def decode(encoder_out, in_lens, predict, W, W_dur, max_duration, blank_id, sos_id, max_symbols_per_frame,
           batch_predict):
    """Runs the batched greedy decoder; returns (hyps, durations or None)."""
    if not (isinstance(encoder_out, torch.Tensor) and encoder_out.is_cuda):
        raise RuntimeError("asr_b200 greedy decoding runs on CUDA tensors only (there is no CPU path)")
    if encoder_out.dim() != 3:
        raise ValueError(f"encoder_out must be (batch, n_frames, d_model), got {tuple(encoder_out.shape)}")
    dev = encoder_out.device
    enc = encoder_out.detach().float().contiguous()  # the systems decode enc.float()
    B, T, D = enc.shape
    V = W.shape[0]
    if W.shape[1] != D:
        raise ValueError(f"joint weight is {tuple(W.shape)}, expected (V, {D})")
    n_dur = 0
    if W_dur is not None:
        n_dur = W_dur.shape[0]
        if W_dur.shape[1] != D:
            raise ValueError(f"joint_dur weight is {tuple(W_dur.shape)}, expected (n_dur, {D})")
        if n_dur > max_duration + 1:
            raise ValueError(f"joint_dur has {n_dur} outputs but durations = range(max_duration + 1) "
                             f"has {max_duration + 1}")
    if not 0 <= blank_id < V:
        raise ValueError(f"blank_id={blank_id} outside the vocabulary of size {V}")
    lens_host = torch.as_tensor(in_lens).detach().to("cpu", torch.int64).reshape(-1)
    if lens_host.numel() != B:
        raise ValueError(f"in_lens has {lens_host.numel()} entries for a batch of {B}")
    if B and (int(lens_host.min()) < 0 or int(lens_host.max()) > T):
        raise ValueError(f"in_lens must lie in [0, {T}]")
    tdt = W_dur is not None
    if B == 0:
        return [], ([] if tdt else None)

    lib = _capi()
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev)
        sp = ctypes.c_void_p(stream.cuda_stream)
        lens = lens_host.to(dev, torch.int32)
        ldw = (V + 3) // 4 * 4
        Wf = W.float().contiguous()
        Wt = torch.empty(D, ldw, device=dev, dtype=torch.float32)
        _check(lib, lib.asr_greedy_pack_weights(Wf.data_ptr(), V, D, Wt.data_ptr(), ldw, sp), "asr_greedy_pack_weights")
        Wd = W_dur.float().contiguous() if tdt else None
        cap = max(T * max(int(max_symbols_per_frame), 0), 1)
        state = torch.empty(B, 4, device=dev, dtype=torch.int32)
        prefix = torch.empty(B, cap + 1, device=dev, dtype=torch.int64)
        durs = torch.empty(B, cap, device=dev, dtype=torch.int32) if tdt else None
        report = torch.empty(B, device=dev, dtype=torch.int32)
        report_h = torch.empty(B, dtype=torch.int32, pin_memory=True)
        # One upload per scan: [active list | utterances that emitted | their prefix lengths].
        active_h = torch.empty(3 * B, dtype=torch.int32, pin_memory=True)
        active_d = torch.empty(3 * B, dtype=torch.int32, device=dev)
        _check(lib, lib.asr_greedy_init(state.data_ptr(), prefix.data_ptr(), B, cap, sos_id, sp), "asr_greedy_init")

        # Every utterance starts from the same prefix [<sos>]: one predictor call.
        start = predict(torch.tensor([[sos_id]], device=dev))[0, -1]
        pred = start.float().reshape(1, D).expand(B, D).contiguous()
        active = np.arange(B, dtype=np.int32)
        active_h[:B].copy_(torch.from_numpy(active))
        active_d[:B].copy_(active_h[:B], non_blocking=True)
        for _ in range(cap * B + 2):
            n = active.size
            _check(lib, lib.asr_greedy_scan(
                enc.data_ptr(), pred.data_ptr(), Wt.data_ptr(), ldw, Wd.data_ptr() if tdt else None, lens.data_ptr(),
                active_d.data_ptr(), n, state.data_ptr(), prefix.data_ptr(), durs.data_ptr() if tdt else None,
                report.data_ptr(), B, T, D, V, n_dur, blank_id, int(max_symbols_per_frame), cap, cap, MAX_WINDOWS, sp),
                "asr_greedy_scan")
            report_h.copy_(report, non_blocking=True)
            stream.synchronize()
            r = report_h.numpy()[active]
            if (r == -1).any():
                raise RuntimeError("asr_greedy_scan: hypothesis buffer overflow")
            keep = (r > 0) | (r == -2)
            emitted = r[keep] > 0
            active, r = active[keep], r[keep]
            if active.size == 0:
                break
            # Utterances that emitted or paused form the next scan's active list;
            # the predictor runs for those that emitted.
            n, Ls = active.size, r[emitted]
            upd = active[emitted]
            m = upd.size
            hb = active_h.numpy()
            hb[:n], hb[n: n + m], hb[n + m: n + 2 * m] = active, upd, Ls
            active_d[: n + 2 * m].copy_(active_h[: n + 2 * m], non_blocking=True)
            if m == 0:
                continue
            if batch_predict is not False:
                idx = active_d[n: n + m].long()
                lens_t = active_d[n + m: n + 2 * m].long()
                rows = prefix[:, : int(Ls.max())].index_select(0, idx)
                if callable(batch_predict):
                    new = batch_predict(rows, lens_t)
                else:
                    new = predict(rows)[torch.arange(upd.size, device=dev), lens_t - 1]
                pred.index_copy_(0, idx, new.float())
            else:
                for b, L in zip(upd.tolist(), Ls.tolist()):
                    out = predict(prefix[b: b + 1, :L])
                    pred[b].copy_(out[0, -1])
        else:
            raise RuntimeError("asr_greedy_scan: decoding did not terminate")

        st = state.cpu().numpy()
        n_tok, n_step = st[:, 2], st[:, 3]
        toks = prefix[:, 1: 1 + int(n_tok.max())].cpu().numpy() if n_tok.max() > 0 else None
        hyps = [toks[b, : n_tok[b]].tolist() if n_tok[b] else [] for b in range(B)]
        if not tdt:
            return hyps, None
        dv = durs[:, : int(n_step.max())].cpu().numpy() if n_step.max() > 0 else None
        return hyps, [dv[b, : n_step[b]].tolist() if n_step[b] else [] for b in range(B)]
