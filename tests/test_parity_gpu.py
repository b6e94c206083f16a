"""Parity of the CUDA path with the reference on identical inputs.

Checked against (a) the committed golden vectors produced by the reference's
own float64 oracles / torch CTC, and (b) the C oracle (oracle/) on seeded
inputs larger than the fixtures. Tolerances (fp32 mode, tf32 = 0):
loss relative error <= 1e-5 and gradient max-abs error <= 1e-4, the bar the
reference's float32 kernels are held to; bf16 tensor-core mode (tf32 = 1) is
held to the bf16 bar measured for it (loss relative error 1.5e-5, gradient
relative-norm error 7.5e-3; tests/test_bf16_parity_gpu.py).
"""

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.golden_io import load_cases
from tests.gpu_cases import ctc_case, transducer_case

pytestmark = pytest.mark.gpu

LOSS_RTOL = 1e-5
LOSS_ATOL = 1e-5
GRAD_ATOL = 1e-4
GRAD_RTOL = 1e-4

CTC = load_cases("ctc")
RNNT = load_cases("rnnt")
TDT = load_cases("tdt")


def cuda(x, dtype=None):
    t = torch.as_tensor(np.ascontiguousarray(x), device="cuda")
    return t if dtype is None else t.to(dtype)


def leaf(x):
    return cuda(x).float().requires_grad_(True)


def assert_loss(got, want):
    got = got.detach().double().cpu().numpy()
    want = np.asarray(want, np.float64)
    np.testing.assert_allclose(got, want, rtol=LOSS_RTOL, atol=LOSS_ATOL)


def assert_grad(got, want, name, atol=GRAD_ATOL, rtol=GRAD_RTOL):
    """|got - want| <= atol + rtol * |want| elementwise: the criterion of the
    reference's own tests (torch.testing.assert_close, atol = rtol = 1e-4).
    Cases drawn from the benchmark distributions pass rtol=0, i.e. a strict
    max-abs bound."""
    g = got.detach().double().cpu().numpy()
    w = np.asarray(want, np.float64)
    if not g.size:
        return
    excess = (np.abs(g - w) - (atol + rtol * np.abs(w))).max()
    err = np.abs(g - w).max()
    assert excess <= 0, f"{name}: max-abs error {err:.3e} exceeds {atol:.0e} + {rtol:.0e}*|ref|"


def assert_bf16_close(got_loss, want_loss, grads, loss_rtol=1.5e-5):
    """The bf16 bar of the tensor-core path (tests/test_bf16_parity_gpu.py): loss
    relative error <= 1.5e-5 per utterance, gradient relative-norm error <= 7.5e-3,
    on the BASELINE activation distribution N(0, 1/d). Activations ~N(0, 1) (tanh
    near saturation, logits about three times larger) measure up to 1.9e-4 on the
    loss and are held to 6e-4."""
    got = got_loss.detach().double().cpu().numpy()
    rel = float((np.abs(got - want_loss) / np.maximum(np.abs(want_loss), 1e-30)).max())
    msg = f"loss {rel:.2e}"
    for name, g, w in grads:
        g = g.detach().double().cpu().numpy()
        msg += f", {name} {np.linalg.norm(g - w) / max(np.linalg.norm(w), 1e-30):.2e}"
    print(" " + msg, end="")
    assert rel <= loss_rtol, msg
    for name, g, w in grads:
        g = g.detach().double().cpu().numpy()
        r = np.linalg.norm(g - w) / max(np.linalg.norm(w), 1e-30)
        assert np.isfinite(g).all() and r <= 7.5e-3, f"{name}: {msg}"


# ---------------------------------------------------------------- CTC


@pytest.mark.parametrize("name", sorted(CTC))
def test_ctc_matches_golden(name):
    from asr_b200.loss.ctc import CTCLossFn

    c = CTC[name]
    x = leaf(c["logits"])
    loss = CTCLossFn.apply(x, cuda(c["targets"]), cuda(c["in_lens"]), cuda(c["tgt_lens"]),
                           bool(c["zero_infinity"]))
    (loss * cuda(c["grad_loss"])).sum().backward()
    np.testing.assert_allclose(loss.detach().double().cpu().numpy(), c["loss"], rtol=1e-5, atol=2e-5)
    assert_grad(x.grad, c["grad_logits"], "grad_logits")


def test_ctc_module_normalises_by_target_length():
    from asr_b200.loss.ctc import CTCLoss, CTCLossFn

    c = CTC["varlen_padded"]
    x = cuda(c["logits"])
    raw = CTCLossFn.apply(x, cuda(c["targets"]), cuda(c["in_lens"]), cuda(c["tgt_lens"]), False)
    out = CTCLoss()(x, cuda(c["targets"]), cuda(c["in_lens"]), cuda(c["tgt_lens"]))
    torch.testing.assert_close(out, raw / cuda(c["tgt_lens"]).clamp_min(1))


def test_ctc_config1_matches_oracle():
    from asr_b200.loss.ctc import CTCLossFn

    c = ctc_case(11, 8, (150, 200), 29, (20, 60))
    x = leaf(c["logits"])
    loss = CTCLossFn.apply(x, cuda(c["targets"]), cuda(c["in_lens"]), cuda(c["tgt_lens"]), False)
    loss.sum().backward()
    lp = torch.log_softmax(torch.tensor(c["logits"]), -1).numpy()
    want, grad = oracle.ctc(lp, c["targets"], c["in_lens"], c["tgt_lens"], grad_loss=c["grad_loss"])
    assert_loss(loss, want)
    assert_grad(x.grad, grad, "grad_logits", rtol=0)


def test_ctc_long_targets():
    """2S+1 = 601 states: the widest register block (16 states per lane)."""
    from asr_b200.loss.ctc import CTCLossFn

    c = ctc_case(12, 3, (650, 700), 40, (280, 300))
    x = leaf(c["logits"])
    loss = CTCLossFn.apply(x, cuda(c["targets"]), cuda(c["in_lens"]), cuda(c["tgt_lens"]), False)
    loss.sum().backward()
    lp = torch.log_softmax(torch.tensor(c["logits"]), -1).numpy()
    want, grad = oracle.ctc(lp, c["targets"], c["in_lens"], c["tgt_lens"], grad_loss=c["grad_loss"])
    assert_loss(loss, want)
    assert_grad(x.grad, grad, "grad_logits")


@pytest.mark.parametrize("S_rng,T_rng,B", [((1400, 1500), (1700, 1800), 2), ((3000, 3100), (3300, 3400), 1)])
def test_ctc_very_long_targets(S_rng, T_rng, B):
    """2S + 1 up to 3001 (8 warps of 16 states) and 6201 (16 warps of 16 states):
    character-level targets of thousands of labels, which the reference's
    state-looping kernels also take (ctc.cu:55-115)."""
    from asr_b200.loss.ctc import CTCLossFn

    c = ctc_case(13, B, T_rng, 40, S_rng)
    x = leaf(c["logits"])
    loss = CTCLossFn.apply(x, cuda(c["targets"]), cuda(c["in_lens"]), cuda(c["tgt_lens"]), False)
    loss.sum().backward()
    lp = torch.log_softmax(torch.tensor(c["logits"]), -1).numpy()
    want, grad = oracle.ctc(lp, c["targets"], c["in_lens"], c["tgt_lens"], grad_loss=c["grad_loss"])
    assert np.isfinite(want).all()
    assert_loss(loss, want)
    assert_grad(x.grad, grad, "grad_logits")


# -------------------------------------------------------------- RNN-T


def run_rnnt(c, tf32=False):
    from asr_b200.loss.rnnt import rnnt_loss

    e, d, w = leaf(c["enc"]), leaf(c["dec"]), leaf(c["W"])
    loss = rnnt_loss(e, d, w, cuda(c["targets"]), cuda(c["in_lens"]), cuda(c["tgt_lens"]), 0, tf32)
    (loss * cuda(c["grad_loss"])).sum().backward()
    return loss, e.grad, d.grad, w.grad


@pytest.mark.parametrize("name", sorted(RNNT))
def test_rnnt_fp32_matches_golden(name):
    c = RNNT[name]
    loss, ge, gd, gw = run_rnnt(c)
    assert_loss(loss, c["loss"])
    assert_grad(ge, c["d_enc"], "d_enc")
    assert_grad(gd, c["d_dec"], "d_dec")
    assert_grad(gw, c["dW"], "dW")


def test_rnnt_char_config_matches_oracle():
    """Config-2 shape family (V=30, d=640), 4 utterances so the oracle stays fast."""
    c = transducer_case(21, 4, (100, 160), (30, 60), 30, 640)
    loss, ge, gd, gw = run_rnnt(c)
    o = oracle.rnnt(c["enc"], c["dec"], c["W"], c["targets"], c["in_lens"], c["tgt_lens"], grad_loss=c["grad_loss"])
    assert_loss(loss, o["loss"])
    assert_grad(ge, o["d_enc"], "d_enc", rtol=0)
    assert_grad(gd, o["d_dec"], "d_dec", rtol=0)
    assert_grad(gw, o["dW"], "dW", rtol=0)


def test_rnnt_wide_labels():
    """U = 300 label positions: 16 positions per lane in the recursions."""
    c = transducer_case(22, 2, (40, 60), (280, 299), 12, 16, act_std=0.5)
    loss, ge, gd, gw = run_rnnt(c)
    o = oracle.rnnt(c["enc"], c["dec"], c["W"], c["targets"], c["in_lens"], c["tgt_lens"], grad_loss=c["grad_loss"])
    assert_loss(loss, o["loss"])
    assert_grad(ge, o["d_enc"], "d_enc")
    assert_grad(gd, o["d_dec"], "d_dec")
    assert_grad(gw, o["dW"], "dW")


def test_rnnt_padding_gets_zero_grad_and_module_normalises():
    from asr_b200.loss.rnnt import RNNTLoss, rnnt_loss

    c = RNNT["padding"]
    loss, ge, gd, gw = run_rnnt(c)
    assert torch.count_nonzero(ge[1, 4:]) == 0
    assert torch.count_nonzero(gd[1, 2:]) == 0
    args = [cuda(c[k]) for k in ("enc", "dec", "W", "targets", "in_lens", "tgt_lens")]
    raw = rnnt_loss(*args)
    torch.testing.assert_close(RNNTLoss()(*args), raw / args[5].clamp_min(1))


def test_rnnt_empty_target_closed_form():
    c = RNNT["empty_target_in_batch"]
    loss, *_ = run_rnnt(c)
    h = np.tanh(c["enc"][1][:, None, :].astype(np.float64) + c["dec"][1][None, :, :].astype(np.float64))
    logits = h @ c["W"].astype(np.float64).T
    logp = logits - np.log(np.exp(logits).sum(-1, keepdims=True))
    expected = -logp[: int(c["in_lens"][1]), 0, 0].sum()
    np.testing.assert_allclose(float(loss[1]), expected, rtol=1e-5)


def test_rnnt_bf16_mode_within_reference_tf32_bar():
    c = transducer_case(23, 4, (20, 30), (6, 10), 32, 64, act_std=1.0)
    loss, ge, gd, gw = run_rnnt(c, tf32=True)
    o = oracle.rnnt(c["enc"], c["dec"], c["W"], c["targets"], c["in_lens"], c["tgt_lens"], grad_loss=c["grad_loss"])
    assert_bf16_close(loss, o["loss"], [("d_enc", ge, o["d_enc"]), ("d_dec", gd, o["d_dec"]), ("dW", gw, o["dW"])],
                      loss_rtol=6e-4)


# ---------------------------------------------------------------- TDT


def run_tdt(c, tf32=False, sigma=None):
    from asr_b200.loss.tdt import tdt_loss

    e, d, w, wd = leaf(c["enc"]), leaf(c["dec"]), leaf(c["W"]), leaf(c["W_dur"])
    s = float(c["sigma"]) if sigma is None else sigma
    loss = tdt_loss(e, d, w, wd, cuda(c["targets"]), cuda(c["in_lens"]), cuda(c["tgt_lens"]),
                    [int(x) for x in c["durations"]], 0, s, tf32)
    (loss * cuda(c["grad_loss"])).sum().backward()
    return loss, e.grad, d.grad, w.grad, wd.grad


@pytest.mark.parametrize("name", sorted(TDT))
def test_tdt_fp32_matches_golden(name):
    c = TDT[name]
    loss, ge, gd, gw, gwd = run_tdt(c)
    assert_loss(loss, c["loss"])
    assert_grad(ge, c["d_enc"], "d_enc")
    assert_grad(gd, c["d_dec"], "d_dec")
    assert_grad(gw, c["dW"], "dW")
    assert_grad(gwd, c["dW_dur"], "dW_dur")


def _tdt_oracle(c, sigma):
    return oracle.tdt(c["enc"], c["dec"], c["W"], c["W_dur"], c["targets"], c["in_lens"], c["tgt_lens"],
                      c["durations"], sigma=sigma, grad_loss=c["grad_loss"])


@pytest.mark.parametrize("sigma", [0.0, 0.05])
def test_tdt_bpe_config_matches_oracle(sigma):
    """Config-3 shape family (V=1024 + 5 durations, d=640), 3 utterances."""
    c = transducer_case(31, 3, (60, 90), (10, 25), 1024, 640, n_dur=5)
    loss, ge, gd, gw, gwd = run_tdt(c, sigma=sigma)
    o = _tdt_oracle(c, sigma)
    assert_loss(loss, o["loss"])
    assert_grad(ge, o["d_enc"], "d_enc", rtol=0)
    assert_grad(gd, o["d_dec"], "d_dec", rtol=0)
    assert_grad(gw, o["dW"], "dW", rtol=0)
    assert_grad(gwd, o["dW_dur"], "dW_dur", rtol=0)


def test_tdt_irregular_durations():
    """Durations [0, 1, 3, 3, 7]: a gap, a duplicate and max_duration 7 (the 8-slot ring)."""
    c = transducer_case(32, 3, (20, 30), (4, 9), 20, 24, n_dur=5, act_std=0.7)
    c["durations"] = np.array([0, 1, 3, 3, 7], np.int32)
    loss, ge, gd, gw, gwd = run_tdt(c, sigma=0.1)
    o = _tdt_oracle(c, 0.1)
    assert_loss(loss, o["loss"])
    for name, g in (("d_enc", ge), ("d_dec", gd), ("dW", gw), ("dW_dur", gwd)):
        assert_grad(g, o[name], name)


def test_tdt_widest_duration_ring():
    """Durations 0..16 (17 classes, the 16-diagonal ring of the recursions)."""
    c = transducer_case(45, 2, (20, 30), (4, 9), 20, 24, n_dur=17, act_std=0.7)
    loss, ge, gd, gw, gwd = run_tdt(c, sigma=0.05)
    o = _tdt_oracle(c, 0.05)
    assert_loss(loss, o["loss"])
    for name, g in (("d_enc", ge), ("d_dec", gd), ("dW", gw), ("dW_dur", gwd)):
        assert_grad(g, o[name], name)


def assert_grad_scaled(name, got, want, rel=2e-5):
    """Long label axes: gradients reach 10^2..10^3 and are sums over thousands of
    lattice nodes in float32 (d_enc over the label axis, dW over every node), so
    they are held to 1e-4 plus `rel` of their largest magnitude (the float32
    summation error grows with that magnitude)."""
    g, w = got.detach().double().cpu().numpy(), np.asarray(want, np.float64)
    err, scale = np.abs(g - w).max(initial=0), np.abs(w).max(initial=0)
    print(f" {name} {err:.1e}/{scale:.1e}", end="")
    assert err <= 1e-4 + rel * scale, f"{name}: max-abs error {err:.3e}, largest magnitude {scale:.3e}"


@pytest.mark.parametrize(
    "durations,U_rng,seed",
    [
        ([0, 1, 2, 3, 4], (880, 899), 47),  # 4 warps of 256 positions, weights staged in shared memory
        ([0, 1, 1, 2, 4], (840, 860), 48),  # repeated duration class: the log-summed duration weights
        ([0, 1, 2, 3, 4], (2000, 2047), 49),  # 8 warps; rings beyond shared memory: global-memory mode
        (list(range(17)), (780, 799), 50),  # durations 0..16, 17 classes: global-memory mode
    ],
)
def test_tdt_long_label_axis(durations, U_rng, seed):
    """Label axes of hundreds to thousands of positions (the reference's TDT
    recursion takes any length, tdt.cu:239-283): several warps per utterance,
    the cross-warp scan of each frame, and, where the rings would not fit one SM,
    the global-memory mode that reads the sources back from the alpha / beta
    arrays."""
    c = transducer_case(seed, 2, (10, 14), U_rng, 16, 32, n_dur=len(durations), act_std=0.7)
    c["durations"] = np.array(durations, np.int32)
    loss, ge, gd, gw, gwd = run_tdt(c, sigma=0.05)
    o = _tdt_oracle(c, 0.05)
    assert_loss(loss, o["loss"])
    for name, g in (("d_enc", ge), ("d_dec", gd), ("dW", gw), ("dW_dur", gwd)):
        assert_grad_scaled(name, g, o[name])


@pytest.mark.parametrize("tf32", [False, True])
def test_rnnt_long_label_axis(tf32):
    """U = 2048 label positions (8 warps of 256): the reference's RNN-T recursion
    strides over any label axis (rnnt.cu:227-229). Both joint paths; the bf16
    path is held to its relative-norm bar (tests/test_bf16_parity_gpu.py)."""
    c = transducer_case(51, 2, (10, 14), (2000, 2047), 16, 32, act_std=0.7)
    loss, ge, gd, gw = run_rnnt(c, tf32=tf32)
    o = oracle.rnnt(c["enc"], c["dec"], c["W"], c["targets"], c["in_lens"], c["tgt_lens"], grad_loss=c["grad_loss"])
    if tf32:
        np.testing.assert_allclose(loss.detach().double().cpu().numpy(), o["loss"], rtol=1.5e-5)
        for name, g in (("d_enc", ge), ("d_dec", gd), ("dW", gw)):
            assert _rel(g.cpu(), torch.as_tensor(o[name])) <= 7.5e-3, name
        return
    assert_loss(loss, o["loss"])
    for name, g in (("d_enc", ge), ("d_dec", gd), ("dW", gw)):
        assert_grad_scaled(name, g, o[name])


def test_label_axis_beyond_the_recursions_is_rejected_cleanly():
    """Past 8192 label positions (32 warps of 256) the recursions report an
    unsupported shape before anything is launched."""
    c = transducer_case(52, 1, (4, 4), (8192, 8192), 8, 8, n_dur=5)
    with pytest.raises(RuntimeError, match="supported kernel range"):
        run_tdt(c, sigma=0.0)


def test_tdt_no_zero_duration():
    c = transducer_case(33, 2, (15, 25), (3, 6), 16, 12, n_dur=3, act_std=0.7)
    c["durations"] = np.array([1, 2, 4], np.int32)
    loss, ge, gd, gw, gwd = run_tdt(c, sigma=0.0)
    o = _tdt_oracle(c, 0.0)
    assert_loss(loss, o["loss"])
    for name, g in (("d_enc", ge), ("d_dec", gd), ("dW", gw), ("dW_dur", gwd)):
        assert_grad(g, o[name], name)


def test_tdt_padding_gets_zero_grad_and_module_normalises():
    from asr_b200.loss.tdt import TDTLoss, tdt_loss

    c = TDT["padding"]
    loss, ge, gd, gw, gwd = run_tdt(c)
    assert torch.count_nonzero(ge[1, 4:]) == 0
    assert torch.count_nonzero(gd[1, 2:]) == 0
    args = [cuda(c[k]) for k in ("enc", "dec", "W", "W_dur", "targets", "in_lens", "tgt_lens")]
    md = int(c["durations"].max())
    raw = tdt_loss(*args, list(range(md + 1)))
    torch.testing.assert_close(TDTLoss(md)(*args), raw / args[6].clamp_min(1))


def test_tdt_bf16_mode_within_reference_tf32_bar():
    c = transducer_case(34, 4, (20, 30), (6, 10), 32, 64, n_dur=5, act_std=1.0)
    loss, ge, gd, gw, gwd = run_tdt(c, tf32=True, sigma=0.0)
    o = _tdt_oracle(c, 0.0)
    assert_bf16_close(loss, o["loss"], [("d_enc", ge, o["d_enc"]), ("d_dec", gd, o["d_dec"]), ("dW", gw, o["dW"]),
                                        ("dW_dur", gwd, o["dW_dur"])], loss_rtol=6e-4)


def test_tdt_bf16_bpe_config_matches_oracle():
    c = transducer_case(35, 3, (60, 90), (10, 25), 1024, 640, n_dur=5)
    loss, ge, gd, gw, gwd = run_tdt(c, tf32=True, sigma=0.05)
    o = _tdt_oracle(c, 0.05)
    assert_bf16_close(loss, o["loss"], [("d_enc", ge, o["d_enc"]), ("d_dec", gd, o["d_dec"]), ("dW", gw, o["dW"]),
                                        ("dW_dur", gwd, o["dW_dur"])])


def _rel(got, want):
    return ((got.double() - want.double()).norm() / want.double().norm().clamp_min(1e-30)).item()


def test_tdt_bf16_backward_tracks_fp32_path():
    """The tensor-core path's gradients stay within 1e-2 (relative norm) of the
    fp32 path on benchmark-distribution inputs: bf16 operand rounding only.
    Label lengths 14..60 exercise both the 16-node groups of the d_hidden
    epilogue (U_b >= 16) and its node-by-node path (U_b < 16)."""
    c = transducer_case(36, 6, (60, 140), (10, 60), 1024, 640, n_dur=5)
    l16, *g16 = run_tdt(c, tf32=True, sigma=0.05)
    l32, *g32 = run_tdt(c, tf32=False, sigma=0.05)
    np.testing.assert_allclose(l16.detach().cpu().numpy(), l32.detach().cpu().numpy(), rtol=2e-3)
    for name, a, b in zip(("d_enc", "d_dec", "dW", "dW_dur"), g16, g32):
        assert _rel(a, b) < 1e-2, f"{name}: {_rel(a, b):.3e}"


def test_tdt_bf16_backward_multi_pass(monkeypatch):
    """Backward split into 700-node passes (boundaries inside frames and
    utterances) gives the single-pass gradients up to fp32 summation order."""
    c = transducer_case(37, 5, (30, 70), (14, 40), 256, 192, n_dur=5)
    l1, *g1 = run_tdt(c, tf32=True, sigma=0.05)
    monkeypatch.setenv("ASR_B200_BWD_PASS_NODES", "700")
    l2, *g2 = run_tdt(c, tf32=True, sigma=0.05)
    torch.testing.assert_close(l2, l1, rtol=0, atol=0)
    for name, a, b in zip(("d_enc", "d_dec", "dW", "dW_dur"), g2, g1):
        assert _rel(a, b) < 1e-5, f"{name}: {_rel(a, b):.3e}"


def test_rnnt_bf16_long_labels():
    """U = 181..200 label positions: the d_hidden kernel's global d_dec path
    (the per-utterance shared rows no longer fit)."""
    c = transducer_case(38, 2, (8, 14), (180, 199), 64, 128)
    l16, *g16 = run_rnnt(c, tf32=True)
    l32, *g32 = run_rnnt(c, tf32=False)
    np.testing.assert_allclose(l16.detach().cpu().numpy(), l32.detach().cpu().numpy(), rtol=2e-3)
    for name, a, b in zip(("d_enc", "d_dec", "dW"), g16, g32):
        assert _rel(a, b) < 1e-2, f"{name}: {_rel(a, b):.3e}"


# ------------------------------------------------------- direct C ABI


def test_capi_tdt_matches_op_path():
    """Calls libasr_b200.so through ctypes with raw device pointers (what any FFI binds)."""
    import ctypes

    from asr_b200 import _lib

    lib = _lib.capi()
    c = TDT["variable_lens_s02"]
    B, T, d = c["enc"].shape
    U = c["dec"].shape[1]
    V = c["W"].shape[0]
    Dn = c["W_dur"].shape[0]
    S = c["targets"].shape[1]
    t = {k: cuda(c[k]) for k in ("enc", "dec", "W", "W_dur", "targets", "in_lens", "tgt_lens", "durations")}
    f32 = dict(device="cuda", dtype=torch.float32)
    loss = torch.empty(B, **f32)
    log_prob = torch.empty(B, **f32)
    alpha = torch.empty(B, T + 1, U, device="cuda", dtype=torch.float64)
    lpb = torch.empty(2, B, T, U, **f32)
    lpy = torch.empty(B, T, U, **f32)
    lpd = torch.empty(B, T, U, Dn, **f32)
    lib.asr_tdt_workspace_bytes.restype = ctypes.c_size_t
    wsb = lib.asr_tdt_workspace_bytes(B, T, U, V, Dn, d, 0, 0)
    ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    P = lambda x: ctypes.c_void_p(x.data_ptr())  # noqa: E731
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    md = int(c["durations"].max())
    rc = lib.asr_tdt_forward(P(t["enc"]), P(t["dec"]), P(t["W"]), P(t["W_dur"]), P(t["targets"]), P(t["in_lens"]),
                             P(t["tgt_lens"]), P(t["durations"]), Dn, md, 1, B, T, U, V, d, S, 0,
                             ctypes.c_float(float(c["sigma"])), 0, P(loss), P(alpha), P(lpb), P(lpy), P(lpd),
                             P(log_prob), P(ws), ctypes.c_size_t(wsb), stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert_loss(loss, c["loss"])
    gl = torch.ones(B, **f32)
    ge, gd = torch.empty(B, T, d, **f32), torch.empty(B, U, d, **f32)
    gw, gwd = torch.empty(V, d, **f32), torch.empty(Dn, d, **f32)
    wsb2 = lib.asr_tdt_workspace_bytes(B, T, U, V, Dn, d, 0, 1)
    ws2 = torch.empty(wsb2, dtype=torch.uint8, device="cuda")
    rc = lib.asr_tdt_backward(P(t["enc"]), P(t["dec"]), P(t["W"]), P(t["W_dur"]), P(t["targets"]), P(t["in_lens"]),
                              P(t["tgt_lens"]), P(t["durations"]), Dn, md, 1, B, T, U, V, d, S, 0, P(alpha), P(lpb),
                              P(lpy), P(lpd), P(log_prob), P(gl), 0, P(ge), P(gd), P(gw), P(gwd), P(ws2),
                              ctypes.c_size_t(wsb2), stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert_grad(ge, c["d_enc"], "d_enc")
    assert_grad(gd, c["d_dec"], "d_dec")
    assert_grad(gw, c["dW"], "dW")
    assert_grad(gwd, c["dW_dur"], "dW_dur")
    clamped = ctypes.c_int(-1)
    assert lib.asr_workspace_status(P(ws2), B, ctypes.byref(clamped), stream) == 0
    assert clamped.value == 0


def test_capi_ctc_direct():
    import ctypes

    from asr_b200 import _lib

    lib = _lib.capi()
    c = CTC["small_fixed"]
    B, T, V = c["log_probs"].shape
    S = c["targets"].shape[1]
    lp = cuda(c["log_probs"])
    tg, il, tl = cuda(c["targets"]), cuda(c["in_lens"]), cuda(c["tgt_lens"])
    alpha = torch.empty(B, T, 2 * S + 1, device="cuda", dtype=torch.float64)
    logz = torch.empty(B, device="cuda")
    P = lambda x: ctypes.c_void_p(x.data_ptr())  # noqa: E731
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.asr_ctc_alpha(P(lp), P(tg), P(il), P(tl), B, T, V, S, P(alpha), P(logz), stream) == 0
    grad = torch.full((B, T, V), float("nan"), device="cuda")
    gl = cuda(c["grad_loss"])
    assert lib.asr_ctc_grad(P(alpha), P(logz), P(lp), P(tg), P(il), P(tl), P(gl), 0, B, T, V, S, P(grad), stream) == 0
    torch.cuda.synchronize()
    np.testing.assert_allclose((-logz).double().cpu().numpy(), c["loss"], rtol=1e-5, atol=2e-5)
    assert_grad(grad, c["grad_logits"], "grad_logits")


def test_rnnt_bf16_wide_hidden_streams_the_hidden_tile():
    """Joint dim 1024 (the large-batch RNN-T configuration): the 128-row hidden
    tile no longer fits in shared memory, so the tensor-core joint streams it
    with the weights; the gradients still track the fp32 path."""
    from asr_b200 import _lib

    assert _lib.joint_uses_tensor_cores(1024, 0, 1024)
    c = transducer_case(39, 3, (30, 60), (20, 40), 1024, 1024)
    l16, *g16 = run_rnnt(c, tf32=True)
    l32, *g32 = run_rnnt(c, tf32=False)
    np.testing.assert_allclose(l16.detach().cpu().numpy(), l32.detach().cpu().numpy(), rtol=2e-3)
    for name, a, b in zip(("d_enc", "d_dec", "dW"), g16, g32):
        assert _rel(a, b) < 1e-2, f"{name}: {_rel(a, b):.3e}"


_PAIR_SCRIPT = r"""
import sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
from tests.gpu_cases import transducer_case
from asr_b200.loss.tdt import tdt_loss
c = transducer_case(40, 5, (40, 90), (10, 40), 1024, 640, n_dur=5)
L = [torch.tensor(c[k], device="cuda", requires_grad=True) for k in ("enc", "dec", "W", "W_dur")]
I = [torch.tensor(c[k], device="cuda") for k in ("targets", "in_lens", "tgt_lens")]
loss = tdt_loss(*L, *I, list(range(5)), 0, 0.05, True)
loss.sum().backward()
np.savez(sys.argv[2], loss=loss.detach().cpu().numpy(), *[t.grad.cpu().numpy() for t in L])
"""


def test_tdt_bf16_joint_variants_agree(tmp_path):
    """The joint kernels' variants compute the same sums: streamed hidden tiles
    (the default), the resident hidden tile (ASR_B200_JOINT_STREAM=0), the
    opt-in CTA pairs of the logits kernel (ASR_B200_JOINT_PAIRS=1, one M = 256
    MMA per pair of SMs) and of the d_hidden kernel (ASR_B200_DH_PAIRS=1: two
    hidden slices per pair, d = 640 leaving one CTA of the last pair without a
    slice). Each runs in its own process: the switches are read once per process."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    root = str(Path(__file__).resolve().parents[1])
    # the logits-kernel variants run the backward's recompute, so they run with the
    # logit stash off and are compared with the streamed kernel without it
    off = {"ASR_B200_LOGIT_STASH_GB": "0"}
    variants = {"stream": {}, "dh_pairs": {"ASR_B200_DH_PAIRS": "1"}, "resident_stash": {"ASR_B200_JOINT_STREAM": "0"},
                "stream_nostash": off,
                "resident": dict(off, ASR_B200_JOINT_STREAM="0"), "pairs": dict(off, ASR_B200_JOINT_PAIRS="1")}
    out = {}
    for name, extra in variants.items():
        f = tmp_path / f"{name}.npz"
        env = {k: v for k, v in os.environ.items()
               if not k.startswith(("ASR_B200_JOINT_", "ASR_B200_DH_", "ASR_B200_LOGIT_"))}
        env.update(extra)
        subprocess.run([sys.executable, "-c", _PAIR_SCRIPT, root, str(f)], check=True, env=env, timeout=300)
        out[name] = np.load(f)
    for name, base in (("dh_pairs", "stream"), ("resident_stash", "stream"), ("resident", "stream_nostash"),
                       ("pairs", "stream_nostash")):
        np.testing.assert_allclose(out[name]["loss"], out[base]["loss"], rtol=1e-6)
        for k in ("arr_0", "arr_1", "arr_2", "arr_3"):
            a, b = out[name][k].astype(np.float64), out[base][k].astype(np.float64)
            assert np.linalg.norm(a - b) <= 1e-5 * np.linalg.norm(b), (name, k)


@pytest.mark.parametrize("tf32", [True, False])
def test_tdt_bf16_activations_match_float32_on_the_same_values(tf32):
    """bf16 encoder / decoder activations (what an autocast system produces) go in
    without float32 copies: the loss equals the float32 path fed the same values,
    the activation gradients come back in bf16 within their rounding, and the
    joint-weight gradients match. Both joint paths: tensor cores read bf16
    directly, the fp32 path reads a float32 copy made in the workspace."""
    from asr_b200.loss.tdt import tdt_loss

    c = transducer_case(41, 4, (40, 90), (10, 40), 1024, 640, n_dur=5)
    enc16 = torch.tensor(c["enc"]).to(torch.bfloat16).cuda()
    dec16 = torch.tensor(c["dec"]).to(torch.bfloat16).cuda()
    args = [cuda(c[k]) for k in ("targets", "in_lens", "tgt_lens")]
    gl = cuda(c["grad_loss"])
    out = {}
    for name, e0, d0 in (("bf16", enc16, dec16), ("f32", enc16.float(), dec16.float())):
        e, d = e0.clone().requires_grad_(True), d0.clone().requires_grad_(True)
        w, wd = leaf(c["W"]), leaf(c["W_dur"])
        loss = tdt_loss(e, d, w, wd, *args, [int(x) for x in c["durations"]], 0, 0.05, tf32)
        (loss * gl).sum().backward()
        out[name] = (loss.detach(), e.grad, d.grad, w.grad, wd.grad)
    lb, eb, db, wb, wdb = out["bf16"]
    lf, ef, df, wf, wdf = out["f32"]
    assert lb.dtype == torch.float32 and eb.dtype == torch.bfloat16 and db.dtype == torch.bfloat16
    torch.testing.assert_close(lb, lf, rtol=1e-6, atol=1e-6)
    assert _rel(eb.float(), ef) < 1e-2 and _rel(db.float(), df) < 1e-2
    assert _rel(wb, wf) < 1e-5 and _rel(wdb, wdf) < 1e-5


def test_rnnt_bf16_activations_module():
    """RNNTLoss on bf16 activations through autograd (tensor-core joint)."""
    from asr_b200.loss.rnnt import RNNTLoss, rnnt_loss

    c = transducer_case(42, 3, (30, 60), (10, 30), 256, 320)
    e = torch.tensor(c["enc"]).to(torch.bfloat16).cuda().requires_grad_(True)
    d = torch.tensor(c["dec"]).to(torch.bfloat16).cuda().requires_grad_(True)
    w = leaf(c["W"])
    args = [cuda(c[k]) for k in ("targets", "in_lens", "tgt_lens")]
    loss = RNNTLoss(tf32=True)(e, d, w, *args)
    loss.sum().backward()
    e32 = e.detach().float().requires_grad_(True)
    d32 = d.detach().float().requires_grad_(True)
    w32 = leaf(c["W"])
    ref = rnnt_loss(e32, d32, w32, *args, 0, True) / args[2].clamp_min(1)
    ref.sum().backward()
    torch.testing.assert_close(loss.detach(), ref.detach(), rtol=1e-6, atol=1e-6)
    assert e.grad.dtype == torch.bfloat16 and _rel(e.grad.float(), e32.grad) < 1e-2
    assert _rel(w.grad, w32.grad) < 1e-5


def _offset_view(x, dtype):
    """`x` as a contiguous CUDA tensor of `dtype` whose data starts one element
    past a 16-byte boundary, so the hidden-row kernels take their scalar path."""
    flat = torch.empty(x.size + 1, dtype=dtype, device="cuda")
    v = flat[1:].view(x.shape)
    v.copy_(torch.as_tensor(np.ascontiguousarray(x)).to(dtype))
    assert v.is_contiguous() and v.data_ptr() % 16 != 0
    return v


@pytest.mark.parametrize(
    "act,d",
    [
        ("f32", 72),  # one 4-column chunk per lane, row-stationary kernel
        ("f32", 640),  # five chunks per lane, three rows in flight
        ("f32", 1100),  # nine chunks per lane: the flat kernel
        ("bf16", 640),  # three 8-column chunks per lane
        ("bf16", 2100),  # nine chunks per lane: the flat kernel
    ],
)
def test_hidden_vector_paths_match_scalar_path(act, d):
    """The vector hidden-row kernels (row-stationary and flat, fp32 and bf16
    activations) write the same H as the element-wise path that unaligned rows
    take: the tensor-core RNN-T loss is identical and the gradients agree to
    accumulation order."""
    from asr_b200 import _lib
    from asr_b200.loss.rnnt import rnnt_loss

    V = 256
    assert _lib.joint_uses_tensor_cores(V, 0, d)
    c = transducer_case(43, 3, (20, 50), (30, 70), V, d)
    dt = torch.bfloat16 if act == "bf16" else torch.float32
    args = [cuda(c[k]) for k in ("targets", "in_lens", "tgt_lens")]
    gl = cuda(c["grad_loss"])
    out = {}
    for name in ("vector", "scalar"):
        if name == "vector":
            e0, d0 = cuda(c["enc"], dt), cuda(c["dec"], dt)
            assert e0.data_ptr() % 16 == 0 and d0.data_ptr() % 16 == 0
        else:
            e0, d0 = _offset_view(c["enc"], dt), _offset_view(c["dec"], dt)
        e, dd = e0.detach().requires_grad_(True), d0.detach().requires_grad_(True)
        w = leaf(c["W"])
        loss = rnnt_loss(e, dd, w, *args, 0, True)
        (loss * gl).sum().backward()
        out[name] = (loss.detach(), e.grad.float(), dd.grad.float(), w.grad)
    lv, *gv = out["vector"]
    ls, *gs = out["scalar"]
    torch.testing.assert_close(lv, ls, rtol=1e-6, atol=1e-6)
    # the backward sums with atomics, in a different order on each run: float32
    # gradients differ by rounding, bf16 activation gradients by the odd bf16 ulp
    # (4e-3 relative) where that rounding crosses a bf16 boundary
    bar = 2e-4 if act == "bf16" else 1e-5
    for name, a, b in zip(("d_enc", "d_dec", "dW"), gv, gs):
        assert _rel(a, b) < bar, f"{name}: {_rel(a, b):.3e}"


_SIMT_SCRIPT = r"""
import sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
from tests.gpu_cases import transducer_case
from asr_b200 import _lib
from asr_b200.loss.tdt import tdt_loss
from asr_b200.loss.rnnt import rnnt_loss
assert not _lib.joint_uses_tensor_cores(1024, 5, 640, tf32=False)
out = {}
c = transducer_case(71, 3, (60, 90), (10, 25), 1024, 640, n_dur=5)
L = [torch.tensor(c[k], device="cuda", requires_grad=True) for k in ("enc", "dec", "W", "W_dur")]
I = [torch.tensor(c[k], device="cuda") for k in ("targets", "in_lens", "tgt_lens")]
loss = tdt_loss(*L, *I, list(range(5)), 0, 0.05, False)
loss.sum().backward()
out.update(tdt_loss=loss.detach().cpu().numpy(), **{f"tdt_{i}": t.grad.cpu().numpy() for i, t in enumerate(L)})
c = transducer_case(72, 3, (60, 90), (10, 25), 30, 640)
L = [torch.tensor(c[k], device="cuda", requires_grad=True) for k in ("enc", "dec", "W")]
I = [torch.tensor(c[k], device="cuda") for k in ("targets", "in_lens", "tgt_lens")]
loss = rnnt_loss(*L, *I, 0, False)
loss.sum().backward()
out.update(rnnt_loss=loss.detach().cpu().numpy(), **{f"rnnt_{i}": t.grad.cpu().numpy() for i, t in enumerate(L)})
np.savez(sys.argv[2], **out)
"""


def test_fp32_simt_path_matches_oracle(tmp_path):
    """tf32 = False runs the tensor cores on split operands by default; the fp32
    SIMT joint (ASR_B200_FP32_SIMT=1, read once per process, and the path for
    shapes the tensor-core kernels do not take) is checked against the oracle in
    a process of its own at the fp32 bars."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    root = str(Path(__file__).resolve().parents[1])
    f = tmp_path / "simt.npz"
    env = dict(os.environ, ASR_B200_FP32_SIMT="1")
    subprocess.run([sys.executable, "-c", _SIMT_SCRIPT, root, str(f)], check=True, env=env, timeout=600)
    got = np.load(f)
    c = transducer_case(71, 3, (60, 90), (10, 25), 1024, 640, n_dur=5)
    o = _tdt_oracle(dict(c, sigma=0.05), 0.05)
    np.testing.assert_allclose(got["tdt_loss"], o["loss"], rtol=LOSS_RTOL, atol=LOSS_ATOL)
    for i, k in enumerate(("d_enc", "d_dec", "dW", "dW_dur")):
        assert np.abs(got[f"tdt_{i}"] - o[k]).max() <= GRAD_ATOL, k
    c = transducer_case(72, 3, (60, 90), (10, 25), 30, 640)
    o = oracle.rnnt(c["enc"], c["dec"], c["W"], c["targets"], c["in_lens"], c["tgt_lens"], grad_loss=c["grad_loss"])
    np.testing.assert_allclose(got["rnnt_loss"], o["loss"], rtol=LOSS_RTOL, atol=LOSS_ATOL)
    for i, k in enumerate(("d_enc", "d_dec", "dW")):
        assert np.abs(got[f"rnnt_{i}"] - o[k]).max() <= GRAD_ATOL, k


def test_fp32_mode_runs_on_tensor_cores():
    """The fp32 mode (tf32 = False) takes the tensor-core joint with split
    operands at the BASELINE shapes (see test_fp32_simt_path_matches_oracle for
    the SIMT path)."""
    from asr_b200 import _lib

    for V, nd, d in ((1024, 5, 640), (30, 0, 640), (1024, 0, 1024)):
        assert _lib.joint_uses_tensor_cores(V, nd, d, tf32=False), (V, nd, d)
