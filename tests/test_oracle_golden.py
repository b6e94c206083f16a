"""Pins the C oracle against the golden vectors computed by the reference's own oracles."""

import numpy as np
import pytest

from oracle import oracle
from tests.golden_io import load_cases

CTC = load_cases("ctc")
RNNT = load_cases("rnnt")
TDT = load_cases("tdt")

# Both sides are float64 arithmetic on the same float32 inputs: agreement to
# ~1e-9 relative is expected (only summation order differs).
RTOL = 1e-8
ATOL = 1e-9


@pytest.mark.parametrize("name", sorted(CTC))
def test_ctc_oracle_matches_reference(name):
    c = CTC[name]
    loss, grad = oracle.ctc(c["log_probs"], c["targets"], c["in_lens"], c["tgt_lens"], grad_loss=c["grad_loss"],
                            zero_infinity=bool(c["zero_infinity"]))
    # golden log_probs were rounded to float32 after log_softmax; torch's reference
    # used the float64 log_softmax, so compare at float32 input precision.
    np.testing.assert_allclose(loss, c["loss"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(grad, c["grad_logits"], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("name", sorted(RNNT))
def test_rnnt_oracle_matches_reference(name):
    c = RNNT[name]
    out = oracle.rnnt(c["enc"], c["dec"], c["W"], c["targets"], c["in_lens"], c["tgt_lens"], grad_loss=c["grad_loss"])
    np.testing.assert_allclose(out["loss"], c["loss"], rtol=RTOL, atol=ATOL)
    for k in ("d_enc", "d_dec", "dW"):
        np.testing.assert_allclose(out[k], c[k], rtol=RTOL, atol=ATOL, err_msg=k)


@pytest.mark.parametrize("name", sorted(TDT))
def test_tdt_oracle_matches_reference(name):
    c = TDT[name]
    out = oracle.tdt(c["enc"], c["dec"], c["W"], c["W_dur"], c["targets"], c["in_lens"], c["tgt_lens"],
                     c["durations"], sigma=float(c["sigma"]), grad_loss=c["grad_loss"])
    np.testing.assert_allclose(out["loss"], c["loss"], rtol=RTOL, atol=ATOL)
    for k in ("d_enc", "d_dec", "dW", "dW_dur"):
        np.testing.assert_allclose(out[k], c[k], rtol=RTOL, atol=ATOL, err_msg=k)


def test_oracle_threads_agree():
    c = TDT["variable_lens_s02"]
    a = oracle.tdt(c["enc"], c["dec"], c["W"], c["W_dur"], c["targets"], c["in_lens"], c["tgt_lens"], c["durations"],
                   sigma=float(c["sigma"]), grad_loss=c["grad_loss"], nthreads=1)
    b = oracle.tdt(c["enc"], c["dec"], c["W"], c["W_dur"], c["targets"], c["in_lens"], c["tgt_lens"], c["durations"],
                   sigma=float(c["sigma"]), grad_loss=c["grad_loss"], nthreads=3)
    for k in a:
        np.testing.assert_allclose(a[k], b[k], rtol=1e-12, atol=1e-14)
