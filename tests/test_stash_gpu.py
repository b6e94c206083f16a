"""The logit stash of the transducer losses (tensor-core joint).

The forward keeps the joint's logits (each minus the row's largest token logit
of its vocabulary chunk: fp16 with tf32 = 1, fp32 with tf32 = 0) in a stash of
at most ASR_B200_LOGIT_STASH_GB, and the backward forms d loss / d logits of the
stashed nodes from it; the nodes past the stash are recomputed by the logits
GEMM as before. The default budget holds every node of these cases, so the
other parity tests (test_parity_gpu, test_bf16_parity_gpu) already run the full
stash. Here:
  * stash off (budget 0): the recompute path, against the float64 oracle;
  * a stash that ends inside a backward pass (small passes, a budget of about
    half the nodes): both kernels in one pass, against the oracle and against
    the full stash;
  * the stash against the recompute path on the same inputs: bf16 mode within
    the fp16 rounding of the stashed logits, fp32 mode within fp32 rounding.
"""

from __future__ import annotations

import numpy as np
import pytest

from tests.gpu_cases import config_draws
from tests.test_bf16_parity_gpu import BF16_GRAD_RELNORM, check_bf16, loss_rel, oracle_of, relnorm, run_ours

pytestmark = pytest.mark.gpu

DRAWS = config_draws()
GRADS = ("d_enc", "d_dec", "dW", "dW_dur")


def _nodes(c):
    return int((c["in_lens"].astype(np.int64) * (c["tgt_lens"] + 1)).sum())


def _budget_gib(c, nodes, tf32):
    """ASR_B200_LOGIT_STASH_GB value whose stash holds `nodes` (a multiple of 256)."""
    vpad = (c["W"].shape[0] + (c["W_dur"].shape[0] if "W_dur" in c else 0) + 15) // 16 * 16
    nch = (vpad + 255) // 256
    cw = ((vpad + nch - 1) // nch + 15) // 16 * 16
    nch = (vpad + cw - 1) // cw
    per = vpad * (2 if tf32 else 4) + 4 * nch
    return (nodes * per + 512 + per // 2) / float(1 << 30)


def _check_fp32(name, got, want):
    rel = loss_rel(got["loss"], want["loss"])
    assert rel <= 1e-5, f"{name}: loss relative error {rel:.3e}"
    for k in [k for k in GRADS if k in got]:
        err, scale = np.abs(got[k] - want[k]).max(), np.abs(want[k]).max()
        assert err <= 1e-4 * max(1.0, scale), f"{name} {k}: max-abs {err:.3e} (|max| {scale:.3e})"


@pytest.mark.parametrize("tf32", [True, False])
@pytest.mark.parametrize("name", ["c3_tdt_bpe", "c2_rnnt_char"])
def test_stash_off_matches_oracle(name, tf32, monkeypatch):
    monkeypatch.setenv("ASR_B200_LOGIT_STASH_GB", "0")
    c = DRAWS[name]
    got, want = run_ours(c, tf32), oracle_of(c)
    if tf32:
        check_bf16(name + "-nostash", got, want)
    else:
        _check_fp32(name + "-nostash", got, want)


@pytest.mark.parametrize("tf32", [True, False])
def test_partial_stash_inside_a_pass(tf32, monkeypatch):
    """Backward passes of 20,480 nodes and a stash of 40 % of the nodes: the
    stash boundary falls inside a pass, whose first nodes come from the stash
    and the rest from the recompute kernel. Compared with the oracle and with
    the full stash over the same passes."""
    c = DRAWS["c3_tdt_bpe"]
    monkeypatch.setenv("ASR_B200_BWD_PASS_NODES", "20480")
    full = run_ours(c, tf32)
    n = _nodes(c)
    m = (int(n * 0.4) // 256) * 256
    assert m % 20480 != 0
    monkeypatch.setenv("ASR_B200_LOGIT_STASH_GB", repr(_budget_gib(c, m, tf32)))
    part = run_ours(c, tf32)
    want = oracle_of(c)
    if tf32:
        check_bf16("c3-partial", part, want)
    else:
        _check_fp32("c3-partial", part, want)
    np.testing.assert_array_equal(part["loss"], full["loss"])
    for k in GRADS:
        assert relnorm(part[k], full[k]) <= (2e-3 if tf32 else 1e-5), f"{k}: {relnorm(part[k], full[k]):.3e}"


@pytest.mark.parametrize("tf32", [True, False])
@pytest.mark.parametrize("name", ["c5_tdt_long", "c4_rnnt_d1024"])
def test_stash_against_recompute(name, tf32, monkeypatch):
    """Same inputs with and without the stash: the losses agree to fp32
    rounding (the stash-writing forward sums each vocabulary chunk relative to
    its own maximum), the gradients differ by the stash's rounding only."""
    c = DRAWS[name]
    with_stash = run_ours(c, tf32)
    monkeypatch.setenv("ASR_B200_LOGIT_STASH_GB", "0")
    without = run_ours(c, tf32)
    assert loss_rel(with_stash["loss"], without["loss"]) <= 1e-6
    errs = {k: relnorm(with_stash[k], without[k]) for k in GRADS if k in without}
    print(f"\n{name} tf32={tf32}: " + ", ".join(f"{k} {v:.2e}" for k, v in errs.items()), end="")
    for k, v in errs.items():
        assert v <= (2e-3 if tf32 else 1e-5), f"{k}: {v:.3e}"


@pytest.mark.parametrize("tf32", [True, False])
def test_stash_one_column_group(tf32, monkeypatch):
    """V + n_dur <= 16: a stash row is a single 16-column group (the kernel's
    row division by one), with the duration columns in the same group."""
    from tests.gpu_cases import transducer_case

    c = transducer_case(73, 3, (20, 40), (10, 30), 11, 64, n_dur=5)
    c.update(kind="tdt", sigma=0.05)
    with_stash = run_ours(c, tf32)
    want = oracle_of(c)
    if tf32:  # off the BASELINE shapes (d = 64): the bf16 loss error measured 3.3e-5
        assert loss_rel(with_stash["loss"], want["loss"]) <= 1e-4
        for k in GRADS:
            assert relnorm(with_stash[k], want[k]) <= BF16_GRAD_RELNORM, k
    else:
        _check_fp32("small-vocab", with_stash, want)
    monkeypatch.setenv("ASR_B200_LOGIT_STASH_GB", "0")
    without = run_ours(c, tf32)
    for k in GRADS:
        assert relnorm(with_stash[k], without[k]) <= (2e-3 if tf32 else 1e-5), k


@pytest.mark.parametrize("tf32", [True, False])
def test_second_backward_over_one_forward(tf32):
    """retain_graph: two backwards over one forward read the same stash (the
    backward leaves it untouched); both match the oracle's gradients at the
    path's bar, and each other."""
    import torch

    from asr_b200.loss.tdt import tdt_loss

    c = DRAWS["c3_tdt_bpe"]
    dev = torch.device("cuda")
    leaves = [torch.tensor(c[k], device=dev, requires_grad=True) for k in ("enc", "dec", "W", "W_dur")]
    ints = [torch.tensor(c[k], device=dev) for k in ("targets", "in_lens", "tgt_lens")]
    loss = tdt_loss(*leaves, *ints, [int(x) for x in c["durations"]], 0, float(c["sigma"]), tf32)
    grads = []
    for _ in range(2):
        g = torch.autograd.grad(loss.sum(), leaves, retain_graph=True)
        grads.append([x.double().cpu().numpy() for x in g])
    want = oracle_of(c)
    for name, a, b in zip(GRADS, grads[0], grads[1]):
        assert relnorm(b, a) <= (2e-3 if tf32 else 1e-5), name
        for got in (a, b):
            if tf32:
                assert relnorm(got, want[name]) <= BF16_GRAD_RELNORM, name
            else:  # the fp32 bar of the other parity tests
                err, scale = np.abs(got - want[name]).max(), np.abs(want[name]).max()
                assert err <= 1e-4 * max(1.0, scale), f"{name}: max-abs {err:.3e}"
