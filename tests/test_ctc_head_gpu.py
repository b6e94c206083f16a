"""Parity of the fused CTC head (asr_b200.loss.ctc_head) with the reference head +
CTC loss: against the golden vectors (torch float64, tests/golden/
make_ctc_head_golden.py) and the float64 oracle (oracle/ctc_head.py) at BPE sizes.

Both sides use the same bf16 operands (RMSNorm output, weight, bias), so the
loss agrees to float32 accumulation (relative 1e-4 here). The backward's dense
part d loss / d logits = grad_loss * softmax is rounded to bf16 before the two
tensor-core GEMMs (the posterior part stays float32), so gradients are held to a
relative-norm bound of 1e-2, the bar the reference holds its own bf16 (tf32 = 1)
loss path to.
"""

import numpy as np
import pytest
import torch

from asr_b200.loss.ctc_head import FusedCTCHead, ctc_head_loss
from oracle import ctc_head as oracle_head
from tests.golden_io import load_cases

pytestmark = pytest.mark.gpu

CASES = load_cases("ctc_head")
LOSS_RTOL = 1e-4
GRAD_REL = 1e-2


def cuda(x, dtype=None):
    t = torch.as_tensor(np.ascontiguousarray(x), device="cuda")
    return t if dtype is None else t.to(dtype)


def rel(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)


def run(c, act=torch.float32):
    enc = cuda(c["enc"]).to(act).requires_grad_(True)
    g = cuda(c["g"]).requires_grad_(True)
    W = cuda(c["W"]).requires_grad_(True)
    b = cuda(c["b"]).requires_grad_(True) if "b" in c else None
    loss = ctc_head_loss(enc, g, W, b, cuda(c["targets"]), cuda(c["in_lens"]), cuda(c["tgt_lens"]),
                         zero_infinity=bool(c["zero_infinity"]))
    (loss * cuda(c["grad_loss"])).sum().backward()
    torch.cuda.synchronize()
    out = {"loss": loss.detach().double().cpu().numpy(), "d_enc": enc.grad.double().cpu().numpy(),
           "dg": g.grad.double().cpu().numpy(), "dW": W.grad.double().cpu().numpy()}
    if b is not None:
        out["db"] = b.grad.double().cpu().numpy()
    return out


def check(out, want, loss_rtol=LOSS_RTOL, grad_rel=GRAD_REL):
    np.testing.assert_allclose(out["loss"], want["loss"], rtol=loss_rtol, atol=loss_rtol)
    for k in ("d_enc", "dg", "dW", "db"):
        if k in want:
            assert rel(out[k], want[k]) < grad_rel, f"{k}: rel {rel(out[k], want[k]):.2e}"


@pytest.mark.parametrize("name", sorted(CASES))
def test_ctc_head_matches_reference_golden(name):
    c = CASES[name]
    check(run(c), c)


def bpe_case(seed, B=12, T=(150, 300), S=(20, 90), V=1024, d=512):
    rng = np.random.default_rng(seed)
    il = rng.integers(T[0], T[1] + 1, size=B).astype(np.int32)
    tl = rng.integers(S[0], S[1] + 1, size=B).astype(np.int32)
    Tm, Sm = int(il.max()), int(tl.max())
    return {"enc": rng.standard_normal((B, Tm, d)).astype(np.float32),
            "g": (1.0 + 0.1 * rng.standard_normal(d)).astype(np.float32),
            "W": (rng.standard_normal((V, d)) / np.sqrt(d)).astype(np.float32),
            "b": (0.1 * rng.standard_normal(V)).astype(np.float32),
            "targets": rng.integers(1, V, size=(B, Sm)).astype(np.int32), "in_lens": il, "tgt_lens": tl,
            "zero_infinity": np.array(1, np.int32), "grad_loss": rng.uniform(0.5, 1.5, B).astype(np.float32)}


def oracle_of(c):
    return oracle_head.ctc_head(c["enc"], c["g"], c["W"], c.get("b"), c["targets"], c["in_lens"], c["tgt_lens"],
                                zero_infinity=bool(c["zero_infinity"]), grad_loss=c["grad_loss"])


def test_ctc_head_matches_oracle_at_bpe_size():
    """BPE-1024 head (d = 512, the reference encoder width), 12 utterances of 150-300 frames."""
    c = bpe_case(1)
    check(run(c), oracle_of(c))


def test_ctc_head_multi_pass(monkeypatch):
    """Node passes of 1024 frames (the per-pass bf16 buffers of the joint kernels)."""
    c = bpe_case(2, B=6, V=300, d=256)
    one = run(c)
    monkeypatch.setenv("ASR_B200_BWD_PASS_NODES", "1024")
    many = run(c)
    np.testing.assert_allclose(many["loss"], one["loss"], rtol=1e-6)
    for k in ("d_enc", "dg", "dW", "db"):
        assert rel(many[k], one[k]) < 1e-5, k


def test_ctc_head_bf16_encoder_output():
    """bf16 activations (the system's autocast encoder output) give the float32
    results on the same values; gradients come back in bf16."""
    c = bpe_case(3, B=4, V=512, d=256)
    c["enc"] = torch.tensor(c["enc"]).bfloat16().float().numpy()
    a = run(c, torch.float32)
    b = run(c, torch.bfloat16)
    np.testing.assert_allclose(b["loss"], a["loss"], rtol=1e-6)
    for k in ("dg", "dW", "db"):
        assert rel(b[k], a[k]) < 1e-5, k
    assert rel(b["d_enc"], a["d_enc"]) < 1e-2


def test_fused_module_matches_unfused_reference_path():
    """FusedCTCHead(enc, targets, ...) against the reference system's own path under
    bf16 autocast: Sequential(RMSNorm, Linear) then fp32 log_softmax + CTC (torch's
    ctc_loss stands for the reference loss op), divided by tgt_lens.clamp_min(1)."""
    c = bpe_case(4, B=6, V=256, d=128)
    head = FusedCTCHead(128, 256, zero_infinity=True).cuda()
    ref = torch.nn.Sequential(torch.nn.RMSNorm(128), torch.nn.Linear(128, 256)).cuda()
    ref.load_state_dict(head.state_dict())
    enc = cuda(c["enc"])
    tg, il, tl = cuda(c["targets"]), cuda(c["in_lens"]), cuda(c["tgt_lens"])
    fused = head(enc, tg, il, tl)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        logits = ref(enc)
    lp = torch.log_softmax(logits.float(), -1)
    want = torch.nn.functional.ctc_loss(lp.transpose(0, 1), tg.long(), il.long(), tl.long(), reduction="none",
                                        zero_infinity=True) / tl.clamp_min(1)
    # the reference rounds its logits to bf16 (autocast output); the fused op keeps them in fp32
    torch.testing.assert_close(fused, want, rtol=5e-3, atol=5e-3)
