"""The CUDA ops on the reference's own recorded outputs (tests/golden/*.pt).

The fixtures were produced by the reference's Triton kernels (CPU interpreter,
tests/golden/make_golden.py). Tolerance: one rounding of the output dtype on
values of order one, as for the oracle pin (tests/test_oracle_golden.py); the
chunked loss compares against the reference's fp16-rounded path with hits
bit-exact and the input gradient within cosine 0.9999.
"""

import os

import pytest
import torch

from auspex_soup_demo_b200.kernels import (_chunked_cross_entropy_fused_kernel, apply_fast_rope,
                                           fast_rms_norm, fast_swiglu,
                                           make_triton_chunked_loss_function)
from helpers import cosine

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    return torch.load(os.path.join(GOLDEN, name), weights_only=False)


def _tol(dtype):
    return {torch.float32: 2e-5, torch.bfloat16: 1.6e-2, torch.float16: 2e-3}[dtype]


@pytest.mark.parametrize("case", _load("rmsnorm.pt"), ids=lambda c: c["tag"])
def test_rmsnorm_golden(case):
    x = case["x"].cuda().requires_grad_(True)
    w = case["w"].cuda().requires_grad_(True)
    y = fast_rms_norm(x, w, case["eps"])
    y.backward(case["dy"].cuda())
    tol = _tol(case["x"].dtype)
    rows = case["x"].numel() // case["x"].shape[-1]
    torch.testing.assert_close(y.float().cpu(), case["y"].float(), rtol=tol, atol=tol)
    torch.testing.assert_close(x.grad.float().cpu(), case["dx"].float(), rtol=tol, atol=tol)
    torch.testing.assert_close(w.grad.float().cpu(), case["dw"].float(), rtol=tol,
                               atol=tol * rows ** 0.5)


@pytest.mark.parametrize("case", _load("swiglu.pt"), ids=lambda c: c["tag"])
def test_swiglu_golden(case):
    g = case["gate"].cuda().requires_grad_(True)
    u = case["up"].cuda().requires_grad_(True)
    out = fast_swiglu(g, u)
    out.backward(case["dy"].cuda())
    tol = _tol(case["gate"].dtype)
    torch.testing.assert_close(out.float().cpu(), case["out"].float(), rtol=tol, atol=tol)
    torch.testing.assert_close(g.grad.float().cpu(), case["dgate"].float(), rtol=tol, atol=tol)
    torch.testing.assert_close(u.grad.float().cpu(), case["dup"].float(), rtol=tol, atol=tol)


@pytest.mark.parametrize("case", _load("rope.pt"), ids=lambda c: c["tag"])
def test_rope_golden(case):
    x = case["x"].cuda().requires_grad_(True)
    out = apply_fast_rope(x, case["cos"].cuda(), case["sin"].cuda())
    out.backward(case["dy"].cuda())
    tol = _tol(case["x"].dtype)
    torch.testing.assert_close(out.float().cpu(), case["out"].float(), rtol=tol, atol=tol)
    torch.testing.assert_close(x.grad.float().cpu(), case["dx"].float(), rtol=tol, atol=tol)


@pytest.mark.parametrize("case", _load("ce_kernel.pt"), ids=lambda c: c["tag"])
def test_ce_kernel_golden(case):
    buf = case["logits"].cuda()
    n = buf.shape[0]
    losses = torch.empty(n, device="cuda")
    ents = torch.empty(n, device="cuda")
    corr = torch.empty(n, device="cuda", dtype=torch.int32)
    _chunked_cross_entropy_fused_kernel[(n,)](
        buf, case["targets"].cuda(), losses, ents, corr, stride_logits_row=buf.stride(0),
        V=buf.shape[1], denominator=case["denominator"], ignore_index=-100, BLOCK_V=4096,
        num_warps=8, num_stages=2)
    torch.testing.assert_close(losses.cpu(), case["losses"], rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(ents.cpu(), case["entropies"], rtol=1e-5, atol=1e-5)
    assert torch.equal(corr.cpu(), case["correct"])
    tol = _tol(case["logits"].dtype)
    torch.testing.assert_close(buf.float().cpu(), case["grad"].float(), rtol=tol, atol=1e-6)


@pytest.mark.parametrize("case", _load("chunked_loss.pt"), ids=lambda c: c["tag"])
def test_chunked_loss_golden(case):
    hidden = case["hidden"]
    head = torch.nn.Linear(hidden.shape[-1], case["weight"].shape[0], bias=False,
                           dtype=hidden.dtype, device="cuda")
    with torch.no_grad():
        head.weight.copy_(case["weight"].cuda())
    head.weight.requires_grad_(False)
    Fn = make_triton_chunked_loss_function()
    h = hidden.cuda().requires_grad_(True)
    loss, ent, tok, corr = Fn.apply(h, head, case["target"].cuda(), case["chunk"],
                                    case["denominator"], -100, True)
    loss.backward()
    torch.testing.assert_close(loss.float().cpu(), case["loss"].float(), rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(ent.cpu(), case["entropy"], rtol=2e-3, atol=2e-3)
    # fp32 activations enter the logits GEMM rounded to fp16, as the reference
    # rounds them (chunked_ce.py:196-199); bf16 ones as they are
    torch.testing.assert_close(tok.cpu(), case["token_loss"], rtol=2e-3, atol=2e-3)
    assert int(corr) == int(case["correct"])
    assert cosine(h.grad, case["dhidden"]) >= 0.9999
    assert h.grad.dtype == hidden.dtype
