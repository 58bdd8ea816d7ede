"""Pin the CPU oracle against the reference's own kernel outputs (CPU only).

The fixtures in tests/golden were produced by running the reference's Triton
kernels through Triton's CPU interpreter (tests/golden/make_golden.py). Each
oracle function must reproduce them to within one rounding of the output dtype.
"""

import os

import pytest
import torch

import oracle

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    return torch.load(os.path.join(GOLDEN, name), weights_only=False)


def _ulp_tol(dtype):
    # one rounding of the output dtype on values of order one
    return {torch.float32: 2e-5, torch.bfloat16: 1.6e-2, torch.float16: 2e-3}[dtype]


@pytest.mark.parametrize("case", _load("rmsnorm.pt"), ids=lambda c: c["tag"])
def test_rmsnorm_oracle_matches_reference(case):
    x, w, dy = case["x"], case["w"], case["dy"]
    y, rstd = oracle.rmsnorm_fwd(x, w, case["eps"])
    dx, dw = oracle.rmsnorm_bwd(dy, x, w, rstd)
    tol = _ulp_tol(x.dtype)
    torch.testing.assert_close(y.float(), case["y"].float(), rtol=tol, atol=tol)
    torch.testing.assert_close(dx.float(), case["dx"].float(), rtol=tol, atol=tol)
    # dw sums over rows: scale the tolerance by the magnitude of the sum
    rows = x.numel() // x.shape[-1]
    torch.testing.assert_close(dw.float(), case["dw"].float(), rtol=tol, atol=tol * rows ** 0.5)


@pytest.mark.parametrize("case", _load("swiglu.pt"), ids=lambda c: c["tag"])
def test_swiglu_oracle_matches_reference(case):
    out = oracle.swiglu_fwd(case["gate"], case["up"])
    dg, du = oracle.swiglu_bwd(case["dy"], case["gate"], case["up"])
    tol = _ulp_tol(case["gate"].dtype)
    torch.testing.assert_close(out.float(), case["out"].float(), rtol=tol, atol=tol)
    torch.testing.assert_close(dg.float(), case["dgate"].float(), rtol=tol, atol=tol)
    torch.testing.assert_close(du.float(), case["dup"].float(), rtol=tol, atol=tol)


@pytest.mark.parametrize("case", _load("rope.pt"), ids=lambda c: c["tag"])
def test_rope_oracle_matches_reference(case):
    out = oracle.rope_fwd(case["x"], case["cos"], case["sin"])
    dx = oracle.rope_bwd(case["dy"], case["cos"], case["sin"])
    tol = _ulp_tol(case["x"].dtype)
    torch.testing.assert_close(out.float(), case["out"].float(), rtol=tol, atol=tol)
    torch.testing.assert_close(dx.float(), case["dx"].float(), rtol=tol, atol=tol)


def test_rope_oracle_equals_hf_formula():
    """With HF-built tables the kernel formula equals q*cos + rotate_half(q)*sin."""
    g = torch.Generator().manual_seed(7)
    x = torch.randn(2, 3, 11, 128, generator=g)
    cos, sin = oracle.rope_cos_sin(11, 128, 1e6)
    rot = torch.cat((-x[..., 64:], x[..., :64]), dim=-1)
    hf = x * cos + rot * sin
    torch.testing.assert_close(oracle.rope_fwd(x, cos, sin), hf, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("case", _load("ce_kernel.pt"), ids=lambda c: c["tag"])
def test_ce_rows_oracle_matches_reference(case):
    loss, ent, corr, grad, _ = oracle.ce_rows(case["logits"], case["targets"], case["denominator"])
    torch.testing.assert_close(loss, case["losses"], rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(ent, case["entropies"], rtol=1e-5, atol=1e-5)
    assert torch.equal(corr, case["correct"])
    tol = _ulp_tol(case["logits"].dtype)
    torch.testing.assert_close(grad.to(case["logits"].dtype).float(), case["grad"].float(),
                               rtol=tol, atol=1e-6)


@pytest.mark.parametrize("case", _load("chunked_loss.pt"), ids=lambda c: c["tag"])
def test_chunked_ce_oracle_matches_reference(case):
    """The reference rounds logits and grads to fp16; the oracle stays in fp32."""
    loss, ent, tok, corr, dh, _ = oracle.chunked_ce(
        case["hidden"], case["weight"], case["target"], case["chunk"], case["denominator"],
        compute_dw=False)
    torch.testing.assert_close(loss, case["loss"].float(), rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(ent, case["entropy"], rtol=2e-3, atol=2e-3)
    torch.testing.assert_close(tok, case["token_loss"], rtol=2e-3, atol=2e-3)
    assert int(corr) == int(case["correct"])
    ref_dh = case["dhidden"].float()
    cos = torch.nn.functional.cosine_similarity(dh.flatten(), ref_dh.flatten(), dim=0)
    assert cos > 0.9999, float(cos)
