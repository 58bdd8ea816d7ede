"""Comparison helpers shared by the GPU parity tests."""

import torch


def bf16_ulp(x: torch.Tensor) -> torch.Tensor:
    """Spacing of bf16 numbers around |x| (8 significant bits)."""
    a = x.float().abs().clamp_min(2.0 ** -126)
    return torch.exp2(torch.floor(torch.log2(a)) - 7)


def assert_lowp_matches(actual: torch.Tensor, expected_fp32: torch.Tensor, dtype=None,
                        max_ulp: int = 1, min_exact: float = 0.97, name: str = ""):
    """actual (bf16/fp16) vs the fp32 oracle rounded once to the same dtype.

    A kernel computing the same fp32 formula rounds to the same value except
    where an fp32 difference of a few ulps straddles a rounding boundary; such
    elements differ by one ulp of the output dtype. Checks: every element
    within `max_ulp` ulps, and at least `min_exact` of them bit-identical.
    """
    dtype = dtype or actual.dtype
    exp = expected_fp32.to(dtype).float().cpu()
    act = actual.float().cpu()
    assert act.shape == exp.shape, (act.shape, exp.shape)
    diff = (act - exp).abs()
    if dtype == torch.bfloat16:
        ulp = bf16_ulp(exp)
    elif dtype == torch.float16:
        a = exp.abs().clamp_min(2.0 ** -14)
        ulp = torch.exp2(torch.floor(torch.log2(a)) - 10)
    else:
        ulp = exp.abs().clamp_min(1e-30) * 2.0 ** -23
    worst = float((diff / ulp).max()) if diff.numel() else 0.0
    exact = float((diff == 0).float().mean()) if diff.numel() else 1.0
    assert worst <= max_ulp + 1e-6, f"{name}: max {worst:.2f} ulp (> {max_ulp})"
    assert exact >= min_exact, f"{name}: only {exact:.4f} of elements bit-identical"
    return worst, exact


def max_rel_err(actual: torch.Tensor, expected: torch.Tensor) -> float:
    """max|a - b| / max|b| (norm-relative error)."""
    a = actual.float().cpu()
    b = expected.float().cpu()
    den = float(b.abs().max())
    return float((a - b).abs().max()) / (den if den > 0 else 1.0)


def cosine(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.double().flatten().cpu()
    b = b.double().flatten().cpu()
    return float((a @ b) / (a.norm() * b.norm()).clamp_min(1e-300))
