"""GPU parity of RMSNorm, SwiGLU and RoPE against the CPU oracle.

Shapes follow the reference's own tests (solution/test_kernels.py) plus the
benchmark configurations and ragged / strided edge cases. fp32 outputs are
compared with relative tolerance 1e-4 (the reference's fp32 tolerance); bf16 /
fp16 outputs must equal the oracle rounded once to the output dtype, up to
one ulp where an fp32 rounding difference straddles a boundary
(helpers.assert_lowp_matches).
"""

import pytest
import torch

import oracle
from auspex_soup_demo_b200.kernels import (FastRMSNormFunction, apply_fast_rope,
                                           apply_fast_rope_qk, fast_rms_norm, fast_swiglu)
from helpers import assert_lowp_matches, max_rel_err

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-4


def _check(actual, expected, name):
    if actual.dtype == torch.float32:
        err = max_rel_err(actual, expected)
        assert err <= FP32_TOL, f"{name}: max rel err {err:.3e}"
    else:
        assert_lowp_matches(actual, expected, name=name)


# ------------------------------------------------------------------ RMSNorm --
RMS_CASES = [
    ((2048, 1536), torch.float32),   # benchmark configuration
    ((4, 512, 1536), torch.float16), ((4, 512, 1536), torch.float32),  # reference test shapes
    ((2, 128, 1536), torch.float16), ((2, 128, 1536), torch.float32),
    ((1, 16, 1536), torch.float16), ((1, 16, 1536), torch.float32),
    ((4, 512, 1536), torch.bfloat16),
    ((7, 96), torch.float32),        # short rows, lanes idle
    ((5, 100), torch.bfloat16),      # cols % 8 != 0: generic path
    ((3, 4096), torch.bfloat16),     # longest vector path
    ((3, 5000), torch.float32),      # beyond the vector path
]


@pytest.mark.parametrize("shape,dtype", RMS_CASES, ids=lambda v: str(v))
def test_rmsnorm_fwd_bwd(shape, dtype):
    g = torch.Generator().manual_seed(0)
    D = shape[-1]
    x = torch.randn(shape, generator=g).to(dtype)
    w = (1.0 + 0.1 * torch.randn(D, generator=g)).to(dtype)
    dy = torch.randn(shape, generator=g).to(dtype)
    y_ref, rstd = oracle.rmsnorm_fwd(x, w, 1e-6)
    dx_ref, dw_ref = oracle.rmsnorm_bwd(dy, x, w, rstd)
    # fp32 reference values before the final rounding
    xf, wf, dyf = x.float(), w.float(), dy.float()
    y32, r32 = oracle.rmsnorm_fwd(xf, wf, 1e-6)
    dx32, dw32 = oracle.rmsnorm_bwd(dyf, xf, wf, r32)

    xg = x.cuda().requires_grad_(True)
    wg = w.cuda().requires_grad_(True)
    y = fast_rms_norm(xg, wg, 1e-6)
    y.backward(dy.cuda())
    torch.cuda.synchronize()
    _check(y, y32, "y")
    _check(xg.grad, dx32, "dx")
    # dw sums over all rows: norm-relative error against the fp32 sum
    err = max_rel_err(wg.grad, dw32)
    assert err <= (FP32_TOL if dtype == torch.float32 else 8e-3), f"dw rel err {err:.3e}"


def test_rmsnorm_strided_rows_and_frozen_weight():
    x_full = torch.randn(64, 2048).cuda()
    x = x_full[:, :1536]  # row stride 2048, no copy
    w = torch.randn(1536).cuda()
    xg = x.detach().requires_grad_(True)
    y = fast_rms_norm(xg, w, 1e-5)
    dy = torch.randn_like(y)
    y.backward(dy)
    y_ref, r = oracle.rmsnorm_fwd(x.cpu(), w.cpu(), 1e-5)
    dx_ref, _ = oracle.rmsnorm_bwd(dy.cpu(), x.cpu(), w.cpu(), r)
    assert max_rel_err(y, y_ref) < FP32_TOL
    assert max_rel_err(xg.grad, dx_ref) < FP32_TOL


def test_rmsnorm_dw_is_deterministic():
    x = torch.randn(2048, 1536, device="cuda", requires_grad=True)
    w = torch.randn(1536, device="cuda", requires_grad=True)
    dy = torch.randn(2048, 1536, device="cuda")
    grads = []
    for _ in range(3):
        w.grad = None
        fast_rms_norm(x, w).backward(dy)
        grads.append(w.grad.clone())
    assert torch.equal(grads[0], grads[1]) and torch.equal(grads[1], grads[2])


# ------------------------------------------------------------------- SwiGLU --
SWIGLU_CASES = [
    ((2048, 8960), torch.bfloat16),  # benchmark configuration
    ((4, 512, 8960), torch.float16), ((4, 512, 8960), torch.float32),  # reference test shapes
    ((2, 64, 1024), torch.float16), ((2, 64, 1024), torch.float32),
    ((1, 16, 512), torch.float16), ((1, 16, 512), torch.float32),
    ((3, 7, 1000), torch.bfloat16),  # cols % 8 == 0 but odd row count
    ((5, 333), torch.bfloat16),      # ragged: scalar path
]


@pytest.mark.parametrize("shape,dtype", SWIGLU_CASES, ids=lambda v: str(v))
def test_swiglu_fwd_bwd(shape, dtype):
    g = torch.Generator().manual_seed(1)
    gate = torch.randn(shape, generator=g).to(dtype)
    up = torch.randn(shape, generator=g).to(dtype)
    dy = torch.randn(shape, generator=g).to(dtype)
    out32 = oracle.swiglu_fwd(gate.float(), up.float())
    dg32, du32 = oracle.swiglu_bwd(dy.float(), gate.float(), up.float())
    gg = gate.cuda().requires_grad_(True)
    ug = up.cuda().requires_grad_(True)
    out = fast_swiglu(gg, ug)
    out.backward(dy.cuda())
    torch.cuda.synchronize()
    _check(out, out32, "out")
    _check(gg.grad, dg32, "dgate")
    _check(ug.grad, du32, "dup")


def test_swiglu_column_slices_of_fused_projection():
    gu = torch.randn(256, 2 * 1024, device="cuda", dtype=torch.bfloat16)
    gate, up = gu[:, :1024], gu[:, 1024:]  # row stride 2048, no copy
    out = fast_swiglu(gate, up)
    ref = oracle.swiglu_fwd(gate.float().cpu(), up.float().cpu())
    assert_lowp_matches(out, ref, name="slices")


# --------------------------------------------------------------------- RoPE --
def _tables(S, D, theta, dtype, B=1):
    cos, sin = oracle.rope_cos_sin(S, D, theta, dtype)
    return cos[None].expand(B, S, D).contiguous(), sin[None].expand(B, S, D).contiguous()


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("shape", [(4, 12, 128, 128), (2, 2, 64, 128)])
def test_rope_reference_test_shapes(shape, dtype):
    B, H, S, D = shape
    g = torch.Generator().manual_seed(2)
    x = torch.randn(shape, generator=g).to(dtype)
    dy = torch.randn(shape, generator=g).to(dtype)
    cos, sin = oracle.rope_cos_sin(S, D, 10000.0, dtype)
    cos4, sin4 = cos[None, None], sin[None, None]
    y32 = oracle.rope_fwd(x.float(), cos4.float(), sin4.float())
    dx32 = oracle.rope_bwd(dy.float(), cos4.float(), sin4.float())
    xg = x.cuda().requires_grad_(True)
    y = apply_fast_rope(xg, cos4.cuda(), sin4.cuda())
    y.backward(dy.cuda())
    _check(y, y32, "y")
    _check(xg.grad, dx32, "dx")


def test_rope_qk_benchmark_config_hf_layout():
    """Q [4,12,512,128] and K [4,2,512,128] bf16 as strided views of [B,S,H,D], theta 1e6."""
    B, S, Hq, Hk, D = 4, 512, 12, 2, 128
    g = torch.Generator().manual_seed(3)
    q = torch.randn(B, S, Hq, D, generator=g).to(torch.bfloat16).cuda().transpose(1, 2)
    k = torch.randn(B, S, Hk, D, generator=g).to(torch.bfloat16).cuda().transpose(1, 2)
    cos, sin = _tables(S, D, 1e6, torch.bfloat16, B)
    cos4, sin4 = cos.cuda()[:, None], sin.cuda()[:, None]
    qg = q.detach().requires_grad_(True)
    kg = k.detach().requires_grad_(True)
    qo, ko = apply_fast_rope_qk(qg, kg, cos4, sin4)
    dq = torch.randn_like(qo)
    dk = torch.randn_like(ko)
    torch.autograd.backward([qo, ko], [dq, dk])
    c32, s32 = cos4.float().cpu(), sin4.float().cpu()
    _check(qo, oracle.rope_fwd(q.float().cpu(), c32, s32), "q")
    _check(ko, oracle.rope_fwd(k.float().cpu(), c32, s32), "k")
    _check(qg.grad, oracle.rope_bwd(dq.float().cpu(), c32, s32), "dq")
    _check(kg.grad, oracle.rope_bwd(dk.float().cpu(), c32, s32), "dk")
    # the output keeps the input's strides (empty_like, as the reference)
    assert qo.stride() == q.stride()


def test_rope_matches_hf_apply_rotary_pos_emb():
    from transformers.models.qwen2 import modeling_qwen2 as m

    original = getattr(m.apply_rotary_pos_emb, "_soup_original", m.apply_rotary_pos_emb)
    B, S, D = 2, 64, 128
    q = torch.randn(B, 12, S, D, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(B, 2, S, D, device="cuda", dtype=torch.bfloat16)
    cos, sin = _tables(S, D, 1e6, torch.bfloat16, B)
    ref_q, ref_k = original(q.float(), k.float(), cos.cuda().float(), sin.cuda().float())
    qo, ko = apply_fast_rope_qk(q, k, cos.cuda()[:, None], sin.cuda()[:, None])
    assert_lowp_matches(qo, ref_q, name="q")
    assert_lowp_matches(ko, ref_k, name="k")


def test_rope_fp32_tables_with_bf16_activations_and_odd_shapes():
    B, H, S, D = 3, 5, 17, 64
    x = torch.randn(B, H, S, D, device="cuda", dtype=torch.bfloat16)
    cos, sin = oracle.rope_cos_sin(S, D, 1e6, torch.float32)
    y = apply_fast_rope(x, cos.cuda(), sin.cuda())  # 2-D tables
    ref = oracle.rope_fwd(x.float().cpu(), cos, sin)
    assert_lowp_matches(y, ref, name="y")
