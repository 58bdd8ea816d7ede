"""tcgen05 GEMM engine through the C ABI (soup_gemm_bf16, soup_gemm_bf16_lora) vs
an fp32 matmul.

Covers the four operand layouts the fused CE uses (K-major / MN-major A and B),
ragged edges in M, N and K, alpha, accumulate, fp32 and bf16 outputs, and the
trailing rank-r K segment with bias that the QLoRA linears use.
"""

import pytest
import torch

from auspex_soup_demo_b200 import _lib

pytestmark = pytest.mark.gpu


def run_gemm(a_store, a_mn, b_store, b_mn, m, n, k, c_dtype=torch.float32, alpha=1.0, c=None,
             accumulate=False):
    dev = a_store.device
    if c is None:
        c = torch.zeros(m, n, dtype=c_dtype, device=dev)
    _lib.call("soup_gemm_bf16", dev, a_store.data_ptr(), a_store.stride(0), int(a_mn),
              b_store.data_ptr(), b_store.stride(0), int(b_mn), c.data_ptr(), c.stride(0),
              _lib.dtype_code(c.dtype), m, n, k, float(alpha), int(accumulate), _lib.stream_of(c))
    torch.cuda.synchronize()
    assert _lib.device_error(dev) == 0
    return c


def operands(m, n, k, a_mn, b_mn, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    B = torch.randn(n, k, device="cuda", generator=g).to(torch.bfloat16)
    a_store = A.t().contiguous() if a_mn else A
    b_store = B.t().contiguous() if b_mn else B
    ref = A.float() @ B.float().t()
    return a_store, b_store, ref


@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 512, 128), (200, 328, 192), (1000, 1536, 704)])
def test_gemm_layouts(a_mn, b_mn, m, n, k):
    a, b, ref = operands(m, n, k, a_mn, b_mn)
    c = run_gemm(a, a_mn, b, b_mn, m, n, k)
    err = (c - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-5, err


def test_gemm_bf16_out_alpha_accumulate():
    m, n, k = 384, 768, 256
    a, b, ref = operands(m, n, k, 0, 1, seed=3)
    c0 = torch.randn(m, n, device="cuda").to(torch.bfloat16)
    c = run_gemm(a, 0, b, 1, m, n, k, alpha=0.5, c=c0.clone(), accumulate=True)
    exp = (0.5 * ref + c0.float())
    err = (c.float() - exp).abs().max().item() / exp.abs().max().item()
    assert err < 8e-3, err


def test_gemm_many_tiles_persistent():
    # more tiles than SMs: every CTA walks several tiles and both TMEM buffers
    m, n, k = 2048, 4096, 512
    a, b, ref = operands(m, n, k, 0, 0, seed=5)
    c = run_gemm(a, 0, b, 0, m, n, k)
    err = (c - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-5, err


def test_gemm_leading_dimension_padding():
    m, n, k = 256, 256, 128
    g = torch.Generator(device="cuda").manual_seed(9)
    A = torch.randn(m, k + 64, device="cuda", generator=g).to(torch.bfloat16)[:, :k]
    B = torch.randn(n, k + 8, device="cuda", generator=g).to(torch.bfloat16)[:, :k]
    c = torch.zeros(m, n + 16, device="cuda")[:, :n]
    run_gemm(A, 0, B, 0, m, n, k, c=c)
    ref = A.float() @ B.float().t()
    assert (c - ref).abs().max().item() / ref.abs().max().item() < 1e-5


@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("m,n,k", [(64, 128, 64), (104, 136, 128), (136, 256, 64), (264, 384, 320)])
def test_gemm_pair_tile_edges(a_mn, b_mn, m, n, k):
    # a 256-row tile split over two CTAs: the second CTA's rows (m <= 128) or
    # its half of the B columns (n <= 128) may lie wholly outside the matrix
    a, b, ref = operands(m, n, k, a_mn, b_mn, seed=11)
    c = run_gemm(a, a_mn, b, b_mn, m, n, k)
    err = (c - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-5, err


@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (1, 1)])
@pytest.mark.parametrize("m,n,k", [(64, 128, 64), (104, 136, 128), (136, 256, 64), (264, 392, 320)])
def test_gemm_pair_tile_edges_bf16_tma_store(a_mn, b_mn, m, n, k):
    # bf16 outputs leave through TMA stores clipped to the matrix: every element
    # inside is written (C starts as NaN) and nothing outside the view is touched
    a, b, ref = operands(m, n, k, a_mn, b_mn, seed=17)
    pad = torch.full((m + 8, n + 16), 7.0, dtype=torch.bfloat16, device="cuda")
    c = pad[:m, :n]
    c.fill_(float("nan"))
    run_gemm(a, a_mn, b, b_mn, m, n, k, c=c)
    err = (c.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err < 8e-3, err
    assert bool((pad[m:, :] == 7.0).all()) and bool((pad[:, n:] == 7.0).all())


def test_gemm_many_tiles_mn_major():
    m, n, k = 3000, 2048, 448
    a, b, ref = operands(m, n, k, 1, 1, seed=13)
    c = run_gemm(a, 1, b, 1, m, n, k)
    err = (c - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-5, err


def run_lora_gemm(a, b, b_mn, a2, b2, m, n, k, r, bias=None, c_dtype=torch.float32, alpha=1.0):
    c = torch.full((m, n), float("nan"), dtype=c_dtype, device=a.device)
    _lib.call("soup_gemm_bf16_lora", a.device, a.data_ptr(), a.stride(0), 0, b.data_ptr(), b.stride(0),
              int(b_mn), a2.data_ptr(), a2.stride(0), b2.data_ptr(), b2.stride(0), r,
              None if bias is None else bias.data_ptr(), c.data_ptr(), c.stride(0),
              _lib.dtype_code(c.dtype), m, n, k, float(alpha), 0, _lib.stream_of(c))
    torch.cuda.synchronize()
    assert _lib.device_error(a.device) == 0
    return c


@pytest.mark.parametrize("b_mn", [0, 1])
@pytest.mark.parametrize("m,n,k,r", [(256, 512, 128, 16), (1000, 1536, 704, 16), (520, 264, 1536, 48),
                                     (2048, 1536, 1536, 80)])
@pytest.mark.parametrize("with_bias,c_bf16", [(False, False), (True, True)])
def test_gemm_lora_segment(b_mn, m, n, k, r, with_bias, c_bf16):
    # C = alpha (A B^T + A2 B2^T) + bias: the rank-r term is the GEMM's trailing
    # k-block(s), zero-filled by TMA past r (r = 16, 48: one block; 80: two)
    g = torch.Generator(device="cuda").manual_seed(11)
    A = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    B = torch.randn(n, k, device="cuda", generator=g).to(torch.bfloat16)
    A2 = torch.randn(m, r, device="cuda", generator=g).to(torch.bfloat16)
    B2 = torch.randn(n, r, device="cuda", generator=g).to(torch.bfloat16)
    bias = torch.randn(n, device="cuda", generator=g).to(torch.bfloat16) if with_bias else None
    b = B.t().contiguous() if b_mn else B
    b2 = B2.t().contiguous() if b_mn else B2
    c = run_lora_gemm(A, b, b_mn, A2, b2, m, n, k, r, bias, torch.bfloat16 if c_bf16 else torch.float32,
                      alpha=0.5)
    ref = 0.5 * (A.float() @ B.float().t() + A2.float() @ B2.float().t())
    if with_bias:
        ref = ref + bias.float()
    err = (c.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err < (8e-3 if c_bf16 else 1e-5), err
    # r = 0 is the plain GEMM
    if r == 16 and not with_bias:
        c0 = run_lora_gemm(A, b, b_mn, A2, b2, m, n, k, 0)
        ref0 = A.float() @ B.float().t()
        assert (c0 - ref0).abs().max().item() / ref0.abs().max().item() < 1e-5


_SINGLE_CTA_SCRIPT = r"""
import torch
from auspex_soup_demo_b200 import _lib
torch.manual_seed(0)
for (m, n, k, a_mn, b_mn) in [(200, 328, 192, 0, 0), (1000, 1536, 704, 0, 1), (384, 512, 256, 1, 1)]:
    A = torch.randn(m, k, device="cuda").to(torch.bfloat16)
    B = torch.randn(n, k, device="cuda").to(torch.bfloat16)
    a = A.t().contiguous() if a_mn else A
    b = B.t().contiguous() if b_mn else B
    c = torch.zeros(m, n, device="cuda")
    _lib.call("soup_gemm_bf16", a.device, a.data_ptr(), a.stride(0), a_mn, b.data_ptr(),
              b.stride(0), b_mn, c.data_ptr(), c.stride(0), _lib.dtype_code(c.dtype), m, n, k,
              1.0, 0, _lib.stream_of(c))
    torch.cuda.synchronize()
    assert _lib.device_error(a.device) == 0
    ref = A.float() @ B.float().t()
    err = (c - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-5, (m, n, k, a_mn, b_mn, err)
for (m, n, k) in [(200, 328, 192), (1000, 1536, 704)]:  # bf16 out: TMA-store epilogue
    A = torch.randn(m, k, device="cuda").to(torch.bfloat16)
    B = torch.randn(n, k, device="cuda").to(torch.bfloat16)
    c = torch.full((m, n), float("nan"), device="cuda", dtype=torch.bfloat16)
    _lib.call("soup_gemm_bf16", A.device, A.data_ptr(), A.stride(0), 0, B.data_ptr(), B.stride(0), 0,
              c.data_ptr(), c.stride(0), _lib.dtype_code(c.dtype), m, n, k, 1.0, 0, _lib.stream_of(c))
    torch.cuda.synchronize()
    assert _lib.device_error(A.device) == 0
    ref = A.float() @ B.float().t()
    err = (c.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err < 8e-3, ("bf16", m, n, k, err)
m, n, k, r = 1000, 1536, 704, 16
A = torch.randn(m, k, device="cuda").to(torch.bfloat16)
B = torch.randn(k, n, device="cuda").to(torch.bfloat16)
A2 = torch.randn(m, r, device="cuda").to(torch.bfloat16)
B2 = torch.randn(r, n, device="cuda").to(torch.bfloat16)
c = torch.zeros(m, n, device="cuda")
_lib.call("soup_gemm_bf16_lora", A.device, A.data_ptr(), A.stride(0), 0, B.data_ptr(), B.stride(0), 1,
          A2.data_ptr(), A2.stride(0), B2.data_ptr(), B2.stride(0), r, None, c.data_ptr(), c.stride(0),
          _lib.dtype_code(c.dtype), m, n, k, 1.0, 0, _lib.stream_of(c))
torch.cuda.synchronize()
assert _lib.device_error(A.device) == 0
ref = A.float() @ B.float() + A2.float() @ B2.float()
err = (c - ref).abs().max().item() / ref.abs().max().item()
assert err < 1e-5, ("lora", err)
print("single-cta ok")
"""


def test_gemm_single_cta_mode():
    # SOUP_GEMM_PAIRS=0 selects the 128-row single-CTA kernel (read once per process)
    import os
    import subprocess
    import sys

    env = dict(os.environ, SOUP_GEMM_PAIRS="0")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _SINGLE_CTA_SCRIPT], env=env, cwd=root,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "single-cta ok" in r.stdout


@pytest.mark.parametrize("m,inter,k,with_bias", [(300, 384, 192, True), (2048, 8960, 1536, False)])
def test_swiglu_epilogue_gemm_equals_gemm_plus_swiglu_kernels(m, inter, k, with_bias):
    # soup_gemm_bf16_lora_swiglu (SwiGLU in the tcgen05 GEMM epilogue, interleaved
    # gate/up rows) against the same GEMM with a plain store followed by the SwiGLU
    # kernels: bit-identical h, [g | u] and [dg | du]
    from auspex_soup_demo_b200 import qlora
    from auspex_soup_demo_b200.kernels.swiglu import swiglu_backward, swiglu_forward

    g = torch.Generator(device="cuda").manual_seed(m + k)
    x = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = (0.05 * torch.randn(2 * inter, k, device="cuda", generator=g)).bfloat16()
    xa = torch.randn(m, 32, device="cuda", generator=g).bfloat16()
    bblk = (0.05 * torch.randn(2 * inter, 32, device="cuda", generator=g)).bfloat16()
    bias = (0.1 * torch.randn(2 * inter, device="cuda", generator=g)).bfloat16() if with_bias else None
    dh = torch.randn(m, inter, device="cuda", generator=g).bfloat16()
    y_ref = qlora.lora_gemm(x, w, False, xa, bblk, torch.empty(m, 2 * inter, device="cuda",
                                                               dtype=torch.bfloat16), bias)
    y2 = y_ref.view(-1, 256)
    gv, uv = y2[:, :128], y2[:, 128:]
    h_ref = swiglu_forward(gv, uv).view(m, inter)
    dy_ref = torch.empty_like(y_ref)
    d2 = dy_ref.view(-1, 256)
    swiglu_backward(dh.view(-1, 128), gv, uv, dg=d2[:, :128], du=d2[:, 128:])
    h = torch.empty(m, inter, device="cuda", dtype=torch.bfloat16)
    y = torch.empty_like(y_ref)
    qlora.swiglu_gemm(x, w, xa, bblk, bias, 0, h, y)
    h_only = torch.empty_like(h)
    qlora.swiglu_gemm(x, w, xa, bblk, bias, 0, h_only)
    dy = torch.empty_like(y_ref)
    qlora.swiglu_gemm(x, w, xa, bblk, bias, 1, dh, dy)
    torch.cuda.synchronize()
    assert torch.equal(y, y_ref)
    assert torch.equal(h, h_ref) and torch.equal(h_only, h_ref)
    assert torch.equal(dy, dy_ref)
    assert _lib.device_error(torch.device("cuda")) == 0


@pytest.mark.parametrize("m,inter,k,r", [(300, 640, 1536, 16), (2048, 8960, 1536, 16), (129, 256, 64, 0)])
def test_dswiglu_epilogue_gemm_equals_gemm_plus_swiglu_backward(m, inter, k, r):
    # soup_gemm_bf16_lora_dswiglu (the down projection's dX GEMM dh = d W + dxa As
    # with the SwiGLU backward in its epilogue, [dg | du] over [g | u] in place)
    # against the plain dX GEMM followed by the SwiGLU backward kernel: bit-identical
    from auspex_soup_demo_b200 import qlora
    from auspex_soup_demo_b200.kernels.swiglu import swiglu_backward

    g = torch.Generator(device="cuda").manual_seed(m + inter + r)
    d = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = (0.05 * torch.randn(k, inter, device="cuda", generator=g)).bfloat16()  # down weight [out, in]
    rr = max(r, 1)
    dxa = torch.randn(m, rr, device="cuda", generator=g).bfloat16()[:, :r].contiguous() if r else None
    As = (0.05 * torch.randn(rr, inter, device="cuda", generator=g)).bfloat16()[:r].contiguous() if r else None
    y = torch.randn(m, 2 * inter, device="cuda", generator=g).bfloat16()  # [g | u], interleaved blocks
    if r:
        dh = qlora.lora_gemm(d, w, True, dxa, As, torch.empty(m, inter, device="cuda", dtype=torch.bfloat16))
    else:
        dh = (d.float() @ w.float()).bfloat16()
        # the dX GEMM alone, through the library (no rank term)
        _lib.call("soup_gemm_bf16", d.device, d.data_ptr(), k, 0, w.data_ptr(), inter, 1, dh.data_ptr(),
                  inter, _lib.dtype_code(dh.dtype), m, inter, k, 1.0, 0, _lib.stream_of(d))
    y2 = y.view(-1, 256)
    dy_ref = torch.empty_like(y)
    d2 = dy_ref.view(-1, 256)
    swiglu_backward(dh.view(-1, 128), y2[:, :128], y2[:, 128:], dg=d2[:, :128], du=d2[:, 128:])
    yy = y.clone()
    if r:
        qlora.dswiglu_gemm(d, w, dxa, As, yy)
    else:
        _lib.call("soup_gemm_bf16_lora_dswiglu", d.device, d.data_ptr(), k, w.data_ptr(), inter, None, 0,
                  None, 0, 0, yy.data_ptr(), 2 * inter, m, inter, k, _lib.stream_of(d))
    torch.cuda.synchronize()
    assert _lib.device_error(torch.device("cuda")) == 0
    assert torch.equal(yy, dy_ref)
