"""Stream-K tail of the tcgen05 pair GEMM (soup_gemm_set_stream_k_workspace).

When the tiles of a launch do not fill whole waves of CTA pairs, the k blocks
of the leftover tiles are spread over the pairs and the pair holding a tile's
last k block adds the other parts' fp32 partials before its epilogue. The
shapes below give every case of that split: fewer tiles than pairs (every
tile in parts), whole waves plus a tail, tails whose tiles have only a few k
blocks (a tile in several short parts), the rank-r k-block of the LoRA GEMM
inside a part, ragged edges, fp32 and bf16 (TMA-store) outputs, accumulate,
the SwiGLU epilogue (whose warps read two separate column runs of a tile),
the fused CE's logits and dW epilogues and the fused MLP backward. Each result is checked against an fp32 matmul, against the same launch
with the stream-K tail turned off, and for bitwise repeatability.
"""

import pytest
import torch

from auspex_soup_demo_b200 import _lib, qlora

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _every_tail_as_stream_k():
    """By default a tail runs as stream-K only when that saves >= 24 k blocks;
    here every tail that can be split is, so the short-K shapes test it too."""
    _lib.lib().soup_gemm_set_stream_k_min_saved(0)
    yield
    _lib.lib().soup_gemm_set_stream_k_min_saved(-1)


def _lora_gemm(A, b, b_mn, A2, b2, r, bias, c, accumulate=False, alpha=1.0):
    m, k = A.shape
    n = c.shape[1]
    _lib.call("soup_gemm_bf16_lora", A.device, A.data_ptr(), A.stride(0), 0, b.data_ptr(), b.stride(0),
              int(b_mn), None if r == 0 else A2.data_ptr(), A2.stride(0) if r else 0,
              None if r == 0 else b2.data_ptr(), b2.stride(0) if r else 0, r,
              None if bias is None else bias.data_ptr(), c.data_ptr(), c.stride(0),
              _lib.dtype_code(c.dtype), m, n, k, float(alpha), int(accumulate), _lib.stream_of(c))
    return c


def _both(fn):
    """fn() with the stream-K tail on (twice) and off; the device error word stays 0."""
    try:
        _lib.set_stream_k(True)
        dev = torch.device("cuda")
        on1 = fn()
        on2 = fn()
        torch.cuda.synchronize()
        assert _lib.device_error(dev) == 0
        _lib.set_stream_k(False)
        off = fn()
        torch.cuda.synchronize()
        assert _lib.device_error(dev) == 0
    finally:
        _lib.set_stream_k(True)
    return on1, on2, off


def _rel(a, b):
    return (a.float() - b.float()).abs().max().item() / b.float().abs().max().item()


# (m, n, k, r, b_mn): tiles of 256 x 256 against 74 CTA pairs on a B200
SHAPES = [
    (2048, 1536, 2048, 48, 1),  # 48 tiles: all of them in k parts
    (8192, 1536, 1536, 16, 0),  # 192 tiles: two whole waves, 44 tiles in parts
    (8192, 1536, 8960, 16, 0),  # the same with K = 8960
    (2560, 2560, 384, 0, 0),    # 100 tiles of 6 k blocks: 26 tiles cut in up to 4 short parts
    (600, 1000, 192, 16, 1),    # 12 ragged tiles of 4 k blocks (the last one the rank block)
    (8192, 2048, 1536, 48, 0),  # 256 tiles: three whole waves, 34 in parts
]


@pytest.mark.parametrize("m,n,k,r,b_mn", SHAPES)
def test_stream_k_tail_matches_fp32_and_partial_wave(m, n, k, r, b_mn):
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    A = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    B = torch.randn(n, k, device="cuda", generator=g).to(torch.bfloat16)
    A2 = torch.randn(m, r, device="cuda", generator=g).to(torch.bfloat16) if r else None
    B2 = torch.randn(n, r, device="cuda", generator=g).to(torch.bfloat16) if r else None
    b = B.t().contiguous() if b_mn else B
    b2 = (B2.t().contiguous() if b_mn else B2) if r else None
    ref = A.float() @ B.float().t()
    if r:
        ref = ref + A2.float() @ B2.float().t()
    # fp32 outputs: 1e-5 of the largest entry at K ~ 1536, growing with the
    # square root of the number of fp32 additions (K = 8960: 2.4e-5)
    fp32_tol = 1e-5 * max(1.0, ((k + r) / 1536) ** 0.5)
    for dtype, tol in ((torch.float32, fp32_tol), (torch.bfloat16, 8e-3)):
        on1, on2, off = _both(lambda: _lora_gemm(A, b, b_mn, A2, b2, r, None,
                                                  torch.empty(m, n, device="cuda", dtype=dtype)))
        assert torch.equal(on1, on2), "stream-K results must not vary from run to run"
        assert _rel(on1, ref) < tol, (dtype, _rel(on1, ref))
        assert _rel(off, ref) < tol, (dtype, _rel(off, ref))
        if dtype == torch.float32:
            assert _rel(on1, off) < fp32_tol


def test_stream_k_tail_with_bias_alpha_and_accumulate():
    m, n, k, r = 2048, 1536, 1536, 16
    g = torch.Generator(device="cuda").manual_seed(7)
    A = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    B = torch.randn(n, k, device="cuda", generator=g).to(torch.bfloat16)
    A2 = torch.randn(m, r, device="cuda", generator=g).to(torch.bfloat16)
    B2 = torch.randn(n, r, device="cuda", generator=g).to(torch.bfloat16)
    bias = torch.randn(n, device="cuda", generator=g).to(torch.bfloat16)
    c0 = torch.randn(m, n, device="cuda", generator=g)
    on1, on2, off = _both(lambda: _lora_gemm(A, B, 0, A2, B2, r, None, c0.clone(), accumulate=True, alpha=0.5))
    ref = c0 + 0.5 * (A.float() @ B.float().t() + A2.float() @ B2.float().t())
    assert torch.equal(on1, on2)
    assert _rel(on1, ref) < 1e-5 and _rel(off, ref) < 1e-5
    on1, on2, off = _both(lambda: _lora_gemm(A, B, 0, A2, B2, r, bias,
                                              torch.empty(m, n, device="cuda", dtype=torch.bfloat16)))
    ref = A.float() @ B.float().t() + A2.float() @ B2.float().t() + bias.float()
    assert torch.equal(on1, on2)
    assert _rel(on1, ref) < 8e-3 and _rel(off, ref) < 8e-3


@pytest.mark.parametrize("m", [2048, 8192])
def test_stream_k_tail_swiglu_epilogue_equals_plain_gemm_plus_swiglu(m):
    """The SwiGLU-epilogue GEMM and the plain GEMM have the same tiles, hence the
    same stream-K parts: h and [g | u] must agree bit for bit with the plain GEMM
    followed by the SwiGLU kernel, with the tail on."""
    from auspex_soup_demo_b200.kernels.swiglu import swiglu_forward

    inter, k, R = 1024, 1536, 32
    g_ = torch.Generator(device="cuda").manual_seed(m)
    x = torch.randn(m, k, device="cuda", generator=g_).to(torch.bfloat16)
    w = (0.05 * torch.randn(2 * inter, k, device="cuda", generator=g_)).to(torch.bfloat16)
    xa = torch.randn(m, R, device="cuda", generator=g_).to(torch.bfloat16)
    Bblk = (0.05 * torch.randn(2 * inter, R, device="cuda", generator=g_)).to(torch.bfloat16)
    _lib.set_stream_k(True)
    h = torch.empty(m, inter, device="cuda", dtype=torch.bfloat16)
    y = torch.empty(m, 2 * inter, device="cuda", dtype=torch.bfloat16)
    qlora.swiglu_gemm(x, w, xa, Bblk, None, 0, h, y)
    plain = qlora.lora_gemm(x, w, False, xa, Bblk, torch.empty(m, 2 * inter, device="cuda",
                                                                 dtype=torch.bfloat16))
    torch.cuda.synchronize()
    assert _lib.device_error(x.device) == 0
    assert torch.equal(y, plain)
    y2 = plain.view(-1, 2 * qlora.IL_BLOCK)
    h_ref = swiglu_forward(y2[:, :qlora.IL_BLOCK], y2[:, qlora.IL_BLOCK:]).view(m, inter)
    assert torch.equal(h, h_ref)


def test_stream_k_tail_fused_ce_logits_and_dweight():
    """The fused head CE with every GEMM tail forced to stream-K (the logits GEMM's
    online-softmax epilogue, the dW GEMM) against the same call with the tail off:
    per-token losses and entropies within fp32 accumulation error, hits equal,
    dhidden and dW at cosine >= 0.9999 (the fp32 sums differ only in order)."""
    from auspex_soup_demo_b200.kernels.chunked_ce import fused_linear_cross_entropy

    n, v, d = 1000, 33000, 1536  # logits 4 x 129 tiles, dW 129 x 6 tiles: both leave a partial wave
    g = torch.Generator(device="cuda").manual_seed(21)
    h = torch.randn(n, d, device="cuda", generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn(v, d, device="cuda", generator=g)).to(torch.bfloat16)
    t = torch.randint(0, v, (n,), device="cuda", generator=g)
    t[::10] = -100

    def run():
        return fused_linear_cross_entropy(h, w, t, denominator=float((t != -100).sum()), compute_dw=True)

    on1, on2, off = _both(run)
    for a, b in zip(on1, on2):
        assert torch.equal(a, b)
    loss_on, ent_on, hit_on, _, dh_on, dw_on = on1
    loss_off, ent_off, hit_off, _, dh_off, dw_off = off
    assert (loss_on - loss_off).abs().max().item() <= 1e-4 * loss_off.abs().max().item()
    assert (ent_on - ent_off).abs().max().item() <= 1e-4 * ent_off.abs().max().item()
    assert torch.equal(hit_on, hit_off)
    cos = torch.nn.functional.cosine_similarity
    assert cos(dh_on.float().flatten(), dh_off.float().flatten(), dim=0).item() >= 0.9999
    assert cos(dw_on.float().flatten(), dw_off.float().flatten(), dim=0).item() >= 0.9999


def test_stream_k_tail_fused_mlp_backward_epilogue():
    """The down projection's dX GEMM with the SwiGLU backward in its epilogue, tail
    forced to stream-K, against the same GEMM with a plain epilogue (also forced)
    followed by the SwiGLU backward kernel: bit-identical [dg | du]."""
    from auspex_soup_demo_b200.kernels.swiglu import swiglu_backward

    m, inter, k, r = 2048, 2048, 1536, 16  # 8 x 8 tiles < 74 CTA pairs: every tile in k parts
    g = torch.Generator(device="cuda").manual_seed(33)
    d = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = (0.05 * torch.randn(k, inter, device="cuda", generator=g)).bfloat16()
    dxa = torch.randn(m, r, device="cuda", generator=g).bfloat16()
    As = (0.05 * torch.randn(r, inter, device="cuda", generator=g)).bfloat16()
    y = torch.randn(m, 2 * inter, device="cuda", generator=g).bfloat16()
    _lib.set_stream_k(True)
    dh = qlora.lora_gemm(d, w, True, dxa, As, torch.empty(m, inter, device="cuda", dtype=torch.bfloat16))
    y2 = y.view(-1, 256)
    dy_ref = torch.empty_like(y)
    d2 = dy_ref.view(-1, 256)
    swiglu_backward(dh.view(-1, 128), y2[:, :128], y2[:, 128:], dg=d2[:, :128], du=d2[:, 128:])
    yy = y.clone()
    qlora.dswiglu_gemm(d, w, dxa, As, yy)
    torch.cuda.synchronize()
    assert _lib.device_error(torch.device("cuda")) == 0
    assert torch.equal(yy, dy_ref)
