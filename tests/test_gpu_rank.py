"""soup_lora_rank_gemm / soup_lora_rank_grad_group: the rank-r products of the
LoRA linears (x As^T, dy B and the gradient products dxa^T x, dy^T xa) against
fp32 PyTorch products of the same bf16 operands.

Tolerance: the kernel accumulates in fp32 on the tensor cores (a different
summation order from the fp32 reference); bf16 outputs are compared within
1 % of the largest magnitude (bf16 rounding is 0.4 %), fp32 gradient
accumulations within 1e-4 relative to the largest magnitude.
"""
import pytest
import torch

from auspex_soup_demo_b200 import _lib

pytestmark = pytest.mark.gpu


def _close(got, ref, tol):
    err = (got.float() - ref.float()).abs().max().item()
    scale = ref.float().abs().max().item()
    assert err <= tol * scale, f"max error {err:.3e} against scale {scale:.3e}"


@pytest.mark.parametrize("t,k,r", [(8192, 1536, 48), (2048, 1536, 16), (2048, 1536, 32), (300, 200, 16),
                                   (2048, 8960, 16), (136, 64, 8), (1024, 1536, 64)])
def test_rank_product_and_transpose(t, k, r):
    from auspex_soup_demo_b200 import qlora

    g = torch.Generator(device="cuda").manual_seed(t + k + r)
    x = torch.randn(t, k, device="cuda", generator=g).bfloat16()
    a = (0.05 * torch.randn(r, k, device="cuda", generator=g)).bfloat16()
    c = torch.empty(t, r, device="cuda", dtype=torch.bfloat16)
    ct = torch.empty(r, t, device="cuda", dtype=torch.bfloat16)
    qlora.rank_gemm(x, a, c=c, ct=ct)
    _close(c, x.float() @ a.float().t(), 1e-2)
    assert torch.equal(ct, c.t())


@pytest.mark.parametrize("t,k,r", [(8192, 1536, 48), (2048, 1536, 16), (304, 200, 16), (2048, 8960, 16)])
def test_rank_gradient_accumulation_transposed_and_deterministic(t, k, r):
    """gA += s dxa^T x written into A.grad [r, k] (the product's transpose),
    twice from the same start: bitwise equal."""
    from auspex_soup_demo_b200 import qlora

    g = torch.Generator(device="cuda").manual_seed(7 * t + k + r)
    x = torch.randn(t, k, device="cuda", generator=g).bfloat16()
    dxa = torch.randn(t, r, device="cuda", generator=g).bfloat16()
    g0 = torch.randn(r, k, device="cuda", generator=g)
    g1, g2 = g0.clone(), g0.clone()
    qlora.rank_gemm(x, dxa.t().contiguous(), a_mn_major=True, g=g1, g_trans=True, alpha=0.5)
    qlora.rank_gemm(x, dxa.t().contiguous(), a_mn_major=True, g=g2, g_trans=True, alpha=0.5)
    assert torch.equal(g1, g2)
    _close(g1 - g0, 0.5 * (dxa.float().t() @ x.float()), 1e-4)
    # untransposed: gB [n, r] += dy^T xa
    gb = torch.zeros(k, r, device="cuda")
    qlora.rank_gemm(x, dxa.t().contiguous(), a_mn_major=True, g=gb)
    _close(gb, x.float().t() @ dxa.float(), 1e-4)


@pytest.mark.parametrize("outs,interleaved", [([1536, 256, 256], False), ([896, 896], True),
                                              ([8960, 8960], True)])
def test_rank_group_gradient_members(outs, interleaved):
    """Each member's gB from one pass over the group's dy: its rows (row blocks
    in turn when interleaved) and its rank columns of dy^T xa."""
    from auspex_soup_demo_b200 import qlora

    t, r = 2048, 16
    g = torch.Generator(device="cuda").manual_seed(len(outs) + int(interleaved))
    n, rr = sum(outs), r * len(outs)
    dy = torch.randn(t, n, device="cuda", generator=g).bfloat16()
    xa = torch.randn(t, rr, device="cuda", generator=g).bfloat16()
    grads = [torch.randn(o, r, device="cuda", generator=g) for o in outs]
    start = [x.clone() for x in grads]
    row_off = [0]
    col_off = [0]
    for o in outs:
        row_off.append(row_off[-1] + o)
        col_off.append(col_off[-1] + r)
    qlora.rank_grad_group(dy, xa.t().contiguous(), row_off, col_off, grads, interleaved)
    G = dy.float().t() @ xa.float()
    for j, o in enumerate(outs):
        if interleaved:
            part = G.view(outs[0] // 128, len(outs), 128, rr)[:, j, :, col_off[j]:col_off[j + 1]]
            part = part.reshape(o, r)
        else:
            part = G[row_off[j]:row_off[j + 1], col_off[j]:col_off[j + 1]]
        _close(grads[j] - start[j], part, 1e-4)


def test_rank_product_argument_errors():
    from auspex_soup_demo_b200 import _lib, qlora

    x = torch.randn(256, 128, device="cuda").bfloat16()
    wide = torch.randn(80, 128, device="cuda").bfloat16()  # n > 64
    with pytest.raises(_lib.SoupError):
        qlora.rank_gemm(x, wide, c=torch.empty(256, 80, device="cuda", dtype=torch.bfloat16))
    a = torch.randn(16, 128, device="cuda").bfloat16()
    with pytest.raises(_lib.SoupError):  # no output
        qlora.rank_gemm(x, a)
    assert _lib.device_error(x.device) == 0


@pytest.mark.parametrize("m,n,r", [(8192, 17920, 32), (1000, 3000, 16), (304, 704, 48), (2048, 4096, 64),
                                   (136, 144, 8)])
def test_rank_dual_matches_fp32(m, n, r):
    """soup_lora_rank_dual: dxa = dy B and G = dy^T xa from one pass over dy,
    against fp32 products of the same bf16 operands (dxa rounded once to bf16,
    G in fp32), ragged edges and ranks 8-64; results bitwise repeatable."""
    from auspex_soup_demo_b200 import qlora

    # TMA operands: rows of dy, B^T and xa^T 16-byte aligned (m, n multiples of 8)
    g = torch.Generator(device="cuda").manual_seed(m + n + r)
    dy = torch.randn(m, n, device="cuda", generator=g).bfloat16()
    B = (0.05 * torch.randn(n, r, device="cuda", generator=g)).bfloat16()
    xa = torch.randn(m, r, device="cuda", generator=g).bfloat16()
    bt, xt = B.t().contiguous(), xa.t().contiguous()
    dxa, G = qlora.rank_dual(dy, bt, xt)
    dxa2, G2 = qlora.rank_dual(dy, bt, xt)
    torch.cuda.synchronize()
    assert _lib.device_error(dy.device) == 0
    assert torch.equal(dxa, dxa2) and torch.equal(G, G2)
    ref_dxa = dy.float() @ B.float()
    ref_G = dy.float().t() @ xa.float()
    # bf16 output: within one rounding of the fp32 result (8e-3 of the largest entry)
    assert (dxa.float() - ref_dxa).abs().max().item() <= 8e-3 * ref_dxa.abs().max().item()
    tol = 1e-5 * max(1.0, (m / 1536) ** 0.5)
    assert (G - ref_G).abs().max().item() <= tol * ref_G.abs().max().item()


def test_rank_dual_rejects_unaligned_rows():
    from auspex_soup_demo_b200 import qlora

    dy = torch.zeros(300, 700, device="cuda", dtype=torch.bfloat16)
    bt = torch.zeros(16, 700, device="cuda", dtype=torch.bfloat16)
    xt = torch.zeros(16, 300, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(_lib.SoupError):
        qlora.rank_dual(dy, bt, xt)
