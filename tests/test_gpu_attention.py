"""The tcgen05 flash attention against PyTorch fp32 attention on the GPU.

Reference: softmax(scale q k^T + causal mask) v computed in fp32 from the same
bf16 inputs (torch SDPA's math, with the KV heads repeated per query group).
The kernel rounds P to bf16 before the P V product, as flash attention does, so
the bf16 outputs are compared by relative error (max |a - b| / max |b| <= 1e-2,
rms <= 4e-3 relative) and cosine >= 0.9999; the log-sum-exp within 1e-3.
"""

import math

import pytest
import torch

from auspex_soup_demo_b200 import _lib
from auspex_soup_demo_b200.kernels.attention import attention_forward
from helpers import cosine

pytestmark = pytest.mark.gpu


def _ref(q, k, v, scale, causal):
    """fp32 attention with repeated KV heads: (out [B, S, H, D], lse [B, H, S])."""
    B, H, S, D = q.shape
    rep = H // k.shape[1]
    kf = k.float().repeat_interleave(rep, dim=1)
    vf = v.float().repeat_interleave(rep, dim=1)
    s = (q.float() @ kf.transpose(-1, -2)) * scale
    if causal:
        mask = torch.ones(S, S, dtype=torch.bool, device=q.device).triu(1)
        s = s.masked_fill(mask, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    o = torch.softmax(s, dim=-1) @ vf
    return o.transpose(1, 2), lse


def _inputs(B, H, Hk, S, seed, hf_layout=True):
    g = torch.Generator(device="cuda").manual_seed(seed)
    D = 128
    if hf_layout:  # [B, S, heads, D] projections viewed as [B, heads, S, D]
        q = torch.randn(B, S, H, D, device="cuda", generator=g).to(torch.bfloat16).transpose(1, 2)
        k = torch.randn(B, S, Hk, D, device="cuda", generator=g).to(torch.bfloat16).transpose(1, 2)
        v = torch.randn(B, S, Hk, D, device="cuda", generator=g).to(torch.bfloat16).transpose(1, 2)
    else:
        q = torch.randn(B, H, S, D, device="cuda", generator=g).to(torch.bfloat16)
        k = torch.randn(B, Hk, S, D, device="cuda", generator=g).to(torch.bfloat16)
        v = torch.randn(B, Hk, S, D, device="cuda", generator=g).to(torch.bfloat16)
    return q, k, v


def _close(out, ref):
    a, b = out.float(), ref.float()
    mx = float((a - b).abs().max()) / float(b.abs().max())
    rms = float((a - b).pow(2).mean().sqrt()) / float(b.pow(2).mean().sqrt())
    return mx, rms


@pytest.mark.parametrize("B,H,Hk,S,causal,hf", [
    (2, 12, 2, 384, True, True),    # Qwen2.5-1.5B heads, three query tiles
    (1, 12, 2, 300, True, True),    # ragged last tile
    (2, 4, 4, 256, False, False),   # no causal mask, MHA, contiguous [B, H, S, D]
    (1, 6, 1, 77, False, True),     # one ragged tile, no mask
    (1, 2, 2, 1024, True, False),   # eight tiles: the max is rescaled lazily across tiles
])
def test_attention_forward_matches_fp32(B, H, Hk, S, causal, hf):
    q, k, v = _inputs(B, H, Hk, S, seed=S + H, hf_layout=hf)
    scale = 1.0 / math.sqrt(128)
    out, lse = attention_forward(q, k, v, scale, causal)
    torch.cuda.synchronize()
    assert _lib.device_error(torch.device("cuda")) == 0
    ref_o, ref_lse = _ref(q, k, v, scale, causal)
    assert out.shape == (B, S, H, 128) and out.dtype == torch.bfloat16
    mx, rms = _close(out, ref_o)
    assert mx <= 1e-2 and rms <= 4e-3, (mx, rms)
    assert cosine(out, ref_o) >= 0.9999
    torch.testing.assert_close(lse, ref_lse, rtol=1e-3, atol=1e-3)


def test_attention_forward_large_logits():
    """Rows whose logits span ~60 nats with the maximum late in the row: the lazily
    kept maximum must be raised (O and the row sum rescaled) without overflow."""
    B, H, Hk, S = 1, 2, 1, 512
    q, k, v = _inputs(B, H, Hk, S, seed=5, hf_layout=False)
    q = (q.float() * 4.0).to(torch.bfloat16)
    k = k.clone()
    k[:, :, 300:310] = (k[:, :, 300:310].float() * 6.0).to(torch.bfloat16)
    scale = 1.0 / math.sqrt(128)
    out, lse = attention_forward(q, k, v, scale, True)
    ref_o, ref_lse = _ref(q, k, v, scale, True)
    assert bool(torch.isfinite(out.float()).all())
    mx, rms = _close(out, ref_o)
    assert mx <= 1e-2 and rms <= 4e-3, (mx, rms)
    torch.testing.assert_close(lse, ref_lse, rtol=1e-3, atol=2e-3)


def _ref_grads(q, k, v, dout, scale, causal):
    qf = q.detach().float().requires_grad_(True)
    kf = k.detach().float().requires_grad_(True)
    vf = v.detach().float().requires_grad_(True)
    o, _ = _ref(qf, kf, vf, scale, causal)
    o.backward(dout.float())
    return qf.grad, kf.grad, vf.grad


@pytest.mark.parametrize("B,H,Hk,S,causal,hf", [
    (2, 12, 2, 384, True, True),    # Qwen2.5-1.5B heads: dK / dV summed over groups of 6
    (1, 12, 2, 300, True, True),    # ragged last tile
    (1, 4, 4, 256, False, False),   # no mask, MHA
    (1, 2, 1, 1024, True, False),   # eight key tiles
])
def test_attention_backward_matches_fp32_autograd(B, H, Hk, S, causal, hf):
    from auspex_soup_demo_b200.kernels.attention import flash_attention

    q, k, v = _inputs(B, H, Hk, S, seed=7 * S + H, hf_layout=hf)
    scale = 1.0 / math.sqrt(128)
    g = torch.Generator(device="cuda").manual_seed(3)
    dout = torch.randn(B, S, H, 128, device="cuda", generator=g).to(torch.bfloat16)
    qg, kg, vg = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
    out = flash_attention(qg, kg, vg, scale, causal)
    out.backward(dout)
    torch.cuda.synchronize()
    assert _lib.device_error(torch.device("cuda")) == 0
    rq, rk, rv = _ref_grads(q, k, v, dout, scale, causal)
    for name, got, ref in (("dq", qg.grad, rq), ("dk", kg.grad, rk), ("dv", vg.grad, rv)):
        assert got.shape == ref.shape and got.dtype == torch.bfloat16, name
        assert cosine(got, ref) >= 0.9999, (name, cosine(got, ref))
        mx, rms = _close(got, ref)
        assert mx <= 2e-2 and rms <= 8e-3, (name, mx, rms)


def test_attention_backward_is_reproducible():
    from auspex_soup_demo_b200.kernels.attention import flash_attention

    q, k, v = _inputs(1, 12, 2, 512, seed=11)
    dout = torch.randn(1, 512, 12, 128, device="cuda").to(torch.bfloat16)
    grads = []
    for _ in range(2):
        qg, kg, vg = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
        flash_attention(qg, kg, vg, 128 ** -0.5, True).backward(dout)
        grads.append((qg.grad, kg.grad, vg.grad))
    for a, b in zip(*grads):
        assert torch.equal(a, b)


def test_qwen2_attention_through_the_interface_matches_sdpa():
    """transformers' Qwen2 attention with config._attn_implementation = "soup_b200"
    against the same module on transformers' SDPA path (bf16 both)."""
    from transformers.models.qwen2.modeling_qwen2 import Qwen2Attention, Qwen2RotaryEmbedding

    from auspex_soup_demo_b200 import qlora
    from auspex_soup_demo_b200.kernels import attention

    name = attention.register()
    cfg = qlora.qwen2_1p5b_config(num_layers=1)
    torch.manual_seed(0)
    attn = Qwen2Attention(cfg, 0).cuda().to(torch.bfloat16)
    rot = Qwen2RotaryEmbedding(cfg).cuda()
    B, S = 2, 640
    x = (0.5 * torch.randn(B, S, cfg.hidden_size, device="cuda")).to(torch.bfloat16)
    pos = torch.arange(S, device="cuda")[None].expand(B, -1)
    cos, sin = rot(x, pos)
    outs, grads = {}, {}
    for impl in ("sdpa", name):
        cfg._attn_implementation = impl
        xi = x.detach().clone().requires_grad_(True)
        y, _ = attn(xi, (cos, sin), None)
        y.float().pow(2).mean().backward()
        outs[impl], grads[impl] = y.detach(), xi.grad
    assert cosine(outs[name], outs["sdpa"]) >= 0.9999
    assert cosine(grads[name], grads["sdpa"]) >= 0.999
