"""Causal grouped-query flash attention on B200 (tcgen05 kernels via the C ABI).

No counterpart kernel in the reference: its Qwen2 attention runs through torch's
``scaled_dot_product_attention`` (transformers' ``sdpa_attention_forward``,
called from ``Qwen2Attention.forward``). This module provides the same call for
the QLoRA step:

* :func:`attention_forward` / :class:`FlashAttentionFunction` - q [B, H, S, 128],
  k / v [B, Hk, S, 128] bf16 with any b / h / s strides (transformers' transposed
  [B, S, H, D] projections are read in place) -> out [B, S, H, 128] bf16 (the
  layout the o_proj consumes, no transpose copy) and the row log-sum-exp for
  the backward;
* :func:`soup_attention` - an attention function with transformers'
  ``AttentionInterface`` signature, registered under the name ``"soup_b200"``
  by :func:`register`. Calls the kernels have no form for (an attention mask,
  dropout, a head dim other than 128, non-bf16 or CPU tensors) go to
  transformers' SDPA function unchanged.
"""

from __future__ import annotations

import torch

from .. import _lib

HEAD_DIM = 128
INTERFACE_NAME = "soup_b200"


def _strides(t: torch.Tensor):
    return _lib.i64_array([t.stride(0), t.stride(1), t.stride(2)])


def _check(q, k, v):
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("attention: q, k, v must be [B, heads, S, D]")
    B, H, S, D = q.shape
    if k.shape != v.shape or k.shape[0] != B or k.shape[2] != S or k.shape[3] != D:
        raise ValueError(f"attention: shapes q {tuple(q.shape)} k {tuple(k.shape)} v {tuple(v.shape)}")
    if H % k.shape[1]:
        raise ValueError("attention: query heads must be a multiple of the KV heads")
    for t in (q, k, v):
        if t.dtype != torch.bfloat16 or not t.is_cuda or t.stride(-1) != 1:
            raise ValueError("attention: q, k, v must be bf16 CUDA tensors with a contiguous last dim")
    return B, H, k.shape[1], S, D


def _s_pad(S: int) -> int:
    return -(-S // 128) * 128


def attention_forward(q, k, v, scale: float, causal: bool = True):
    """(out [B, S, H, D] bf16, lse [B, H, S] fp32) of softmax(scale q k^T) v.

    lse is a view of a [B, H, S rounded up to 128] buffer (the layout the
    backward reads)."""
    B, H, Hk, S, D = _check(q, k, v)
    out = torch.empty(B, S, H, D, dtype=torch.bfloat16, device=q.device)
    lse = torch.empty(B, H, _s_pad(S), dtype=torch.float32, device=q.device)
    _lib.call("soup_attention_fwd", q.device, q.data_ptr(), _strides(q), k.data_ptr(), _strides(k),
              v.data_ptr(), _strides(v), B, H, Hk, S, D, float(scale), int(bool(causal)),
              out.data_ptr(), lse.data_ptr(), _lib.stream_of(q))
    return out, lse[..., :S]


def attention_backward(q, k, v, out, lse, dout, scale: float, causal: bool = True):
    """(dq [B, H, S, D], dk, dv [B, Hk, S, D]) as transposed views of contiguous
    [B, S, heads, D] buffers; lse as returned by :func:`attention_forward`."""
    B, H, Hk, S, D = _check(q, k, v)
    if dout.shape != (B, S, H, D):
        raise ValueError(f"attention: dout must be [B, S, H, D], got {tuple(dout.shape)}")
    dout = dout.to(torch.bfloat16).contiguous()
    base = lse._base if lse._base is not None else lse
    if base.shape != (B, H, _s_pad(S)) or base.dtype != torch.float32 or not base.is_contiguous():
        raise ValueError("attention: lse must come from attention_forward")
    dq = torch.empty(B, S, H, D, dtype=torch.bfloat16, device=q.device)
    dk = torch.empty(B, S, Hk, D, dtype=torch.bfloat16, device=q.device)
    dv = torch.empty(B, S, Hk, D, dtype=torch.bfloat16, device=q.device)
    nbytes = _lib.lib().soup_attention_bwd_workspace_bytes(B, H, S)
    ws = _lib.scratch(q.device, nbytes)
    _lib.call("soup_attention_bwd", q.device, q.data_ptr(), _strides(q), k.data_ptr(), _strides(k),
              v.data_ptr(), _strides(v), out.data_ptr(), dout.data_ptr(), base.data_ptr(), B, H, Hk,
              S, D, float(scale), int(bool(causal)), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
              ws.data_ptr(), nbytes, _lib.stream_of(q))
    return dq.transpose(1, 2), dk.transpose(1, 2), dv.transpose(1, 2)


class FlashAttentionFunction(torch.autograd.Function):
    """out [B, S, H, D] = attention(q, k, v) with the tcgen05 kernels; backward
    recomputes P from the saved log-sum-exp."""

    @staticmethod
    def forward(ctx, q, k, v, scale: float, causal: bool):
        out, lse = attention_forward(q, k, v, scale, causal)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.scale = scale
        ctx.causal = causal
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse = ctx.saved_tensors
        dq, dk, dv = attention_backward(q, k, v, out, lse, dout, ctx.scale, ctx.causal)
        return dq, dk, dv, None, None


def flash_attention(q, k, v, scale: float, causal: bool = True):
    return FlashAttentionFunction.apply(q, k, v, scale, causal)


def _supported(module, query, key, value, attention_mask, dropout) -> bool:
    return (attention_mask is None and not dropout and query.is_cuda
            and query.dtype == key.dtype == value.dtype == torch.bfloat16
            and query.shape[-1] == HEAD_DIM and query.stride(-1) == 1 and key.stride(-1) == 1
            and value.stride(-1) == 1 and query.shape[2] == key.shape[2]
            and all(t.stride(i) % 8 == 0 for t in (query, key, value) for i in range(3))
            and all(t.data_ptr() % 16 == 0 for t in (query, key, value)))


def soup_attention(module, query, key, value, attention_mask, dropout: float = 0.0,
                   scaling=None, is_causal=None, **kwargs):
    """transformers ``AttentionInterface`` function: (attn_output [B, S, H, D], None).

    Causal when the module is (and the query is longer than one token), as
    transformers' SDPA path decides (``integrations/sdpa_attention.py``). Calls
    outside the kernels' form go to transformers' SDPA function."""
    if not _supported(module, query, key, value, attention_mask, dropout):
        from transformers.integrations.sdpa_attention import sdpa_attention_forward

        return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout,
                                      scaling=scaling, is_causal=is_causal, **kwargs)
    causal = is_causal if is_causal is not None else getattr(module, "is_causal", True)
    causal = bool(causal) and query.shape[2] > 1
    scale = scaling if scaling is not None else query.shape[-1] ** -0.5
    return flash_attention(query, key, value, float(scale), causal), None


def register() -> str:
    """Register :func:`soup_attention` with transformers under ``INTERFACE_NAME``."""
    from transformers import AttentionInterface

    AttentionInterface.register(INTERFACE_NAME, soup_attention)
    return INTERFACE_NAME
