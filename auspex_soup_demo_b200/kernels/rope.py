"""Fused rotate-half RoPE on B200 (sm_100a CUDA via the C ABI).

Drop-in for the reference's ``solution/kernels/rope.py``: ``FastRoPEFunction``
(one [B, H, S, D] tensor, any b/h/s strides, last dim contiguous),
``apply_fast_rope``, ``patch_qwen2_rope`` and the kernel handles
``_fused_rope_2d_fwd_kernel`` / ``_fused_rope_2d_bwd_kernel``. The arithmetic is
``rope.py:20-117``. The Qwen2 patch rotates Q and K in ONE launch
(:class:`FastRoPEQKFunction`) where the reference launches twice
(``rope.py:217-218``).
"""

from __future__ import annotations

import torch

from .. import _lib
from ._shim import LaunchShim


def _cos_view(cos: torch.Tensor, sin: torch.Tensor, x: torch.Tensor):
    """Return (cos, sin, stride_b, stride_s) as the kernel indexes them.

    Accepts [B|1, 1, S, D] and [B|1, S, D] (reference ``rope.py:132-133``) and
    [S, D]. cos/sin must share strides; dtype is x's dtype or fp32.
    """
    if cos.dtype not in (x.dtype, torch.float32):
        cos = cos.to(x.dtype)
        sin = sin.to(x.dtype)
    if sin.dtype != cos.dtype:
        sin = sin.to(cos.dtype)
    if cos.stride(-1) != 1 or sin.stride() != cos.stride():
        cos = cos.contiguous()
        sin = sin.contiguous()
    if cos.dim() == 4:
        sb = cos.stride(0) if cos.shape[0] > 1 else 0
        ss = cos.stride(2)
    elif cos.dim() == 3:
        sb = cos.stride(0) if cos.shape[0] > 1 else 0
        ss = cos.stride(1)
    elif cos.dim() == 2:
        sb, ss = 0, cos.stride(0)
    else:
        raise ValueError(f"cos/sin must be 2-D, 3-D or 4-D, got shape {tuple(cos.shape)}")
    return cos, sin, sb, ss


def rope_tables(seq_len: int, head_dim: int, theta: float, dtype=torch.bfloat16, device=None):
    """cos/sin [S, D] for positions 0..S-1 as transformers' Qwen2 rotary embedding
    builds them: fp32 inverse frequencies and angles, ``cat(freqs, freqs)``, cast
    to the activation dtype."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64, device=device).float()
                           / head_dim))
    freqs = torch.arange(seq_len, device=device).float()[:, None] * inv[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def _check_x(x: torch.Tensor):
    if x.dim() != 4:
        raise ValueError(f"RoPE input must be [B, H, S, D], got {tuple(x.shape)}")
    if x.shape[-1] % 2:
        raise ValueError("head_dim must be even")
    if x.stride(-1) != 1:
        raise ValueError("RoPE input must have a contiguous last dimension")


def rope_apply(q, k, cos, sin, inverse: bool, q_out=None, k_out=None):
    """Rotate q (and k, if given) in one launch; returns (q_out, k_out)."""
    _check_x(q)
    B, Hq, S, D = q.shape
    if k is not None:
        _check_x(k)
        if k.shape[0] != B or k.shape[2] != S or k.shape[3] != D or k.dtype != q.dtype:
            raise ValueError("q and k must share batch, seq, head_dim and dtype")
    cos, sin, sb, ss = _cos_view(cos, sin, q)
    if q_out is None:
        q_out = torch.empty_like(q)
    if k is not None and k_out is None:
        k_out = torch.empty_like(k)
    qs = _lib.i64_array([q.stride(0), q.stride(1), q.stride(2)])
    qos = _lib.i64_array([q_out.stride(0), q_out.stride(1), q_out.stride(2)])
    if k is not None:
        ks = _lib.i64_array([k.stride(0), k.stride(1), k.stride(2)])
        kos = _lib.i64_array([k_out.stride(0), k_out.stride(1), k_out.stride(2)])
        hk = k.shape[1]
    else:
        ks = kos = None
        hk = 0
    _lib.call("soup_rope", q.device, q.data_ptr(), qs, q_out.data_ptr(), qos, Hq, _lib.ptr(k), ks,
              _lib.ptr(k_out), kos, hk, cos.data_ptr(), sin.data_ptr(), sb, ss, B, S, D,
              _lib.dtype_code(q.dtype), _lib.dtype_code(cos.dtype), 1 if inverse else 0,
              _lib.stream_of(q))
    return q_out, k_out


class FastRoPEFunction(torch.autograd.Function):
    """RoPE on one [B, H, S, D] tensor (reference: ``rope.py:120-191``)."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
        out, _ = rope_apply(x, None, cos, sin, inverse=False)
        ctx.save_for_backward(cos, sin)
        return out

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        cos, sin = ctx.saved_tensors
        g = grad_output if grad_output.stride(-1) == 1 else grad_output.contiguous()
        dx, _ = rope_apply(g, None, cos, sin, inverse=True)
        return dx, None, None


class FastRoPEQKFunction(torch.autograd.Function):
    """RoPE on Q and K together: one launch forward, one launch backward."""

    @staticmethod
    def forward(ctx, q, k, cos, sin):
        q_out, k_out = rope_apply(q, k, cos, sin, inverse=False)
        ctx.save_for_backward(cos, sin)
        ctx.meta = ((q.shape, q.dtype, q.device), (k.shape, k.dtype, k.device))
        return q_out, k_out

    @staticmethod
    def backward(ctx, dq, dk):
        cos, sin = ctx.saved_tensors
        (qs, qd, qdev), (ks, kd, kdev) = ctx.meta
        if dq is None:
            dq = torch.zeros(qs, dtype=qd, device=qdev)
        if dk is None:
            dk = torch.zeros(ks, dtype=kd, device=kdev)
        dq = dq if dq.stride(-1) == 1 else dq.contiguous()
        dk = dk if dk.stride(-1) == 1 else dk.contiguous()
        gq, gk = rope_apply(dq, dk, cos, sin, inverse=True)
        return gq, gk, None, None


def apply_fast_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate one tensor (reference: ``rope.py:194-196``)."""
    return FastRoPEFunction.apply(x, cos, sin)


def apply_fast_rope_qk(q, k, cos, sin):
    """Rotate Q and K in one fused launch."""
    return FastRoPEQKFunction.apply(q, k, cos, sin)


def patch_qwen2_rope():
    """Route ``modeling_qwen2.apply_rotary_pos_emb`` on CUDA tensors to the fused op.

    Mirrors ``rope.py:199-223``: cos/sin [B, S, D] are unsqueezed at dim 1;
    Q and K are rotated in one launch. CPU tensors use the original function.
    """
    try:
        from transformers.models.qwen2 import modeling_qwen2
    except ImportError:
        return
    if getattr(modeling_qwen2.apply_rotary_pos_emb, "_soup_b200", False):
        return
    original_apply_rotary = modeling_qwen2.apply_rotary_pos_emb

    def apply_rotary_pos_emb_patched(q, k, cos, sin, position_ids=None, unsqueeze_dim=1):
        if not q.is_cuda:
            return original_apply_rotary(q, k, cos, sin, unsqueeze_dim=unsqueeze_dim)
        if cos.dim() == 3 and unsqueeze_dim == 1:
            cos = cos.unsqueeze(1)
            sin = sin.unsqueeze(1)
        return apply_fast_rope_qk(q, k, cos, sin)

    apply_rotary_pos_emb_patched._soup_b200 = True
    apply_rotary_pos_emb_patched._soup_original = original_apply_rotary
    modeling_qwen2.apply_rotary_pos_emb = apply_rotary_pos_emb_patched


# ---- kernel handles with the reference's launch signatures ---------------------
def _launch(inverse, x_ptr, cos_ptr, sin_ptr, out_ptr, s_xb, s_xh, s_xs, stride_cb, stride_cs, s_ob,
            s_oh, s_os, H, S, HALF_DIM, grid_bh):
    B = grid_bh // int(H)
    xs = _lib.i64_array([int(s_xb), int(s_xh), int(s_xs)])
    os_ = _lib.i64_array([int(s_ob), int(s_oh), int(s_os)])
    _lib.call("soup_rope", x_ptr.device, x_ptr.data_ptr(), xs, out_ptr.data_ptr(), os_, int(H), 0,
              None, 0, None, 0, cos_ptr.data_ptr(), sin_ptr.data_ptr(), int(stride_cb),
              int(stride_cs), B, int(S), 2 * int(HALF_DIM), _lib.dtype_code(x_ptr.dtype),
              _lib.dtype_code(cos_ptr.dtype), 1 if inverse else 0, _lib.stream_of(x_ptr))


class _RopeShim(LaunchShim):
    def __getitem__(self, grid):
        inner = super().__getitem__(grid)

        def run(*args, **kwargs):
            kwargs["_grid_bh"] = int(grid[0])
            return inner(*args, **kwargs)

        return run


def _fwd(x_ptr, cos_ptr, sin_ptr, out_ptr, stride_xb, stride_xh, stride_xs, stride_cb, stride_cs,
         stride_ob, stride_oh, stride_os, H, S, HALF_DIM, _grid_bh, **_triton_only):
    _launch(False, x_ptr, cos_ptr, sin_ptr, out_ptr, stride_xb, stride_xh, stride_xs, stride_cb,
            stride_cs, stride_ob, stride_oh, stride_os, H, S, HALF_DIM, _grid_bh)


def _bwd(grad_ptr, cos_ptr, sin_ptr, dx_ptr, stride_gb, stride_gh, stride_gs, stride_cb, stride_cs,
         stride_dxb, stride_dxh, stride_dxs, H, S, HALF_DIM, _grid_bh, **_triton_only):
    _launch(True, grad_ptr, cos_ptr, sin_ptr, dx_ptr, stride_gb, stride_gh, stride_gs, stride_cb,
            stride_cs, stride_dxb, stride_dxh, stride_dxs, H, S, HALF_DIM, _grid_bh)


_fused_rope_2d_fwd_kernel = _RopeShim(
    "_fused_rope_2d_fwd_kernel",
    ["x_ptr", "cos_ptr", "sin_ptr", "out_ptr", "stride_xb", "stride_xh", "stride_xs", "stride_cb",
     "stride_cs", "stride_ob", "stride_oh", "stride_os", "H", "S", "HALF_DIM"],
    _fwd)
_fused_rope_2d_bwd_kernel = _RopeShim(
    "_fused_rope_2d_bwd_kernel",
    ["grad_ptr", "cos_ptr", "sin_ptr", "dx_ptr", "stride_gb", "stride_gh", "stride_gs", "stride_cb",
     "stride_cs", "stride_dxb", "stride_dxh", "stride_dxs", "H", "S", "HALF_DIM"],
    _bwd)
