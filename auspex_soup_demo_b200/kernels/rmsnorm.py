"""Fused RMSNorm forward and backward on B200 (sm_100a CUDA via the C ABI).

Drop-in for the reference's ``solution/kernels/rmsnorm.py``: same public names
(``FastRMSNormFunction``, ``fast_rms_norm``, ``patch_qwen2_rmsnorm`` and the
kernel handles ``_rms_norm_fwd_kernel`` / ``_rms_norm_bwd_dx_kernel``) and the
same arithmetic (``rmsnorm.py:22-96``). The backward computes dx and, when the
weight needs a gradient, dw in the same pass (the reference runs dw as eager
PyTorch, ``rmsnorm.py:161-167``); the dw reduction is deterministic.
"""

from __future__ import annotations

import torch

from .. import _lib
from ._shim import LaunchShim


def _rows_view(t: torch.Tensor, d: int) -> torch.Tensor:
    """[..., d] -> [rows, d] without a copy when the last dim is contiguous."""
    t2 = t.reshape(-1, d)
    if t2.stride(-1) != 1:
        t2 = t2.contiguous()
    return t2


def rmsnorm_forward(x2: torch.Tensor, weight: torch.Tensor, eps: float, out=None, rstd=None):
    rows, d = x2.shape
    if out is None:
        out = torch.empty((rows, d), dtype=x2.dtype, device=x2.device)
    if rstd is None:
        rstd = torch.empty(rows, dtype=torch.float32, device=x2.device)
    _lib.call("soup_rmsnorm_fwd", x2.device, x2.data_ptr(), x2.stride(0), weight.data_ptr(),
              out.data_ptr(), out.stride(0), rstd.data_ptr(), rows, d, float(eps),
              _lib.dtype_code(x2.dtype), _lib.dtype_code(weight.dtype), _lib.stream_of(x2))
    return out, rstd


def rmsnorm_backward(dy2: torch.Tensor, x2: torch.Tensor, weight: torch.Tensor, rstd: torch.Tensor,
                     need_dw: bool, dx=None):
    rows, d = x2.shape
    if dx is None:
        dx = torch.empty((rows, d), dtype=x2.dtype, device=x2.device)
    dw = None
    ws, ws_bytes = 0, 0
    if need_dw:
        dw = torch.empty(d, dtype=weight.dtype, device=weight.device)
        ws_bytes = _lib.lib().soup_rmsnorm_bwd_workspace_bytes(rows, d)
        ws = _lib.scratch(x2.device, ws_bytes).data_ptr()
    _lib.call("soup_rmsnorm_bwd", x2.device, dy2.data_ptr(), dy2.stride(0), x2.data_ptr(),
              x2.stride(0), weight.data_ptr(), rstd.data_ptr(), dx.data_ptr(), dx.stride(0),
              _lib.ptr(dw), ws, ws_bytes, rows, d, _lib.dtype_code(x2.dtype),
              _lib.dtype_code(weight.dtype), _lib.stream_of(x2))
    return dx, dw


class FastRMSNormFunction(torch.autograd.Function):
    """RMSNorm autograd Function (reference: ``rmsnorm.py:99-169``)."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6):
        orig_shape = x.shape
        d = orig_shape[-1]
        x2 = _rows_view(x, d)
        weight = weight.contiguous()
        out, rstd = rmsnorm_forward(x2, weight, eps)
        ctx.save_for_backward(x2, weight, rstd)
        ctx.eps = eps
        ctx.orig_shape = orig_shape
        return out.view(orig_shape)

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        x2, weight, rstd = ctx.saved_tensors
        d = x2.shape[1]
        dy2 = _rows_view(grad_output, d)
        if dy2.dtype != x2.dtype:
            dy2 = dy2.to(x2.dtype)
        dx, dw = rmsnorm_backward(dy2, x2, weight, rstd, need_dw=ctx.needs_input_grad[1])
        return dx.view(ctx.orig_shape), dw, None


def fast_rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """Entry point for the fused RMSNorm (reference: ``rmsnorm.py:172-174``)."""
    return FastRMSNormFunction.apply(x, weight, eps)


def patch_qwen2_rmsnorm():
    """Route ``Qwen2RMSNorm.forward`` on CUDA tensors to :func:`fast_rms_norm`.

    Mirrors ``rmsnorm.py:177-194``. CPU tensors keep the original forward.
    Unlike the reference, errors on CUDA tensors propagate instead of
    silently falling back to the eager module.
    """
    try:
        from transformers.models.qwen2 import modeling_qwen2
    except ImportError:
        return
    cls = modeling_qwen2.Qwen2RMSNorm
    if getattr(cls.forward, "_soup_b200", False):
        return
    original_forward = cls.forward

    def forward(self, hidden_states):
        if not hidden_states.is_cuda or self.weight is None or not self.weight.is_cuda:
            return original_forward(self, hidden_states)
        return fast_rms_norm(hidden_states, self.weight, self.variance_epsilon)

    forward._soup_b200 = True
    forward._soup_original = original_forward
    cls.forward = forward


# ---- kernel handles with the reference's launch signatures ---------------------
def _launch_fwd(x_ptr, weight_ptr, out_ptr, rstd_ptr, stride_x_row, stride_out_row, D, eps,
                **_triton_only):
    rows = rstd_ptr.numel()
    _lib.call("soup_rmsnorm_fwd", x_ptr.device, x_ptr.data_ptr(), int(stride_x_row),
              weight_ptr.data_ptr(), out_ptr.data_ptr(), int(stride_out_row), rstd_ptr.data_ptr(),
              rows, int(D), float(eps), _lib.dtype_code(x_ptr.dtype),
              _lib.dtype_code(weight_ptr.dtype), _lib.stream_of(x_ptr))


def _launch_bwd_dx(grad_ptr, x_ptr, weight_ptr, rstd_ptr, dx_ptr, stride_grad_row, stride_x_row,
                   stride_dx_row, D, **_triton_only):
    rows = rstd_ptr.numel()
    _lib.call("soup_rmsnorm_bwd", x_ptr.device, grad_ptr.data_ptr(), int(stride_grad_row),
              x_ptr.data_ptr(), int(stride_x_row), weight_ptr.data_ptr(), rstd_ptr.data_ptr(),
              dx_ptr.data_ptr(), int(stride_dx_row), 0, 0, 0, rows, int(D),
              _lib.dtype_code(x_ptr.dtype), _lib.dtype_code(weight_ptr.dtype),
              _lib.stream_of(x_ptr))


_rms_norm_fwd_kernel = LaunchShim(
    "_rms_norm_fwd_kernel",
    ["x_ptr", "weight_ptr", "out_ptr", "rstd_ptr", "stride_x_row", "stride_out_row", "D", "eps"],
    _launch_fwd)
_rms_norm_bwd_dx_kernel = LaunchShim(
    "_rms_norm_bwd_dx_kernel",
    ["grad_ptr", "x_ptr", "weight_ptr", "rstd_ptr", "dx_ptr", "stride_grad_row", "stride_x_row",
     "stride_dx_row", "D"],
    _launch_bwd_dx)
