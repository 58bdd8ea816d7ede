"""Fused SwiGLU forward and recompute-backward on B200 (sm_100a CUDA via the C ABI).

Drop-in for the reference's ``solution/kernels/swiglu.py``: ``FastSwiGLUFunction``,
``fast_swiglu``, ``patch_qwen2_mlp`` and the kernel handles
``_custom_swiglu_fwd_kernel`` / ``_custom_swiglu_bwd_kernel``; arithmetic of
``swiglu.py:20-95`` (sigmoid recomputed from the saved gate in backward).
The MLP patch keeps the reference's selective recompute: gate/up projections
and SwiGLU run under ``torch.utils.checkpoint``, ``down_proj`` outside it
(``swiglu.py:173-221``).
"""

from __future__ import annotations

import torch
import torch.utils.checkpoint

from .. import _lib
from ._shim import LaunchShim


def _rows(t: torch.Tensor, n: int) -> torch.Tensor:
    t2 = t.reshape(-1, n)
    if t2.stride(-1) != 1:
        t2 = t2.contiguous()
    return t2


def swiglu_forward(g2: torch.Tensor, u2: torch.Tensor, out=None) -> torch.Tensor:
    rows, n = g2.shape
    if out is None:
        out = torch.empty((rows, n), dtype=g2.dtype, device=g2.device)
    _lib.call("soup_swiglu_fwd", g2.device, g2.data_ptr(), g2.stride(0), u2.data_ptr(), u2.stride(0),
              out.data_ptr(), out.stride(0), rows, n, _lib.dtype_code(g2.dtype), _lib.stream_of(g2))
    return out


def swiglu_backward(dy2, g2, u2, dg=None, du=None):
    rows, n = g2.shape
    if dg is None:
        dg = torch.empty((rows, n), dtype=g2.dtype, device=g2.device)
    if du is None:
        du = torch.empty((rows, n), dtype=u2.dtype, device=u2.device)
    _lib.call("soup_swiglu_bwd", g2.device, dy2.data_ptr(), dy2.stride(0), g2.data_ptr(),
              g2.stride(0), u2.data_ptr(), u2.stride(0), dg.data_ptr(), dg.stride(0), du.data_ptr(),
              du.stride(0), rows, n, _lib.dtype_code(g2.dtype), _lib.stream_of(g2))
    return dg, du


class FastSwiGLUFunction(torch.autograd.Function):
    """SwiGLU autograd Function (reference: ``swiglu.py:98-165``)."""

    @staticmethod
    def forward(ctx, gate: torch.Tensor, up: torch.Tensor):
        if up.dtype != gate.dtype:
            raise TypeError(f"gate and up dtypes differ: {gate.dtype} vs {up.dtype}")
        orig_shape = gate.shape
        n = orig_shape[-1]
        g2 = _rows(gate, n)
        u2 = _rows(up, n)
        out = swiglu_forward(g2, u2)
        ctx.save_for_backward(g2, u2)
        ctx.orig_shape = orig_shape
        return out.view(orig_shape)

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        g2, u2 = ctx.saved_tensors
        n = g2.shape[1]
        dy2 = _rows(grad_output, n)
        if dy2.dtype != g2.dtype:
            dy2 = dy2.to(g2.dtype)
        dg, du = swiglu_backward(dy2, g2, u2)
        return dg.view(ctx.orig_shape), du.view(ctx.orig_shape)


def fast_swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up (reference: ``swiglu.py:168-170``)."""
    return FastSwiGLUFunction.apply(gate, up)


#: Recompute gate/up + SwiGLU in backward (the reference's selective recompute,
#: ``swiglu.py:197-214``). False keeps the activations instead: more memory
#: (2 x tokens x intermediate bf16 per layer), no second gate/up GEMM pass.
RECOMPUTE = True


def patch_qwen2_mlp():
    """Route ``Qwen2MLP.forward`` on CUDA tensors through the fused SwiGLU.

    Training with grad: gate/up projections + SwiGLU are checkpointed and
    recomputed in backward, ``down_proj`` stays outside the checkpoint
    (``swiglu.py:197-214``). Eval / no-grad: direct call. CPU tensors and
    non-SiLU activations keep the original forward. Errors on CUDA tensors
    propagate (the reference falls back to eager silently).
    """
    try:
        from transformers.models.qwen2 import modeling_qwen2
    except ImportError:
        return
    cls = modeling_qwen2.Qwen2MLP
    if getattr(cls.forward, "_soup_b200", False):
        return
    original_forward = cls.forward

    def forward(self, x):
        act = getattr(getattr(self, "config", None), "hidden_act", "silu")
        if act != "silu" or not x.is_cuda:
            return original_forward(self, x)
        recompute = (RECOMPUTE and self.training and torch.is_grad_enabled()
                     and getattr(x, "requires_grad", False))
        group = getattr(self.gate_proj, "lora_group", None)
        if (group is not None and group.kind == "gate_up" and group.members[0] is self.gate_proj
                and group.members[1] is self.up_proj and group.usable(x)):
            # gate/up as one GEMM feeding the fused SwiGLU; same recompute policy
            # (without recompute the SwiGLU backward joins down_proj's dX GEMM)
            return group.mlp(x, self.down_proj, recompute)
        if not recompute:
            return self.down_proj(fast_swiglu(self.gate_proj(x), self.up_proj(x)))

        def _swiglu_forward(hidden_states):
            return fast_swiglu(self.gate_proj(hidden_states), self.up_proj(hidden_states))

        # the recomputed region has no random ops: skip the RNG state save/restore,
        # which also keeps the step capturable in a CUDA graph
        swiglu_out = torch.utils.checkpoint.checkpoint(_swiglu_forward, x, use_reentrant=False,
                                                       preserve_rng_state=False)
        return self.down_proj(swiglu_out)

    forward._soup_b200 = True
    forward._soup_original = original_forward
    cls.forward = forward


# ---- kernel handles with the reference's launch signatures ---------------------
def _launch_fwd(gate_ptr, up_ptr, out_ptr, stride_g_row, stride_u_row, stride_o_row, N_cols,
                **_triton_only):
    rows = gate_ptr.numel() // max(int(N_cols), 1) if gate_ptr.dim() < 2 else gate_ptr.shape[0]
    _lib.call("soup_swiglu_fwd", gate_ptr.device, gate_ptr.data_ptr(), int(stride_g_row),
              up_ptr.data_ptr(), int(stride_u_row), out_ptr.data_ptr(), int(stride_o_row), rows,
              int(N_cols), _lib.dtype_code(gate_ptr.dtype), _lib.stream_of(gate_ptr))


def _launch_bwd(grad_ptr, gate_ptr, up_ptr, dgate_ptr, dup_ptr, stride_grad_row, stride_g_row,
                stride_u_row, stride_dg_row, stride_du_row, N_cols, **_triton_only):
    rows = gate_ptr.numel() // max(int(N_cols), 1) if gate_ptr.dim() < 2 else gate_ptr.shape[0]
    _lib.call("soup_swiglu_bwd", gate_ptr.device, grad_ptr.data_ptr(), int(stride_grad_row),
              gate_ptr.data_ptr(), int(stride_g_row), up_ptr.data_ptr(), int(stride_u_row),
              dgate_ptr.data_ptr(), int(stride_dg_row), dup_ptr.data_ptr(), int(stride_du_row),
              rows, int(N_cols), _lib.dtype_code(gate_ptr.dtype), _lib.stream_of(gate_ptr))


_custom_swiglu_fwd_kernel = LaunchShim(
    "_custom_swiglu_fwd_kernel",
    ["gate_ptr", "up_ptr", "out_ptr", "stride_g_row", "stride_u_row", "stride_o_row", "N_cols"],
    _launch_fwd)
_custom_swiglu_bwd_kernel = LaunchShim(
    "_custom_swiglu_bwd_kernel",
    ["grad_ptr", "gate_ptr", "up_ptr", "dgate_ptr", "dup_ptr", "stride_grad_row", "stride_g_row",
     "stride_u_row", "stride_dg_row", "stride_du_row", "N_cols"],
    _launch_bwd)
