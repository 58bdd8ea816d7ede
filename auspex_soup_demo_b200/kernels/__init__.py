"""sm_100a fused ops behind the reference's kernel-package names.

Mirrors the export list of the reference's ``solution/kernels/__init__.py:3-51``.
"""

from .chunked_ce import (
    _chunked_cross_entropy_fused_kernel,
    chunk_cross_entropy_triton,
    make_triton_chunked_loss_function,
    patch_soup_chunked_loss,
    fused_linear_cross_entropy,
)
from .rmsnorm import (
    _rms_norm_fwd_kernel,
    _rms_norm_bwd_dx_kernel,
    FastRMSNormFunction,
    fast_rms_norm,
    patch_qwen2_rmsnorm,
)
from .rope import (
    _fused_rope_2d_fwd_kernel,
    _fused_rope_2d_bwd_kernel,
    FastRoPEFunction,
    FastRoPEQKFunction,
    apply_fast_rope,
    apply_fast_rope_qk,
    patch_qwen2_rope,
)
from .swiglu import (
    _custom_swiglu_fwd_kernel,
    _custom_swiglu_bwd_kernel,
    FastSwiGLUFunction,
    fast_swiglu,
    patch_qwen2_mlp,
)

__all__ = [
    "_chunked_cross_entropy_fused_kernel",
    "chunk_cross_entropy_triton",
    "make_triton_chunked_loss_function",
    "patch_soup_chunked_loss",
    "fused_linear_cross_entropy",
    "_rms_norm_fwd_kernel",
    "_rms_norm_bwd_dx_kernel",
    "FastRMSNormFunction",
    "fast_rms_norm",
    "patch_qwen2_rmsnorm",
    "_fused_rope_2d_fwd_kernel",
    "_fused_rope_2d_bwd_kernel",
    "FastRoPEFunction",
    "FastRoPEQKFunction",
    "apply_fast_rope",
    "apply_fast_rope_qk",
    "patch_qwen2_rope",
    "_custom_swiglu_fwd_kernel",
    "_custom_swiglu_bwd_kernel",
    "FastSwiGLUFunction",
    "fast_swiglu",
    "patch_qwen2_mlp",
]
