"""B200-native (sm_100a) fused ops for Qwen2.5 QLoRA training.

Drop-in for the reference solution package (``solution/__init__.py``): the same
``CONFIG`` toggles and ``apply()`` entry point, which installs the fused
chunked cross-entropy into Soup (when ``soup_cli`` is importable) and patches
transformers' Qwen2 RMSNorm, rotary embedding and MLP to the fused CUDA ops.

Unlike the reference, ``apply()`` first loads the compiled library and raises
if it is missing, and the patched modules do not fall back to eager PyTorch on
CUDA tensors: a failure is an error, never a silent slow path.
"""

import sys

from . import _lib
from .kernels.chunked_ce import patch_soup_chunked_loss
from .kernels.rmsnorm import patch_qwen2_rmsnorm
from .kernels.rope import patch_qwen2_rope
from .kernels.swiglu import patch_qwen2_mlp

CONFIG = {
    # 1. fused lm_head cross-entropy with loss / entropy / accuracy (chunk size for Soup)
    "chunked_ce": True,
    # 2. fused RMSNorm forward and backward
    "rmsnorm": True,
    # 3. fused RoPE (Q and K in one launch)
    "rope": True,
    # 4. fused SwiGLU with selective recompute of gate/up
    "swiglu": True,
}


def apply():
    """Install the patches selected in CONFIG (reference: ``solution/__init__.py:42-70``)."""
    _lib.lib()  # fail loudly when the CUDA library is absent
    steps = [
        ("chunked_ce", "Chunked Loss", lambda: patch_soup_chunked_loss(chunk_size=64)),
        ("rmsnorm", "RMSNorm", patch_qwen2_rmsnorm),
        ("rope", "RoPE", patch_qwen2_rope),
        ("swiglu", "SwiGLU", patch_qwen2_mlp),
    ]
    for key, label, fn in steps:
        if CONFIG.get(key):
            try:
                fn()
            except Exception as exc:  # same reporting as the reference
                print(f"[SOUP-B200] Warning: failed to patch {label}: {exc}", file=sys.stderr)
