"""CPU oracle for the four fused QLoRA ops (test infrastructure only).

This package restates, in plain PyTorch eager on the CPU, the arithmetic of the
reference's RMSNorm, SwiGLU, RoPE and chunked cross-entropy path. It is the
checker for the CUDA kernels in ``auspex_soup_demo_b200``: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import it. The
product path never calls into this package.

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own kernels
(``solution/kernels/*.py``, executed on the CPU by Triton's interpreter) on small
seeded inputs and stores their outputs under ``tests/golden/``;
``tests/test_oracle_golden.py`` checks every function here against them.
"""

from .ops import (  # noqa: F401
    IGNORE_INDEX,
    rmsnorm_fwd,
    rmsnorm_bwd,
    swiglu_fwd,
    swiglu_bwd,
    rope_fwd,
    rope_bwd,
    rope_cos_sin,
    ce_rows,
    chunked_ce,
)
