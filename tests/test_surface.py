"""CPU checks of the drop-in surface: names, launch-handle argument binding,
patch installation, and CPU tensors keeping the original transformers code."""

import pytest
import torch

import auspex_soup_demo_b200 as pkg
from auspex_soup_demo_b200 import kernels
from auspex_soup_demo_b200.kernels._shim import LaunchShim

# The export list of the reference's solution/kernels/__init__.py:3-51.
REFERENCE_EXPORTS = [
    "_chunked_cross_entropy_fused_kernel", "chunk_cross_entropy_triton",
    "make_triton_chunked_loss_function", "patch_soup_chunked_loss",
    "_rms_norm_fwd_kernel", "_rms_norm_bwd_dx_kernel", "FastRMSNormFunction", "fast_rms_norm",
    "patch_qwen2_rmsnorm", "_fused_rope_2d_fwd_kernel", "_fused_rope_2d_bwd_kernel",
    "FastRoPEFunction", "apply_fast_rope", "patch_qwen2_rope", "_custom_swiglu_fwd_kernel",
    "_custom_swiglu_bwd_kernel", "FastSwiGLUFunction", "fast_swiglu", "patch_qwen2_mlp",
]


def test_reference_exports_present():
    for name in REFERENCE_EXPORTS:
        assert hasattr(kernels, name), name
        assert name in kernels.__all__


def test_config_and_apply_match_reference_shape():
    assert set(pkg.CONFIG) == {"chunked_ce", "rmsnorm", "rope", "swiglu"}
    assert callable(pkg.apply)


def test_launch_shim_binds_reference_arguments():
    seen = {}

    def launch(a, b, c, **extra):
        seen.update(a=a, b=b, c=c, extra=extra)

    k = LaunchShim("k", ["a", "b", "c"], launch)
    k[(4,)](1, 2, c=3, BLOCK_V=4096, num_warps=8, num_stages=2)
    assert seen["a"] == 1 and seen["b"] == 2 and seen["c"] == 3
    assert seen["extra"] == {"BLOCK_V": 4096, "num_warps": 8, "num_stages": 2}
    with pytest.raises(TypeError):
        k[(1,)](1, 2)
    with pytest.raises(TypeError):
        k[(1,)](1, 2, 3, 4)
    with pytest.raises(TypeError):
        k[(1,)](1, 2, 3, a=5)


def test_apply_patches_and_cpu_tensors_keep_original_code():
    from transformers.models.qwen2 import modeling_qwen2 as m
    from transformers import Qwen2Config

    cfg = Qwen2Config(hidden_size=64, intermediate_size=128, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=16, vocab_size=100, num_hidden_layers=1)
    torch.manual_seed(0)
    norm = m.Qwen2RMSNorm(64, eps=1e-6)
    mlp = m.Qwen2MLP(cfg)
    x = torch.randn(2, 5, 64)
    ref_norm = norm(x)
    ref_mlp = mlp(x)
    q = torch.randn(2, 4, 5, 16)
    k = torch.randn(2, 2, 5, 16)
    cos = torch.randn(2, 5, 16)
    sin = torch.randn(2, 5, 16)
    ref_q, ref_k = m.apply_rotary_pos_emb(q, k, cos, sin)
    pkg.apply()
    assert getattr(m.Qwen2RMSNorm.forward, "_soup_b200", False)
    assert getattr(m.Qwen2MLP.forward, "_soup_b200", False)
    assert getattr(m.apply_rotary_pos_emb, "_soup_b200", False)
    pkg.apply()  # idempotent
    assert m.Qwen2RMSNorm.forward._soup_original is not m.Qwen2RMSNorm.forward
    torch.testing.assert_close(norm(x), ref_norm)
    torch.testing.assert_close(mlp(x), ref_mlp)
    q2, k2 = m.apply_rotary_pos_emb(q, k, cos, sin)
    torch.testing.assert_close(q2, ref_q)
    torch.testing.assert_close(k2, ref_k)


def test_extract_head_weight_lookup_order():
    from auspex_soup_demo_b200.kernels.chunked_ce import _extract_head_weight

    lin = torch.nn.Linear(4, 3, bias=False)
    assert _extract_head_weight(lin) is lin.weight

    class M(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.head = torch.nn.Linear(4, 3, bias=False)

        def get_output_embeddings(self):
            return self.head

        def project(self, h):
            return self.head(h)

    mm = M()
    assert _extract_head_weight(mm.project) is mm.head.weight

    def closure_head(h, _m=mm):
        return _m.head(h)

    def make():
        model = mm

        def head(h):
            return model.head(h)

        return head

    assert _extract_head_weight(make()) is mm.head.weight
    assert _extract_head_weight(lambda h: h) is None


def test_fused_ops_refuse_cpu_tensors():
    from auspex_soup_demo_b200.kernels.chunked_ce import fused_linear_cross_entropy

    with pytest.raises(RuntimeError):
        fused_linear_cross_entropy(torch.zeros(4, 8), torch.zeros(16, 8), torch.zeros(4, dtype=torch.long))
