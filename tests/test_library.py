"""CPU checks of the C ABI: the library loads, exports every declared symbol,
validates arguments before touching the GPU, and sizes its workspaces."""

import ctypes
import os
import re

import pytest

from auspex_soup_demo_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "soupb200.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(soup_[a-z0-9_]+)\s*\(", text)))


def test_library_loads():
    lib = _lib.lib()
    assert lib.soup_version() >= 1


def test_every_declared_symbol_is_exported():
    lib = _lib.lib()
    names = declared_symbols()
    assert len(names) >= 12
    for name in names:
        assert hasattr(lib, name), f"{name} declared in soupb200.h but not exported"


def test_binding_covers_the_header():
    assert sorted(_lib.exported_symbols()) == declared_symbols()


def test_null_pointers_are_rejected_without_a_gpu():
    lib = _lib.lib()
    st = lib.soup_rmsnorm_fwd(None, 8, None, None, 8, None, 4, 8, 1e-6, 0, 0, None)
    assert st == _lib.SOUP_ERR_INVALID
    assert b"rmsnorm" in lib.soup_last_error()
    st = lib.soup_swiglu_fwd(None, 8, None, 8, None, 8, 4, 8, 2, None)
    assert st == _lib.SOUP_ERR_INVALID
    st = lib.soup_ce_rows(None, 8, None, None, None, None, 4, 8, 1.0, -100, 2, 1, None)
    assert st == _lib.SOUP_ERR_INVALID
    st = lib.soup_ce_linear(None, 8, None, 8, _lib.BF16, None, 0, None, 4, 8, 8, 1.0, -100, None,
                            None, None, None, None, _lib.BF16, None, 0, 0, None, 0, None)
    assert st == _lib.SOUP_ERR_INVALID
    st = lib.soup_gemm_bf16(None, 8, 0, None, 8, 0, None, 8, 0, 4, 4, 4, 1.0, 0, None)
    assert st == _lib.SOUP_ERR_INVALID
    strides = _lib.i64_array([1, 1, 1])
    st = lib.soup_rope(None, strides, None, strides, 1, None, None, None, None, 0, None, None, 0, 0,
                       1, 1, 128, 2, 2, 0, None)
    assert st == _lib.SOUP_ERR_INVALID


def test_bad_sizes_are_rejected():
    lib = _lib.lib()
    fake = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    # row stride smaller than the row
    st = lib.soup_rmsnorm_fwd(fake, 4, fake, fake, 8, fake, 4, 8, 1e-6, 0, 0, None)
    assert st == _lib.SOUP_ERR_INVALID
    # odd head_dim
    strides = _lib.i64_array([1, 1, 1])
    st = lib.soup_rope(fake, strides, fake, strides, 1, None, None, None, None, 0, fake, fake, 0, 0,
                       1, 1, 127, 2, 2, 0, None)
    assert st == _lib.SOUP_ERR_INVALID
    # unsupported dtype code
    st = lib.soup_swiglu_fwd(fake, 8, fake, 8, fake, 8, 0, 8, 7, None)
    assert st == _lib.SOUP_OK  # zero rows: nothing to do, accepted before dtype dispatch
    st = lib.soup_swiglu_fwd(fake, 8, fake, 8, fake, 8, 1, 8, 7, None)
    assert st == _lib.SOUP_ERR_INVALID


def test_workspace_sizes():
    lib = _lib.lib()
    n, v, d = 2048, 151936, 1536
    ws = lib.soup_ce_linear_workspace_bytes(n, v, d)
    logits = n * v * 2
    assert logits < ws < logits + 200 * 2 ** 20  # logits + partials + split-K slices
    assert lib.soup_ce_linear_workspace_bytes(0, v, d) == 0
    assert lib.soup_rmsnorm_bwd_workspace_bytes(2048, 1536) >= 1536 * 4
    # workspace grows linearly with rows
    assert lib.soup_ce_linear_workspace_bytes(4096, v, d) > 1.9 * ws


def test_dtype_codes():
    import torch
    assert _lib.dtype_code(torch.float32) == _lib.F32
    assert _lib.dtype_code(torch.float16) == _lib.F16
    assert _lib.dtype_code(torch.bfloat16) == _lib.BF16
    with pytest.raises(TypeError):
        _lib.dtype_code(torch.int32)


def test_ce_gradient_state_entry_points_validate_before_the_gpu():
    """The lm_head-gradient call and the vocab-parallel stages reject bad arguments
    (null pointers, bad dtype codes, a workspace smaller than their layout) before
    any launch."""
    lib = _lib.lib()
    fake = ctypes.c_void_p(16)  # 16-byte aligned, never dereferenced
    n, v, d = 4, 64, 8
    BF = _lib.BF16
    # soup_ce_linear_dweight(workspace, bytes, hidden, h_ld, in_dtype, rows, vocab, dim,
    #                        grad_scale, dweight, dw_dtype, accumulate, stream)
    st = lib.soup_ce_linear_dweight(None, 1 << 20, fake, d, BF, n, v, d, None, fake, _lib.F32, 0, None)
    assert st == _lib.SOUP_ERR_INVALID
    st = lib.soup_ce_linear_dweight(fake, 1 << 20, fake, d, BF, n, v, d, None, fake, 7, 0, None)
    assert st == _lib.SOUP_ERR_INVALID
    st = lib.soup_ce_linear_dweight(fake, 1 << 20, fake, d, _lib.F32, n, v, d, None, fake, _lib.F32,
                                    0, None)
    assert st == _lib.SOUP_ERR_INVALID  # operands are bf16 or fp16
    st = lib.soup_ce_linear_dweight(fake, 1 << 20, fake, d, BF, n, v, 12, None, fake, _lib.F32, 0,
                                    None)
    assert st in (_lib.SOUP_ERR_INVALID, _lib.SOUP_ERR_UNSUPPORTED)  # dim % 8 != 0, h_ld < dim
    need = lib.soup_ce_linear_workspace_bytes(n, v, d)
    st = lib.soup_ce_linear_dweight(fake, need - 1, fake, d, BF, n, v, d, None, fake, _lib.F32, 0,
                                    None)
    assert st == _lib.SOUP_ERR_WORKSPACE
    # soup_ce_linear(hidden, h_ld, weight, w_ld, in_dtype, weight_bwd, wb_ld, targets, rows, vocab,
    #                dim, den, ignore, losses, entropies, correct, sums, dhidden, dh_dtype,
    #                dweight, dw_dtype, accumulate, workspace, bytes, stream)
    st = lib.soup_ce_linear(fake, d, fake, d, _lib.F16, None, 0, fake, n, v, d, 1.0, -100, fake,
                            fake, fake, None, fake, _lib.BF16, None, _lib.F32, 0, fake, need, None)
    assert st == _lib.SOUP_ERR_INVALID  # fp16 operands with dhidden need the bf16 weight copy
    assert b"weight_bwd" in lib.soup_last_error()
    st = lib.soup_ce_linear(fake, d, fake, d, BF, None, 0, fake, n, v, d, 1.0, -100, fake, fake,
                            fake, None, fake, 7, None, _lib.F32, 0, fake, need, None)
    assert st == _lib.SOUP_ERR_INVALID  # bad dhidden dtype
    # soup_ce_vp_forward(hidden, h_ld, weight_shard, w_ld, in_dtype, targets, rows, vocab_shard,
    #                    vocab_offset, dim, states, workspace, bytes, stream)
    st = lib.soup_ce_vp_forward(None, d, fake, d, BF, fake, n, v, 0, d, fake, fake, 1 << 20, None)
    assert st == _lib.SOUP_ERR_INVALID
    st = lib.soup_ce_vp_forward(fake, d, fake, d, BF, fake, n, v, -1, d, fake, fake, 1 << 20, None)
    assert st == _lib.SOUP_ERR_INVALID  # negative vocab offset
    need_vp = lib.soup_ce_vp_workspace_bytes(n, v, d)
    st = lib.soup_ce_vp_forward(fake, d, fake, d, BF, fake, n, v, 0, d, fake, fake, need_vp - 1,
                                None)
    assert st == _lib.SOUP_ERR_WORKSPACE
    # soup_ce_vp_backward(workspace, bytes, hidden, h_ld, weight_shard, w_ld, in_dtype,
    #                     weight_shard_bwd, wb_ld, targets, rows, vocab_shard, vocab_offset, dim,
    #                     lse, denominator, ignore_index, dhidden_partial, dh_dtype,
    #                     dweight_shard, dw_dtype, accumulate, stream)
    st = lib.soup_ce_vp_backward(fake, need_vp, fake, d, fake, d, BF, None, 0, fake, n, v, 0, d,
                                 None, 1.0, -100, fake, _lib.F32, None, BF, 0, None)
    assert st == _lib.SOUP_ERR_INVALID  # no lse
    st = lib.soup_ce_vp_backward(fake, need_vp, fake, d, fake, d, BF, None, 0, fake, n, v, 0, d,
                                 fake, 1.0, -100, fake, 7, None, BF, 0, None)
    assert st == _lib.SOUP_ERR_INVALID  # bad dhidden dtype
    st = lib.soup_ce_vp_backward(fake, need_vp, fake, d, fake, d, _lib.F16, None, 0, fake, n, v, 0,
                                 d, fake, 1.0, -100, fake, _lib.F32, None, BF, 0, None)
    assert st == _lib.SOUP_ERR_INVALID  # fp16 shard without its bf16 copy
    st = lib.soup_ce_vp_backward(fake, need_vp - 1, fake, d, fake, d, BF, None, 0, fake, n, v, 0, d,
                                 fake, 1.0, -100, fake, _lib.F32, None, BF, 0, None)
    assert st == _lib.SOUP_ERR_WORKSPACE


def test_wait_limit_setting_is_validated_on_the_host():
    lib = _lib.lib()
    assert lib.soup_set_wait_limit_ns(500_000) == _lib.SOUP_ERR_INVALID  # below 1 ms
    assert b"wait_limit" in lib.soup_last_error()
    assert lib.soup_set_wait_limit_ns(10_000_000) == _lib.SOUP_OK
    assert lib.soup_set_wait_limit_ns(0) == _lib.SOUP_OK  # back to the 2 s default
    st = lib.soup_gemm_wait_expiry_check(None, None, None, 256, 256, 256, 1_000_000, None)
    assert st == _lib.SOUP_ERR_INVALID


def test_stream_k_and_dual_rank_entry_points_validate_on_the_host():
    lib = _lib.lib()
    # stream-K scratch: one 256 KB fp32 slot per CTA pair plus the ready flags
    # (the library assumes 148 SMs when no GPU is visible)
    assert lib.soup_gemm_stream_k_workspace_bytes() >= 74 * 256 * 1024
    assert lib.soup_gemm_set_stream_k_min_saved(-1) == _lib.SOUP_OK
    fake = ctypes.c_void_p(256)  # never dereferenced: validation fails first
    m, n, r = 8192, 17920, 32
    ws = lib.soup_lora_rank_dual_workspace_bytes(m, n, r)
    # 8 x 8 tiles of 128 x 128 per CTA: dxa partials of 18 column blocks, G partials of 8 row blocks
    assert ws == (18 * m + 8 * n) * 32 * 4
    assert lib.soup_lora_rank_dual_workspace_bytes(m, n, 65) == 0
    args = [fake, n, fake, n, fake, m, m, n, r, fake, r, fake, r, fake, ws, None]

    def call(**over):
        a = list(args)
        for i, v in over.items():
            a[int(i[1:])] = v
        return lib.soup_lora_rank_dual(*a)

    assert call(a0=None) == _lib.SOUP_ERR_INVALID                 # no dy
    assert call(a8=80, a10=80, a12=80) == _lib.SOUP_ERR_INVALID   # rank above 64
    assert call(a1=n - 8) == _lib.SOUP_ERR_INVALID                # dy row stride shorter than a row
    assert call(a5=m - 8) == _lib.SOUP_ERR_INVALID                # xa^T row stride shorter than a row
    assert call(a1=n + 3) == _lib.SOUP_ERR_UNSUPPORTED            # rows not 16-byte aligned
    assert call(a14=ws - 16) == _lib.SOUP_ERR_WORKSPACE           # workspace too small
    assert call(a13=None) == _lib.SOUP_ERR_WORKSPACE              # no workspace
