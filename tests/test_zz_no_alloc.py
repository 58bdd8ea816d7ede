"""The allocation-free RMSNorm backward, called through the C ABI.

soup_rmsnorm_bwd_noalloc serves callers that cannot hand the library scratch
memory (for example code running under an allocator that already owns the
whole GPU, or host code that must not call cudaMalloc because it can
synchronise the device). It keeps its dw partial rows in a 4 MiB array built
into the library. This test compares it with soup_rmsnorm_bwd, which takes a
caller workspace, and with the CPU oracle, on two calls in a row, and checks
the size limit. The file is named so pytest collects it last.
"""

import pytest
import torch

import oracle
from auspex_soup_demo_b200 import _lib

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-4  # the fp32 tolerance of the other RMSNorm tests


def _inputs(seed, rows, cols, dtype):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, cols, device="cuda", generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(cols, device="cuda", generator=g)).to(dtype)
    dy = torch.randn(rows, cols, device="cuda", generator=g).to(dtype)
    y = torch.empty_like(x)
    rstd = torch.empty(rows, device="cuda")
    _lib.call("soup_rmsnorm_fwd", x.device, x.data_ptr(), cols, w.data_ptr(), y.data_ptr(), cols,
              rstd.data_ptr(), rows, cols, 1e-6, _lib.dtype_code(dtype), _lib.dtype_code(dtype),
              _lib.stream_of(x))
    return x, w, dy, rstd


def _with_workspace(x, w, dy, rstd):
    rows, cols = x.shape
    dx = torch.empty_like(x)
    dw = torch.empty_like(w)
    nbytes = _lib.lib().soup_rmsnorm_bwd_workspace_bytes(rows, cols)
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    _lib.call("soup_rmsnorm_bwd", x.device, dy.data_ptr(), cols, x.data_ptr(), cols, w.data_ptr(),
              rstd.data_ptr(), dx.data_ptr(), cols, dw.data_ptr(), ws.data_ptr(), nbytes, rows, cols,
              _lib.dtype_code(x.dtype), _lib.dtype_code(w.dtype), _lib.stream_of(x))
    return dx, dw


def _without_allocation(x, w, dy, rstd):
    rows, cols = x.shape
    dx = torch.empty_like(x)
    dw = torch.empty_like(w)
    status = _lib.lib().soup_rmsnorm_bwd_noalloc(
        dy.data_ptr(), cols, x.data_ptr(), cols, w.data_ptr(), rstd.data_ptr(), dx.data_ptr(), cols,
        dw.data_ptr(), rows, cols, _lib.dtype_code(x.dtype), _lib.dtype_code(w.dtype),
        _lib.stream_of(x))
    _lib.check("soup_rmsnorm_bwd_noalloc", status)
    return dx, dw


def _close(a, b):
    den = float(b.float().abs().max()) or 1.0
    return float((a.float() - b.float()).abs().max()) / den


@pytest.mark.parametrize("rows,cols,dtype", [(2048, 1536, torch.float32), (300, 1000, torch.bfloat16)])
def test_noalloc_matches_workspace_entry_point_twice(rows, cols, dtype):
    for call in range(2):  # the shared array keeps the previous call's contents
        x, w, dy, rstd = _inputs(10 + call, rows, cols, dtype)
        ref_dx, ref_dw = _with_workspace(x, w, dy, rstd)
        dx, dw = _without_allocation(x, w, dy, rstd)
        torch.cuda.synchronize()
        tol = FP32_TOL if dtype == torch.float32 else 8e-3
        assert _close(dx, ref_dx) <= tol, f"call {call}: dx"
        assert _close(dw, ref_dw) <= tol, f"call {call}: dw"
        # and against the CPU restatement of the reference's backward
        o_dx, o_dw = oracle.rmsnorm_bwd(dy.cpu(), x.cpu(), w.cpu(), rstd.cpu())
        assert _close(dx.cpu(), o_dx) <= tol, f"call {call}: dx vs oracle"
        assert _close(dw.cpu(), o_dw) <= tol, f"call {call}: dw vs oracle"


def test_noalloc_rejects_sizes_beyond_its_buffer():
    rows, cols = 4096, 65536  # 148 partial rows of 256 KiB > 4 MiB
    dev = torch.device("cuda")
    x = torch.empty(rows, cols, device=dev, dtype=torch.bfloat16)
    w = torch.empty(cols, device=dev, dtype=torch.bfloat16)
    rstd = torch.empty(rows, device=dev)
    status = _lib.lib().soup_rmsnorm_bwd_noalloc(
        x.data_ptr(), cols, x.data_ptr(), cols, w.data_ptr(), rstd.data_ptr(), x.data_ptr(), cols,
        w.data_ptr(), rows, cols, _lib.BF16, _lib.BF16, _lib.stream_of(x))
    assert status == _lib.SOUP_ERR_WORKSPACE
    assert b"4194304" in _lib.lib().soup_last_error()
