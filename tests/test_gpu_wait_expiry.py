"""The bounded waits of the tcgen05 GEMM end a kernel with an error status, not a hang.

soup_gemm_wait_expiry_check launches the pair GEMM with its producer withholding
one k-block, so the MMA issuer waits for a stage that nothing fills. With a 1 ms
limit the wait expires: the kernel records its code in the device error word,
drains what it issued (each drain wait bounded by the same limit), frees TMEM and
returns. The test reads the code back, checks that reading clears it, and runs a
normal GEMM on the same device afterwards.
"""

import pytest
import torch

from auspex_soup_demo_b200 import _lib

pytestmark = pytest.mark.gpu

WAIT_CODES = {0x101, 0x102, 0x103}


def _gemm(a, b):
    m, k = a.shape
    n = b.shape[0]
    c = torch.empty(m, n, device=a.device, dtype=torch.float32)
    _lib.call("soup_gemm_bf16", a.device, a.data_ptr(), k, 0, b.data_ptr(), k, 0, c.data_ptr(), n,
              _lib.F32, m, n, k, 1.0, 0, _lib.stream_of(a))
    return c


def test_expired_wait_returns_error_and_the_device_stays_usable():
    dev = torch.device("cuda:0")
    assert _lib.device_error(dev) == 0
    g = torch.Generator(device=dev).manual_seed(0)
    m, n, k = 512, 512, 256
    a = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
    b = torch.randn(n, k, device=dev, generator=g).to(torch.bfloat16)
    c = torch.zeros(m, n, device=dev, dtype=torch.bfloat16)
    _lib.call("soup_gemm_wait_expiry_check", dev, a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k,
              1_000_000, _lib.stream_of(a))
    code = _lib.device_error(dev)  # synchronises the stream: the kernel has returned
    assert code in WAIT_CODES, hex(code)
    assert _lib.device_error(dev) == 0  # the read cleared it
    # the same device runs a normal GEMM correctly right after
    out = _gemm(a, b)
    ref = a.float() @ b.float().t()
    torch.cuda.synchronize()
    assert torch.allclose(out, ref, rtol=1e-3, atol=1e-2)
    assert _lib.device_error(dev) == 0


def test_host_set_wait_limit_applies_to_normal_launches():
    dev = torch.device("cuda:0")
    lib = _lib.lib()
    g = torch.Generator(device=dev).manual_seed(1)
    a = torch.randn(300, 192, device=dev, generator=g).to(torch.bfloat16)
    b = torch.randn(260, 192, device=dev, generator=g).to(torch.bfloat16)
    try:
        assert lib.soup_set_wait_limit_ns(5_000_000) == 0
        out = _gemm(a, b)
        torch.cuda.synchronize()
    finally:
        assert lib.soup_set_wait_limit_ns(0) == 0
    assert torch.allclose(out, a.float() @ b.float().t(), rtol=1e-3, atol=1e-2)
    assert _lib.device_error(dev) == 0


def test_expiry_check_rejects_bad_arguments():
    dev = torch.device("cuda:0")
    a = torch.zeros(256, 64, device=dev, dtype=torch.bfloat16)  # k < 128: one k-block only
    with pytest.raises(_lib.SoupError):
        _lib.call("soup_gemm_wait_expiry_check", dev, a.data_ptr(), a.data_ptr(), a.data_ptr(),
                  256, 256, 64, 1_000_000, _lib.stream_of(a))
    b = torch.zeros(256, 256, device=dev, dtype=torch.bfloat16)
    with pytest.raises(_lib.SoupError):  # limit below 1 ms
        _lib.call("soup_gemm_wait_expiry_check", dev, b.data_ptr(), b.data_ptr(), b.data_ptr(),
                  256, 256, 256, 1000, _lib.stream_of(b))
