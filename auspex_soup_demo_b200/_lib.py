"""ctypes binding of the C-ABI library ``libsoupb200.so`` (declared in include/soupb200.h).

The library is built in-tree by ``auspex_soup_demo_b200.build``. Loading fails
loudly (:class:`SoupLibraryError`) when it is missing: there is no fallback
implementation. Every call goes to the CUDA stream torch considers current
for the tensor's device.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libsoupb200.so")

SOUP_OK = 0
SOUP_ERR_INVALID = 1
SOUP_ERR_UNSUPPORTED = 2
SOUP_ERR_CUDA = 3
SOUP_ERR_WORKSPACE = 4
SOUP_ERR_DEVICE = 5

F32, F16, BF16 = 0, 1, 2
_DTYPE = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}


class SoupLibraryError(RuntimeError):
    """The compiled library is missing or does not load."""


class SoupError(RuntimeError):
    """An entry point returned a non-zero status."""

    def __init__(self, fn: str, status: int, detail: str):
        super().__init__(f"{fn} failed with status {status}: {detail}")
        self.status = status


c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_f = ctypes.c_float
c_vp = ctypes.c_void_p
c_sz = ctypes.c_size_t
P_I64 = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes)
_SIGNATURES = {
    "soup_version": (c_int, []),
    "soup_last_error": (ctypes.c_char_p, []),
    "soup_device_error": (c_int, [c_vp, ctypes.POINTER(c_int)]),
    "soup_set_wait_limit_ns": (c_int, [ctypes.c_uint64]),
    "soup_gemm_wait_expiry_check": (c_int, [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, ctypes.c_uint64,
                                            c_vp]),
    "soup_rmsnorm_fwd": (c_int, [c_vp, c_i64, c_vp, c_vp, c_i64, c_vp, c_i64, c_i64, c_f, c_int,
                                 c_int, c_vp]),
    "soup_rmsnorm_bwd_workspace_bytes": (c_sz, [c_i64, c_i64]),
    "soup_rmsnorm_bwd": (c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp, c_i64, c_vp, c_vp,
                                 c_sz, c_i64, c_i64, c_int, c_int, c_vp]),
    "soup_rmsnorm_bwd_noalloc": (c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp, c_i64, c_vp,
                                         c_i64, c_i64, c_int, c_int, c_vp]),
    "soup_swiglu_fwd": (c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_int, c_vp]),
    "soup_swiglu_bwd": (c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64,
                                c_i64, c_i64, c_int, c_vp]),
    "soup_rope": (c_int, [c_vp, P_I64, c_vp, P_I64, c_i64, c_vp, P_I64, c_vp, P_I64, c_i64, c_vp,
                          c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_int, c_int, c_int, c_vp]),
    "soup_ce_rows": (c_int, [c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_f, c_i64, c_int,
                             c_int, c_vp]),
    "soup_ce_linear_workspace_bytes": (c_sz, [c_i64, c_i64, c_i64]),
    "soup_ce_linear": (c_int, [c_vp, c_i64, c_vp, c_i64, c_int, c_vp, c_i64, c_vp, c_i64, c_i64,
                               c_i64, c_f, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_vp, c_int,
                               c_int, c_vp, c_sz, c_vp]),
    "soup_ce_linear_dweight": (c_int, [c_vp, c_sz, c_vp, c_i64, c_int, c_i64, c_i64, c_i64, c_vp,
                                       c_vp, c_int, c_int, c_vp]),
    "soup_ce_vp_workspace_bytes": (c_sz, [c_i64, c_i64, c_i64]),
    "soup_ce_vp_forward": (c_int, [c_vp, c_i64, c_vp, c_i64, c_int, c_vp, c_i64, c_i64, c_i64, c_i64,
                                   c_vp, c_vp, c_sz, c_vp]),
    "soup_ce_vp_combine": (c_int, [c_vp, c_int, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp,
                                   c_vp, c_vp]),
    "soup_ce_vp_backward": (c_int, [c_vp, c_sz, c_vp, c_i64, c_vp, c_i64, c_int, c_vp, c_i64, c_vp,
                                    c_i64, c_i64, c_i64, c_i64, c_vp, c_f, c_i64, c_vp, c_int, c_vp,
                                    c_int, c_int, c_vp]),
    "soup_set_stage_events": (c_int, [ctypes.POINTER(c_vp), c_int]),
    "soup_attention_fwd": (c_int, [c_vp, P_I64, c_vp, P_I64, c_vp, P_I64, c_i64, c_i64, c_i64, c_i64,
                                   c_i64, c_f, c_int, c_vp, c_vp, c_vp]),
    "soup_attention_bwd_workspace_bytes": (c_sz, [c_i64, c_i64, c_i64]),
    "soup_attention_bwd": (c_int, [c_vp, P_I64, c_vp, P_I64, c_vp, P_I64, c_vp, c_vp, c_vp, c_i64,
                                   c_i64, c_i64, c_i64, c_i64, c_f, c_int, c_vp, c_vp, c_vp, c_vp,
                                   c_sz, c_vp]),
    "soup_nf4_quantize": (c_int, [c_vp, c_i64, c_int, c_int, ctypes.POINTER(c_f), c_vp, c_vp, c_vp]),
    "soup_nf4_dequant": (c_int, [c_vp, c_vp, c_i64, c_int, ctypes.POINTER(c_f), c_vp, c_int, c_vp]),
    "soup_gemm_stream_k_workspace_bytes": (c_sz, []),
    "soup_gemm_set_stream_k_workspace": (c_int, [c_vp, c_sz]),
    "soup_gemm_set_stream_k_min_saved": (c_int, [c_int]),
    "soup_gemm_bf16": (c_int, [c_vp, c_i64, c_int, c_vp, c_i64, c_int, c_vp, c_i64, c_int, c_i64,
                               c_i64, c_i64, c_f, c_int, c_vp]),
    "soup_gemm_bf16_lora_swiglu": (c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_i64,
                                           c_vp, c_int, c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_i64,
                                           c_vp]),
    "soup_gemm_bf16_lora_dswiglu": (c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64,
                                            c_i64, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp]),
    "soup_adamw_flat": (c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_vp, c_f, c_f, c_f, c_f, c_f, c_vp,
                                c_int, c_i64, c_f, c_vp]),
    "soup_gemm_bf16_lora": (c_int, [c_vp, c_i64, c_int, c_vp, c_i64, c_int, c_vp, c_i64, c_vp, c_i64,
                                    c_i64, c_vp, c_vp, c_i64, c_int, c_i64, c_i64, c_i64, c_f, c_int,
                                    c_vp]),
    "soup_lora_rank_gemm": (c_int, [c_vp, c_i64, c_int, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_i64,
                                    c_vp, c_i64, c_vp, c_i64, c_int, c_f, c_vp]),
    "soup_lora_rank_dual_workspace_bytes": (c_sz, [c_i64, c_i64, c_i64]),
    "soup_lora_rank_dual": (c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_i64,
                                    c_vp, c_i64, c_vp, c_sz, c_vp]),
    "soup_lora_rank_grad_group": (c_int, [c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_i64, c_int, c_int,
                                          c_vp, c_vp, c_vp, c_vp, c_f, c_vp]),
}

_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """Load (once) and return the library; raise SoupLibraryError if absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise SoupLibraryError(
                f"{LIB_PATH} is not built; run `python -m auspex_soup_demo_b200.build` "
                "(nvcc with sm_100a support is required)")
        try:
            handle = ctypes.CDLL(LIB_PATH)
        except OSError as exc:  # pragma: no cover - depends on the host
            raise SoupLibraryError(f"cannot load {LIB_PATH}: {exc}") from exc
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def exported_symbols():
    """Names the binding expects the library to export."""
    return list(_SIGNATURES)


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE[dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {dtype}; expected float32, float16 or bfloat16") from None


def check(fn: str, status: int) -> None:
    if status != SOUP_OK:
        detail = lib().soup_last_error()
        raise SoupError(fn, status, detail.decode() if detail else "")


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def call(fn: str, device: torch.device, *args) -> None:
    """Invoke entry point `fn` with `device` current; raise on failure."""
    f = getattr(lib(), fn)
    if device.index is not None and device.index != torch.cuda.current_device():
        with torch.cuda.device(device):
            if fn in _GEMM_ENTRY_POINTS:
                _ensure_stream_k()
            check(fn, f(*args))
    else:
        if fn in _GEMM_ENTRY_POINTS:
            _ensure_stream_k()
        check(fn, f(*args))


# --------------------------------------------------------------------------
# Stream-K scratch of the tcgen05 GEMMs: one zero-filled buffer per device,
# registered with the library before the first GEMM on that device (the
# kernels leave it zero-filled). SOUP_STREAM_K=0 in the environment, or
# set_stream_k(False), runs every GEMM's last wave as a partial wave instead.
# Launches on one device share the buffer, so GEMMs of this library must not
# run concurrently on unordered streams of one device.
# --------------------------------------------------------------------------
STREAM_K = os.environ.get("SOUP_STREAM_K", "1") != "0"
_GEMM_ENTRY_POINTS = {
    "soup_gemm_bf16", "soup_gemm_bf16_lora", "soup_gemm_bf16_lora_swiglu",
    "soup_gemm_bf16_lora_dswiglu", "soup_ce_linear", "soup_ce_linear_dweight",
    "soup_ce_vp_forward", "soup_ce_vp_backward",
}
_sk_buffers = {}  # device index -> registered buffer


def _ensure_stream_k() -> None:
    """Register the current device's stream-K buffer, once. Skipped while a
    CUDA graph is being captured (the zero-fill would become part of the
    graph): launches then run without the stream-K tail."""
    idx = torch.cuda.current_device()
    if idx in _sk_buffers or not STREAM_K:
        return
    if torch.cuda.is_current_stream_capturing():
        return
    with _lock:
        if idx in _sk_buffers:
            return
        nbytes = int(lib().soup_gemm_stream_k_workspace_bytes())
        buf = torch.zeros(nbytes, dtype=torch.uint8, device=torch.device("cuda", idx))
        torch.cuda.synchronize(idx)  # zero before any stream's first GEMM reads it
        check("soup_gemm_set_stream_k_workspace",
              lib().soup_gemm_set_stream_k_workspace(buf.data_ptr(), nbytes))
        _sk_buffers[idx] = buf


def set_stream_k(enabled: bool) -> None:
    """Turn the GEMMs' stream-K tail on or off for later launches (devices with
    a registered buffer; the others get one on their next GEMM when enabled).
    Synchronises those devices first."""
    global STREAM_K
    STREAM_K = bool(enabled)
    for idx, buf in list(_sk_buffers.items()):
        with torch.cuda.device(idx):
            torch.cuda.synchronize(idx)
            if enabled:
                check("soup_gemm_set_stream_k_workspace",
                      lib().soup_gemm_set_stream_k_workspace(buf.data_ptr(), buf.numel()))
            else:
                check("soup_gemm_set_stream_k_workspace", lib().soup_gemm_set_stream_k_workspace(None, 0))


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def i64_array(values):
    return (ctypes.c_int64 * len(values))(*values)


def device_error(device: torch.device) -> int:
    """Read and clear the device error word (synchronises the current stream).
    After a GEMM wait error (codes 0x101-0x104) the device's stream-K buffer is
    zeroed again, since an aborted launch may have left ready flags set."""
    out = c_int(0)
    with torch.cuda.device(device):
        check("soup_device_error",
              lib().soup_device_error(torch.cuda.current_stream(device).cuda_stream,
                                      ctypes.byref(out)))
        idx = torch.cuda.current_device()
        if 0x101 <= out.value <= 0x104 and _sk_buffers.get(idx) is not None:
            torch.cuda.synchronize(idx)
            _sk_buffers[idx].zero_()
            torch.cuda.synchronize(idx)
    return out.value


# --------------------------------------------------------------------------
# Scratch buffers, one per (device, stream), grown on demand.
# --------------------------------------------------------------------------
_scratch = {}


def scratch(device: torch.device, nbytes: int) -> torch.Tensor:
    """A uint8 device buffer of at least `nbytes` for the current stream."""
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    buf = _scratch.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
        _scratch[key] = buf
    return buf


def release_scratch() -> None:
    _scratch.clear()
