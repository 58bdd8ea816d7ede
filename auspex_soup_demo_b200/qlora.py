"""QLoRA training step on the Qwen2.5-1.5B architecture, driven through the fused ops.

The reference's workload (``task/task.yaml``): Qwen2.5-1.5B-Instruct, 4-bit NF4
base weights, LoRA r=16 / alpha=32, AdamW 2e-4, trained by Soup (TRL/HF
Trainer) with ``solution.apply()`` patches installed. Soup, PEFT and
bitsandbytes are not available here, so this module provides the pieces of that
step that surround the fused ops:

* :class:`LoRANF4Linear` - a frozen NF4 base weight (blocksize 64, our CUDA
  quantiser/dequantiser) plus trainable LoRA factors; the base weight is
  dequantised to bf16 for each use (forward and backward) and never stored;
  base product and LoRA term are one tcgen05 GEMM whose last k-block is the
  rank-16 term (soup_gemm_bf16_lora), and the LoRA gradients accumulate
  straight into fp32 buffers;
* :func:`build_qwen2_qlora` - the Qwen2.5-1.5B architecture (28 layers, hidden
  1536, MLP 8960, 12 query / 2 KV heads of 128, vocab 151936, tied embeddings,
  rope theta 1e6) randomly initialised (N(0, 0.02)) with LoRA on
  q/k/v/o/gate/up/down;
* :class:`QLoRATrainer` - one optimiser step: transformer body (with the fused
  RMSNorm / RoPE / SwiGLU patches), fused head cross-entropy, backward, AdamW.
  With ``torch.distributed`` initialised (one process per GPU, NCCL), only the
  LoRA gradients exist, and they are averaged over ranks by one all-reduce of
  their flat buffer after the backward pass.
"""

from __future__ import annotations

import ctypes
import math
from typing import Iterable, Optional

import numpy as np
import torch
import torch.nn.functional as F

from . import _lib

LORA_TARGETS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")

_CODE_CACHE = {}


def nf4_code_values() -> np.ndarray:
    """The 16 NF4 code values (QLoRA paper, Appendix E), ascending, fp32.

    Standard-normal quantiles at probabilities evenly spaced from ``offset`` to
    0.5: 8 for the positive half, 7 for the negative half, plus an exact zero,
    normalised to [-1, 1]; offset = 1 - (1/30 + 1/32)/2.
    """
    if "np" not in _CODE_CACHE:
        from scipy.stats import norm

        offset = 1.0 - 0.5 * (1.0 / 30.0 + 1.0 / 32.0)
        pos = norm.ppf(np.linspace(offset, 0.5, 9)[:-1])
        neg = -norm.ppf(np.linspace(offset, 0.5, 8)[:-1])
        vals = np.sort(np.concatenate([pos, [0.0], neg]))
        _CODE_CACHE["np"] = (vals / np.abs(vals).max()).astype(np.float32)
    return _CODE_CACHE["np"]


def _code_ptr():
    import ctypes

    if "c" not in _CODE_CACHE:
        _CODE_CACHE["c"] = (ctypes.c_float * 16)(*[float(v) for v in nf4_code_values()])
    return _CODE_CACHE["c"]


def nf4_quantize(weight: torch.Tensor, blocksize: int = 64):
    """(packed uint8 [n/2], absmax fp32 [n/64]) of a CUDA weight tensor."""
    w = weight.detach().contiguous()
    n = w.numel()
    packed = torch.empty(n // 2, dtype=torch.uint8, device=w.device)
    absmax = torch.empty(n // blocksize, dtype=torch.float32, device=w.device)
    _lib.call("soup_nf4_quantize", w.device, w.data_ptr(), n, _lib.dtype_code(w.dtype), blocksize,
              _code_ptr(), packed.data_ptr(), absmax.data_ptr(), _lib.stream_of(w))
    return packed, absmax


def nf4_dequantize(packed: torch.Tensor, absmax: torch.Tensor, shape, dtype=torch.bfloat16,
                   blocksize: int = 64, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    n = packed.numel() * 2
    if out is None:
        out = torch.empty(shape, dtype=dtype, device=packed.device)
    _lib.call("soup_nf4_dequant", packed.device, packed.data_ptr(), absmax.data_ptr(), n, blocksize,
              _code_ptr(), out.data_ptr(), _lib.dtype_code(out.dtype), _lib.stream_of(packed))
    return out


def _accumulate_grad(param: torch.Tensor, m1: torch.Tensor, m2: torch.Tensor, alpha: float):
    """param.grad += alpha * m1 @ m2, in place when the gradient is an fp32 CUDA
    buffer and the factors are 16-bit (cuBLAS accumulates the bf16 product into
    the fp32 gradient; no cast or add kernels). Returns None in that case, else
    the gradient for autograd to accumulate."""
    g = param.grad
    if (g is not None and g.is_cuda and g.dtype == torch.float32 and m1.dtype in (torch.bfloat16, torch.float16)
            and g.is_contiguous()):
        torch.addmm(g, m1, m2, alpha=alpha, out_dtype=torch.float32, out=g)
        return None
    return (alpha * (m1.float() @ m2.float())).to(param.dtype)


# Contractions longer than this (K = 8960: down forward, K = 17920: gate/up
# backward) run on the tcgen05 GEMM only when their output has at least
# LONG_K_MIN_WAVES waves of 256 x 256 tiles over the CTA pairs and the
# GEMMs' stream-K tail is on (_lib.STREAM_K); otherwise on cuBLAS plus an
# accumulating rank-r GEMM. Measured on B200 (CUDA graphs of 40 launches):
# at 8192 tokens (192 tiles, 2.6 waves) the gate/up backward takes 322-331 us
# against cuBLAS's 340-364 and the down forward 159-168 against 157-165; at
# 2048 tokens (48 tiles) cuBLAS is faster (83 vs 88 us, 43 vs 50 us). Every
# K = 1536 projection is faster on the tcgen05 GEMM at both sizes.
FUSED_MAX_K = 4096
LONG_K_MIN_WAVES = 2

# Row-block size of the interleaved gate/up weight layout (half a GEMM tile).
IL_BLOCK = 128

#: Keep each projection's dequantised 16-bit base weight from its forward to its
#: backward instead of dequantising the NF4 weight again there (bitsandbytes'
#: behaviour). Costs the weights of every layer between the passes (2.6 GB for
#: the 28 Qwen2.5-1.5B layers in bf16) and saves half of the dequantisation.
KEEP_BASE_WEIGHTS = True


def _keep(w: torch.Tensor):
    return w if KEEP_BASE_WEIGHTS else None


def _fused_ok(k: int, *ts: torch.Tensor, n: Optional[int] = None) -> bool:
    """The tcgen05 LoRA GEMM takes these operands: 16-byte aligned bf16 rows;
    for K > FUSED_MAX_K also an output of ts[0].shape[0] x n wide enough (see
    FUSED_MAX_K)."""
    if k > FUSED_MAX_K:
        if n is None or not _lib.STREAM_K or not ts or ts[0] is None or not ts[0].is_cuda:
            return False
        tiles = -(-ts[0].shape[0] // 256) * -(-n // 256)
        pairs = torch.cuda.get_device_properties(ts[0].device).multi_processor_count // 2
        if tiles < LONG_K_MIN_WAVES * pairs:
            return False
    for t in ts:
        if t is None:
            continue
        if (not t.is_cuda or t.dtype != torch.bfloat16 or t.dim() != 2 or t.stride(1) != 1
                or t.stride(0) % 8 or t.data_ptr() % 16):
            return False
    return True


def lora_gemm(a: torch.Tensor, b: torch.Tensor, b_mn_major: bool, a2: torch.Tensor, b2: torch.Tensor,
              out: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[M, N] = a @ op(b) + a2 @ op(b2) (+ bias) in one tcgen05 GEMM (soup_gemm_bf16_lora).

    a [M, K] and a2 [M, r] are row-major; op(b) is b^T for b [N, K]
    (b_mn_major False) or b for b [K, N] (True), and op(b2) likewise for b2
    [N, r] / [r, N]. The rank-r term is the GEMM's last k-block(s).
    """
    m, k = a.shape
    n = out.shape[1]
    r = a2.shape[1]
    _lib.call("soup_gemm_bf16_lora", a.device, a.data_ptr(), a.stride(0), 0, b.data_ptr(), b.stride(0),
              int(b_mn_major), a2.data_ptr(), a2.stride(0), b2.data_ptr(), b2.stride(0), r,
              None if bias is None else bias.data_ptr(), out.data_ptr(), out.stride(0),
              _lib.dtype_code(out.dtype), m, n, k, 1.0, 0, _lib.stream_of(a))
    return out


# A group's output gradient at least this wide, with at least DUAL_MIN_ROWS
# tokens, takes dxa and the B-gradient product from one pass of
# soup_lora_rank_dual: measured on B200 at the gate/up gradient [8192, 17920]
# (rank 32) 76 us against 86.5 us for cuBLAS's two products; at 2048 tokens
# (31 vs 24 us) and for the q/k/v gradient [8192, 2048] (26 vs 18 us) cuBLAS
# is faster.
DUAL_RANK = True
DUAL_MIN_COLS = 8192
DUAL_MIN_ROWS = 4096


def _dual_ok(group, dy: torch.Tensor, xa: torch.Tensor, need_params) -> bool:
    return (DUAL_RANK and dy.is_cuda and dy.dtype == torch.bfloat16 and xa.dtype == torch.bfloat16
            and dy.dim() == 2 and dy.shape[1] >= DUAL_MIN_COLS and dy.shape[0] >= DUAL_MIN_ROWS
            and dy.shape[0] % 8 == 0 and dy.shape[1] % 8 == 0 and dy.stride(1) == 1 and dy.stride(0) % 8 == 0
            and dy.data_ptr() % 16 == 0 and xa.shape[1] <= 64
            and any(need_params[2 * j + 1] for j in range(len(group.members))))


def rank_dual(dy: torch.Tensor, bt: torch.Tensor, xt: torch.Tensor):
    """(dxa = dy bt^T [M, R] bf16, G = dy^T xt^T [N, R] fp32) in one pass over
    dy [M, N] (soup_lora_rank_dual): a LoRA group's dxa = dy B and the product
    whose blocks are its members' B gradients, for bt = B^T [R, N] and
    xt = xa^T [R, M]."""
    m, n = dy.shape
    r = bt.shape[0]
    dxa = torch.empty(m, r, device=dy.device, dtype=torch.bfloat16)
    G = torch.empty(n, r, device=dy.device, dtype=torch.float32)
    nbytes = int(_lib.lib().soup_lora_rank_dual_workspace_bytes(m, n, r))
    ws = _lib.scratch(dy.device, nbytes)
    _lib.call("soup_lora_rank_dual", dy.device, dy.data_ptr(), dy.stride(0), bt.data_ptr(), bt.stride(0),
              xt.data_ptr(), xt.stride(0), m, n, r, dxa.data_ptr(), dxa.stride(0), G.data_ptr(), G.stride(0),
              ws.data_ptr(), nbytes, _lib.stream_of(dy))
    return dxa, G


def rank_gemm(a: torch.Tensor, b: torch.Tensor, a_mn_major: bool = False, c=None, ct=None, g=None,
              g_trans: bool = False, alpha: float = 1.0) -> None:
    """soup_lora_rank_gemm: C = op(a) b^T for a narrow b [n, K] (n <= 64), with
    op(a) = a [M, K] or, with a_mn_major, a^T for a stored [K, M]. Writes
    c = bf16(alpha C) [M, n], ct = its transpose [n, M] and/or g += alpha C
    (fp32; g_trans: g^T += alpha C)."""
    k, m = a.shape if a_mn_major else a.shape[::-1]
    n = b.shape[0]
    _lib.call("soup_lora_rank_gemm", a.device, a.data_ptr(), a.stride(0), int(a_mn_major), b.data_ptr(),
              b.stride(0), m, n, k, _lib.ptr(c), 0 if c is None else c.stride(0), _lib.ptr(ct),
              0 if ct is None else ct.stride(0), _lib.ptr(g), 0 if g is None else g.stride(0), int(g_trans),
              float(alpha), _lib.stream_of(a))


def rank_grad_group(dy: torch.Tensor, xaT: torch.Tensor, row_off, col_off, grads, interleaved: bool,
                    alpha: float = 1.0) -> None:
    """soup_lora_rank_grad_group: the members' gB += alpha dy^T xa in one pass over
    dy [T, N] (member j: rows [row_off[j], row_off[j+1]) of N - 128-row blocks in
    turn when interleaved - and rank columns [col_off[j], col_off[j+1]) of xaT [R, T])."""
    k, m = dy.shape
    nm = len(grads)
    ptrs = (ctypes.c_void_p * nm)(*[g.data_ptr() for g in grads])
    _lib.call("soup_lora_rank_grad_group", dy.device, dy.data_ptr(), dy.stride(0), xaT.data_ptr(),
              xaT.stride(0), m, xaT.shape[0], k, nm, int(interleaved), _lib.i64_array(list(row_off)),
              _lib.i64_array(list(col_off)), ptrs, _lib.i64_array([g.stride(0) for g in grads]),
              float(alpha), _lib.stream_of(dy))


#: Run the rank-r products of the LoRA linears (x As^T, dy B and the gradient
#: products dxa^T x, dy^T xa) on soup_lora_rank_gemm instead of cuBLAS. Off by
#: default: measured on B200 inside the captured Qwen2.5-1.5B step at 8192
#: tokens, cuBLAS runs the 25 MB products in 5-6 us (the kernel 7.5-11 us) and
#: streams the 150-300 MB ones at 6.4 TB/s (the kernel 5 TB/s); the kernel wins
#: only the gradient products of the rank-16 linears (9.7-10.8 us against
#: 12.6-12.9), and the step is 1.3 % slower with it on.
RANK_KERNELS = False


def _rank_ok(*ts) -> bool:
    if not RANK_KERNELS:
        return False
    for t in ts:
        if (t is None or not t.is_cuda or t.dtype != torch.bfloat16 or t.dim() != 2 or t.stride(1) != 1
                or t.stride(0) % 8 or t.data_ptr() % 16):
            return False
    return True


def _grad_ok(g: Optional[torch.Tensor]) -> bool:
    return g is not None and g.is_cuda and g.dtype == torch.float32 and g.is_contiguous()


def _rank_product(a: torch.Tensor, bt: torch.Tensor):
    """(a @ bt^T [M, R], its transpose [R, M] or None): one soup_lora_rank_gemm
    writing both when the operands allow, else cuBLAS."""
    m, r = a.shape[0], bt.shape[0]
    if r <= 64 and m % 8 == 0 and _rank_ok(a, bt):
        c = torch.empty(m, r, device=a.device, dtype=a.dtype)
        ct = torch.empty(r, m, device=a.device, dtype=a.dtype)
        rank_gemm(a, bt, c=c, ct=ct)
        return c, ct
    return a @ bt.t(), None


def _lora_grads(A, B, x2, dy2, xa, xaT, dxa, dxaT, s, need_a: bool, need_b: bool):
    """(gA, gB) of one LoRA linear: accumulated in place into fp32 .grad buffers
    (None returned) by soup_lora_rank_gemm when the transposed rank products
    exist, else through _accumulate_grad."""
    gA = gB = None
    if need_a:
        if dxaT is not None and _grad_ok(A.grad) and _rank_ok(x2):
            rank_gemm(x2, dxaT, a_mn_major=True, g=A.grad, g_trans=True, alpha=s)
        else:
            gA = _accumulate_grad(A, dxa.t(), x2, s)
    if need_b:
        if xaT is not None and _grad_ok(B.grad) and _rank_ok(dy2):
            rank_gemm(dy2, xaT, a_mn_major=True, g=B.grad)
        else:
            gB = _accumulate_grad(B, dy2.t(), xa, 1.0)
    return gA, gB


class _LoRALinearFn(torch.autograd.Function):
    """y = x W^T (+ b) + (x As^T) B^T for a frozen base weight W and LoRA factors
    A [r, in], B [out, r], with As = s A (s = alpha / r).

    ``weight_fn(dtype)`` returns W [out, in] (dequantised from NF4 for each use,
    never stored); ``As16`` and ``B16`` are As and B in the activation dtype.
    Forward: xa = x As^T (a rank-r GEMM), then y = x W^T + xa B^T (+ b) as ONE
    tcgen05 GEMM whose last k-block is the rank-r term (lora_gemm) when the
    output is large enough, else cuBLAS plus an accumulating rank-r GEMM.
    Backward: dxa = dy B, dx = dy W + dxa As (again one GEMM with a rank-r
    k-block), dA += s dxa^T x and dB += dy^T xa straight into fp32 gradient
    buffers when the parameters have them (see _accumulate_grad).
    """

    @staticmethod
    def forward(ctx, x, A, B, As16, B16, scaling, weight_fn, bias, Bt16=None):
        w = weight_fn(x.dtype)
        x2 = x.reshape(-1, x.shape[-1])
        xa, xaT = _rank_product(x2, As16)
        m, n = x2.shape[0], w.shape[0]
        if _fused_ok(x2.shape[1], x2, w, xa, B16, bias.view(1, -1) if bias is not None else None, n=n):
            y2 = lora_gemm(x2, w, False, xa, B16, torch.empty(m, n, device=x.device, dtype=x.dtype), bias)
            y = y2.view(*x.shape[:-1], n)
        else:
            y = F.linear(x, w, bias)
            y.view(-1, n).addmm_(xa, B16.t())
        ctx.save_for_backward(x, xa, As16, B16, xaT, Bt16)
        ctx.params = (A, B)
        ctx.scaling = scaling
        ctx.weight_fn = weight_fn
        ctx.w = _keep(w)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, xa, As16, B16, xaT, Bt16 = ctx.saved_tensors
        A, B = ctx.params
        s = ctx.scaling
        dy2 = dy.reshape(-1, dy.shape[-1])
        if dy2.stride(1) != 1:
            dy2 = dy2.contiguous()
        x2 = x.reshape(-1, x.shape[-1])
        if xaT is not None:
            dxa, dxaT = _rank_product(dy2, Bt16 if Bt16 is not None else B16.t().contiguous())
        else:
            dxa, dxaT = dy2 @ B16, None
        dx = None
        if ctx.needs_input_grad[0]:
            w = ctx.w if ctx.w is not None and ctx.w.dtype == dy.dtype else ctx.weight_fn(dy.dtype)
            ctx.w = None
            m, n = dy2.shape[0], w.shape[1]
            if _fused_ok(dy2.shape[1], dy2, w, dxa, As16, n=w.shape[1]):
                dx2 = lora_gemm(dy2, w, True, dxa, As16, torch.empty(m, n, device=dy.device, dtype=dy.dtype))
            else:
                dx2 = dy2 @ w
                dx2.addmm_(dxa, As16)
            dx = dx2.view(x.shape)
        gA, gB = _lora_grads(A, B, x2, dy2, xa, xaT, dxa, dxaT, s, ctx.needs_input_grad[1],
                             ctx.needs_input_grad[2])
        return dx, gA, gB, None, None, None, None, None, None


class _LoRABase(torch.nn.Module):
    """Trainable LoRA factors (fp32) beside a frozen base weight.

    ``lora_As16`` / ``lora_B16`` may be set to 16-bit copies of (alpha/r) * A
    and of B that the owner refreshes after every optimiser step
    (QLoRATrainer keeps them in one buffer and refreshes them with two
    kernels per step); without them the factors are cast on each use.
    """

    def _init_lora(self, linear: torch.nn.Linear, r: int, alpha: int, lora_dtype: torch.dtype):
        self.in_features = linear.in_features
        self.out_features = linear.out_features
        if linear.bias is not None:
            self.register_buffer("bias", linear.bias.detach().clone())
        else:
            self.bias = None
        dev = linear.weight.device
        self.lora_A = torch.nn.Parameter(torch.empty(r, self.in_features, device=dev, dtype=lora_dtype))
        self.lora_B = torch.nn.Parameter(torch.zeros(self.out_features, r, device=dev, dtype=lora_dtype))
        torch.nn.init.kaiming_uniform_(self.lora_A, a=math.sqrt(5))
        self.scaling = alpha / r
        self.lora_As16 = None
        self.lora_B16 = None
        self.lora_Bt16 = None  # B16 transposed [r, out], refreshed with it (or None)
        self.lora_group = None

    def base_weight(self, dtype) -> torch.Tensor:
        raise NotImplementedError

    def forward(self, x):
        grp = self.lora_group
        if grp is not None and grp.kind == "qkv" and grp.usable(x):
            out = grp.member_output(self, x)
            if out is not None:
                return out
        as16, b16, bt16 = self.lora_As16, self.lora_B16, self.lora_Bt16
        if as16 is None or as16.dtype != x.dtype:
            as16 = (self.lora_A.detach() * self.scaling).to(x.dtype)
            b16 = self.lora_B.detach().to(x.dtype)
            bt16 = None
        bias = None if self.bias is None else self.bias.to(x.dtype)
        return _LoRALinearFn.apply(x, self.lora_A, self.lora_B, as16, b16, self.scaling,
                                   self.base_weight, bias, bt16)


class LoRANF4Linear(_LoRABase):
    """Frozen NF4 base linear + trainable LoRA: y = base(x) + (alpha/r) * B(A(x))."""

    def __init__(self, linear: torch.nn.Linear, r: int = 16, alpha: int = 32,
                 lora_dtype: torch.dtype = torch.float32):
        super().__init__()
        packed, absmax = nf4_quantize(linear.weight)
        self.register_buffer("packed", packed)
        self.register_buffer("absmax", absmax)
        self._init_lora(linear, r, alpha, lora_dtype)

    def dequantized_weight(self, dtype=torch.bfloat16) -> torch.Tensor:
        g = self.lora_group
        if g is not None and g.interleaved:  # the packed rows are a strided view
            return g.member_weight(self, dtype)
        return nf4_dequantize(self.packed, self.absmax, (self.out_features, self.in_features), dtype)

    def base_weight(self, dtype) -> torch.Tensor:
        return self.dequantized_weight(dtype)


class LoRADenseLinear(_LoRABase):
    """Frozen dense base linear + trainable LoRA (for non-quantised runs and CPU tests)."""

    def __init__(self, linear: torch.nn.Linear, r: int = 16, alpha: int = 32,
                 lora_dtype: torch.dtype = torch.float32):
        super().__init__()
        self.register_buffer("weight", linear.weight.detach().clone())
        self._init_lora(linear, r, alpha, lora_dtype)

    def base_weight(self, dtype) -> torch.Tensor:
        return self.weight.reshape(self.out_features, self.in_features).to(dtype)


class LoRAProjectionGroup:
    """Projections of one input (q/k/v, or gate/up) computed as ONE GEMM.

    The members keep their own LoRA parameters, names and buffers (the adapter
    layout does not change), but their frozen base weights live in one
    concatenated buffer - NF4 ``packed``/``absmax`` (the 64-element blocks of
    row-concatenated weights are the members' blocks in order) or a dense
    weight - of which each member's buffer is a view, and likewise the biases.
    One call then does one dequantisation, one rank-R GEMM xa = x As^T
    (R = sum of the members' ranks, As the members' scaled A factors stacked)
    and one tcgen05 GEMM y = x W^T + xa Bblk^T (+ bias) whose rank-R k-block
    uses the block-diagonal Bblk (member j's rows use only member j's xa
    columns). Backward is one dX GEMM with a rank-R k-block, one dxa GEMM,
    one gA GEMM into the stacked A gradients, and one gB GEMM per member.

    On B200 with Qwen2.5-1.5B shapes at 2048 tokens this replaces k_proj /
    v_proj GEMMs with N = 256 (8 of 74 CTA pairs busy) and the separate
    dequantisations, rank-16 GEMMs and autograd gradient sums of each member.

    The members' buffers are views of the group's; build the model on the
    device it will run on (moving it afterwards copies the views apart).
    """

    def __init__(self, members, kind: str):
        self.members = list(members)
        self.kind = kind
        ins = {m.in_features for m in self.members}
        assert len(ins) == 1, "grouped projections must share their input"
        self.in_features = ins.pop()
        self.outs = [m.out_features for m in self.members]
        self.ranks = [m.lora_A.shape[0] for m in self.members]
        self.out_off = [0]
        for n in self.outs:
            self.out_off.append(self.out_off[-1] + n)
        self.rank_off = [0]
        for r in self.ranks:
            self.rank_off.append(self.rank_off[-1] + r)
        self.n_total = self.out_off[-1]
        self.r_total = self.rank_off[-1]
        scal = {m.scaling for m in self.members}
        self.scaling = scal.pop() if len(scal) == 1 else None
        self.nf4 = all(isinstance(m, LoRANF4Linear) for m in self.members)
        # gate/up rows interleaved in blocks of IL_BLOCK (gate block c, then up block
        # c) so every 256-column GEMM tile holds g and u of the same 128 columns and
        # SwiGLU runs in the GEMM epilogue (soup_gemm_bf16_lora_swiglu)
        self.interleaved = (kind == "gate_up" and len(self.members) == 2 and self.outs[0] == self.outs[1]
                            and self.outs[0] % IL_BLOCK == 0 and self.in_features % 64 == 0)
        if self.interleaved:
            self._init_interleaved()
        elif self.nf4:
            self.packed = torch.cat([m.packed for m in self.members])
            self.absmax = torch.cat([m.absmax for m in self.members])
            po = ao = 0
            for m in self.members:
                n_p, n_a = m.packed.numel(), m.absmax.numel()
                m._buffers["packed"] = self.packed[po:po + n_p]
                m._buffers["absmax"] = self.absmax[ao:ao + n_a]
                po += n_p
                ao += n_a
        else:
            assert all(isinstance(m, LoRADenseLinear) for m in self.members)
            self.weight = torch.cat([m.weight for m in self.members])
            for m, a, b in zip(self.members, self.out_off[:-1], self.out_off[1:]):
                m._buffers["weight"] = self.weight[a:b]
        if self.interleaved:
            pass  # bias set by _init_interleaved
        elif any(m.bias is not None for m in self.members):
            self.bias = torch.cat([m.bias if m.bias is not None else
                                   torch.zeros(m.out_features, dtype=self.members[0].lora_A.dtype
                                               if self.members[0].bias is None else self.members[0].bias.dtype,
                                               device=self.members[0].lora_A.device)
                                   for m in self.members])
            for m, a, b in zip(self.members, self.out_off[:-1], self.out_off[1:]):
                if m.bias is not None:
                    m._buffers["bias"] = self.bias[a:b]
        else:
            self.bias = None
        # set by QLoRATrainer: 16-bit stacked As and block-diagonal B (refreshed
        # after every optimiser step) and the fp32 gradient view of the stacked A
        self.As16 = None
        self.Bblk16 = None
        self.BblkT16 = None  # Bblk16 transposed [R, N], refreshed with it
        self.gradA = None
        self._stash = None
        for m in self.members:
            m.lora_group = self

    def _il_view(self, t: torch.Tensor, width: int) -> torch.Tensor:
        """[2 * inter, width] rows in interleaved order viewed as [blocks, 2, IL_BLOCK, width]."""
        return t.view(self.outs[0] // IL_BLOCK, 2, IL_BLOCK, width)

    def _init_interleaved(self):
        nb = self.outs[0] // IL_BLOCK
        k = self.in_features

        def inter(ts, width):
            return torch.stack([t.reshape(nb, IL_BLOCK, width) for t in ts], dim=1).reshape(-1)

        if self.nf4:
            self.packed = inter([m.packed for m in self.members], k // 2)
            self.absmax = inter([m.absmax for m in self.members], k // 64)
            pv, av = self._il_view(self.packed, k // 2), self._il_view(self.absmax, k // 64)
            for j, m in enumerate(self.members):
                m._buffers["packed"] = pv[:, j]
                m._buffers["absmax"] = av[:, j]
        else:
            self.weight = inter([m.weight for m in self.members], k).view(2 * self.outs[0], k)
            wv = self._il_view(self.weight, k)
            for j, m in enumerate(self.members):
                m._buffers["weight"] = wv[:, j]
        if any(m.bias is not None for m in self.members):
            ref = next(m.bias for m in self.members if m.bias is not None)
            self.bias = inter([m.bias if m.bias is not None else torch.zeros_like(ref)
                               for m in self.members], 1)
        else:
            self.bias = None

    def member_weight(self, member, dtype) -> torch.Tensor:
        """One member's base weight [out, in] (dequantised from the group's buffer)."""
        j = self.members.index(member)
        w = self.base_weight(dtype)
        if self.interleaved:
            return self._il_view(w, self.in_features)[:, j].reshape(self.outs[j], self.in_features)
        return w[self.out_off[j]:self.out_off[j + 1]]

    # -- operands ---------------------------------------------------------------
    def base_weight(self, dtype) -> torch.Tensor:
        if self.nf4:
            return nf4_dequantize(self.packed, self.absmax, (self.n_total, self.in_features), dtype)
        return self.weight.to(dtype)

    def factors(self, dtype):
        """(As [R, in], Bblk [N, R]) in ``dtype``."""
        if self.As16 is not None and self.As16.dtype == dtype:
            return self.As16, self.Bblk16
        As = torch.cat([(m.lora_A.detach() * m.scaling).to(dtype) for m in self.members])
        Bblk = torch.zeros(self.n_total, self.r_total, dtype=dtype, device=As.device)
        for j, m in enumerate(self.members):
            r0, r1 = self.rank_off[j], self.rank_off[j + 1]
            if self.interleaved:
                self._il_view(Bblk, self.r_total)[:, j, :, r0:r1] = \
                    m.lora_B.detach().to(dtype).view(-1, IL_BLOCK, r1 - r0)
            else:
                Bblk[self.out_off[j]:self.out_off[j + 1], r0:r1] = m.lora_B.detach().to(dtype)
        return As, Bblk

    def factors_t(self, Bblk: torch.Tensor) -> torch.Tensor:
        """Bblk^T [R, N]: the owner's refreshed copy when Bblk is its buffer."""
        t = self.BblkT16
        if t is not None and self.Bblk16 is not None and Bblk.data_ptr() == self.Bblk16.data_ptr():
            return t
        return Bblk.t().contiguous()

    def out_features_of(self, j: int) -> int:
        return self.outs[j]

    def usable(self, x: torch.Tensor) -> bool:
        return (x.is_cuda and x.dtype == torch.bfloat16 and x.shape[-1] == self.in_features
                and all(m.lora_group is self for m in self.members))

    def params(self):
        out = []
        for m in self.members:
            out += [m.lora_A, m.lora_B]
        return out

    # -- calls ------------------------------------------------------------------
    def project(self, x: torch.Tensor):
        """The members' outputs for input x (a tuple, member order)."""
        return _LoRAGroupFn.apply(x, self, *self.params())

    def member_output(self, member, x: torch.Tensor) -> Optional[torch.Tensor]:
        """Output of ``member`` for x: the first member's call computes every
        member's output and keeps the others until they are asked for with
        the same input tensor (HF's attention calls q_proj, k_proj, v_proj on
        one hidden-state tensor in turn). None means: compute it alone."""
        st = self._stash
        if st is not None and st[0] is x and st[1] == x._version and member in st[2]:
            out = st[2].pop(member)
            if not st[2]:
                self._stash = None
            return out
        if member is not self.members[0]:
            return None
        outs = self.project(x)
        self._stash = (x, x._version, dict(zip(self.members[1:], outs[1:])))
        return outs[0]

    def swiglu(self, x: torch.Tensor, recompute: bool) -> torch.Tensor:
        """silu(gate(x)) * up(x) for a gate/up group, with the gate/up GEMM
        recomputed in backward when ``recompute`` (the reference's selective
        recompute of the MLP, solution/kernels/swiglu.py:197-214)."""
        return _LoRAGateUpFn.apply(x, self, bool(recompute), *self.params())

    def mlp(self, x: torch.Tensor, down, recompute: bool) -> torch.Tensor:
        """down(silu(gate(x)) * up(x)) for a gate/up group; one Function with the
        SwiGLU backward fused into down's input-gradient GEMM (FUSE_MLP_BACKWARD)
        when the activations are kept, bf16, and down is an ungrouped LoRA linear."""
        if (FUSE_MLP_BACKWARD and not recompute and self.interleaved
                and isinstance(down, _LoRABase) and down.lora_group is None
                and x.dtype == torch.bfloat16 and down.in_features == self.outs[0]):
            return _LoRAMLPFn.apply(x, self, down, down.lora_A, down.lora_B, *self.params())
        return down(self.swiglu(x, recompute))


def _group_gemm(group: LoRAProjectionGroup, x2: torch.Tensor, w: torch.Tensor, As16, Bblk,
                xa: Optional[torch.Tensor] = None):
    """(y = x2 W^T + (x2 As^T) Bblk^T + bias [M, N], xa = x2 As^T); a given xa is reused."""
    if xa is None:
        xa = x2 @ As16.t()
    m = x2.shape[0]
    n = group.n_total
    bias = None if group.bias is None else group.bias.to(x2.dtype)
    if _fused_ok(x2.shape[1], x2, w, xa, Bblk, bias.view(1, -1) if bias is not None else None, n=n):
        y = lora_gemm(x2, w, False, xa, Bblk, torch.empty(m, n, device=x2.device, dtype=x2.dtype), bias)
    else:
        y = F.linear(x2, w, bias)
        y.addmm_(xa, Bblk.t())
    return y, xa


def _group_backward(group: LoRAProjectionGroup, dy: torch.Tensor, x2: torch.Tensor, xa: torch.Tensor,
                    w: torch.Tensor, As16, Bblk, need_dx: bool, need_params, xaT=None):
    """dx (or None) and the LoRA gradients for a group GEMM's output gradient
    dy [M, N]. Gradients go straight into fp32 ``.grad`` buffers where the
    parameters have them (None is returned for those). With xaT (= xa^T from
    the forward's soup_lora_rank_gemm) the rank products run on that kernel:
    dxa and dxa^T in one pass over dy, gA into the stacked A gradient, and
    every member's gB in one more pass over dy."""
    G = None
    if xaT is not None:
        dxa, dxaT = _rank_product(dy, group.factors_t(Bblk))
    elif _dual_ok(group, dy, xa, need_params):
        # dxa and G = dy^T xa (the members' B gradients) in one pass over dy
        dxa, G = rank_dual(dy, group.factors_t(Bblk), xa.t().contiguous())
        dxaT = None
    else:
        dxa, dxaT = dy @ Bblk, None
    dx = None
    if need_dx:
        m, n = dy.shape[0], w.shape[1]
        if _fused_ok(dy.shape[1], dy, w, dxa, As16, n=w.shape[1]):
            dx = lora_gemm(dy, w, True, dxa, As16, torch.empty(m, n, device=dy.device, dtype=dy.dtype))
        else:
            dx = dy @ w
            dx.addmm_(dxa, As16)
    grads = []
    gA_done = False
    if group.gradA is not None and group.scaling is not None and all(
            need_params[2 * j] and group.members[j].lora_A.grad is not None
            and group.members[j].lora_A.grad.data_ptr() == group.gradA[group.rank_off[j]].data_ptr()
            for j in range(len(group.members))):
        if dxaT is not None and _rank_ok(x2) and _grad_ok(group.gradA):
            rank_gemm(x2, dxaT, a_mn_major=True, g=group.gradA, g_trans=True, alpha=group.scaling)
        else:
            torch.addmm(group.gradA, dxa.t(), x2, alpha=group.scaling, out_dtype=torch.float32, out=group.gradA)
        gA_done = True
    gB_done = False
    nm = len(group.members)
    if (xaT is not None and nm <= 4 and _rank_ok(dy) and xaT.shape[0] <= 64
            and all(need_params[2 * j + 1] and _grad_ok(group.members[j].lora_B.grad) for j in range(nm))):
        rank_grad_group(dy, xaT, group.out_off, group.rank_off, [mm.lora_B.grad for mm in group.members],
                        group.interleaved)
        gB_done = True
    # one product G = dy^T xa [N, R] reads dy once for all members' B gradients
    # (member j's gradient is its output rows - row blocks when interleaved - and
    # rank columns of G); one accumulating product per member would re-read dy and
    # costs cuBLAS ~14 us each at 8192 tokens even for the 4 MB k / v gradients
    if G is None and not gB_done and any(need_params[2 * j + 1] for j in range(len(group.members))):
        G = torch.mm(dy.t(), xa, out_dtype=torch.float32)
    for j, mem in enumerate(group.members):
        r0, r1 = group.rank_off[j], group.rank_off[j + 1]
        o0, o1 = group.out_off[j], group.out_off[j + 1]
        gA = gB = None
        if need_params[2 * j] and not gA_done:
            gA = _accumulate_grad(mem.lora_A, dxa[:, r0:r1].t(), x2, mem.scaling)
        if need_params[2 * j + 1] and not gB_done:
            if G is not None:
                if group.interleaved:
                    part = group._il_view(G, group.r_total)[:, j, :, r0:r1]
                else:
                    part = G[o0:o1, r0:r1]
                g = mem.lora_B.grad
                if g is not None and g.is_cuda and g.dtype == torch.float32 and g.is_contiguous():
                    g.view(part.shape).add_(part)
                else:
                    gB = part.reshape(group.outs[j], r1 - r0).to(mem.lora_B.dtype)
            else:
                gB = _accumulate_grad(mem.lora_B, dy[:, o0:o1].t(), xa[:, r0:r1], 1.0)
        grads += [gA, gB]
    return dx, grads


class _LoRAGroupFn(torch.autograd.Function):
    """Outputs of a projection group (see LoRAProjectionGroup) for input x."""

    @staticmethod
    def forward(ctx, x, group, *params):
        k = group.in_features
        x2 = x.reshape(-1, k)
        w = group.base_weight(x.dtype)
        As16, Bblk = group.factors(x.dtype)
        xa, xaT = _rank_product(x2, As16)
        y, xa = _group_gemm(group, x2, w, As16, Bblk, xa)
        ctx.save_for_backward(x2, xa, As16, Bblk, xaT)
        ctx.w = _keep(w)
        ctx.group = group
        ctx.lead = x.shape[:-1]
        outs = tuple(y[:, a:b].view(*x.shape[:-1], b - a)
                     for a, b in zip(group.out_off[:-1], group.out_off[1:]))
        return outs

    @staticmethod
    def backward(ctx, *douts):
        x2, xa, As16, Bblk, xaT = ctx.saved_tensors
        group = ctx.group
        m = x2.shape[0]
        parts = [d.reshape(m, n) if d is not None else torch.zeros(m, n, device=x2.device, dtype=x2.dtype)
                 for d, n in zip(douts, group.outs)]
        dy = torch.cat(parts, dim=1)
        w = None
        if ctx.needs_input_grad[0]:
            w = ctx.w if ctx.w is not None and ctx.w.dtype == dy.dtype else group.base_weight(dy.dtype)
        ctx.w = None
        dx, grads = _group_backward(group, dy, x2, xa, w, As16, Bblk, ctx.needs_input_grad[0],
                                    ctx.needs_input_grad[2:], xaT)
        if dx is not None:
            dx = dx.view(*ctx.lead, x2.shape[1])
        return (dx, None, *grads)


def _gu_views(group: LoRAProjectionGroup, y: torch.Tensor):
    """(g, u) row views of a gate/up output [M, 2 * inter]: column halves, or, with
    interleaved rows, [M * blocks, 2 * IL_BLOCK] rows split in half."""
    inter = group.outs[0]
    if group.interleaved:
        y2 = y.view(-1, 2 * IL_BLOCK)
        return y2[:, :IL_BLOCK], y2[:, IL_BLOCK:]
    return y[:, :inter], y[:, inter:]


def swiglu_gemm(x2, w, xa, Bblk, bias, mode: int, h, y=None):
    """soup_gemm_bf16_lora_swiglu: the interleaved gate/up GEMM with SwiGLU (mode 0:
    h = silu(g) u, optionally [g | u] into y) or its backward (mode 1: h holds dh,
    dg / du into y) in the epilogue."""
    m, k = x2.shape
    inter = w.shape[0] // 2
    _lib.call("soup_gemm_bf16_lora_swiglu", x2.device, x2.data_ptr(), x2.stride(0), w.data_ptr(),
              w.stride(0), xa.data_ptr(), xa.stride(0), Bblk.data_ptr(), Bblk.stride(0), xa.shape[1],
              None if bias is None else bias.data_ptr(), mode, h.data_ptr(), h.stride(0),
              None if y is None else y.data_ptr(), 0 if y is None else y.stride(0), m, inter, k,
              _lib.stream_of(x2))


def dswiglu_gemm(d2, w, dxa, As16, y):
    """soup_gemm_bf16_lora_dswiglu: dh = d2 W + dxa As (the down projection's input
    gradient) with the SwiGLU backward in the epilogue: [g | u] in y (the
    interleaved layout of swiglu_gemm) is overwritten by [dg | du]."""
    m, k = d2.shape
    inter = w.shape[1]
    _lib.call("soup_gemm_bf16_lora_dswiglu", d2.device, d2.data_ptr(), d2.stride(0), w.data_ptr(),
              w.stride(0), dxa.data_ptr(), dxa.stride(0), As16.data_ptr(), As16.stride(0),
              dxa.shape[1], y.data_ptr(), y.stride(0), m, inter, k, _lib.stream_of(d2))


def _swiglu_fused_ok(group, x2, w, xa, Bblk, bias, *outs) -> bool:
    return (group.interleaved and _fused_ok(x2.shape[1], x2, w, xa, Bblk,
                                            bias.view(1, -1) if bias is not None else None, *outs))


class _LoRAGateUpFn(torch.autograd.Function):
    """h = silu(g) * u with [g | u] = one group GEMM of x (gate/up group).

    With interleaved gate/up rows the SwiGLU runs in the GEMM epilogue
    (soup_gemm_bf16_lora_swiglu): the forward writes only h, and the
    recompute-backward turns dh straight into [dg | du] without storing g, u.
    With ``recompute`` the forward keeps only x and the rank-R product xa; the
    backward dequantises the weights once for the recompute and dx. Without it
    [g | u] is kept from the forward.
    """

    @staticmethod
    def forward(ctx, x, group, recompute, *params):
        from .kernels.swiglu import swiglu_forward

        k = group.in_features
        inter = group.outs[0]
        x2 = x.reshape(-1, k)
        m = x2.shape[0]
        w = group.base_weight(x.dtype)
        As16, Bblk = group.factors(x.dtype)
        bias = None if group.bias is None else group.bias.to(x2.dtype)
        h = torch.empty(m, inter, device=x.device, dtype=x.dtype)
        y = None
        xa, xaT = _rank_product(x2, As16)
        if _swiglu_fused_ok(group, x2, w, xa, Bblk, bias, h):
            if not recompute:
                y = torch.empty(m, group.n_total, device=x.device, dtype=x.dtype)
            swiglu_gemm(x2, w, xa, Bblk, bias, 0, h, y)
        else:
            y, _ = _group_gemm(group, x2, w, As16, Bblk, xa)
            g, u = _gu_views(group, y)
            swiglu_forward(g, u, out=h.view(g.shape[0], g.shape[1]))
        ctx.recompute = recompute
        ctx.w = _keep(w)
        if recompute:
            ctx.save_for_backward(x2, xa, As16, Bblk, xaT)
        else:
            ctx.save_for_backward(x2, xa, As16, Bblk, xaT, y)
        ctx.group = group
        ctx.lead = x.shape[:-1]
        return h.view(*x.shape[:-1], inter)

    @staticmethod
    def backward(ctx, dh):
        from .kernels.swiglu import swiglu_backward

        group = ctx.group
        saved = ctx.saved_tensors
        x2, xa, As16, Bblk, xaT = saved[:5]
        inter = group.outs[0]
        w = ctx.w if ctx.w is not None and ctx.w.dtype == x2.dtype else group.base_weight(x2.dtype)
        ctx.w = None
        dh2 = dh.reshape(-1, inter)
        if dh2.stride(1) != 1 or dh2.stride(0) != inter:
            dh2 = dh2.contiguous()
        if dh2.dtype != x2.dtype:
            dh2 = dh2.to(x2.dtype)
        bias = None if group.bias is None else group.bias.to(x2.dtype)
        dy = torch.empty(x2.shape[0], group.n_total, device=x2.device, dtype=x2.dtype)
        if ctx.recompute and _swiglu_fused_ok(group, x2, w, xa, Bblk, bias, dh2, dy):
            swiglu_gemm(x2, w, xa, Bblk, bias, 1, dh2, dy)
        else:
            if ctx.recompute:
                y, _ = _group_gemm(group, x2, w, As16, Bblk, xa)
            else:
                y = saved[5]
            g, u = _gu_views(group, y)
            dg, du = _gu_views(group, dy)
            swiglu_backward(dh2.view(g.shape[0], g.shape[1]), g, u, dg=dg, du=du)
        dx, grads = _group_backward(group, dy, x2, xa, w, As16, Bblk, ctx.needs_input_grad[0],
                                    ctx.needs_input_grad[3:], xaT)
        if dx is not None:
            dx = dx.view(*ctx.lead, x2.shape[1])
        return (dx, None, None, *grads)


#: Run the MLP (gate/up + SwiGLU + down_proj) as one autograd Function whose
#: backward puts the SwiGLU backward into the epilogue of the down projection's
#: input-gradient GEMM, when the MLP keeps [g | u] (no recompute). False keeps
#: two Functions (down_proj's backward writes dh, the gate/up backward runs the
#: SwiGLU backward as an elementwise pass); results are bit-identical.
FUSE_MLP_BACKWARD = True


class _LoRAMLPFn(torch.autograd.Function):
    """out = down(silu(g) u) with [g | u] = the gate/up group GEMM of x and down a
    LoRA linear, as one Function (see FUSE_MLP_BACKWARD).

    Forward: the gate/up GEMM with the SwiGLU epilogue writes h and keeps [g | u]
    (soup_gemm_bf16_lora_swiglu), then down's GEMM as in _LoRALinearFn. Backward:
    dxa_down = dout B_down, then [dg | du] = SwiGLU'(dout W_down + dxa_down As_down)
    in place of [g | u] (soup_gemm_bf16_lora_dswiglu: dh never reaches memory),
    down's LoRA gradients, then the gate/up group backward.
    """

    @staticmethod
    def forward(ctx, x, group, down, A_d, B_d, *params):
        k = group.in_features
        inter = group.outs[0]
        x2 = x.reshape(-1, k)
        m = x2.shape[0]
        w = group.base_weight(x.dtype)
        As16, Bblk = group.factors(x.dtype)
        bias = None if group.bias is None else group.bias.to(x2.dtype)
        h = torch.empty(m, inter, device=x.device, dtype=x.dtype)
        y = torch.empty(m, group.n_total, device=x.device, dtype=x.dtype)
        xa, xaT = _rank_product(x2, As16)
        if _swiglu_fused_ok(group, x2, w, xa, Bblk, bias, h, y):
            swiglu_gemm(x2, w, xa, Bblk, bias, 0, h, y)
        else:
            from .kernels.swiglu import swiglu_forward

            y, _ = _group_gemm(group, x2, w, As16, Bblk, xa)
            g, u = _gu_views(group, y)
            swiglu_forward(g, u, out=h.view(g.shape[0], g.shape[1]))
        # down: as _LoRALinearFn.forward
        as16_d, b16_d, bt16_d = down.lora_As16, down.lora_B16, down.lora_Bt16
        if as16_d is None or as16_d.dtype != x.dtype:
            as16_d = (down.lora_A.detach() * down.scaling).to(x.dtype)
            b16_d = down.lora_B.detach().to(x.dtype)
            bt16_d = None
        bias_d = None if down.bias is None else down.bias.to(x.dtype)
        w_d = down.base_weight(x.dtype)
        xa_d, xa_dT = _rank_product(h, as16_d)
        n_out = w_d.shape[0]
        if _fused_ok(inter, h, w_d, xa_d, b16_d, bias_d.view(1, -1) if bias_d is not None else None,
                     n=n_out):
            out = lora_gemm(h, w_d, False, xa_d, b16_d,
                            torch.empty(m, n_out, device=x.device, dtype=x.dtype), bias_d)
        else:
            out = F.linear(h, w_d, bias_d)
            out.addmm_(xa_d, b16_d.t())
        ctx.save_for_backward(x2, xa, As16, Bblk, y, h, xa_d, as16_d, b16_d, xaT, xa_dT, bt16_d)
        ctx.w = _keep(w)
        ctx.w_d = _keep(w_d)
        ctx.group = group
        ctx.down = down
        ctx.lead = x.shape[:-1]
        return out.view(*x.shape[:-1], n_out)

    @staticmethod
    def backward(ctx, dout):
        from .kernels.swiglu import swiglu_backward

        x2, xa, As16, Bblk, y, h, xa_d, as16_d, b16_d, xaT, xa_dT, bt16_d = ctx.saved_tensors
        group, down = ctx.group, ctx.down
        d2 = dout.reshape(-1, dout.shape[-1])
        if d2.stride(1) != 1 or d2.stride(0) != d2.shape[1]:
            d2 = d2.contiguous()
        if d2.dtype != x2.dtype:
            d2 = d2.to(x2.dtype)
        w_d = ctx.w_d if ctx.w_d is not None and ctx.w_d.dtype == x2.dtype else down.base_weight(x2.dtype)
        w = ctx.w if ctx.w is not None and ctx.w.dtype == x2.dtype else group.base_weight(x2.dtype)
        ctx.w = ctx.w_d = None
        if xa_dT is not None:
            dxa_d, dxa_dT = _rank_product(d2, bt16_d if bt16_d is not None else b16_d.t().contiguous())
        else:
            dxa_d, dxa_dT = d2 @ b16_d, None
        if _fused_ok(d2.shape[1], d2, w_d, dxa_d, as16_d, y):
            dswiglu_gemm(d2, w_d, dxa_d, as16_d, y)
            dy = y  # [dg | du] over [g | u]
        else:
            dh = d2 @ w_d
            dh.addmm_(dxa_d, as16_d)
            dy = torch.empty_like(y)
            g, u = _gu_views(group, y)
            dg, du = _gu_views(group, dy)
            swiglu_backward(dh.view(g.shape[0], g.shape[1]), g, u, dg=dg, du=du)
        gA_d, gB_d = _lora_grads(down.lora_A, down.lora_B, h, d2, xa_d, xa_dT, dxa_d, dxa_dT, down.scaling,
                                 ctx.needs_input_grad[3], ctx.needs_input_grad[4])
        dx, grads = _group_backward(group, dy, x2, xa, w, As16, Bblk, ctx.needs_input_grad[0],
                                    ctx.needs_input_grad[5:], xaT)
        if dx is not None:
            dx = dx.view(*ctx.lead, x2.shape[1])
        return (dx, None, None, gA_d, gB_d, *grads)


def group_projections(model, kinds=("qkv", "gate_up")):
    """Group each decoder layer's q/k/v and gate/up LoRA projections (see
    LoRAProjectionGroup). Returns the groups."""
    groups = []
    for layer in model.model.layers:
        sets = []
        if "qkv" in kinds:
            sets.append(("qkv", [getattr(layer.self_attn, n, None) for n in ("q_proj", "k_proj", "v_proj")]))
        if "gate_up" in kinds:
            sets.append(("gate_up", [getattr(layer.mlp, n, None) for n in ("gate_proj", "up_proj")]))
        for kind, mods in sets:
            if all(isinstance(m, (LoRANF4Linear, LoRADenseLinear)) for m in mods) and \
                    len({type(m) for m in mods}) == 1 and \
                    len({m.in_features for m in mods}) == 1 and \
                    all(getattr(m, "lora_group", None) is None for m in mods):
                groups.append(LoRAProjectionGroup(mods, kind))
    return groups


def qwen2_1p5b_config(num_layers: int = 28, attention: str = "sdpa", **overrides):
    """Qwen2.5-1.5B shapes with ``num_layers`` decoder layers.

    attention: ``"sdpa"`` (transformers' SDPA, cuDNN on B200; the default: it is
    faster than this library's kernels at the step's shapes) or ``"soup"``
    (the tcgen05 flash attention of ``kernels.attention``, registered with
    transformers under its interface name)."""
    from transformers import Qwen2Config

    kw = dict(hidden_size=1536, intermediate_size=8960, num_hidden_layers=num_layers,
              num_attention_heads=12, num_key_value_heads=2, vocab_size=151936,
              tie_word_embeddings=True, rms_norm_eps=1e-6, max_position_embeddings=32768,
              rope_parameters={"rope_theta": 1000000.0, "rope_type": "default"},
              initializer_range=0.02, hidden_act="silu", use_cache=False)
    kw.update(overrides)
    cfg = Qwen2Config(**kw)
    if attention == "soup":
        from .kernels.attention import register

        cfg._attn_implementation = register()
    elif attention == "sdpa":
        cfg._attn_implementation = "sdpa"
    else:
        raise ValueError(f"attention must be 'sdpa' or 'soup', not {attention!r}")
    return cfg


def build_qwen2_qlora(config=None, device="cuda", seed: int = 0, r: int = 16, alpha: int = 32,
                      targets: Iterable[str] = LORA_TARGETS, quantize: bool = True,
                      dtype: torch.dtype = torch.bfloat16, group: bool = True):
    """Randomly initialised Qwen2 model with (NF4 +) LoRA on the target linears.

    quantize=False keeps dense frozen base weights (CPU runs and tests).
    group=True computes each layer's q/k/v and gate/up projections as one GEMM
    each on CUDA (LoRAProjectionGroup); parameters and names are unchanged.
    """
    from transformers import Qwen2ForCausalLM

    cfg = config or qwen2_1p5b_config()
    torch.manual_seed(seed)
    with torch.device(device):
        model = Qwen2ForCausalLM(cfg)
    model.to(dtype)
    wrap = LoRANF4Linear if quantize else LoRADenseLinear
    # LoRA factors get their own seed point, independent of how much of the
    # global RNG the model construction consumed; every rank starts from the
    # same adapters.
    torch.manual_seed(seed + 1)
    for p in model.parameters():
        p.requires_grad_(False)
    targets = list(dict.fromkeys(targets))  # fixed order: the LoRA init draws depend on it
    for layer in model.model.layers:
        for parent in (layer.self_attn, layer.mlp):
            for name in targets:
                lin = getattr(parent, name, None)
                if isinstance(lin, torch.nn.Linear):
                    setattr(parent, name, wrap(lin, r, alpha))
    if group:
        group_projections(model)
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    return model


def lora_parameters(model) -> list:
    return [p for p in model.parameters() if p.requires_grad]


def causal_labels(input_ids: torch.Tensor, ignore_index: int = -100) -> torch.Tensor:
    """Next-token labels: labels[:, t] = ids[:, t+1], the last position ignored."""
    labels = torch.full_like(input_ids, ignore_index)
    labels[:, :-1] = input_ids[:, 1:]
    return labels


class QLoRATrainer:
    """Forward (fused ops) -> fused head CE -> backward -> gradient all-reduce -> AdamW.

    The LoRA gradients live in one flat fp32 buffer (each parameter's ``.grad``
    is a view of it). With ``ddp=True`` (an initialised process group, one
    process per GPU) the whole buffer is averaged over ranks by a single
    all-reduce after backward: 73.9 MB for the 1.5B model's 18.5 M LoRA
    parameters, a fraction of a millisecond over NVLink, so it is not worth
    overlapping with the backward pass. Everything in :meth:`step` is GPU work
    with no host synchronisation, so :meth:`capture` can record one whole step
    (forward, backward, all-reduce, AdamW) as a CUDA graph and :meth:`replay`
    re-launches it with a single call.
    """

    def __init__(self, model, lr: float = 2e-4, chunk: int = 64, ddp: bool = False,
                 loss_fn=None, fused_adamw: Optional[bool] = None, weight_decay: float = 0.0,
                 optimizer: str = "auto"):
        from .kernels import make_triton_chunked_loss_function

        self.model = model
        self.params = lora_parameters(model)
        self.body = model.model
        self.ddp = ddp
        if ddp:
            import torch.distributed as dist

            assert dist.is_initialized(), "ddp=True needs an initialised process group"
            self.world = dist.get_world_size()
            self.nccl = dist.get_backend() == "nccl"
            for p in self.params:  # every rank starts from rank 0's adapters
                dist.broadcast(p.data, src=0)
        else:
            self.world = 1
        dev = self.params[0].device
        # Parameters, gradients and the 16-bit copies the forward uses are views
        # of flat buffers: one all-reduce for the gradients, two kernels per
        # step to refresh the copies. The A factors come first (their copies
        # hold (alpha/r) * A), then everything else.
        lora = [m for m in model.modules() if isinstance(m, _LoRABase) and m.lora_A.requires_grad]
        a_ids = {id(m.lora_A) for m in lora}
        order = [p for p in self.params if id(p) in a_ids] + [p for p in self.params if id(p) not in a_ids]
        self.n_a = sum(p.numel() for p in order if id(p) in a_ids)
        scalings = {m.scaling for m in lora}
        self.scaling = scalings.pop() if len(scalings) == 1 else None
        total = sum(p.numel() for p in order)
        self.flat_param = torch.empty(total, dtype=torch.float32, device=dev)
        self.flat_grad = torch.zeros(total, dtype=torch.float32, device=dev)
        act_dtype = model.get_input_embeddings().weight.dtype
        self.flat_param16 = (torch.empty(total, dtype=act_dtype, device=dev)
                             if act_dtype in (torch.bfloat16, torch.float16) and self.scaling is not None
                             else None)
        views16 = {}
        offsets = {}
        off = 0
        for p in order:
            n = p.numel()
            self.flat_param[off:off + n].copy_(p.data.reshape(-1))
            p.data = self.flat_param[off:off + n].view_as(p)
            p.grad = self.flat_grad[off:off + n].view_as(p)
            offsets[id(p)] = off
            if self.flat_param16 is not None:
                views16[id(p)] = self.flat_param16[off:off + n].view_as(p)
            off += n
        self._bblk_copies = []
        self._t_copies = []
        if self.flat_param16 is not None:
            for m in lora:
                if id(m.lora_B) in views16:
                    m.lora_As16 = views16[id(m.lora_A)]
                    m.lora_B16 = views16[id(m.lora_B)]
            self._setup_groups(lora, offsets)
            self._setup_bt(lora, offsets)
            self._refresh_param16()
        on_cuda = self.params[0].is_cuda
        # AdamW (HF Trainer defaults: betas 0.9 / 0.999, eps 1e-8, weight decay 0).
        # "soup": one soup_adamw_flat launch over the flat buffers that also
        # writes the 16-bit copies; "torch": torch.optim.AdamW; "auto": soup on CUDA.
        if optimizer not in ("auto", "soup", "torch"):
            raise ValueError(f"optimizer must be auto, soup or torch, not {optimizer!r}")
        self.lr, self.betas, self.eps, self.weight_decay = lr, (0.9, 0.999), 1e-8, weight_decay
        if optimizer == "soup" or (optimizer == "auto" and on_cuda):
            if not on_cuda:
                raise ValueError("optimizer='soup' needs CUDA parameters")
            self.exp_avg = torch.zeros_like(self.flat_param)
            self.exp_avg_sq = torch.zeros_like(self.flat_param)
            self.step_t = torch.zeros((), dtype=torch.float32, device=dev)
            self.opt = None
        else:
            fused = on_cuda if fused_adamw is None else fused_adamw
            self.opt = torch.optim.AdamW(self.params, lr=lr, betas=self.betas, eps=self.eps,
                                         weight_decay=weight_decay, fused=fused, capturable=on_cuda)
        # loss_fn: an autograd Function with the reference's chunked-loss signature
        self.loss_fn = loss_fn or make_triton_chunked_loss_function()
        self.chunk = chunk
        self.graph = None
        # prepared per-layer-type masks: None = plain causal (full attention only)
        types = set(getattr(model.config, "layer_types", None) or ["full_attention"])
        self._no_mask = {"full_attention": None} if types == {"full_attention"} else None
        model.train()

    def _allreduce_grads(self):
        import torch.distributed as dist

        if self.nccl:
            dist.all_reduce(self.flat_grad, op=dist.ReduceOp.AVG)
        else:  # gloo has no AVG
            dist.all_reduce(self.flat_grad, op=dist.ReduceOp.SUM)
            self.flat_grad.mul_(1.0 / self.world)

    def step(self, input_ids: torch.Tensor, labels: torch.Tensor, denominator: float):
        self.flat_grad.zero_()
        self._refresh_param16()  # the factors may have been changed outside the trainer
        # Batches here are unpadded single sequences, so the attention mask is
        # exactly the causal pattern. Handing transformers a prepared "no mask"
        # keeps SDPA on is_causal with grouped K/V heads also while a CUDA graph
        # is captured: its own mask builder cannot inspect position ids during
        # stream capture and then materialises a [B, 1, S, S] mask, which makes
        # SDPA expand K/V to every query head and use a masked kernel (about 3x
        # slower on B200 at S=2048).
        out = self.body(input_ids=input_ids, attention_mask=self._no_mask)
        hidden = out.last_hidden_state if hasattr(out, "last_hidden_state") else out[0]
        loss, entropy, token_loss, correct = self.loss_fn.apply(
            hidden, self.model.lm_head, labels, self.chunk, denominator, -100, True)
        loss.backward()
        if self.ddp:
            self._allreduce_grads()
        if self.opt is None:
            self._adamw_step()  # also rewrites the 16-bit copies
            self._refresh_bblk()
        else:
            self.opt.step()
            self._refresh_param16()  # forwards outside the trainer see the updated factors
        return loss.detach(), correct

    def _adamw_step(self):
        self.step_t.add_(1.0)
        p16 = self.flat_param16
        b1, b2 = self.betas
        dev = self.flat_param.device
        _lib.call("soup_adamw_flat", dev, self.flat_param.data_ptr(), self.flat_grad.data_ptr(),
                  self.exp_avg.data_ptr(), self.exp_avg_sq.data_ptr(), self.flat_param.numel(),
                  self.step_t.data_ptr(), self.lr, b1, b2, self.eps, self.weight_decay,
                  None if p16 is None else p16.data_ptr(),
                  _lib.dtype_code(p16.dtype) if p16 is not None else _lib.BF16,
                  self.n_a if p16 is not None else 0, float(self.scaling or 1.0),
                  _lib.stream_of(self.flat_param))

    def _setup_groups(self, lora, offsets):
        """Give every projection group (LoRAProjectionGroup) views of the flat
        buffers: its stacked 16-bit scaled A factors and their fp32 gradient
        (the members' A factors are adjacent in the flat order), and a
        block-diagonal 16-bit B. Groups of one structure (every decoder layer's
        q/k/v, every layer's gate/up) share one [layers, N, R] buffer, and when
        their members' B factors sit at a fixed stride in the flat buffer the
        refresh is one strided copy per member position for all layers."""
        groups = []
        for m in lora:
            g = m.lora_group
            if g is not None and all(x is not g for x in groups):
                groups.append(g)
        dev = self.flat_param.device
        self._bblk_copies = []
        kinds = {}
        for g in groups:
            a_offs = [offsets.get(id(mm.lora_A)) for mm in g.members]
            b_offs = [offsets.get(id(mm.lora_B)) for mm in g.members]
            if any(o is None for o in a_offs + b_offs) or any(
                    a_offs[j + 1] != a_offs[j] + g.members[j].lora_A.numel() for j in range(len(a_offs) - 1)):
                continue
            n_a = g.r_total * g.in_features
            g.As16 = self.flat_param16[a_offs[0]:a_offs[0] + n_a].view(g.r_total, g.in_features)
            g.gradA = self.flat_grad[a_offs[0]:a_offs[0] + n_a].view(g.r_total, g.in_features)
            key = (g.kind, tuple(g.outs), tuple(g.ranks), g.in_features, g.interleaved)
            kinds.setdefault(key, []).append((g, b_offs))
        for key, items in kinds.items():
            g0 = items[0][0]
            buf = torch.zeros(len(items), g0.n_total, g0.r_total, dtype=self.flat_param16.dtype, device=dev)
            buf_t = torch.zeros(len(items), g0.r_total, g0.n_total, dtype=self.flat_param16.dtype, device=dev)
            for l, (g, _) in enumerate(items):
                g.Bblk16 = buf[l]
                g.BblkT16 = buf_t[l]
            self._t_copies.append((buf_t, buf.transpose(1, 2)))
            L, R = len(items), g0.r_total
            for j in range(len(g0.members)):
                n_j, r_j = g0.outs[j], g0.ranks[j]
                o0, c0 = g0.out_off[j], g0.rank_off[j]
                offs = [b[j] for _, b in items]
                stride = offs[1] - offs[0] if len(offs) > 1 else n_j * r_j
                # member j's rows of the block-diagonal B: a contiguous row range, or
                # (interleaved gate/up) every other block of IL_BLOCK rows
                if g0.interleaved:
                    nb = n_j // IL_BLOCK
                    dst_all = buf.view(L, nb, 2, IL_BLOCK, R)[:, :, j, :, c0:c0 + r_j]
                    src_shape = (nb, IL_BLOCK, r_j)
                else:
                    dst_all = buf[:, o0:o0 + n_j, c0:c0 + r_j]
                    src_shape = (n_j, r_j)
                if all(offs[l] == offs[0] + l * stride for l in range(len(offs))):
                    inner = tuple(int(np.prod(src_shape[d + 1:])) for d in range(len(src_shape)))
                    src = self.flat_param16.as_strided((L, *src_shape), (stride, *inner), offs[0])
                    self._bblk_copies.append((dst_all, src))
                else:
                    for l, off in enumerate(offs):
                        src = self.flat_param16[off:off + n_j * r_j].view(src_shape)
                        self._bblk_copies.append((dst_all[l], src))

    def _setup_bt(self, lora, offsets):
        """Transposed 16-bit B copies [r, out] of the ungrouped LoRA linears (the
        operand of dxa = dy B in soup_lora_rank_gemm): one [layers, r, out] buffer
        per shape, refreshed by one strided copy when the factors sit at a fixed
        stride in the flat buffer."""
        kinds = {}
        for m in lora:
            if m.lora_group is None and m.lora_B16 is not None and id(m.lora_B) in offsets:
                kinds.setdefault((m.out_features, m.lora_B.shape[1]), []).append(m)
        dev = self.flat_param.device
        for (n, r), mods in kinds.items():
            L = len(mods)
            buf = torch.empty(L, r, n, dtype=self.flat_param16.dtype, device=dev)
            for l, m in enumerate(mods):
                m.lora_Bt16 = buf[l]
            offs = [offsets[id(m.lora_B)] for m in mods]
            stride = offs[1] - offs[0] if L > 1 else n * r
            if all(offs[l] == offs[0] + l * stride for l in range(L)):
                src = self.flat_param16.as_strided((L, n, r), (stride, r, 1), offs[0])
                self._t_copies.append((buf, src.transpose(1, 2)))
            else:
                for l, m in enumerate(mods):
                    self._t_copies.append((buf[l], m.lora_B16.t()))

    def _refresh_param16(self):
        if self.flat_param16 is not None:
            na = self.n_a
            torch.mul(self.flat_param[:na], self.scaling, out=self.flat_param16[:na])
            self.flat_param16[na:].copy_(self.flat_param[na:])
            self._refresh_bblk()

    def _refresh_bblk(self):
        for dst, src in self._bblk_copies:
            dst.copy_(src)
        # the transposed copies: operands of the rank kernels and of the dual
        # product (after the block-diagonal copies they read)
        if RANK_KERNELS or DUAL_RANK:
            for dst, src in self._t_copies:
                dst.copy_(src)

    def capture(self, input_ids: torch.Tensor, labels: torch.Tensor, denominator: float,
                warmup: int = 3):
        """Record one step on static `input_ids`/`labels` buffers as a CUDA graph.

        Later batches are copied into the same buffers before :meth:`replay`.
        `denominator` is baked into the graph (the count of non-ignored labels
        is the same for every batch of fixed shape without padding).
        """
        self.static_ids = input_ids
        self.static_labels = labels
        side = torch.cuda.Stream(input_ids.device)
        side.wait_stream(torch.cuda.current_stream(input_ids.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.step(input_ids, labels, denominator)
        torch.cuda.current_stream(input_ids.device).wait_stream(side)
        torch.cuda.synchronize(input_ids.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.static_loss, self.static_correct = self.step(input_ids, labels, denominator)
        return self.static_loss

    def replay(self):
        self.graph.replay()
        return self.static_loss, self.static_correct

    def save_adapter(self, directory: str, base_model_name_or_path: str = "Qwen/Qwen2.5-1.5B-Instruct"):
        """Write the LoRA factors as a PEFT adapter directory (see ``adapter.save_adapter``)."""
        from .adapter import save_adapter

        return save_adapter(self.model, directory, base_model_name_or_path)

    def release_graph(self):
        """Drop the captured graph (do this before destroying the process group)."""
        self.graph = None
