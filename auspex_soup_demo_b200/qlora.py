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


# Contractions longer than this stay on cuBLAS plus an accumulating rank-r
# GEMM: measured on B200 at 2048 and 8192 tokens, the one-GEMM tcgen05 path
# wins for every Qwen2.5-1.5B projection with K = 1536 (q/k/v/o, gate/up
# forward, down backward) and loses for K = 8960 (down forward, gate/up
# backward), where the output is narrow, the extra pass over it cheap, and
# the persistent kernel's last wave of 256 x 256 tiles mostly idle.
FUSED_MAX_K = 4096


def _fused_ok(k: int, *ts: torch.Tensor) -> bool:
    if k > FUSED_MAX_K:
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
    def forward(ctx, x, A, B, As16, B16, scaling, weight_fn, bias):
        w = weight_fn(x.dtype)
        x2 = x.reshape(-1, x.shape[-1])
        xa = x2 @ As16.t()
        m, n = x2.shape[0], w.shape[0]
        if _fused_ok(x2.shape[1], x2, w, xa, B16, bias.view(1, -1) if bias is not None else None):
            y2 = lora_gemm(x2, w, False, xa, B16, torch.empty(m, n, device=x.device, dtype=x.dtype), bias)
            y = y2.view(*x.shape[:-1], n)
        else:
            y = F.linear(x, w, bias)
            y.view(-1, n).addmm_(xa, B16.t())
        ctx.save_for_backward(x, xa, As16, B16)
        ctx.params = (A, B)
        ctx.scaling = scaling
        ctx.weight_fn = weight_fn
        return y

    @staticmethod
    def backward(ctx, dy):
        x, xa, As16, B16 = ctx.saved_tensors
        A, B = ctx.params
        s = ctx.scaling
        dy2 = dy.reshape(-1, dy.shape[-1])
        if dy2.stride(1) != 1:
            dy2 = dy2.contiguous()
        x2 = x.reshape(-1, x.shape[-1])
        dxa = dy2 @ B16
        dx = gA = gB = None
        if ctx.needs_input_grad[0]:
            w = ctx.weight_fn(dy.dtype)
            m, n = dy2.shape[0], w.shape[1]
            if _fused_ok(dy2.shape[1], dy2, w, dxa, As16):
                dx2 = lora_gemm(dy2, w, True, dxa, As16, torch.empty(m, n, device=dy.device, dtype=dy.dtype))
            else:
                dx2 = dy2 @ w
                dx2.addmm_(dxa, As16)
            dx = dx2.view(x.shape)
        if ctx.needs_input_grad[1]:
            gA = _accumulate_grad(A, dxa.t(), x2, s)
        if ctx.needs_input_grad[2]:
            gB = _accumulate_grad(B, dy2.t(), xa, 1.0)
        return dx, gA, gB, None, None, None, None, None


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

    def base_weight(self, dtype) -> torch.Tensor:
        raise NotImplementedError

    def forward(self, x):
        as16, b16 = self.lora_As16, self.lora_B16
        if as16 is None or as16.dtype != x.dtype:
            as16 = (self.lora_A.detach() * self.scaling).to(x.dtype)
            b16 = self.lora_B.detach().to(x.dtype)
        bias = None if self.bias is None else self.bias.to(x.dtype)
        return _LoRALinearFn.apply(x, self.lora_A, self.lora_B, as16, b16, self.scaling,
                                   self.base_weight, bias)


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
        return self.weight.to(dtype)


def qwen2_1p5b_config(num_layers: int = 28, **overrides):
    from transformers import Qwen2Config

    kw = dict(hidden_size=1536, intermediate_size=8960, num_hidden_layers=num_layers,
              num_attention_heads=12, num_key_value_heads=2, vocab_size=151936,
              tie_word_embeddings=True, rms_norm_eps=1e-6, max_position_embeddings=32768,
              rope_parameters={"rope_theta": 1000000.0, "rope_type": "default"},
              initializer_range=0.02, hidden_act="silu", use_cache=False)
    kw.update(overrides)
    cfg = Qwen2Config(**kw)
    cfg._attn_implementation = "sdpa"
    return cfg


def build_qwen2_qlora(config=None, device="cuda", seed: int = 0, r: int = 16, alpha: int = 32,
                      targets: Iterable[str] = LORA_TARGETS, quantize: bool = True,
                      dtype: torch.dtype = torch.bfloat16):
    """Randomly initialised Qwen2 model with (NF4 +) LoRA on the target linears.

    quantize=False keeps dense frozen base weights (CPU runs and tests).
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
                 loss_fn=None, fused_adamw: Optional[bool] = None):
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
        off = 0
        for p in order:
            n = p.numel()
            self.flat_param[off:off + n].copy_(p.data.reshape(-1))
            p.data = self.flat_param[off:off + n].view_as(p)
            p.grad = self.flat_grad[off:off + n].view_as(p)
            if self.flat_param16 is not None:
                views16[id(p)] = self.flat_param16[off:off + n].view_as(p)
            off += n
        if self.flat_param16 is not None:
            for m in lora:
                if id(m.lora_B) in views16:
                    m.lora_As16 = views16[id(m.lora_A)]
                    m.lora_B16 = views16[id(m.lora_B)]
            self._refresh_param16()
        on_cuda = self.params[0].is_cuda
        fused = on_cuda if fused_adamw is None else fused_adamw
        self.opt = torch.optim.AdamW(self.params, lr=lr, fused=fused, capturable=on_cuda)
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
        self.opt.step()
        self._refresh_param16()  # forwards outside the trainer see the updated factors
        return loss.detach(), correct

    def _refresh_param16(self):
        if self.flat_param16 is not None:
            na = self.n_a
            torch.mul(self.flat_param[:na], self.scaling, out=self.flat_param16[:na])
            self.flat_param16[na:].copy_(self.flat_param[na:])

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
