"""QLoRA training step on the Qwen2.5-1.5B architecture, driven through the fused ops.

The reference's workload (``task/task.yaml``): Qwen2.5-1.5B-Instruct, 4-bit NF4
base weights, LoRA r=16 / alpha=32, AdamW 2e-4, trained by Soup (TRL/HF
Trainer) with ``solution.apply()`` patches installed. Soup, PEFT and
bitsandbytes are not available here, so this module provides the pieces of that
step that surround the fused ops:

* :class:`LoRANF4Linear` - a frozen NF4 base weight (blocksize 64, our CUDA
  quantiser/dequantiser) plus trainable LoRA factors; the base weight is
  dequantised to bf16 for each use (forward and backward) and never stored;
* :func:`build_qwen2_qlora` - the Qwen2.5-1.5B architecture (28 layers, hidden
  1536, MLP 8960, 12 query / 2 KV heads of 128, vocab 151936, tied embeddings,
  rope theta 1e6) randomly initialised (N(0, 0.02)) with LoRA on
  q/k/v/o/gate/up/down;
* :class:`QLoRATrainer` - one optimiser step: transformer body (with the fused
  RMSNorm / RoPE / SwiGLU patches), fused head cross-entropy, backward, AdamW.
  With ``torch.distributed`` initialised (one process per GPU, NCCL), the body
  is wrapped in DistributedDataParallel: only the LoRA gradients exist, so only
  they are all-reduced, in buckets overlapped with the backward pass.
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


class _NF4LinearFn(torch.autograd.Function):
    """y = x W^T + b with W dequantised from NF4 on each use; W is frozen."""

    @staticmethod
    def forward(ctx, x, packed, absmax, bias, out_features, in_features):
        w = nf4_dequantize(packed, absmax, (out_features, in_features), dtype=x.dtype)
        y = F.linear(x, w, bias)
        ctx.save_for_backward(packed, absmax)
        ctx.shape = (out_features, in_features)
        return y

    @staticmethod
    def backward(ctx, dy):
        packed, absmax = ctx.saved_tensors
        dx = None
        if ctx.needs_input_grad[0]:
            w = nf4_dequantize(packed, absmax, ctx.shape, dtype=dy.dtype)
            dx = dy @ w
        return dx, None, None, None, None, None


def _add_lora(y: torch.Tensor, x: torch.Tensor, lora_a: torch.Tensor, lora_b: torch.Tensor,
              scaling: float) -> torch.Tensor:
    """y + scaling * (x A^T) B^T with the addition done by the GEMM (beta = 1).

    The scale is folded into the [out, r] factor and the rank-r product is
    accumulated onto y by one addmm, so no pass over the [tokens, out]
    activations is spent on scaling or adding.
    """
    xa = F.linear(x, lora_a.to(x.dtype))
    b = (lora_b * scaling).to(x.dtype)
    out = torch.addmm(y.reshape(-1, y.shape[-1]), xa.reshape(-1, xa.shape[-1]), b.t())
    return out.view(y.shape)


class LoRANF4Linear(torch.nn.Module):
    """Frozen NF4 base linear + trainable LoRA: y = base(x) + (alpha/r) * B(A(x))."""

    def __init__(self, linear: torch.nn.Linear, r: int = 16, alpha: int = 32,
                 lora_dtype: torch.dtype = torch.float32):
        super().__init__()
        self.in_features = linear.in_features
        self.out_features = linear.out_features
        packed, absmax = nf4_quantize(linear.weight)
        self.register_buffer("packed", packed)
        self.register_buffer("absmax", absmax)
        if linear.bias is not None:
            self.register_buffer("bias", linear.bias.detach().clone())
        else:
            self.bias = None
        dev = linear.weight.device
        self.lora_A = torch.nn.Parameter(torch.empty(r, self.in_features, device=dev, dtype=lora_dtype))
        self.lora_B = torch.nn.Parameter(torch.zeros(self.out_features, r, device=dev, dtype=lora_dtype))
        torch.nn.init.kaiming_uniform_(self.lora_A, a=math.sqrt(5))
        self.scaling = alpha / r

    def dequantized_weight(self, dtype=torch.bfloat16) -> torch.Tensor:
        return nf4_dequantize(self.packed, self.absmax, (self.out_features, self.in_features), dtype)

    def forward(self, x):
        y = _NF4LinearFn.apply(x, self.packed, self.absmax, self.bias, self.out_features,
                               self.in_features)
        return _add_lora(y, x, self.lora_A, self.lora_B, self.scaling)


class LoRADenseLinear(torch.nn.Module):
    """Frozen dense base linear + trainable LoRA (for non-quantised runs and CPU tests)."""

    def __init__(self, linear: torch.nn.Linear, r: int = 16, alpha: int = 32,
                 lora_dtype: torch.dtype = torch.float32):
        super().__init__()
        self.in_features = linear.in_features
        self.out_features = linear.out_features
        self.register_buffer("weight", linear.weight.detach().clone())
        if linear.bias is not None:
            self.register_buffer("bias", linear.bias.detach().clone())
        else:
            self.bias = None
        dev = linear.weight.device
        self.lora_A = torch.nn.Parameter(torch.empty(r, self.in_features, device=dev, dtype=lora_dtype))
        self.lora_B = torch.nn.Parameter(torch.zeros(self.out_features, r, device=dev, dtype=lora_dtype))
        torch.nn.init.kaiming_uniform_(self.lora_A, a=math.sqrt(5))
        self.scaling = alpha / r

    def forward(self, x):
        y = F.linear(x, self.weight.to(x.dtype), None if self.bias is None else self.bias.to(x.dtype))
        return _add_lora(y, x, self.lora_A, self.lora_B, self.scaling)


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
        total = sum(p.numel() for p in self.params)
        dev = self.params[0].device
        self.flat_grad = torch.zeros(total, dtype=torch.float32, device=dev)
        off = 0
        for p in self.params:
            p.grad = self.flat_grad[off:off + p.numel()].view_as(p)
            off += p.numel()
        on_cuda = self.params[0].is_cuda
        fused = on_cuda if fused_adamw is None else fused_adamw
        self.opt = torch.optim.AdamW(self.params, lr=lr, fused=fused, capturable=on_cuda)
        # loss_fn: an autograd Function with the reference's chunked-loss signature
        self.loss_fn = loss_fn or make_triton_chunked_loss_function()
        self.chunk = chunk
        self.graph = None
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
        out = self.body(input_ids=input_ids)
        hidden = out.last_hidden_state if hasattr(out, "last_hidden_state") else out[0]
        loss, entropy, token_loss, correct = self.loss_fn.apply(
            hidden, self.model.lm_head, labels, self.chunk, denominator, -100, True)
        loss.backward()
        if self.ddp:
            self._allreduce_grads()
        self.opt.step()
        return loss.detach(), correct

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
