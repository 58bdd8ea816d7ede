"""CPU eager formulation of the QLoRA train step (test infrastructure and CPU baseline only).

The reference trains Qwen2.5-1.5B-Instruct with 4-bit NF4 base weights and LoRA
r=16 / alpha=32 on q/k/v/o/gate/up/down (``task/task.yaml:3-22``) through the HF
Trainer, with ``solution.apply()`` installing its fused ops
(``solution/__init__.py:42-70``). Every patched forward falls back to
transformers' own eager code when its kernel cannot run
(``solution/kernels/rmsnorm.py:187-192``, ``rope.py:209-221``,
``swiglu.py:193-219``): that eager code is the reference's own CPU
implementation of the step. This module builds it in plain PyTorch on the host:

* ``Qwen2ForCausalLM`` with transformers' eager RMSNorm, rotate-half RoPE,
  SwiGLU MLP and SDPA attention (no patch installed);
* LoRA linears ``y = x W^T + (alpha/r) (x A^T) B^T`` over frozen dense bf16 base
  weights (bitsandbytes' per-use NF4 dequantisation is left out, which only
  makes this baseline faster);
* the head loss as the reference's chunked loop (``chunked_ce.py:267-313``):
  per 64-token chunk, logits ``h W^T`` in fp32, ``F.cross_entropy(sum)`` over
  the non-ignored labels, divided by their count;
* ``torch.optim.AdamW`` (lr 2e-4, the HF Trainer defaults otherwise).

It is the CPU arm that ``bench.py`` times; nothing in the package imports it.
"""

from __future__ import annotations

import math
import time

import torch
import torch.nn.functional as F

LORA_TARGETS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")

# Qwen2.5-1.5B shapes
HIDDEN, INTER, HEADS, KV_HEADS, HEAD_DIM, VOCAB = 1536, 8960, 12, 2, 128, 151936


class EagerLoRALinear(torch.nn.Module):
    """Frozen base linear + trainable LoRA factors, plain PyTorch ops."""

    def __init__(self, linear: torch.nn.Linear, r: int = 16, alpha: int = 32):
        super().__init__()
        self.weight = torch.nn.Parameter(linear.weight.detach().clone(), requires_grad=False)
        self.bias = (torch.nn.Parameter(linear.bias.detach().clone(), requires_grad=False)
                     if linear.bias is not None else None)
        self.lora_A = torch.nn.Parameter(torch.empty(r, linear.in_features))
        self.lora_B = torch.nn.Parameter(torch.zeros(linear.out_features, r))
        torch.nn.init.kaiming_uniform_(self.lora_A, a=math.sqrt(5))
        self.scaling = alpha / r

    def forward(self, x):
        y = F.linear(x, self.weight, self.bias)
        xa = F.linear(x, self.lora_A.to(x.dtype))
        return y + self.scaling * F.linear(xa, self.lora_B.to(x.dtype))


def qwen2_config(num_layers: int = 28):
    from transformers import Qwen2Config

    cfg = Qwen2Config(hidden_size=HIDDEN, intermediate_size=INTER, num_hidden_layers=num_layers,
                      num_attention_heads=HEADS, num_key_value_heads=KV_HEADS, vocab_size=VOCAB,
                      tie_word_embeddings=True, rms_norm_eps=1e-6, max_position_embeddings=32768,
                      rope_parameters={"rope_theta": 1000000.0, "rope_type": "default"},
                      initializer_range=0.02, hidden_act="silu", use_cache=False)
    cfg._attn_implementation = "sdpa"
    return cfg


def _fill_normal(t: torch.Tensor, std: float, gen: torch.Generator, block: int = 1 << 20):
    """t ~ N(0, std^2) from one random block of `block` values repeated over t.

    The host's random generator makes ~30 M values/s, so drawing the 1.5 B base
    weights one by one would take minutes; the step's timing and arithmetic do
    not depend on the weights being independent draws.
    """
    flat = t.view(-1)
    src = (torch.randn(min(block, flat.numel()), generator=gen) * std).to(t.dtype)
    for s in range(0, flat.numel(), src.numel()):
        n = min(src.numel(), flat.numel() - s)
        flat[s:s + n].copy_(src[:n])


def build_model(num_layers: int = 28, seed: int = 0, dtype=torch.bfloat16):
    """Random-init Qwen2.5-1.5B-architecture model on the CPU with LoRA on the 7 projections.

    Linear and embedding weights ~ N(0, 0.02) (repeated random blocks, see
    _fill_normal), RMSNorm weights 1, biases 0, as the model's own initialiser
    would set them.
    """
    from transformers import Qwen2ForCausalLM
    from transformers.models.qwen2.modeling_qwen2 import Qwen2RotaryEmbedding

    cfg = qwen2_config(num_layers)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(dtype)
    try:
        with torch.device("meta"):
            model = Qwen2ForCausalLM(cfg)
    finally:
        torch.set_default_dtype(prev)
    model = model.to_empty(device="cpu")
    gen = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("layernorm.weight") or name.endswith("norm.weight"):
                p.fill_(1.0)
            elif name.endswith(".bias"):
                p.zero_()
            else:
                _fill_normal(p, 0.02, gen)
    model.model.rotary_emb = Qwen2RotaryEmbedding(config=cfg)
    model.tie_weights()
    for p in model.parameters():
        p.requires_grad_(False)
    torch.manual_seed(seed + 1)
    for layer in model.model.layers:
        for parent in (layer.self_attn, layer.mlp):
            for name in LORA_TARGETS:
                lin = getattr(parent, name, None)
                if isinstance(lin, torch.nn.Linear):
                    setattr(parent, name, EagerLoRALinear(lin))
    model.train()
    return model


def chunked_head_loss(hidden, head_weight, labels, chunk: int = 64, ignore_index: int = -100):
    """Mean CE over the non-ignored labels, computed per sequence chunk on fp32 logits."""
    den = max(int((labels != ignore_index).sum()), 1)
    total = hidden.new_zeros((), dtype=torch.float32)
    for s in range(0, hidden.shape[1], chunk):
        h = hidden[:, s:s + chunk].reshape(-1, hidden.shape[-1])
        logits = F.linear(h, head_weight).float()
        total = total + F.cross_entropy(logits, labels[:, s:s + chunk].reshape(-1),
                                        ignore_index=ignore_index, reduction="sum")
    return total / den


class EagerQLoRAStep:
    """forward -> chunked head CE -> backward -> AdamW on the LoRA factors."""

    def __init__(self, model, lr: float = 2e-4):
        self.model = model
        self.params = [p for p in model.parameters() if p.requires_grad]
        self.opt = torch.optim.AdamW(self.params, lr=lr, betas=(0.9, 0.999), eps=1e-8,
                                     weight_decay=0.0)

    def step(self, input_ids, labels):
        self.opt.zero_grad(set_to_none=True)
        out = self.model.model(input_ids=input_ids)
        loss = chunked_head_loss(out.last_hidden_state, self.model.lm_head.weight, labels)
        loss.backward()
        self.opt.step()
        return float(loss.detach())


def causal_labels(input_ids, ignore_index: int = -100):
    labels = torch.full_like(input_ids, ignore_index)
    labels[:, :-1] = input_ids[:, 1:]
    return labels


def train_flop_per_token(seq: int, num_layers: int = 28, r: int = 16) -> float:
    """Algorithmic FLOPs of one trained token of the QLoRA step (frozen base, tied head).

    Base projections and the head: forward + input gradient, 2 x 2 x params.
    Causal attention: forward 4 * heads * head_dim * (seq + 1) / 2 per layer
    (QK^T and PV over the mean causal context), backward twice that. LoRA:
    forward 2 r (in + out) per projection, backward (dx, dA, dB) twice that
    again plus the forward's share: 6 r (in + out). MLP recompute, NF4
    dequantisation and the optimiser are not counted.
    """
    kv = KV_HEADS * HEAD_DIM
    lin = [(HIDDEN, HIDDEN), (HIDDEN, kv), (HIDDEN, kv), (HIDDEN, HIDDEN),
           (HIDDEN, INTER), (HIDDEN, INTER), (INTER, HIDDEN)]
    base = sum(i * o for i, o in lin)
    lora = sum(r * (i + o) for i, o in lin)
    attn_fwd = 4.0 * HEADS * HEAD_DIM * (seq + 1) / 2.0
    per_layer = 4.0 * base + 3.0 * attn_fwd + 6.0 * lora
    return num_layers * per_layer + 4.0 * VOCAB * HIDDEN


def time_steps(num_layers: int, batch: int, seq: int, steps: int, warmup: int, seed: int = 0,
               threads: int = 0):
    """Seconds per step of the eager CPU step on uniform random token ids."""
    if threads:
        torch.set_num_threads(threads)
    model = build_model(num_layers, seed)
    runner = EagerQLoRAStep(model)
    g = torch.Generator().manual_seed(1234)
    ids = torch.randint(0, VOCAB, (batch, seq), generator=g)
    labels = causal_labels(ids)
    loss = None
    for _ in range(warmup):
        loss = runner.step(ids, labels)
    t0 = time.perf_counter()
    for _ in range(steps):
        loss = runner.step(ids, labels)
    return (time.perf_counter() - t0) / max(steps, 1), loss
