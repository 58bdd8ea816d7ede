"""CPU restatement of the reference's fused-op arithmetic (test infrastructure only).

Every function computes in float32 from its (possibly lower-precision) inputs
and rounds once to the output dtype, in the operation order of the reference
kernel it cites. Reference paths are relative to the reference project root
(``solution/kernels/...``); ``modeling_qwen2.py`` lines refer to transformers
5.5.0 ``transformers/models/qwen2/modeling_qwen2.py``.

Parity status: pinned. ``tests/golden/make_golden.py`` runs the reference's own
Triton kernels on the CPU (Triton interpreter) on seeded inputs; the fixtures it
writes are checked against these functions in ``tests/test_oracle_golden.py``.
"""

from __future__ import annotations

import torch

IGNORE_INDEX = -100


# --------------------------------------------------------------------------
# RMSNorm
# --------------------------------------------------------------------------
def rmsnorm_fwd(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6):
    """y = (x * rstd) * w with rstd = 1 / sqrt(mean(x^2) + eps), fp32 math.

    Follows ``solution/kernels/rmsnorm.py:43-57`` (forward kernel) and the
    reference test formula ``solution/test_kernels.py:69-73``. Returns
    ``(y in x.dtype, rstd fp32 [rows])``; ``x`` is viewed as [rows, D].
    """
    shape = x.shape
    xf = x.reshape(-1, shape[-1]).float()
    var = (xf * xf).sum(-1) / shape[-1]
    rstd = 1.0 / torch.sqrt(var + eps)
    y = (xf * rstd[:, None]) * weight.float()[None, :]
    return y.to(x.dtype).reshape(shape), rstd


def rmsnorm_bwd(dy: torch.Tensor, x: torch.Tensor, weight: torch.Tensor, rstd: torch.Tensor):
    """dx = rstd * (dy*w - (x/D) * rstd^2 * sum(dy*w*x)); dw = sum_rows dy * x * rstd.

    dx follows ``solution/kernels/rmsnorm.py:83-96``; dw follows the eager
    reduction at ``rmsnorm.py:161-167`` (fp32, cast to the weight dtype).
    """
    shape = x.shape
    D = shape[-1]
    dyf = dy.reshape(-1, D).float()
    xf = x.reshape(-1, D).float()
    wf = weight.float()[None, :]
    r = rstd.float()[:, None]
    dyw = dyf * wf
    s = (dyw * xf).sum(-1, keepdim=True)
    dx = r * (dyw - (xf / D) * (r * r) * s)
    dw = (dyf * (xf * r)).sum(0)
    return dx.to(x.dtype).reshape(shape), dw.to(weight.dtype)


# --------------------------------------------------------------------------
# SwiGLU
# --------------------------------------------------------------------------
def swiglu_fwd(gate: torch.Tensor, up: torch.Tensor):
    """out = g * sigmoid(g) * u in fp32 (``solution/kernels/swiglu.py:36-44``)."""
    g = gate.float()
    u = up.float()
    sig = torch.sigmoid(g)
    return ((g * sig) * u).to(gate.dtype)


def swiglu_bwd(dy: torch.Tensor, gate: torch.Tensor, up: torch.Tensor):
    """du = dy * g * sig; dg = dy * u * sig * (1 + g * (1 - sig)).

    Follows ``solution/kernels/swiglu.py:75-89`` (sigmoid recomputed from gate).
    Returns ``(dgate, dup)`` in the input dtypes.
    """
    d = dy.float()
    g = gate.float()
    u = up.float()
    sig = torch.sigmoid(g)
    du = d * (g * sig)
    dg = d * u * sig * (1.0 + g * (1.0 - sig))
    return dg.to(gate.dtype), du.to(up.dtype)


# --------------------------------------------------------------------------
# RoPE (rotate-half layout)
# --------------------------------------------------------------------------
def rope_cos_sin(seq_len: int, head_dim: int, theta: float, dtype=torch.float32, positions=None):
    """cos/sin tables [S, D] as Qwen2RotaryEmbedding builds them.

    fp32 inverse frequencies and angles, ``cat(freqs, freqs)``, then a cast to
    the activation dtype (``modeling_qwen2.py:89-113``).
    """
    if positions is None:
        positions = torch.arange(seq_len)
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    freqs = positions.float()[:, None] * inv_freq[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def _rope_tables(cos: torch.Tensor, x: torch.Tensor):
    """Broadcast cos/sin ([B|1,1,S,D], [B|1,S,D] or [S,D]) to [B,1,S,D/2] fp32.

    Only the first half of the last dim is used, exactly as the reference
    kernel indexes ``cos_ptr + cols`` with ``cols < HALF_DIM``
    (``solution/kernels/rope.py:45-55``).
    """
    B, H, S, D = x.shape
    c = cos
    if c.dim() == 2:
        c = c[None, None]
    elif c.dim() == 3:
        c = c[:, None]
    c = c[..., : D // 2].float()
    return c.expand(B, 1, S, D // 2)


def rope_fwd(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """y1 = x1*c - x2*s, y2 = x1*s + x2*c (``solution/kernels/rope.py:52-67``).

    x is [B, H, S, D] (any strides). Equal to ``modeling_qwen2.py:144``
    ``q*cos + rotate_half(q)*sin`` when cos/sin halves are equal, as HF builds them.
    """
    D = x.shape[-1]
    h = D // 2
    c = _rope_tables(cos, x)
    s = _rope_tables(sin, x)
    xf = x.float()
    x1, x2 = xf[..., :h], xf[..., h:]
    y = torch.cat((x1 * c - x2 * s, x1 * s + x2 * c), dim=-1)
    return y.to(x.dtype)


def rope_bwd(dy: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """dx1 = g1*c + g2*s, dx2 = g2*c - g1*s (``solution/kernels/rope.py:102-117``)."""
    D = dy.shape[-1]
    h = D // 2
    c = _rope_tables(cos, dy)
    s = _rope_tables(sin, dy)
    g = dy.float()
    g1, g2 = g[..., :h], g[..., h:]
    dx = torch.cat((g1 * c + g2 * s, g2 * c - g1 * s), dim=-1)
    return dx.to(dy.dtype)


# --------------------------------------------------------------------------
# Cross-entropy with online metrics
# --------------------------------------------------------------------------
def ce_rows(logits: torch.Tensor, targets: torch.Tensor, denominator: float = 1.0,
            ignore_index: int = IGNORE_INDEX):
    """Per-row CE loss, Shannon entropy, top-1 hit and (p - onehot)/denominator.

    Semantics of ``solution/kernels/chunked_ce.py:46-128``:
      * loss = logsumexp(z) - z[target]; 0 for ignored rows (``:100,105``);
        a target outside [0, V) that is not ignore_index contributes z_t = 0
        (``:92-93``);
      * entropy = max(0, lse - sum(p*z)), stored for every row, ignored
        rows included (``:102,109-110``);
      * correct = (first-index argmax == target), 0 for ignored rows
        (``:71-73,86-88,103,106``);
      * grad = (softmax - onehot) / denominator, 0 for ignored rows (``:116-128``).
    All arithmetic in fp32 on ``logits.float()``. Returns
    ``(loss fp32 [N], entropy fp32 [N], correct int32 [N], grad fp32 [N, V], lse fp32 [N])``.
    """
    z = logits.float()
    N, V = z.shape
    t = targets.reshape(-1).long()
    ignored = t == ignore_index
    in_range = (t >= 0) & (t < V)
    lse = torch.logsumexp(z, dim=-1)
    safe_t = torch.where(in_range, t, torch.zeros_like(t))
    zt = torch.where(in_range, z.gather(1, safe_t[:, None])[:, 0], torch.zeros_like(lse))
    p = torch.exp(z - lse[:, None])
    loss = torch.where(ignored, torch.zeros_like(lse), lse - zt)
    entropy = torch.clamp(lse - (p * z).sum(-1), min=0.0)
    amax = z.argmax(dim=-1)
    correct = ((amax == t) & ~ignored).to(torch.int32)
    onehot = torch.zeros_like(z)
    onehot[in_range, safe_t[in_range]] = 1.0
    grad = (p - onehot) / float(denominator)
    grad[ignored] = 0.0
    return loss, entropy, correct, grad, lse


def chunked_ce(hidden: torch.Tensor, weight: torch.Tensor, target: torch.Tensor, chunk: int = 32,
               denominator: float = 1.0, ignore_index: int = IGNORE_INDEX, with_grad: bool = True,
               compute_dw: bool = True):
    """Full chunked lm_head CE of ``TritonChunkedHeadLoss.forward`` in fp32.

    hidden [B, S, D], weight [V, D], target [B, S]. Mirrors
    ``solution/kernels/chunked_ce.py:271-304``: per sequence chunk the logits
    ``piece @ W^T`` (``:199``), the per-row CE of :func:`ce_rows`, the input
    gradient ``grad_logits @ W`` (``:249``); the mean loss is total / den with
    den = denominator if > 0 else 1 (``:303-304``). The logits are kept in fp32
    (the reference rounds them to fp16 at ``:197-199``). The lm_head gradient
    ``grad_logits^T @ piece`` has no reference counterpart (the reference head
    is frozen); it is returned when ``compute_dw``.

    Returns ``(mean_loss, token_entropy [B,S], token_loss [B,S], correct int64,
    dhidden fp32 [B,S,D] or None, dW fp32 [V,D] or None)``.
    """
    B, S, D = hidden.shape
    den = float(denominator) if float(denominator) > 0 else 1.0
    Wf = weight.float()
    ent_parts, loss_parts = [], []
    total = torch.zeros((), dtype=torch.float32)
    hits = torch.zeros((), dtype=torch.int64)
    dh = torch.zeros(B, S, D, dtype=torch.float32) if with_grad else None
    dW = torch.zeros_like(Wf) if (with_grad and compute_dw) else None
    for start in range(0, S, chunk):
        stop = min(start + chunk, S)
        piece = hidden[:, start:stop].reshape(-1, D).float()
        lab = target[:, start:stop].reshape(-1)
        logits = piece @ Wf.t()
        loss, ent, corr, grad, _ = ce_rows(logits, lab, den, ignore_index)
        total = total + loss.sum()
        hits = hits + corr.sum().to(torch.int64)
        ent_parts.append(ent.view(B, stop - start))
        loss_parts.append(loss.view(B, stop - start))
        if with_grad:
            dh[:, start:stop] = (grad @ Wf).view(B, stop - start, D)
            if dW is not None:
                dW += grad.t() @ piece
    entropy = torch.cat(ent_parts, dim=1)
    token_loss = torch.cat(loss_parts, dim=1)
    return total / den, entropy, token_loss, hits, dh, dW
