"""Fused lm_head cross-entropy with online metrics on B200 (tcgen05 GEMMs via the C ABI).

Drop-in for the reference's ``solution/kernels/chunked_ce.py``:
``make_triton_chunked_loss_function`` (autograd Function with the signature
``forward(ctx, hidden, head, target, chunk, denominator, ignore_index, with_grad)``
returning ``(loss/den, token_entropy, token_loss, correct)``),
``chunk_cross_entropy_triton`` (one chunk, 5-tuple), ``patch_soup_chunked_loss``
and the kernel handle ``_chunked_cross_entropy_fused_kernel``.

How the B200 path differs from the reference's per-chunk loop (same results):
the reference runs, per 32/64-token sequence chunk, an fp16 cuBLAS logits GEMM,
one Triton CE kernel and an fp16 dhidden GEMM (``chunked_ce.py:183-264``),
re-streaming the 467 MB lm_head twice per chunk. Here all tokens of a call go
through one ``soup_ce_linear`` launch sequence (tcgen05 logits GEMM with the
online-softmax epilogue storing row-shifted exponentials exp(z - c), a per-row
statistics pass, split-K dX GEMM with the per-row gradient factor applied in
its reduce, dW GEMM) with fp32 accumulation and fp32 metrics; no pass
rewrites the [rows, vocab] buffer between the GEMMs. bf16 activations with a
bf16 head are multiplied as they are; other dtypes enter the logits GEMM as
fp16, as in the reference (see :func:`ce_operands`). ``chunk``
stays in the signature; token rows are processed in blocks sized by
``CE_WORKSPACE_BYTES`` instead, which bounds the logits buffer the way
``chunk`` bounds it in the reference. With a trainable head the lm_head
gradient GEMM runs in backward, scaled by the upstream gradient inside its
epilogue, and accumulates into ``weight.grad`` in the weight's dtype.
"""

from __future__ import annotations

from typing import Any, Optional, Tuple

import torch

from .. import _lib
from ._shim import LaunchShim

IGNORE_INDEX = -100

#: Largest scratch buffer (bytes) one fused CE launch sequence may use; rows
#: are processed in blocks that fit. 0 selects all rows at once.
CE_WORKSPACE_BYTES = 8 << 30

# dtype -> (key of the weight it was cast from, cast copy); one entry per dtype
_HEAD_CACHE = {}


def _extract_head_weight(head: Any) -> Optional[torch.Tensor]:
    """Find the lm_head weight behind a module, bound method or closure.

    Same lookup order as the reference (``chunked_ce.py:131-167``).
    """
    w = getattr(head, "weight", None)
    if isinstance(w, torch.Tensor):
        return w
    self_obj = getattr(head, "__self__", None)
    if self_obj is not None:
        w = getattr(self_obj, "weight", None)
        if isinstance(w, torch.Tensor):
            return w
        if hasattr(self_obj, "get_output_embeddings"):
            try:
                w = getattr(self_obj.get_output_embeddings(), "weight", None)
                if isinstance(w, torch.Tensor):
                    return w
            except Exception:
                pass
    closure = getattr(head, "__closure__", None)
    if closure:
        for cell in closure:
            val = getattr(cell, "cell_contents", None)
            w = getattr(val, "weight", None)
            if isinstance(w, torch.Tensor):
                return w
            if hasattr(val, "get_output_embeddings"):
                try:
                    w = getattr(val.get_output_embeddings(), "weight", None)
                    if isinstance(w, torch.Tensor):
                        return w
                except Exception:
                    pass
    return None


def _tma_rows_ok(t: torch.Tensor) -> bool:
    return (t.dim() == 2 and t.stride(1) == 1 and (t.stride(0) * t.element_size()) % 16 == 0
            and t.data_ptr() % 16 == 0)


def _cached_cast(weight: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """The head weight in `dtype`: the tensor itself when it already is (with
    TMA-ready rows), else a cast copy kept while the weight is unchanged (the
    reference keeps its fp16 copy the same way, ``chunked_ce.py:170-180``)."""
    w = weight.detach()
    if w.dtype == dtype and _tma_rows_ok(w):
        return w
    key = (id(weight), weight._version, weight.data_ptr(), weight.dtype)
    ent = _HEAD_CACHE.get(dtype)
    if ent is None or ent[0] != key:
        ent = (key, w.to(dtype).contiguous())
        _HEAD_CACHE[dtype] = ent
    return ent[1]


def ce_operands(hidden2d: torch.Tensor, weight: torch.Tensor, need_dx: bool):
    """``(h, w, w_bwd, in_dtype)`` for the fused CE entry points.

    bf16 hidden rows with a bf16 weight are used as they are. Anything else goes
    through the logits GEMM as fp16 operands, the reference's own arithmetic
    (``chunked_ce.py:196-199`` rounds the chunk and a cached copy of W to fp16):
    the rows rounded to fp16 and a cached fp16 copy of W, plus a cached bf16 copy
    of W for the dX GEMM (the logits' gradient is kept in bf16).
    """
    if hidden2d.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16:
        h = hidden2d.detach()
        if not _tma_rows_ok(h):
            h = h.contiguous()
        return h, _cached_cast(weight, torch.bfloat16), None, _lib.BF16
    h = hidden2d.detach()
    if h.dtype != torch.float16 or not _tma_rows_ok(h):
        h = h.to(torch.float16).contiguous()
    w = _cached_cast(weight, torch.float16)
    wb = _cached_cast(weight, torch.bfloat16) if need_dx else None
    return h, w, wb, _lib.F16


def _rows_per_block(rows: int, vocab: int, dim: int, budget: int) -> int:
    if budget <= 0:
        return rows
    lib = _lib.lib()
    full = lib.soup_ce_linear_workspace_bytes(rows, vocab, dim)
    if full <= budget:
        return rows
    per_row = max(1, full // rows)
    r = max(128, (budget // per_row) // 128 * 128)
    return min(rows, r)


def fused_linear_cross_entropy(hidden: torch.Tensor, weight: torch.Tensor, targets: torch.Tensor,
                               denominator: float = 1.0, ignore_index: int = IGNORE_INDEX,
                               with_grad: bool = True, compute_dw: bool = False,
                               dw_dtype: torch.dtype = torch.float32,
                               workspace_bytes: Optional[int] = None,
                               dh_dtype: Optional[torch.dtype] = None):
    """Tensor-level fused head CE over hidden [N, D] and weight [V, D].

    Returns ``(losses [N] f32, entropies [N] f32, correct [N] i32, sums [2] f32
    = (sum loss, hits), dhidden [N, D] | None, dW [V, D] | None)``. dhidden is
    ``dh_dtype`` (bf16 or fp32; default bf16 for bf16 hidden states, fp32
    otherwise). Operands: see :func:`ce_operands`. Gradients are scaled by
    1/denominator (denominator <= 0 counts as 1).
    """
    if not hidden.is_cuda:
        raise RuntimeError("fused_linear_cross_entropy needs CUDA tensors")
    n, d = hidden.shape
    v = weight.shape[0]
    if dh_dtype is None:
        dh_dtype = torch.bfloat16 if hidden.dtype == torch.bfloat16 else torch.float32
    h, w, wb, in_dt = ce_operands(hidden, weight, with_grad)
    t = targets.reshape(-1)
    if t.dtype != torch.int64 or not t.is_contiguous():
        t = t.to(torch.int64).contiguous()
    dev = hidden.device
    losses = torch.empty(n, dtype=torch.float32, device=dev)
    ents = torch.empty(n, dtype=torch.float32, device=dev)
    corr = torch.empty(n, dtype=torch.int32, device=dev)
    dh = torch.empty(n, d, dtype=dh_dtype, device=dev) if with_grad else None
    dw = torch.empty(v, d, dtype=dw_dtype, device=dev) if (with_grad and compute_dw) else None
    budget = CE_WORKSPACE_BYTES if workspace_bytes is None else workspace_bytes
    rb = _rows_per_block(n, v, d, budget)
    nblk = (n + rb - 1) // rb
    sums = torch.empty(nblk, 2, dtype=torch.float32, device=dev)
    lib = _lib.lib()
    stream = _lib.stream_of(hidden)
    for b in range(nblk):
        r0 = b * rb
        r = min(rb, n - r0)
        ws_bytes = lib.soup_ce_linear_workspace_bytes(r, v, d)
        ws = _lib.scratch(dev, ws_bytes)
        _lib.call("soup_ce_linear", dev, h[r0].data_ptr(), h.stride(0), w.data_ptr(), w.stride(0),
                  in_dt, _lib.ptr(wb), wb.stride(0) if wb is not None else 0, t[r0:].data_ptr(), r,
                  v, d, float(denominator), int(ignore_index), losses[r0:].data_ptr(),
                  ents[r0:].data_ptr(), corr[r0:].data_ptr(), sums[b].data_ptr(),
                  _lib.ptr(dh[r0] if dh is not None else None), _lib.dtype_code(dh_dtype),
                  _lib.ptr(dw), _lib.dtype_code(dw_dtype), 1 if b > 0 else 0, ws.data_ptr(),
                  ws_bytes, stream)
    total = sums.sum(0) if nblk > 1 else sums[0]
    return losses, ents, corr, total, dh, dw


def _fused_forward_keep_grad_state(hidden: torch.Tensor, weight: torch.Tensor, targets: torch.Tensor,
                                denominator: float, ignore_index: int,
                                dh_dtype: Optional[torch.dtype] = None):
    """Forward + dhidden in one pass, leaving the gradient state in a workspace owned by the caller.

    Returns ``(losses, ents, corr, sums, dh, state)`` where ``state`` holds the
    workspace and the operand-typed hidden rows needed by :func:`_dweight_from_state`.
    """
    n, d = hidden.shape
    v = weight.shape[0]
    if dh_dtype is None:
        dh_dtype = torch.bfloat16 if hidden.dtype == torch.bfloat16 else torch.float32
    h, w, wb, in_dt = ce_operands(hidden, weight, True)
    t = targets.reshape(-1)
    if t.dtype != torch.int64 or not t.is_contiguous():
        t = t.to(torch.int64).contiguous()
    dev = hidden.device
    lib = _lib.lib()
    ws_bytes = lib.soup_ce_linear_workspace_bytes(n, v, d)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    losses = torch.empty(n, dtype=torch.float32, device=dev)
    ents = torch.empty(n, dtype=torch.float32, device=dev)
    corr = torch.empty(n, dtype=torch.int32, device=dev)
    sums = torch.empty(2, dtype=torch.float32, device=dev)
    dh = torch.empty(n, d, dtype=dh_dtype, device=dev)
    _lib.call("soup_ce_linear", dev, h.data_ptr(), h.stride(0), w.data_ptr(), w.stride(0), in_dt,
              _lib.ptr(wb), wb.stride(0) if wb is not None else 0, t.data_ptr(), n, v, d,
              float(denominator), int(ignore_index), losses.data_ptr(), ents.data_ptr(),
              corr.data_ptr(), sums.data_ptr(), dh.data_ptr(), _lib.dtype_code(dh_dtype), 0,
              _lib.F32, 0, ws.data_ptr(), ws_bytes, _lib.stream_of(hidden))
    return losses, ents, corr, sums, dh, {"ws": ws, "h": h, "in_dtype": in_dt, "rows": n,
                                          "vocab": v, "dim": d}


def _dweight_from_state(state, weight: torch.Tensor, grad_scale: torch.Tensor) -> None:
    """weight.grad (+)= grad_scale * dL^T H, in the weight's dtype, one GEMM launch."""
    scale = grad_scale.detach().to(torch.float32).reshape(1).contiguous()
    dev = weight.device
    if weight.dtype in (torch.bfloat16, torch.float32):
        target = weight.grad
        accumulate = 1
        if target is None:
            target = torch.empty_like(weight)
            accumulate = 0
        _lib.call("soup_ce_linear_dweight", dev, state["ws"].data_ptr(), state["ws"].numel(),
                  state["h"].data_ptr(), state["h"].stride(0), state["in_dtype"], state["rows"],
                  state["vocab"], state["dim"], scale.data_ptr(), target.data_ptr(),
                  _lib.dtype_code(weight.dtype), accumulate, _lib.stream_of(weight))
        if weight.grad is None:
            weight.grad = target
        return
    tmp = torch.empty(weight.shape, dtype=torch.float32, device=dev)
    _lib.call("soup_ce_linear_dweight", dev, state["ws"].data_ptr(), state["ws"].numel(),
              state["h"].data_ptr(), state["h"].stride(0), state["in_dtype"], state["rows"],
              state["vocab"], state["dim"], scale.data_ptr(), tmp.data_ptr(), _lib.F32, 0,
              _lib.stream_of(weight))
    g = tmp.to(weight.dtype)
    weight.grad = g if weight.grad is None else weight.grad.add_(g)


def chunk_cross_entropy_triton(head: Any, piece: torch.Tensor, target: torch.Tensor,
                               ignore_index: int = IGNORE_INDEX, denominator: float = 1.0,
                               with_grad: bool = True
                               ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                                          Optional[torch.Tensor]]:
    """CE loss, metrics and input gradient of one chunk (reference ``chunked_ce.py:183-264``).

    Returns ``(total_loss, entropy, token_loss, hits, piece_grad)`` as the
    reference does: total_loss the fp32 sum of the per-token losses (not
    divided by the denominator), entropy/token_loss fp32 shaped
    ``piece.shape[:-1]``, hits an int64 count, and piece_grad (None without
    gradient) the input gradient ``(softmax - onehot) / denominator @ W`` in
    fp16 like the reference's fp16 GEMM result (``chunked_ce.py:246-249``),
    here rounded once from fp32.
    """
    weight = _extract_head_weight(head)
    shape = piece.shape
    if weight is not None and piece.is_cuda:
        flat = piece.reshape(-1, shape[-1])
        losses, ents, corr, sums, dh, _ = fused_linear_cross_entropy(
            flat, weight, target.reshape(-1), denominator, ignore_index, with_grad,
            dh_dtype=torch.float32)
        hits = corr.sum()
        grad = dh.view(shape).to(torch.float16) if dh is not None else None
        return sums[0], ents.view(shape[:-1]), losses.view(shape[:-1]), hits, grad
    # A head that is a plain callable: its own logits, then the CE kernel in place.
    if with_grad:
        piece_in = piece.detach().requires_grad_(True)
        with torch.enable_grad():
            logits = head(piece_in)
    else:
        piece_in = None
        logits = head(piece)
    flat_logits = logits.detach().reshape(-1, logits.shape[-1])
    if flat_logits.stride(-1) != 1:
        flat_logits = flat_logits.contiguous()
    n = flat_logits.shape[0]
    losses = torch.empty(n, dtype=torch.float32, device=piece.device)
    ents = torch.empty(n, dtype=torch.float32, device=piece.device)
    corr = torch.empty(n, dtype=torch.int32, device=piece.device)
    t = target.reshape(-1).to(torch.int64).contiguous()
    ce_rows(flat_logits, t, losses, ents, corr, float(denominator), ignore_index, write_grad=with_grad)
    grad = None
    if with_grad:
        grad = torch.autograd.grad(logits, piece_in, grad_outputs=flat_logits.view(logits.shape),
                                   retain_graph=False)[0]
    return (losses.sum(), ents.view(shape[:-1]), losses.view(shape[:-1]), corr.sum(), grad)


def ce_rows(logits: torch.Tensor, targets: torch.Tensor, losses, entropies, correct,
            denominator: float, ignore_index: int = IGNORE_INDEX, write_grad: bool = True):
    """Per-row CE metrics over a logits buffer; optionally its in-place gradient."""
    rows, vocab = logits.shape
    _lib.call("soup_ce_rows", logits.device, logits.data_ptr(), logits.stride(0), targets.data_ptr(),
              losses.data_ptr(), entropies.data_ptr(), correct.data_ptr(), rows, vocab,
              float(denominator), int(ignore_index), _lib.dtype_code(logits.dtype),
              1 if write_grad else 0, _lib.stream_of(logits))


def make_triton_chunked_loss_function():
    """Autograd Function for the chunked head loss (reference ``chunked_ce.py:267-313``).

    With a head whose weight can be found, every token row goes through the
    fused tcgen05 path; the input gradient is precomputed in forward (as in
    the reference) and scaled by ``grad_loss`` in backward. When the head
    weight itself requires grad, its gradient is computed too and accumulated
    into ``weight.grad`` in backward (the reference treats the head as frozen).
    """

    class B200ChunkedHeadLoss(torch.autograd.Function):
        @staticmethod
        def forward(ctx, hidden, head, target, chunk, denominator, ignore_index, with_grad):
            den = float(denominator) if float(denominator) > 0 else 1.0
            weight = _extract_head_weight(head)
            ctx.with_grad = with_grad
            ctx.weight = None
            ctx.dw_state = None
            if weight is not None and hidden.is_cuda:
                B, S, D = hidden.shape
                want_dw = bool(with_grad and weight.requires_grad)
                h2 = hidden.reshape(-1, D)
                state = None
                if want_dw and _rows_per_block(h2.shape[0], weight.shape[0], D,
                                               CE_WORKSPACE_BYTES) == h2.shape[0]:
                    # dW is deferred to backward, where grad_loss scales it in the epilogue
                    losses, ents, corr, sums, dh, state = _fused_forward_keep_grad_state(
                        h2, weight, target.reshape(-1), den, ignore_index)
                    dw = None
                else:
                    losses, ents, corr, sums, dh, dw = fused_linear_cross_entropy(
                        h2, weight, target.reshape(-1), den, ignore_index, with_grad,
                        compute_dw=want_dw)
                token_entropy = ents.view(B, S)
                token_loss = losses.view(B, S)
                correct = corr.sum()
                total = sums[0]
                if with_grad:
                    grad = dh.view(B, S, D)
                    if grad.dtype != hidden.dtype:
                        grad = grad.to(hidden.dtype)
                    ctx.save_for_backward(grad)
                    if want_dw:
                        ctx.weight = weight
                        ctx.dw = dw
                        ctx.dw_state = state
            else:
                grad = torch.zeros_like(hidden) if with_grad else None
                total = torch.zeros((), dtype=torch.float32, device=hidden.device)
                entropies, losses_l = [], []
                correct = torch.zeros((), dtype=torch.long, device=hidden.device)
                for start in range(0, hidden.shape[1], chunk):
                    stop = start + chunk
                    part, ent, tok, hits, pg = chunk_cross_entropy_triton(
                        head, hidden[:, start:stop], target[:, start:stop],
                        ignore_index=ignore_index, denominator=den, with_grad=with_grad)
                    if with_grad:
                        grad[:, start:stop] = pg.to(hidden.dtype)
                    total = total + part
                    entropies.append(ent)
                    losses_l.append(tok)
                    correct = correct + hits
                token_entropy = torch.cat(entropies, dim=1)
                token_loss = torch.cat(losses_l, dim=1)
                if with_grad:
                    ctx.save_for_backward(grad)
            ctx.mark_non_differentiable(token_entropy, token_loss, correct)
            return total / den, token_entropy, token_loss, correct

        @staticmethod
        def backward(ctx, grad_loss, _grad_entropy, _grad_token_loss, _grad_correct):
            if not ctx.with_grad:
                return (None,) * 7
            (grad,) = ctx.saved_tensors
            if ctx.weight is not None:
                w = ctx.weight
                if ctx.dw_state is not None:
                    _dweight_from_state(ctx.dw_state, w, grad_loss)
                else:
                    g = (ctx.dw * grad_loss).to(w.dtype)
                    if w.grad is None:
                        w.grad = g
                    else:
                        w.grad.add_(g)
                ctx.dw = None
                ctx.dw_state = None
            return ((grad * grad_loss).to(grad.dtype), None, None, None, None, None, None)

    return B200ChunkedHeadLoss


def patch_soup_chunked_loss(chunk_size: int = 64):
    """Install the fused loss into Soup's streaming head loss (reference ``chunked_ce.py:316-350``).

    A no-op when ``soup_cli`` is not importable, as in the reference.
    """
    try:
        from soup_cli.trainer.sft import SFTTrainerWrapper
        from soup_cli.utils.stream_loss_chunk import ChunkedHeadLoss, causal_lm_of
        import soup_cli.utils.stream_loss_chunk as slc
    except ImportError:
        return
    slc._chunked_function = make_triton_chunked_loss_function
    original_setup = SFTTrainerWrapper._setup_transformers

    def _setup_transformers_with_custom_chunk(self, cfg, tcfg):
        result = original_setup(self, cfg, tcfg)
        model = getattr(self, "model", None)
        if model is None or not isinstance(model, torch.nn.Module):
            return result
        has_cuda = any(p.is_cuda for p in model.parameters()) if hasattr(model, "parameters") else False
        if not has_cuda:
            return result
        if getattr(self, "_stream_loss_chunk_hook", None) is None:
            self._stream_loss_chunk_hook = ChunkedHeadLoss(causal_lm_of(model), chunk_size)
        return result

    SFTTrainerWrapper._setup_transformers = _setup_transformers_with_custom_chunk


# ---- kernel handle with the reference's launch signature -----------------------
def _launch_ce(logits_ptr, targets_ptr, losses_ptr, entropies_ptr, correct_ptr, stride_logits_row,
               V, denominator, ignore_index=IGNORE_INDEX, **_triton_only):
    rows = losses_ptr.numel()
    _lib.call("soup_ce_rows", logits_ptr.device, logits_ptr.data_ptr(), int(stride_logits_row),
              targets_ptr.data_ptr(), losses_ptr.data_ptr(), entropies_ptr.data_ptr(),
              correct_ptr.data_ptr(), rows, int(V), float(denominator), int(ignore_index),
              _lib.dtype_code(logits_ptr.dtype), 1, _lib.stream_of(logits_ptr))


_chunked_cross_entropy_fused_kernel = LaunchShim(
    "_chunked_cross_entropy_fused_kernel",
    ["logits_ptr", "targets_ptr", "losses_ptr", "entropies_ptr", "correct_ptr",
     "stride_logits_row", "V", "denominator"],
    _launch_ce)
