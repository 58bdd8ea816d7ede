"""Vocab-parallel fused head cross-entropy (lm_head rows sharded over GPUs).

No counterpart in the reference, which runs on one GPU. Rank r holds rows
``[offset_r, offset_r + V_r)`` of the [V, D] head weight and every token's
hidden state. Per step:

1. ``soup_ce_vp_forward``: tcgen05 logits GEMM over the shard with the
   online-softmax epilogue -> one record per token (max, sum exp, sum z*exp,
   global argmax, target logit or 0);
2. one NCCL all-gather of the records (rows x 20 bytes per rank);
3. ``soup_ce_vp_combine``: merge the ranks' records in rank order -> loss,
   entropy, hit, global lse (identical on every rank);
4. ``soup_ce_vp_backward``: the shard's per-row gradient factors from the
   global lse (the forward stored exp(z - c) per row, so no pass rewrites
   the shard's [rows, V_r] buffer), the rank's partial dhidden and its dW
   shard (local);
5. one NCCL reduce-scatter (sum) of the bf16 partial dhidden over token
   blocks, so each rank receives the rows it owns (or, on request, an fp32
   all-reduce that leaves every row on every rank).

Row semantics match the single-GPU path (reference ``chunked_ce.py:46-128``).
"""

from __future__ import annotations

from typing import Optional

import torch

from .. import _lib
from .chunked_ce import IGNORE_INDEX, _tma_rows_ok


def shard_range(vocab: int, rank: int, world: int):
    """(offset, size) of rank's contiguous vocabulary shard; sizes differ by at most 1."""
    base, rem = divmod(vocab, world)
    size = base + (1 if rank < rem else 0)
    offset = rank * base + min(rank, rem)
    return offset, size


class ShardState:
    """Workspace and inputs one rank keeps between its forward and backward stages."""

    def __init__(self, hidden, weight_shard, targets, offset, ws, weight_bwd=None, in_dtype=None):
        self.hidden = hidden
        self.weight_shard = weight_shard
        self.targets = targets
        self.offset = offset
        self.ws = ws
        self.weight_bwd = weight_bwd
        self.in_dtype = _lib.BF16 if in_dtype is None else in_dtype


def _prep(hidden, weight_shard, targets):
    """(h, w, w_bwd, in_dtype, t): operands as the single-GPU path takes them
    (bf16 hidden with a bf16 shard as they are; otherwise fp16 operands for the
    logits GEMM and a bf16 copy of the shard for the dX GEMM)."""
    if hidden.dtype == torch.bfloat16 and weight_shard.dtype == torch.bfloat16:
        h = hidden.detach()
        if not _tma_rows_ok(h):
            h = h.contiguous()
        w = weight_shard.detach()
        if not _tma_rows_ok(w):
            w = w.contiguous()
        wb, in_dt = None, _lib.BF16
    else:
        h = hidden.detach()
        if h.dtype != torch.float16 or not _tma_rows_ok(h):
            h = h.to(torch.float16).contiguous()
        w = weight_shard.detach()
        if w.dtype != torch.float16 or not _tma_rows_ok(w):
            w = w.to(torch.float16).contiguous()
        wb = weight_shard.detach().to(torch.bfloat16).contiguous()
        in_dt = _lib.F16
    t = targets.reshape(-1)
    if t.dtype != torch.int64 or not t.is_contiguous():
        t = t.to(torch.int64).contiguous()
    return h, w, wb, in_dt, t


def vp_forward_shard(hidden, weight_shard, targets, offset: int, workspace: Optional[torch.Tensor] = None):
    """Stage 1 on one rank: returns (records [rows, 5] fp32, ShardState)."""
    h, w, wb, in_dt, t = _prep(hidden, weight_shard, targets)
    n, d = h.shape
    v = w.shape[0]
    nbytes = _lib.lib().soup_ce_vp_workspace_bytes(n, v, d)
    if workspace is None or workspace.numel() < nbytes:
        workspace = torch.empty(nbytes, dtype=torch.uint8, device=h.device)
    states = torch.empty(n, 5, dtype=torch.float32, device=h.device)
    _lib.call("soup_ce_vp_forward", h.device, h.data_ptr(), h.stride(0), w.data_ptr(), w.stride(0),
              in_dt, t.data_ptr(), n, v, int(offset), d, states.data_ptr(), workspace.data_ptr(),
              workspace.numel(), _lib.stream_of(h))
    return states, ShardState(h, w, t, int(offset), workspace, wb, in_dt)


def vp_combine(states_all: torch.Tensor, targets: torch.Tensor, vocab_total: int,
               ignore_index: int = IGNORE_INDEX):
    """Stage 3: states_all [nranks, rows, 5] -> (losses, entropies, correct, lse, sums)."""
    nranks, n, _ = states_all.shape
    sa = states_all.contiguous()
    t = targets.reshape(-1).to(torch.int64).contiguous()
    dev = sa.device
    losses = torch.empty(n, dtype=torch.float32, device=dev)
    ents = torch.empty(n, dtype=torch.float32, device=dev)
    corr = torch.empty(n, dtype=torch.int32, device=dev)
    lse = torch.empty(n, dtype=torch.float32, device=dev)
    sums = torch.empty(2, dtype=torch.float32, device=dev)
    _lib.call("soup_ce_vp_combine", dev, sa.data_ptr(), nranks, t.data_ptr(), n, int(vocab_total),
              int(ignore_index), losses.data_ptr(), ents.data_ptr(), corr.data_ptr(), lse.data_ptr(),
              sums.data_ptr(), _lib.stream_of(sa))
    return losses, ents, corr, lse, sums


def vp_backward_shard(state: ShardState, lse: torch.Tensor, denominator: float,
                      ignore_index: int = IGNORE_INDEX, dh_dtype=torch.float32,
                      compute_dw: bool = True, dw_dtype=torch.bfloat16):
    """Stage 4 on one rank: returns (partial dhidden [rows, D], dW shard [V_r, D] | None)."""
    h, w = state.hidden, state.weight_shard
    n, d = h.shape
    v = w.shape[0]
    dh = torch.empty(n, d, dtype=dh_dtype, device=h.device)
    dw = torch.empty(v, d, dtype=dw_dtype, device=h.device) if compute_dw else None
    wb = state.weight_bwd
    _lib.call("soup_ce_vp_backward", h.device, state.ws.data_ptr(), state.ws.numel(), h.data_ptr(),
              h.stride(0), w.data_ptr(), w.stride(0), state.in_dtype, _lib.ptr(wb),
              wb.stride(0) if wb is not None else 0, state.targets.data_ptr(), n, v, state.offset, d,
              lse.data_ptr(), float(denominator), int(ignore_index), dh.data_ptr(),
              _lib.dtype_code(dh_dtype), _lib.ptr(dw), _lib.dtype_code(dw_dtype), 0,
              _lib.stream_of(h))
    return dh, dw


def token_block(rows: int, rank: int, world: int):
    """(start, count) of the token rows whose dhidden rank keeps after the
    reduce-scatter: blocks of ceil(rows / world) rows in rank order, the last
    one(s) shorter when rows is not a multiple of world."""
    per = -(-rows // world)
    start = min(rank * per, rows)
    return start, min(per, rows - start)


def _host_staged(group) -> bool:
    """True when the group's backend moves host tensors only (gloo): the
    collectives are then staged through host copies of the device buffers."""
    import torch.distributed as dist

    return dist.get_backend(group) == "gloo"


def _all_gather_records(states: torch.Tensor, world: int, group) -> torch.Tensor:
    import torch.distributed as dist

    if _host_staged(group):
        parts = [torch.empty_like(states, device="cpu") for _ in range(world)]
        dist.all_gather(parts, states.cpu(), group=group)
        return torch.stack(parts).to(states.device)
    out = torch.empty(world, *states.shape, dtype=states.dtype, device=states.device)
    dist.all_gather_into_tensor(out, states, group=group)
    return out


def _reduce_scatter_rows(dh: torch.Tensor, rank: int, world: int, group) -> torch.Tensor:
    """Sum of every rank's dh [rows, D], of which this rank receives its token block."""
    import torch.distributed as dist

    rows = dh.shape[0]
    start, count = token_block(rows, rank, world)
    if _host_staged(group):
        h = dh.cpu()
        dist.all_reduce(h, op=dist.ReduceOp.SUM, group=group)
        return h[start:start + count].to(dh.device)
    per = -(-rows // world)
    src = dh
    if per * world != rows:  # zero rows pad the last block to the common size
        src = torch.zeros(per * world, dh.shape[1], dtype=dh.dtype, device=dh.device)
        src[:rows].copy_(dh)
    out = torch.empty(per, dh.shape[1], dtype=dh.dtype, device=dh.device)
    dist.reduce_scatter_tensor(out, src, op=dist.ReduceOp.SUM, group=group)
    return out[:count]


def vocab_parallel_cross_entropy(hidden: torch.Tensor, weight_shard: torch.Tensor, vocab_offset: int,
                                 vocab_total: int, targets: torch.Tensor, denominator: float = 1.0,
                                 ignore_index: int = IGNORE_INDEX, group=None, with_grad: bool = True,
                                 compute_dw: bool = True, workspace: Optional[torch.Tensor] = None,
                                 dh_reduce: str = "scatter", timers: Optional[dict] = None):
    """All stages on this rank with collectives over `group` (NCCL; a gloo group
    stages them through host memory).

    Returns ``(losses, entropies, correct, sums, dhidden | None, dW shard | None)``;
    dW covers this rank's vocabulary rows. dhidden:

    * ``dh_reduce="scatter"`` (default): the bf16 partials are reduce-scattered
      over token blocks; this rank gets rows ``token_block(rows, rank, world)``
      of the summed dhidden (bf16), a quarter of the bytes of an fp32
      all-reduce;
    * ``dh_reduce="all"``: fp32 partials all-reduced, every rank gets all rows.

    ``timers``: when a dict is given, (start, end) CUDA events of each stage
    (forward, all_gather, combine, backward, dh_reduce) are stored in it.
    """
    import torch.distributed as dist

    if dh_reduce not in ("scatter", "all"):
        raise ValueError(f"dh_reduce must be 'scatter' or 'all', not {dh_reduce!r}")
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    stream = torch.cuda.current_stream(hidden.device)

    def mark(name, start=True):
        if timers is None:
            return
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(stream)
        timers[name] = (ev, None) if start else (timers[name][0], ev)

    mark("forward")
    states, st = vp_forward_shard(hidden, weight_shard, targets, vocab_offset, workspace)
    mark("forward", False)
    mark("all_gather")
    states_all = _all_gather_records(states, world, group) if world > 1 else states.unsqueeze(0)
    mark("all_gather", False)
    mark("combine")
    losses, ents, corr, lse, sums = vp_combine(states_all, st.targets, vocab_total, ignore_index)
    mark("combine", False)
    dh = dw = None
    if with_grad:
        mark("backward")
        dh_dtype = torch.bfloat16 if dh_reduce == "scatter" else torch.float32
        dh, dw = vp_backward_shard(st, lse, denominator, ignore_index, dh_dtype=dh_dtype,
                                   compute_dw=compute_dw)
        mark("backward", False)
        mark("dh_reduce")
        if dh_reduce == "scatter":
            dh = _reduce_scatter_rows(dh, rank, world, group) if world > 1 else dh
        elif world > 1:
            if _host_staged(group):
                h = dh.cpu()
                dist.all_reduce(h, op=dist.ReduceOp.SUM, group=group)
                dh = h.to(dh.device)
            else:
                dist.all_reduce(dh, op=dist.ReduceOp.SUM, group=group)
        mark("dh_reduce", False)
    return losses, ents, corr, sums, dh, dw
