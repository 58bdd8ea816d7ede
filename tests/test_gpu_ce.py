"""GPU parity of the cross-entropy paths against the CPU oracle.

* the reference-compatible CE kernel over a logits buffer (in-place grad),
  launched exactly as the reference's test launches its Triton kernel;
* the fused tcgen05 head CE (logits GEMM + online-softmax epilogue, row statistics,
  dX and dW GEMMs) through the reference's autograd-Function signature.

Tolerances follow the reference's targets: fp32 loss within 1e-4 relative,
entropy 2e-3, gradients cosine >= 0.9999, accuracy counts bit-exact (a row
may only differ where the oracle's own top-2 logits are closer than the fp32
accumulation error, which is reported, not hidden).
"""

import pytest
import torch

import oracle
from auspex_soup_demo_b200 import _lib
from auspex_soup_demo_b200.kernels import (_chunked_cross_entropy_fused_kernel,
                                           make_triton_chunked_loss_function)
from auspex_soup_demo_b200.kernels.chunked_ce import fused_linear_cross_entropy
from helpers import cosine

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("N_rows, V", [(16, 151936), (32, 4096), (4, 1000)])
def test_ce_kernel_reference_launch(N_rows, V):
    """Same inputs and launch form as the reference test (solution/test_kernels.py:92-145)."""
    torch.manual_seed(42)
    logits = torch.randn(N_rows, V, device="cuda", dtype=torch.float16)
    targets = torch.randint(0, V, (N_rows,), device="cuda", dtype=torch.long)
    targets[0] = -100
    mask = targets != -100
    denom = mask.sum().clamp(min=1).float()
    loss, ent, corr, grad, _ = oracle.ce_rows(logits.cpu(), targets.cpu(), float(denom))
    buf = logits.clone()
    losses = torch.empty(N_rows, device="cuda", dtype=torch.float32)
    entropies = torch.empty(N_rows, device="cuda", dtype=torch.float32)
    correct = torch.empty(N_rows, device="cuda", dtype=torch.int32)
    _chunked_cross_entropy_fused_kernel[(N_rows,)](
        buf, targets, losses, entropies, correct, stride_logits_row=buf.stride(0), V=V,
        denominator=denom.item(), ignore_index=-100, BLOCK_V=4096, num_warps=8, num_stages=2)
    torch.cuda.synchronize()
    torch.testing.assert_close(losses.sum().cpu() / denom.cpu(), loss.sum() / denom.cpu(),
                               rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(entropies.cpu(), ent, rtol=2e-3, atol=2e-3)
    assert torch.equal(correct.cpu(), corr)
    torch.testing.assert_close(buf.float().cpu(), grad.half().float(), rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_ce_kernel_ignored_rows_and_ties(dtype):
    N, V = 6, 5003
    g = torch.Generator().manual_seed(4)
    logits = torch.randn(N, V, generator=g).to(dtype)
    targets = torch.randint(0, V, (N,), generator=g)
    targets[0] = -100
    logits[1, 17] = logits[1, 4000] = 11.0  # tie: first index wins
    targets[1] = 17
    logits[2, 5] = logits[2, 6] = 11.0
    targets[2] = 6  # tie, target is the second index -> miss
    loss, ent, corr, grad, _ = oracle.ce_rows(logits, targets, 5.0)
    buf = logits.cuda()
    out = [torch.empty(N, device="cuda"), torch.empty(N, device="cuda"),
           torch.empty(N, device="cuda", dtype=torch.int32)]
    _chunked_cross_entropy_fused_kernel[(N,)](buf, targets.cuda(), *out, buf.stride(0), V, 5.0,
                                              ignore_index=-100)
    torch.testing.assert_close(out[0].cpu(), loss, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(out[1].cpu(), ent, rtol=1e-4, atol=1e-4)
    assert out[2].cpu().tolist() == corr.tolist() == [0, 1, 0] + corr.tolist()[3:]
    assert float(buf[0].float().abs().max()) == 0.0  # ignored row: zero grad
    tol = 2e-3 if dtype == torch.bfloat16 else 1e-5
    torch.testing.assert_close(buf.float().cpu(), grad.to(dtype).float(), rtol=tol, atol=1e-6)


def _inputs(n, v, d, seed=0, ignore_frac=0.1):
    g = torch.Generator().manual_seed(seed)
    hidden = torch.randn(n, d, generator=g).to(torch.bfloat16)
    weight = (0.02 * torch.randn(v, d, generator=g)).to(torch.bfloat16)
    targets = torch.randint(0, v, (n,), generator=g)
    targets[torch.rand(n, generator=g) < ignore_frac] = -100
    return hidden, weight, targets


def _check_fused(n, v, d, seed, workspace_bytes=None, dw_dtype=torch.float32, inputs=None):
    hidden, weight, targets = inputs if inputs is not None else _inputs(n, v, d, seed)
    den = float((targets != -100).sum())
    logits = hidden.float() @ weight.float().t()
    loss, ent, corr, grad, lse = oracle.ce_rows(logits, targets, den)
    dh_ref = grad @ weight.float()
    dw_ref = grad.t() @ hidden.float()
    losses, ents, hits, sums, dh, dw = fused_linear_cross_entropy(
        hidden.cuda(), weight.cuda(), targets.cuda(), den, -100, True, compute_dw=True,
        dw_dtype=dw_dtype, workspace_bytes=workspace_bytes)
    torch.cuda.synchronize()
    assert _lib.device_error(torch.device("cuda")) == 0
    # loss: fp32, 1e-4 relative
    tot = float(sums[0])
    assert abs(tot - float(loss.sum())) <= 1e-4 * abs(float(loss.sum())), (tot, float(loss.sum()))
    torch.testing.assert_close(losses.cpu(), loss, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(ents.cpu(), ent, rtol=2e-3, atol=2e-3)
    # accuracy: bit-exact, except provable near-ties of the oracle's own logits
    diff = (hits.cpu() != corr).nonzero().flatten()
    if diff.numel():
        top2 = logits[diff].topk(2, dim=-1).values
        gap = (top2[:, 0] - top2[:, 1]).abs()
        assert bool((gap < 1e-4 * top2[:, 0].abs().clamp_min(1)).all()), (diff, gap)
    assert int(sums[1]) == int(hits.sum())
    assert cosine(dh, dh_ref) >= 0.9999
    assert cosine(dw, dw_ref) >= 0.9999
    return diff.numel()


def test_fused_ce_small_ragged():
    # vocab not a multiple of the 256-column tile, rows not a multiple of 128
    _check_fused(200, 4099, 192, seed=1)


def test_fused_ce_medium():
    _check_fused(512, 32000, 512, seed=2)


def test_fused_ce_full_vocab_and_dim():
    # the benchmark's vocab and hidden size at 512 tokens (oracle runs in seconds)
    assert _check_fused(512, 151936, 1536, seed=3) <= 1


def test_fused_ce_targets_far_below_the_maximum():
    # half of the rows have logits ~100 wide with the target at the row minimum
    # (loss ~100): above the stored exponentials' shift window, so the overflow
    # flag is raised and the gated second logits GEMM rewrites them with shift = lse
    hidden, weight, targets = _inputs(256, 4099, 192, seed=11)
    hidden[:128] = (hidden[:128].float() * 60.0).to(torch.bfloat16)
    logits = hidden.float() @ weight.float().t()
    targets[:128] = logits[:128].argmin(dim=-1)
    targets[3] = -100
    assert float((logits[:128].max(-1).values - logits[:128].min(-1).values).min()) > 80.0
    _check_fused(256, 4099, 192, seed=11, inputs=(hidden, weight, targets))


def test_fused_ce_row_blocks_accumulate_dw():
    # a small workspace budget forces several row blocks; dW accumulates across them
    _check_fused(384, 8192, 256, seed=4, workspace_bytes=2 * 1024 * 1024)


def test_fused_ce_bf16_dw():
    _check_fused(256, 4096, 256, seed=5, dw_dtype=torch.bfloat16)


def test_fused_ce_all_rows_ignored():
    hidden, weight, targets = _inputs(130, 1000, 64, seed=6)
    targets[:] = -100
    losses, ents, hits, sums, dh, dw = fused_linear_cross_entropy(
        hidden.cuda(), weight.cuda(), targets.cuda(), 0.0, -100, True, compute_dw=True)
    assert float(losses.abs().max()) == 0.0
    assert int(hits.sum()) == 0
    assert float(dh.float().abs().max()) == 0.0
    assert float(dw.abs().max()) == 0.0
    assert bool(torch.isfinite(ents).all())


def test_autograd_function_reference_signature():
    """make_triton_chunked_loss_function() drives the fused path; dhidden via backward."""
    B, S, D, V = 2, 96, 256, 5000
    g = torch.Generator().manual_seed(7)
    hidden = torch.randn(B, S, D, generator=g).to(torch.bfloat16)
    head = torch.nn.Linear(D, V, bias=False).to(torch.bfloat16)
    with torch.no_grad():
        head.weight.copy_((0.05 * torch.randn(V, D, generator=g)).to(torch.bfloat16))
    head.weight.requires_grad_(False)
    target = torch.randint(0, V, (B, S), generator=g)
    target[:, :3] = -100
    den = float((target != -100).sum())
    ref = oracle.chunked_ce(hidden, head.weight, target, 32, den, compute_dw=False)
    Fn = make_triton_chunked_loss_function()
    h = hidden.cuda().requires_grad_(True)
    loss, ent, tok, corr = Fn.apply(h, head.cuda(), target.cuda(), 32, den, -100, True)
    (2.0 * loss).backward()
    assert abs(float(loss) - float(ref[0])) <= 1e-4 * abs(float(ref[0]))
    torch.testing.assert_close(ent.cpu(), ref[1], rtol=2e-3, atol=2e-3)
    torch.testing.assert_close(tok.cpu(), ref[2], rtol=1e-4, atol=1e-4)
    assert int(corr) == int(ref[3])
    assert cosine(h.grad, 2.0 * ref[4]) >= 0.9999
    assert h.grad.shape == hidden.shape and h.grad.dtype == torch.bfloat16


def test_autograd_function_trainable_head_accumulates_weight_grad():
    B, S, D, V = 1, 130, 128, 3000
    g = torch.Generator().manual_seed(8)
    hidden = torch.randn(B, S, D, generator=g).to(torch.bfloat16)
    W = (0.05 * torch.randn(V, D, generator=g)).to(torch.bfloat16)
    target = torch.randint(0, V, (B, S), generator=g)
    den = float(S)
    ref = oracle.chunked_ce(hidden, W, target, 64, den, compute_dw=True)
    head = torch.nn.Linear(D, V, bias=False, dtype=torch.bfloat16, device="cuda")
    with torch.no_grad():
        head.weight.copy_(W.cuda())
    Fn = make_triton_chunked_loss_function()
    h = hidden.cuda().requires_grad_(True)
    loss, *_ = Fn.apply(h, head, target.cuda(), 64, den, -100, True)
    (3.0 * loss).backward()  # upstream gradient 3 is applied inside the dW GEMM epilogue
    assert head.weight.grad is not None and head.weight.grad.dtype == torch.bfloat16
    assert cosine(head.weight.grad, ref[5]) >= 0.999  # bf16-stored weight grad
    g1 = head.weight.grad.float().cpu()
    ratio = float((g1 * ref[5]).sum() / (ref[5] * ref[5]).sum())
    assert abs(ratio - 3.0) < 0.02, ratio
    # a second backward accumulates into the existing gradient
    h2 = hidden.cuda().requires_grad_(True)
    loss2, *_ = Fn.apply(h2, head, target.cuda(), 64, den, -100, True)
    loss2.backward()
    g2 = head.weight.grad.float().cpu()
    ratio2 = float((g2 * ref[5]).sum() / (ref[5] * ref[5]).sum())
    assert abs(ratio2 - 4.0) < 0.03, ratio2


def test_autograd_function_trainable_head_after_overflow_fallback():
    # rows whose target is ~100 nats below the row maximum: the forward takes the
    # gated fallback GEMM, and the backward's dW (soup_ce_linear_dweight, scaling the
    # hidden rows by the stored per-row factors) must still match the oracle
    B, S, D, V = 1, 130, 128, 3000
    g = torch.Generator().manual_seed(12)
    hidden = torch.randn(B, S, D, generator=g)
    hidden[0, :64] *= 90.0
    hidden = hidden.to(torch.bfloat16)
    W = (0.05 * torch.randn(V, D, generator=g)).to(torch.bfloat16)
    target = torch.randint(0, V, (B, S), generator=g)
    logits = hidden[0].float() @ W.float().t()
    target[0, :64] = logits[:64].argmin(dim=-1)
    assert float((logits[:64].max(-1).values - logits[:64].min(-1).values).min()) > 80.0
    den = float(S)
    ref = oracle.chunked_ce(hidden, W, target, 64, den, compute_dw=True)
    head = torch.nn.Linear(D, V, bias=False, dtype=torch.bfloat16, device="cuda")
    with torch.no_grad():
        head.weight.copy_(W.cuda())
    Fn = make_triton_chunked_loss_function()
    h = hidden.cuda().requires_grad_(True)
    loss, *_ = Fn.apply(h, head, target.cuda(), 64, den, -100, True)
    loss.backward()
    assert abs(float(loss.detach()) - float(ref[0])) <= 1e-4 * abs(float(ref[0]))
    assert cosine(h.grad, ref[4]) >= 0.9999
    assert cosine(head.weight.grad, ref[5]) >= 0.999  # bf16-stored weight grad


def test_autograd_function_callable_head_path():
    """A head without a findable weight: its logits + the CE kernel + autograd (reference :200-210)."""
    B, S, D, V = 2, 40, 64, 1000
    g = torch.Generator().manual_seed(9)
    hidden = torch.randn(B, S, D, generator=g)
    W = 0.1 * torch.randn(V, D, generator=g)
    target = torch.randint(0, V, (B, S), generator=g)
    Wc = W.cuda()

    def head(x):
        return x @ Wc.t()

    ref = oracle.chunked_ce(hidden, W, target, 16, float(B * S), compute_dw=False)
    Fn = make_triton_chunked_loss_function()
    h = hidden.cuda().requires_grad_(True)
    loss, ent, tok, corr = Fn.apply(h, head, target.cuda(), 16, float(B * S), -100, True)
    loss.backward()
    assert abs(float(loss) - float(ref[0])) <= 1e-4 * abs(float(ref[0]))
    assert int(corr) == int(ref[3])
    assert cosine(h.grad, ref[4]) >= 0.9999


@pytest.mark.parametrize("world, far", [(1, False), (3, False), (8, False), (3, True)])
def test_vocab_parallel_ce_emulated_ranks(world, far):
    """Shards processed one after another on one GPU, records combined as the
    all-gather would, partial dhidden summed as the all-reduce would. far: half
    of the rows have logits ~100+ wide with the target at the row minimum, so
    the shards' stored exponentials overflow their shift window and the gated
    fallback GEMM of the backward rewrites them."""
    from auspex_soup_demo_b200.kernels.vocab_parallel import (shard_range, vp_backward_shard,
                                                              vp_combine, vp_forward_shard)

    n, v, d = 384, 20011, 256  # vocab not divisible by the rank count or the tile width
    hidden, weight, targets = _inputs(n, v, d, seed=11)
    if far:
        hidden[:192] = (hidden[:192].float() * 60.0).to(torch.bfloat16)
        targets[:192] = (hidden[:192].float() @ weight.float().t()).argmin(dim=-1)
        targets[3] = -100
    targets[5] = v - 1          # last vocabulary row (last shard)
    targets[6] = 0              # first row (first shard)
    den = float((targets != -100).sum())
    logits = hidden.float() @ weight.float().t()
    loss, ent, corr, grad, lse_ref = oracle.ce_rows(logits, targets, den)
    hc, wc, tc = hidden.cuda(), weight.cuda(), targets.cuda()
    states, shard_states = [], []
    for r in range(world):
        off, size = shard_range(v, r, world)
        s, st = vp_forward_shard(hc, wc[off:off + size], tc, off)
        states.append(s)
        shard_states.append(st)
    losses, ents, hits, lse, sums = vp_combine(torch.stack(states), tc, v)
    dh = torch.zeros(n, d, device="cuda")
    dws = []
    for st in shard_states:
        p, dw = vp_backward_shard(st, lse, den)
        dh += p
        dws.append(dw)
    torch.cuda.synchronize()
    torch.testing.assert_close(losses.cpu(), loss, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(ents.cpu(), ent, rtol=2e-3, atol=2e-3)
    torch.testing.assert_close(lse.cpu(), lse_ref, rtol=1e-5, atol=1e-5)
    assert torch.equal(hits.cpu(), corr)
    assert abs(float(sums[0]) - float(loss.sum())) <= 1e-4 * float(loss.sum())
    assert cosine(dh, grad @ weight.float()) >= 0.9999
    assert cosine(torch.cat(dws), grad.t() @ hidden.float()) >= 0.9999


def test_fused_ce_ragged_rows_over_several_pair_tiles():
    # 700 rows: two full 256-row pair tiles and a ragged third
    _check_fused(700, 8192, 256, seed=8)


def test_fused_ce_benchmark_configuration_against_torch_fp32():
    # the benchmark's exact workload (2048 tokens, V 151936, D 1536, its seeded inputs)
    # against plain PyTorch fp32 on the GPU: logits, log-softmax, dlogits, dH and dW
    import bench

    dev = torch.device("cuda")
    hidden_cpu, labels_cpu, weight = bench.make_inputs(0, dev)
    hidden, labels = hidden_cpu.to(dev), labels_cpu.to(dev)
    den = float((labels_cpu != -100).sum())
    losses, ents, hits, sums, dh, dw = fused_linear_cross_entropy(
        hidden, weight, labels, den, -100, True, compute_dw=True, dw_dtype=torch.float32)
    torch.cuda.synchronize()
    assert _lib.device_error(dev) == 0
    h32, w32 = hidden.float(), weight.float()
    logits = h32 @ w32.t()
    logp = torch.log_softmax(logits, dim=-1)
    valid = labels != -100
    t = labels.clamp_min(0)
    loss_ref = torch.where(valid, -logp.gather(1, t[:, None])[:, 0], torch.zeros_like(logp[:, 0]))
    ent_ref = -(logp.exp() * logp).sum(-1)
    top2 = logits.topk(2, dim=-1)
    hit_ref = valid & (top2.indices[:, 0] == labels)
    dl = logp.exp()
    dl[valid.nonzero()[:, 0], t[valid]] -= 1.0
    dl[~valid] = 0.0
    dl /= den
    dh_ref = dl @ w32
    dw_ref = dl.t() @ h32
    del logits, logp, dl
    torch.testing.assert_close(losses, loss_ref, rtol=1e-4, atol=1e-4)
    assert abs(float(sums[0]) - float(loss_ref.sum())) <= 1e-4 * abs(float(loss_ref.sum()))
    torch.testing.assert_close(ents, ent_ref, rtol=2e-3, atol=2e-3)
    diff = (hits.bool() != hit_ref).nonzero().flatten()
    if diff.numel():  # only provable near-ties of the fp32 logits may differ
        gap = (top2.values[diff, 0] - top2.values[diff, 1]).abs()
        assert bool((gap < 1e-4 * top2.values[diff, 0].abs().clamp_min(1)).all()), (diff, gap)
    assert diff.numel() <= 2
    assert int(sums[1]) == int(hits.sum())
    assert cosine(dh, dh_ref) >= 0.9999
    assert cosine(dw, dw_ref) >= 0.9999


def _planted_chunk(dtype, seed):
    """One 128-row chunk (B=4 x chunk 32) at the benchmark's vocab and dim; a third
    of the labelled rows have their target at the row's arg-max, so the hit count
    is far from zero and must agree exactly."""
    B, C, D, V = 4, 32, 1536, 151936
    g = torch.Generator(device="cuda").manual_seed(seed)  # the host generator is slow at this size
    piece = torch.randn(B, C, D, device="cuda", generator=g).to(dtype)
    W = (0.02 * torch.randn(V, D, device="cuda", generator=g)).to(dtype)
    target = torch.randint(0, V, (B, C), device="cuda", generator=g)
    opd = torch.bfloat16 if dtype == torch.bfloat16 else torch.float16
    logits = piece.to(opd).float().reshape(-1, D) @ W.to(opd).float().t()
    am = logits.argmax(-1).view(B, C)
    plant = torch.rand(B, C, device="cuda", generator=g) < 0.35
    target[plant] = am[plant]
    target[torch.rand(B, C, device="cuda", generator=g) < 0.1] = -100
    target[0, 0] = -100
    return piece.cpu(), W.cpu(), target.cpu(), logits


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_chunk_cross_entropy_triton_fused_branch(dtype):
    """The reference's one-chunk entry point with a module head (chunked_ce.py:183-264):
    total_loss = sum of the per-token losses (fp32), entropy / token_loss fp32 of
    the piece's leading shape, hits an int64 count, piece_grad fp16 (the reference's
    fp16 GEMM output) and None without gradient. The oracle gets the operands the
    GEMM multiplies: bf16 as given, other dtypes rounded to fp16 as the reference
    rounds them (chunked_ce.py:196-199)."""
    from auspex_soup_demo_b200.kernels import chunk_cross_entropy_triton

    piece, W, target, logits = _planted_chunk(dtype, seed=21 + int(dtype.itemsize))
    den = float((target != -100).sum())
    opd = torch.bfloat16 if dtype == torch.bfloat16 else torch.float16
    ref = oracle.chunked_ce(piece.to(opd), W.to(opd), target, 32, den, compute_dw=False)
    ref_total = float(ref[2].sum())
    head = torch.nn.Linear(W.shape[1], W.shape[0], bias=False, dtype=dtype, device="cuda")
    with torch.no_grad():
        head.weight.copy_(W.cuda())
    total, ent, tok, hits, grad = chunk_cross_entropy_triton(head, piece.cuda(), target.cuda(),
                                                             -100, den, True)
    torch.cuda.synchronize()
    assert total.dtype == torch.float32 and total.dim() == 0
    assert abs(float(total) - ref_total) <= 1e-4 * abs(ref_total), (float(total), ref_total)
    assert abs(float(total) - float(tok.sum())) <= 1e-5 * abs(ref_total)
    assert ent.shape == tok.shape == target.shape
    assert ent.dtype == tok.dtype == torch.float32
    torch.testing.assert_close(tok.cpu(), ref[2], rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(ent.cpu(), ref[1], rtol=2e-3, atol=2e-3)
    assert hits.dtype == torch.int64
    assert int(hits) == int(ref[3]) and int(hits) > 20
    assert grad.shape == piece.shape and grad.dtype == torch.float16
    assert cosine(grad, ref[4]) >= 0.9999
    # without gradient: same metrics, no piece_grad
    total2, _, tok2, hits2, grad2 = chunk_cross_entropy_triton(head, piece.cuda(), target.cuda(),
                                                               -100, den, False)
    assert grad2 is None
    assert int(hits2) == int(hits)
    torch.testing.assert_close(tok2, tok, rtol=1e-6, atol=1e-6)
    assert _lib.device_error(torch.device("cuda")) == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_fused_ce_fp16_operands_match_the_reference_rounding(dtype):
    """fp16 / fp32 activations enter the logits GEMM as fp16 operands (kind::f16 with
    the f16 format), the reference's own rounding: against the oracle on the
    fp16-rounded operands the loss is within 1e-4, hits bit-exact, and dhidden (fp32
    for fp32 input) within cosine 0.9999."""
    piece, W, target, _ = _planted_chunk(dtype, seed=33)
    B, C, D = piece.shape
    den = float((target != -100).sum())
    ref = oracle.chunked_ce(piece.half(), W.half(), target, 32, den, compute_dw=False)
    head = torch.nn.Linear(D, W.shape[0], bias=False, dtype=dtype, device="cuda")
    with torch.no_grad():
        head.weight.copy_(W.cuda())
    head.weight.requires_grad_(False)
    Fn = make_triton_chunked_loss_function()
    h = piece.cuda().requires_grad_(True)
    loss, ent, tok, corr = Fn.apply(h, head, target.cuda(), 32, den, -100, True)
    loss.backward()
    assert abs(float(loss.detach()) - float(ref[0])) <= 1e-4 * abs(float(ref[0]))
    torch.testing.assert_close(tok.cpu(), ref[2], rtol=1e-4, atol=1e-4)
    assert int(corr) == int(ref[3])
    assert h.grad.dtype == dtype
    assert cosine(h.grad, ref[4]) >= 0.9999
