"""GPU checks of the QLoRA step: NF4 kernels vs the oracle (bit-exact), the
NF4 + LoRA linear vs a dense reference, and a small Qwen2 model trained with
the fused patches vs the same model on the original transformers code."""

import contextlib

import pytest
import torch

import oracle.nf4 as onf4
from auspex_soup_demo_b200 import _lib, apply, qlora
from helpers import cosine

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape,dtype", [((1536, 256), torch.bfloat16), ((8960, 64), torch.float32),
                                         ((64, 64), torch.float16)])
def test_nf4_quantize_dequantize_bit_exact(shape, dtype):
    g = torch.Generator().manual_seed(1)
    w = (0.02 * torch.randn(shape, generator=g)).to(dtype)
    w[0, :64] = 0.0  # an all-zero block
    code = onf4.nf4_code()
    p_ref, a_ref = onf4.nf4_quantize(w, code)
    p, a = qlora.nf4_quantize(w.cuda())
    assert torch.equal(a.cpu(), a_ref)
    assert torch.equal(p.cpu(), p_ref)
    d = qlora.nf4_dequantize(p, a, shape, dtype=torch.bfloat16)
    d_ref = onf4.nf4_dequantize(p_ref, a_ref, code, dtype=torch.bfloat16).view(shape)
    assert torch.equal(d.cpu(), d_ref)
    d32 = qlora.nf4_dequantize(p, a, shape, dtype=torch.float32)
    assert torch.equal(d32.cpu(), onf4.nf4_dequantize(p_ref, a_ref, code, dtype=torch.float32).view(shape))


@pytest.mark.parametrize("fused_max_k", [10 ** 9, 0])  # tcgen05 rank-r GEMM / cuBLAS path
def test_lora_nf4_linear_forward_backward(fused_max_k, monkeypatch):
    monkeypatch.setattr(qlora, "FUSED_MAX_K", fused_max_k)
    torch.manual_seed(0)
    lin = torch.nn.Linear(512, 384, bias=True, device="cuda", dtype=torch.bfloat16)
    mod = qlora.LoRANF4Linear(lin, r=16, alpha=32)
    torch.nn.init.normal_(mod.lora_B, std=0.05)
    x = torch.randn(3, 40, 512, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    y = mod(x)
    dy = torch.randn_like(y)
    y.backward(dy)
    # dense fp32 reference on the dequantised base weight
    wq = mod.dequantized_weight(torch.float32)
    xr = x.detach().float().requires_grad_(True)
    A = mod.lora_A.detach().clone().requires_grad_(True)
    B = mod.lora_B.detach().clone().requires_grad_(True)
    yr = xr @ wq.t() + mod.bias.float() + (xr @ A.t() @ B.t()) * mod.scaling
    yr.backward(dy.float())
    assert cosine(y, yr) > 0.9999
    assert cosine(x.grad, xr.grad) > 0.9999
    assert cosine(mod.lora_A.grad, A.grad) > 0.9999
    assert cosine(mod.lora_B.grad, B.grad) > 0.9999


@contextlib.contextmanager
def original_transformers_code():
    """Temporarily restore the unpatched Qwen2 functions."""
    from transformers.models.qwen2 import modeling_qwen2 as m

    saved = (m.Qwen2RMSNorm.forward, m.Qwen2MLP.forward, m.apply_rotary_pos_emb)
    m.Qwen2RMSNorm.forward = getattr(saved[0], "_soup_original", saved[0])
    m.Qwen2MLP.forward = getattr(saved[1], "_soup_original", saved[1])
    m.apply_rotary_pos_emb = getattr(saved[2], "_soup_original", saved[2])
    try:
        yield
    finally:
        m.Qwen2RMSNorm.forward, m.Qwen2MLP.forward, m.apply_rotary_pos_emb = saved


class EagerHeadLoss(torch.autograd.Function):
    """Unfused head CE with the reference's chunked-loss signature (fp32 logits)."""

    @staticmethod
    def forward(ctx, hidden, head, target, chunk, denominator, ignore_index, with_grad):
        with torch.enable_grad():
            h = hidden.detach().requires_grad_(True)
            logits = (h @ head.weight.t()).float()
            loss = torch.nn.functional.cross_entropy(
                logits.view(-1, logits.shape[-1]), target.view(-1), ignore_index=ignore_index,
                reduction="sum") / denominator
            (g,) = torch.autograd.grad(loss, h)
        ctx.save_for_backward(g)
        z = torch.zeros(hidden.shape[:2], device=hidden.device)
        return loss.detach(), z, z, torch.zeros((), dtype=torch.long, device=hidden.device)

    @staticmethod
    def backward(ctx, gl, *_):
        (g,) = ctx.saved_tensors
        return g * gl, None, None, None, None, None, None


def _small_model(seed=0):
    cfg = qlora.qwen2_1p5b_config(num_layers=2, hidden_size=256, intermediate_size=640,
                                  num_attention_heads=4, num_key_value_heads=2, vocab_size=2048)
    model = qlora.build_qwen2_qlora(cfg, device="cuda", seed=seed)
    for m in model.modules():  # non-zero B so all LoRA factors receive gradients
        if isinstance(m, qlora.LoRANF4Linear):
            torch.nn.init.normal_(m.lora_B, std=0.02)
    return model


def _grads(model, ids, labels, loss_fn):
    model.zero_grad(set_to_none=True)
    hidden = model.model(input_ids=ids).last_hidden_state
    den = float((labels != -100).sum())
    loss, *_ = loss_fn.apply(hidden, model.lm_head, labels, 64, den, -100, True)
    loss.backward()
    return float(loss), {n: p.grad.detach().clone() for n, p in model.named_parameters()
                         if p.requires_grad}


def test_patched_qwen2_matches_original_code():
    from auspex_soup_demo_b200.kernels import make_triton_chunked_loss_function

    apply()
    model = _small_model()
    model.train()
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(0, 2048, (2, 96), generator=g).cuda()
    labels = qlora.causal_labels(ids)
    loss_fused, g_fused = _grads(model, ids, labels, make_triton_chunked_loss_function())
    with original_transformers_code():
        loss_ref, g_ref = _grads(model, ids, labels, EagerHeadLoss)
    assert abs(loss_fused - loss_ref) <= 2e-3 * abs(loss_ref), (loss_fused, loss_ref)
    worst = min(cosine(g_fused[k], g_ref[k]) for k in g_ref)
    assert worst > 0.99, worst
    assert sum(cosine(g_fused[k], g_ref[k]) for k in g_ref) / len(g_ref) > 0.999


@contextlib.contextmanager
def _fp32_activations(model):
    """Run the model in fp32: the 16-bit parameters and buffers (embedding, norms,
    biases) are swapped for fp32 copies (the NF4 base weights dequantise to the
    activation dtype; the LoRA factors are fp32 already), then restored."""
    saved = []
    for t in list(model.parameters()) + list(model.buffers()):
        if t.dtype in (torch.bfloat16, torch.float16):
            saved.append((t, t.data))
            t.data = t.data.float()
    try:
        yield
    finally:
        for t, d in saved:
            t.data = d


def test_patched_qwen2_is_as_accurate_as_the_original_bf16_code():
    """The fused bf16 step and transformers' own bf16 step, both against the same
    model run in fp32 on transformers' code: per LoRA parameter, the fused step's
    gradient error (1 - cosine to fp32) is at most twice the unfused bf16 step's
    plus 1e-5, and its loss error at most twice the unfused one's plus 1e-4
    relative. Two bf16 paths that differ only in rounding order agree with each
    other only to the size of their common error, which this bounds instead."""
    from auspex_soup_demo_b200.kernels import make_triton_chunked_loss_function

    apply()
    model = _small_model(seed=2)
    model.train()
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, 2048, (2, 96), generator=g).cuda()
    labels = qlora.causal_labels(ids)
    loss_fused, g_fused = _grads(model, ids, labels, make_triton_chunked_loss_function())
    with original_transformers_code():
        loss_bf16, g_bf16 = _grads(model, ids, labels, EagerHeadLoss)
        with _fp32_activations(model):
            loss_32, g_32 = _grads(model, ids, labels, EagerHeadLoss)
    err_f = abs(loss_fused - loss_32) / abs(loss_32)
    err_b = abs(loss_bf16 - loss_32) / abs(loss_32)
    assert err_f <= 2 * err_b + 1e-4, (err_f, err_b)
    worst = []
    for k in g_32:
        e_f = 1 - cosine(g_fused[k], g_32[k])
        e_b = 1 - cosine(g_bf16[k], g_32[k])
        worst.append((e_f - 2 * e_b, k, e_f, e_b))
        assert e_f <= 2 * e_b + 1e-5, (k, e_f, e_b)
    assert sum(1 - e for _, _, e, _ in worst) / len(worst) > 0.999


def test_qlora_trainer_reduces_loss():
    apply()
    model = _small_model(seed=1)
    trainer = qlora.QLoRATrainer(model, lr=2e-3)
    g = torch.Generator().manual_seed(4)
    ids = torch.randint(0, 2048, (4, 64), generator=g).cuda()
    labels = qlora.causal_labels(ids)
    den = float((labels != -100).sum())
    losses = [float(trainer.step(ids, labels, den)[0]) for _ in range(8)]
    assert losses[-1] < losses[0] - 0.05, losses


def test_trained_adapter_saves_and_reloads_as_peft(tmp_path):
    from auspex_soup_demo_b200 import adapter

    apply()
    model = _small_model(seed=2)
    trainer = qlora.QLoRATrainer(model, lr=2e-3)
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, 2048, (2, 64), generator=g).cuda()
    labels = qlora.causal_labels(ids)
    den = float((labels != -100).sum())
    for _ in range(3):
        trainer.step(ids, labels, den)
    out = trainer.save_adapter(str(tmp_path / "adapter"))
    listing = adapter.header_listing(str(tmp_path / "adapter" / "adapter_model.safetensors"))
    assert len(listing) == 2 * 7 * 2 and all(v[0] == "F32" for v in listing.values())
    fresh = _small_model(seed=2)  # same NF4 base, different (perturbed) LoRA B
    adapter.load_adapter(fresh, out)
    model.eval()
    fresh.eval()
    with torch.no_grad():
        a = model(input_ids=ids).logits
        b = fresh(input_ids=ids).logits
    assert torch.equal(a, b)


def test_captured_step_matches_eager_steps():
    # the whole train step (fused ops, head CE, backward, AdamW) recorded as one CUDA
    # graph and replayed on new batches
    apply()
    g = torch.Generator().manual_seed(6)
    batches = [torch.randint(0, 2048, (2, 256), generator=g).cuda() for _ in range(3)]
    labels = [qlora.causal_labels(b) for b in batches]
    den = float((labels[0] != -100).sum())

    eager = qlora.QLoRATrainer(_small_model(seed=3), lr=1e-3)
    ref = []
    for _ in range(4):  # the capture's 3 warm-up steps + the captured step, on batch 0
        ref.append(float(eager.step(batches[0], labels[0], den)[0]))
    for b, lab in zip(batches[1:], labels[1:]):
        ref.append(float(eager.step(b, lab, den)[0]))

    graphed = qlora.QLoRATrainer(_small_model(seed=3), lr=1e-3)
    init = {n: p.detach().clone() for n, p in graphed.model.named_parameters() if p.requires_grad}
    ids = batches[0].clone()
    lab = labels[0].clone()
    graphed.capture(ids, lab, den, warmup=3)
    got = []
    loss, _ = graphed.replay()
    got.append(float(loss))
    for b, l2 in zip(batches[1:], labels[1:]):
        ids.copy_(b)
        lab.copy_(l2)
        loss, _ = graphed.replay()
        got.append(float(loss))
    torch.cuda.synchronize()
    graphed.release_graph()
    assert _lib.device_error(torch.device("cuda")) == 0
    # Replays follow the eager steps to 1e-4 of the loss (the attention backward's
    # accumulation order varies between runs and AdamW magnifies it); the batches'
    # losses differ from one another by ~5e-3, so stale graph inputs would show.
    for a, b in zip(ref[3:], got):
        assert abs(a - b) <= 1e-4 * abs(a), (ref[3:], got)
    assert abs(got[1] - got[2]) > 1e-3, got
    pa = dict(eager.model.named_parameters())
    for n, p in graphed.model.named_parameters():
        if p.requires_grad:  # the 6 updates agree in direction
            assert cosine(p - init[n], pa[n] - init[n]) > 0.99, n


def _small_model_grouped(seed, group):
    cfg = qlora.qwen2_1p5b_config(num_layers=2, hidden_size=256, intermediate_size=640,
                                  num_attention_heads=4, num_key_value_heads=2, vocab_size=2048)
    model = qlora.build_qwen2_qlora(cfg, device="cuda", seed=seed, group=group)
    torch.manual_seed(seed + 7)
    for m in model.modules():
        if isinstance(m, qlora.LoRANF4Linear):
            torch.nn.init.normal_(m.lora_B, std=0.02)
    return model


@pytest.mark.parametrize("recompute", [True, False])
def test_grouped_projections_match_separate_modules(recompute, monkeypatch):
    # q/k/v and gate/up as one GEMM each (LoRAProjectionGroup) vs every projection
    # on its own: same loss and LoRA gradients up to bf16 accumulation order
    from auspex_soup_demo_b200.kernels import make_triton_chunked_loss_function
    from auspex_soup_demo_b200.kernels import swiglu as sw

    apply()
    monkeypatch.setattr(sw, "RECOMPUTE", recompute)
    g = torch.Generator().manual_seed(11)
    ids = torch.randint(0, 2048, (2, 96), generator=g).cuda()
    labels = qlora.causal_labels(ids)
    fn = make_triton_chunked_loss_function()
    grouped = _small_model_grouped(5, True)
    assert grouped.model.layers[0].self_attn.k_proj.lora_group is not None
    separate = _small_model_grouped(5, False)
    grouped.train()
    separate.train()
    l1, g1 = _grads(grouped, ids, labels, fn)
    l2, g2 = _grads(separate, ids, labels, fn)
    assert abs(l1 - l2) <= 1e-3 * abs(l2), (l1, l2)
    worst = min(cosine(g1[k], g2[k]) for k in g2)
    assert worst > 0.999, worst
    # through the trainer (stacked As, block-diagonal B and gradient views of the flat buffers)
    den = float((labels != -100).sum())
    t1 = qlora.QLoRATrainer(_small_model_grouped(6, True), lr=1e-3)
    t2 = qlora.QLoRATrainer(_small_model_grouped(6, False), lr=1e-3)
    a = [float(t1.step(ids, labels, den)[0]) for _ in range(3)]
    b = [float(t2.step(ids, labels, den)[0]) for _ in range(3)]
    for x, y in zip(a, b):
        assert abs(x - y) <= 2e-3 * abs(y), (a, b)
    assert a[-1] < a[0]
    p1 = dict(t1.model.named_parameters())
    for n, p in t2.model.named_parameters():
        if p.requires_grad:
            assert cosine(p1[n].grad, p.grad) > 0.99, n


def test_mlp_recompute_and_kept_activations_give_identical_gradients(monkeypatch):
    # the reference recomputes gate/up in the MLP backward (swiglu.py:197-214); keeping
    # [g | u] from the forward instead runs the same kernels on the same inputs, so the
    # loss and every LoRA gradient must agree bit for bit
    from auspex_soup_demo_b200.kernels import make_triton_chunked_loss_function
    from auspex_soup_demo_b200.kernels import swiglu as sw

    apply()
    g = torch.Generator().manual_seed(12)
    ids = torch.randint(0, 2048, (2, 160), generator=g).cuda()
    labels = qlora.causal_labels(ids)
    fn = make_triton_chunked_loss_function()
    out = {}
    for group in (True, False):
        for recompute in (True, False):
            monkeypatch.setattr(sw, "RECOMPUTE", recompute)
            model = _small_model_grouped(9, group)
            model.train()
            out[(group, recompute)] = _grads(model, ids, labels, fn)
    for group in (True, False):
        l1, g1 = out[(group, True)]
        l2, g2 = out[(group, False)]
        assert l1 == l2, (group, l1, l2)
        assert g1.keys() == g2.keys()
        for k in g1:
            assert torch.equal(g1[k], g2[k]), (group, k)


def test_fused_mlp_backward_gives_identical_gradients(monkeypatch):
    # the MLP as one Function (SwiGLU backward in the down projection's dX GEMM
    # epilogue, [dg | du] written over the kept [g | u]) against gate/up and down
    # as two Functions with the SwiGLU backward as an elementwise pass
    from auspex_soup_demo_b200.kernels import make_triton_chunked_loss_function
    from auspex_soup_demo_b200.kernels import swiglu as sw

    apply()
    monkeypatch.setattr(sw, "RECOMPUTE", False)
    g = torch.Generator().manual_seed(13)
    ids = torch.randint(0, 2048, (2, 200), generator=g).cuda()
    labels = qlora.causal_labels(ids)
    fn = make_triton_chunked_loss_function()
    out = {}
    for fused in (True, False):
        monkeypatch.setattr(qlora, "FUSE_MLP_BACKWARD", fused)
        model = _small_model_grouped(10, True)
        model.train()
        out[fused] = _grads(model, ids, labels, fn)
    (l1, g1), (l2, g2) = out[True], out[False]
    assert l1 == l2, (l1, l2)
    assert g1.keys() == g2.keys()
    for k in g1:
        assert torch.equal(g1[k], g2[k]), k


@pytest.mark.parametrize("n,n_scaled,wd", [(4096 * 37, 4096 * 5, 0.0), (100003, 77, 0.01)])
def test_adamw_flat_matches_torch_adamw(n, n_scaled, wd):
    # the fused flat-buffer AdamW (vector path for n % 4 == 0, scalar otherwise)
    # against torch.optim.AdamW on the same parameters and gradients, 3 steps
    g = torch.Generator(device="cuda").manual_seed(21)
    p0 = torch.randn(n, device="cuda", generator=g)
    grads = [torch.randn(n, device="cuda", generator=g) * (i + 1) for i in range(3)]
    lr, scale = 2e-3, 2.0
    ref = p0.clone().requires_grad_(True)
    opt = torch.optim.AdamW([ref], lr=lr, weight_decay=wd, foreach=False, fused=False)
    p, m, v = p0.clone(), torch.zeros_like(p0), torch.zeros_like(p0)
    p16 = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    step = torch.zeros((), device="cuda")
    for gr in grads:
        ref.grad = gr.clone()
        opt.step()
        step.add_(1.0)
        _lib.call("soup_adamw_flat", p.device, p.data_ptr(), gr.data_ptr(), m.data_ptr(), v.data_ptr(), n,
                  step.data_ptr(), lr, 0.9, 0.999, 1e-8, wd, p16.data_ptr(), _lib.BF16, n_scaled, scale,
                  _lib.stream_of(p))
    torch.cuda.synchronize()
    st = opt.state[ref]
    torch.testing.assert_close(p, ref.detach(), rtol=1e-5, atol=1e-7)
    # the kernel rounds m + (1 - beta1) (g - m) once (FMA), torch twice: moments of
    # O(1) differ by up to an ulp of their inputs where the update nearly cancels
    torch.testing.assert_close(m, st["exp_avg"], rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(v, st["exp_avg_sq"], rtol=1e-5, atol=1e-6)
    want16 = torch.cat([p[:n_scaled] * scale, p[n_scaled:]]).to(torch.bfloat16)
    assert torch.equal(p16, want16)


def test_qlora_model_with_soup_attention_matches_sdpa():
    """The same small model (head dim 128) with the tcgen05 attention and with
    transformers' SDPA: loss and LoRA gradients agree."""
    from auspex_soup_demo_b200.kernels import make_triton_chunked_loss_function

    apply()
    results = []
    for attention in ("sdpa", "soup"):
        cfg = qlora.qwen2_1p5b_config(num_layers=2, hidden_size=512, intermediate_size=1024,
                                      num_attention_heads=4, num_key_value_heads=2,
                                      vocab_size=2048, attention=attention)
        model = qlora.build_qwen2_qlora(cfg, device="cuda", seed=6)
        torch.manual_seed(7)  # the same non-zero B factors in both models
        for m in model.modules():
            if isinstance(m, qlora.LoRANF4Linear):
                torch.nn.init.normal_(m.lora_B, std=0.02)
        model.train()
        g = torch.Generator().manual_seed(8)
        ids = torch.randint(0, 2048, (2, 256), generator=g).cuda()
        labels = qlora.causal_labels(ids)
        results.append(_grads(model, ids, labels, make_triton_chunked_loss_function()))
    (l_sdpa, g_sdpa), (l_soup, g_soup) = results
    assert abs(l_soup - l_sdpa) <= 2e-3 * abs(l_sdpa), (l_soup, l_sdpa)
    cos = [cosine(g_soup[k], g_sdpa[k]) for k in g_sdpa]
    assert min(cos) > 0.99 and sum(cos) / len(cos) > 0.999, min(cos)


@pytest.mark.parametrize("group", [True, False])
def test_rank_kernels_give_matching_gradients(group, monkeypatch):
    # the LoRA rank products (xa, dxa and the gA / gB accumulations) on
    # soup_lora_rank_gemm against cuBLAS, through the trainer (fp32 gradient
    # views, transposed 16-bit B copies). Both paths round xa and dxa to bf16
    # after fp32 sums taken in a different order, so single elements differ by
    # one bf16 ulp and that propagates through the model: the second step's
    # gradients agree to a cosine of ~0.99989 (0.9995 asserted)
    apply()
    g = torch.Generator().manual_seed(14)
    ids = torch.randint(0, 2048, (2, 96), generator=g).cuda()
    labels = qlora.causal_labels(ids)
    den = float((labels != -100).sum())
    out = {}
    for rank in (True, False):
        monkeypatch.setattr(qlora, "RANK_KERNELS", rank)
        trainer = qlora.QLoRATrainer(_small_model_grouped(15, group), lr=1e-3)
        losses = [float(trainer.step(ids, labels, den)[0]) for _ in range(2)]
        grads = {n: p.grad.clone() for n, p in trainer.model.named_parameters() if p.requires_grad}
        out[rank] = (losses, grads)
    (l1, g1), (l2, g2) = out[True], out[False]
    for a, b in zip(l1, l2):
        assert abs(a - b) <= 1e-3 * abs(b), (l1, l2)
    worst = min(cosine(g1[k], g2[k]) for k in g2)
    assert worst > 0.9995, worst


def test_dual_rank_product_gives_matching_gradients(monkeypatch):
    # the gate/up group's dxa and B-gradient product from one pass over its
    # output gradient (soup_lora_rank_dual) against cuBLAS's two products,
    # through the trainer; the width limits are lowered so the small model's
    # gate/up gradient [192, 1280] takes the kernel. dxa is rounded to bf16 after
    # fp32 sums in a different order, as in the rank-kernel comparison above
    apply()
    monkeypatch.setattr(qlora, "DUAL_MIN_COLS", 1024)
    monkeypatch.setattr(qlora, "DUAL_MIN_ROWS", 128)
    g = torch.Generator().manual_seed(15)
    ids = torch.randint(0, 2048, (2, 96), generator=g).cuda()
    labels = qlora.causal_labels(ids)
    den = float((labels != -100).sum())
    out = {}
    for dual in (True, False):
        monkeypatch.setattr(qlora, "DUAL_RANK", dual)
        trainer = qlora.QLoRATrainer(_small_model_grouped(16, True), lr=1e-3)
        losses = [float(trainer.step(ids, labels, den)[0]) for _ in range(2)]
        grads = {n: p.grad.clone() for n, p in trainer.model.named_parameters() if p.requires_grad}
        out[dual] = (losses, grads)
    (l1, g1), (l2, g2) = out[True], out[False]
    for a, b in zip(l1, l2):
        assert abs(a - b) <= 1e-3 * abs(b), (l1, l2)
    worst = min(cosine(g1[k], g2[k]) for k in g2)
    assert worst > 0.9995, worst
