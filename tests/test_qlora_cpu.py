"""CPU checks of the QLoRA step's host logic: NF4 code table, labels, and the
data-parallel plumbing (DDP over the LoRA factors) with two gloo ranks."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

import oracle.nf4 as onf4
from auspex_soup_demo_b200 import qlora


def test_nf4_code_table_matches_the_oracle_construction():
    a = torch.tensor(qlora.nf4_code_values())
    b = onf4.nf4_code()
    assert torch.equal(a, b)
    assert a[0] == -1.0 and a[-1] == 1.0 and (a == 0).sum() == 1
    assert bool((a[1:] > a[:-1]).all())


def test_nf4_oracle_round_trip_error():
    code = onf4.nf4_code()
    w = torch.randn(64 * 512) * 0.02
    packed, absmax = onf4.nf4_quantize(w, code)
    assert packed.numel() == w.numel() // 2 and absmax.numel() == w.numel() // 64
    back = onf4.nf4_dequantize(packed, absmax, code, dtype=torch.float32)
    rel = float((back - w).norm() / w.norm())
    assert rel < 0.12, rel
    # every block's largest-magnitude element is exact (code +-1 times absmax)
    blocks = w.view(-1, 64)
    i = blocks.abs().argmax(dim=1)
    assert torch.allclose(back.view(-1, 64).gather(1, i[:, None]), blocks.gather(1, i[:, None]))


def test_causal_labels():
    ids = torch.tensor([[5, 6, 7, 8]])
    assert qlora.causal_labels(ids).tolist() == [[6, 7, 8, -100]]


class EagerChunkedLoss(torch.autograd.Function):
    """CPU stand-in with the reference's chunked-loss signature (for host-logic tests)."""

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
        z = torch.zeros(hidden.shape[:2])
        return loss.detach(), z, z, torch.zeros((), dtype=torch.long)

    @staticmethod
    def backward(ctx, gl, *_):
        (g,) = ctx.saved_tensors
        return g * gl, None, None, None, None, None, None


def _tiny_cfg():
    return qlora.qwen2_1p5b_config(num_layers=2, hidden_size=64, intermediate_size=128,
                                   num_attention_heads=4, num_key_value_heads=2, vocab_size=97)


def _batch(seed, n=2, s=12):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, 97, (n, s), generator=g)
    return ids, qlora.causal_labels(ids)


def _worker(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.manual_seed(0)
    model = qlora.build_qwen2_qlora(_tiny_cfg(), device="cpu", seed=0, quantize=False,
                                    dtype=torch.float32)
    for m in model.modules():  # non-zero B so every LoRA factor gets a gradient
        if isinstance(m, qlora.LoRADenseLinear):
            torch.nn.init.normal_(m.lora_B, std=0.02)
    trainer = qlora.QLoRATrainer(model, lr=1e-2, ddp=True, loss_fn=EagerChunkedLoss)
    ids, labels = _batch(100 + rank)
    total_valid = sum(int((_batch(100 + r)[1] != -100).sum()) for r in range(world))
    # DDP averages gradients over ranks: each rank's loss is scaled so the
    # average equals the mean loss over the union of the ranks' batches
    trainer.step(ids, labels, total_valid / world)
    state = {n: p.detach().clone() for n, p in model.named_parameters() if p.requires_grad}
    torch.save(state, f"{out_path}.{rank}")
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_data_parallel_lora_step_matches_single_process(tmp_path):
    world = 2
    out = str(tmp_path / "state")
    mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, join=True,
                       start_method="spawn")
    s0 = torch.load(f"{out}.0")
    s1 = torch.load(f"{out}.1")
    for k in s0:
        assert torch.equal(s0[k], s1[k]), f"ranks diverged on {k}"
    # single process on the union batch
    torch.manual_seed(0)
    model = qlora.build_qwen2_qlora(_tiny_cfg(), device="cpu", seed=0, quantize=False,
                                    dtype=torch.float32)
    for m in model.modules():
        if isinstance(m, qlora.LoRADenseLinear):
            torch.nn.init.normal_(m.lora_B, std=0.02)
    trainer = qlora.QLoRATrainer(model, lr=1e-2, ddp=False, loss_fn=EagerChunkedLoss)
    b0, b1 = _batch(100), _batch(101)
    ids = torch.cat([b0[0], b1[0]])
    labels = torch.cat([b0[1], b1[1]])
    trainer.step(ids, labels, float((labels != -100).sum()))
    ref = {n: p.detach() for n, p in model.named_parameters() if p.requires_grad}
    assert set(ref) == {k.replace("module.", "") for k in s0} or set(ref) == set(s0)
    # Adam's first step is lr * g / (|g| + eps): gradients that differ only by
    # fp32 summation order (two half-batch sums vs one) can move a near-zero
    # gradient's update; allow 1 % of the learning rate.
    for k, v in s0.items():
        kk = k.replace("module.", "")
        torch.testing.assert_close(v, ref[kk], rtol=1e-3, atol=1e-4)


def test_projection_groups_share_buffers_and_trainer_views():
    # q/k/v and gate/up groups: the members' base weights and biases are views of
    # the group's concatenated buffers, and the trainer's stacked As / gradient
    # views and block-diagonal B equal what the group builds from its members
    cfg = qlora.qwen2_1p5b_config(num_layers=2, hidden_size=256, intermediate_size=640,
                                  num_attention_heads=4, num_key_value_heads=2, vocab_size=512)
    model = qlora.build_qwen2_qlora(cfg, device="cpu", quantize=False, seed=0)
    for m in model.modules():
        if isinstance(m, qlora.LoRADenseLinear):
            torch.nn.init.normal_(m.lora_B, std=0.02)
    layer = model.model.layers[1]
    qkv = layer.self_attn.q_proj.lora_group
    gu = layer.mlp.gate_proj.lora_group
    assert qkv.kind == "qkv" and qkv.members == [layer.self_attn.q_proj, layer.self_attn.k_proj,
                                                 layer.self_attn.v_proj]
    assert gu.kind == "gate_up" and gu.n_total == 2 * 640 and gu.bias is None
    assert layer.self_attn.o_proj.lora_group is None and layer.mlp.down_proj.lora_group is None
    assert layer.self_attn.k_proj.weight.data_ptr() == qkv.weight[256].data_ptr()
    assert layer.self_attn.v_proj.bias.data_ptr() == qkv.bias[384:].data_ptr()
    As_ref, B_ref = qkv.factors(torch.bfloat16)  # built from the members (no trainer yet)
    trainer = qlora.QLoRATrainer(model, lr=1e-3, loss_fn=EagerChunkedLoss)
    for g in (qkv, gu):
        assert g.As16 is not None and g.Bblk16.shape == (g.n_total, g.r_total)
        g_as, g_b = g.As16, g.Bblk16
        g.As16 = None  # rebuild from the members for comparison
        a2, b2 = g.factors(torch.bfloat16)
        g.As16 = g_as
        assert torch.equal(g_as, a2) and torch.equal(g_b, b2)
        assert g.gradA.data_ptr() == g.members[0].lora_A.grad.data_ptr()
    assert torch.equal(qkv.As16, As_ref) and torch.equal(qkv.Bblk16, B_ref)
    # after an optimiser step the copies follow the fp32 factors
    ids = torch.randint(0, 512, (2, 16))
    labels = qlora.causal_labels(ids)
    trainer.step(ids, labels, float((labels != -100).sum()))
    g_b = gu.Bblk16.clone()
    gu_as = gu.As16
    gu.As16 = None
    _, b2 = gu.factors(torch.bfloat16)
    gu.As16 = gu_as
    assert torch.equal(g_b, b2)


def test_interleaved_gate_up_members_keep_their_weights():
    # gate/up rows are stored interleaved in blocks of 128 inside the group; each
    # member still returns its own [out, in] base weight
    cfg = qlora.qwen2_1p5b_config(num_layers=1, hidden_size=256, intermediate_size=384,
                                  num_attention_heads=4, num_key_value_heads=2, vocab_size=512)
    grouped = qlora.build_qwen2_qlora(cfg, device="cpu", quantize=False, seed=3)
    plain = qlora.build_qwen2_qlora(cfg, device="cpu", quantize=False, seed=3, group=False)
    g = grouped.model.layers[0].mlp.gate_proj.lora_group
    assert g.interleaved and g.weight.shape == (768, 256)
    for name in ("gate_proj", "up_proj"):
        a = getattr(grouped.model.layers[0].mlp, name).base_weight(torch.float32)
        b = getattr(plain.model.layers[0].mlp, name).base_weight(torch.float32)
        assert torch.equal(a, b), name
    # block c of the group's rows: gate rows [128c, 128c+128), then the same up rows
    gw = plain.model.layers[0].mlp.gate_proj.weight
    uw = plain.model.layers[0].mlp.up_proj.weight
    assert torch.equal(g.weight[128:256], uw[:128]) and torch.equal(g.weight[256:384], gw[128:256])
