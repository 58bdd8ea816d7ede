"""PEFT adapter files: names, dtypes and shapes as the reference harness reads them
(``harness/run_task.py:62-72``), the LoraConfig fields it compares
(``harness/check_rules.py:171-183``), and save -> load round trips."""

import json
import os
import struct

import pytest
import torch

from auspex_soup_demo_b200 import adapter, qlora

TARGETS = sorted(qlora.LORA_TARGETS)


def small_model(seed=0, layers=2):
    cfg = qlora.qwen2_1p5b_config(num_layers=layers, hidden_size=64, intermediate_size=96,
                                  num_attention_heads=4, num_key_value_heads=2, vocab_size=128)
    cfg._attn_implementation = "eager"
    return qlora.build_qwen2_qlora(cfg, device="cpu", seed=seed, quantize=False,
                                   dtype=torch.float32)


def harness_listing(adapter_dir):
    # the reference harness's reader: 8-byte little-endian header size, JSON header
    with open(os.path.join(adapter_dir, "adapter_model.safetensors"), "rb") as fh:
        n = struct.unpack("<Q", fh.read(8))[0]
        header = json.loads(fh.read(n))
    return {k: [v.get("dtype"), v.get("shape")] for k, v in sorted(header.items())
            if k != "__metadata__"}


def test_full_size_names_and_shapes_match_peft_layout():
    # Qwen2.5-1.5B with r=16 on the seven projections: 18,464,768 LoRA parameters
    model = qlora.build_qwen2_qlora(qlora.qwen2_1p5b_config(), device="meta", quantize=False)
    mods = adapter.lora_modules(model)
    assert len(mods) == 28 * 7
    total = sum(m.lora_A.numel() + m.lora_B.numel() for m in mods.values())
    assert total == 18_464_768
    shapes = {p: (tuple(m.lora_A.shape), tuple(m.lora_B.shape)) for p, m in mods.items()}
    assert shapes["model.layers.0.self_attn.q_proj"] == ((16, 1536), (1536, 16))
    assert shapes["model.layers.0.self_attn.k_proj"] == ((16, 1536), (256, 16))
    assert shapes["model.layers.27.mlp.down_proj"] == ((16, 8960), (1536, 16))
    assert shapes["model.layers.5.mlp.gate_proj"] == ((16, 1536), (8960, 16))


def test_saved_files_as_the_harness_reads_them(tmp_path):
    model = small_model()
    out = adapter.save_adapter(model, str(tmp_path / "adapter"))
    listing = harness_listing(out)
    assert listing == adapter.header_listing(os.path.join(out, "adapter_model.safetensors"))
    assert len(listing) == 2 * 7 * 2
    k = "base_model.model.model.layers.1.self_attn.v_proj.lora_B.weight"
    assert listing[k] == ["F32", [32, 16]]  # 2 kv heads x head_dim 16
    assert listing["base_model.model.model.layers.0.mlp.down_proj.lora_A.weight"] == ["F32", [16, 96]]
    assert all(name.startswith("base_model.model.model.layers.") for name in listing)
    assert all(name.endswith((".lora_A.weight", ".lora_B.weight")) for name in listing)
    cfg = json.load(open(os.path.join(out, "adapter_config.json")))
    assert cfg["peft_type"] == "LORA" and cfg["task_type"] == "CAUSAL_LM"
    assert cfg["r"] == 16 and cfg["lora_alpha"] == 32 and cfg["bias"] == "none"
    assert sorted(cfg["target_modules"]) == TARGETS
    assert cfg["use_rslora"] is False and cfg["use_dora"] is False
    assert cfg["base_model_name_or_path"] == "Qwen/Qwen2.5-1.5B-Instruct"


def test_round_trip_restores_factors_and_outputs(tmp_path):
    a = small_model(seed=0)
    with torch.no_grad():
        for m in adapter.lora_modules(a).values():
            m.lora_B.normal_(0, 0.05)  # trained-looking B (init is zero)
    out = adapter.save_adapter(a, str(tmp_path / "ad"))
    b = small_model(seed=0)  # same frozen base, LoRA factors scrambled before the load
    with torch.no_grad():
        for m in adapter.lora_modules(b).values():
            m.lora_A.uniform_(-1, 1)
            m.lora_B.uniform_(-1, 1)
    cfg = adapter.load_adapter(b, out)
    assert cfg["r"] == 16
    for (pa, ma), (pb, mb) in zip(adapter.lora_modules(a).items(), adapter.lora_modules(b).items()):
        assert pa == pb
        assert torch.equal(ma.lora_A, mb.lora_A) and torch.equal(ma.lora_B, mb.lora_B)
    ids = torch.randint(0, 128, (2, 12), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        assert torch.equal(a(input_ids=ids).logits, b(input_ids=ids).logits)


def test_load_rejects_mismatches(tmp_path):
    from safetensors.torch import load_file, save_file

    model = small_model()
    out = adapter.save_adapter(model, str(tmp_path / "ad"))
    path = os.path.join(out, "adapter_model.safetensors")
    sd = {k: v.clone() for k, v in load_file(path).items()}  # detach from the mapped file
    # a missing tensor
    drop = dict(sd)
    drop.pop(next(iter(drop)))
    save_file(drop, path)
    with pytest.raises(KeyError):
        adapter.load_adapter(small_model(), out)
    adapter.load_adapter(small_model(), out, strict=False)
    # a different rank in the config
    save_file(sd, path)
    cfg_path = os.path.join(out, "adapter_config.json")
    cfg = json.load(open(cfg_path))
    cfg["r"] = 8
    json.dump(cfg, open(cfg_path, "w"))
    with pytest.raises(ValueError):
        adapter.load_adapter(small_model(), out)
    # a different scale
    cfg["r"] = 16
    cfg["lora_alpha"] = 16
    json.dump(cfg, open(cfg_path, "w"))
    with pytest.raises(ValueError):
        adapter.load_adapter(small_model(), out)
