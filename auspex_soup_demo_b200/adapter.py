"""PEFT-format LoRA adapter files for the QLoRA path.

The reference trains through Soup + PEFT and its harness reads the result as a
standard PEFT LoRA adapter directory (``harness/run_task.py:62-72`` lists the
tensor names, dtypes and shapes from the ``adapter_model.safetensors`` header;
``harness/check_rules.py:171-183`` compares ``adapter_config.json`` key by key;
``harness/eval_adapter.py:29-34`` loads it with ``PeftModel.from_pretrained``).
This module writes and reads that layout for models built by
``qlora.build_qwen2_qlora``:

* ``adapter_model.safetensors``: for every LoRA-wrapped linear at module path
  ``P`` of the causal-LM model, ``base_model.model.P.lora_A.weight`` [r, in] and
  ``base_model.model.P.lora_B.weight`` [out, r] (PEFT's saved names: the
  ``base_model.model.`` prefix of ``PeftModelForCausalLM``, adapter name removed),
  in the parameters' dtype (fp32 here, as PEFT keeps LoRA factors of 4-bit
  models);
* ``adapter_config.json``: the ``LoraConfig`` fields PEFT writes for a plain
  LoRA adapter (``peft_type`` LORA, ``task_type`` CAUSAL_LM, ``r``,
  ``lora_alpha``, ``target_modules``, ...).

The LoRA scale is alpha / r in both (no rsLoRA), so ``y = base(x) + (alpha/r) B A x``
means the same thing when PEFT loads the factors.
"""

from __future__ import annotations

import json
import os
import re
from typing import Dict, Optional

import torch

ADAPTER_WEIGHTS = "adapter_model.safetensors"
ADAPTER_CONFIG = "adapter_config.json"
_PREFIX = "base_model.model."
_KEY = re.compile(r"^base_model\.model\.(.+)\.lora_([AB])\.weight$")


def lora_modules(model) -> Dict[str, torch.nn.Module]:
    """Module path -> LoRA-wrapped linear (anything with lora_A / lora_B parameters)."""
    out = {}
    for name, mod in model.named_modules():
        if isinstance(getattr(mod, "lora_A", None), torch.nn.Parameter) and \
                isinstance(getattr(mod, "lora_B", None), torch.nn.Parameter):
            out[name] = mod
    return out


def adapter_state_dict(model) -> Dict[str, torch.Tensor]:
    """PEFT-named LoRA tensors (CPU, contiguous, the parameters' dtype)."""
    sd = {}
    for path, mod in lora_modules(model).items():
        sd[f"{_PREFIX}{path}.lora_A.weight"] = mod.lora_A.detach().to("cpu").contiguous()
        sd[f"{_PREFIX}{path}.lora_B.weight"] = mod.lora_B.detach().to("cpu").contiguous()
    return sd


def adapter_config(model, base_model_name_or_path: str, r: Optional[int] = None,
                   lora_alpha: Optional[float] = None, lora_dropout: float = 0.0) -> dict:
    """The LoraConfig dictionary PEFT stores beside the weights."""
    mods = lora_modules(model)
    if not mods:
        raise ValueError("model has no LoRA-wrapped modules")
    first = next(iter(mods.values()))
    r = int(r if r is not None else first.lora_A.shape[0])
    if lora_alpha is None:
        lora_alpha = first.scaling * r
    alpha = float(lora_alpha)
    if alpha.is_integer():
        alpha = int(alpha)
    targets = sorted({path.rsplit(".", 1)[-1] for path in mods})
    return {
        "alpha_pattern": {},
        "base_model_name_or_path": base_model_name_or_path,
        "bias": "none",
        "fan_in_fan_out": False,
        "inference_mode": True,
        "init_lora_weights": True,
        "layers_pattern": None,
        "layers_to_transform": None,
        "lora_alpha": alpha,
        "lora_dropout": float(lora_dropout),
        "modules_to_save": None,
        "peft_type": "LORA",
        "r": r,
        "rank_pattern": {},
        "revision": None,
        "target_modules": targets,
        "task_type": "CAUSAL_LM",
        "use_dora": False,
        "use_rslora": False,
    }


def save_adapter(model, directory: str, base_model_name_or_path: str = "Qwen/Qwen2.5-1.5B-Instruct",
                 lora_dropout: float = 0.0) -> str:
    """Write ``adapter_model.safetensors`` + ``adapter_config.json``; returns the directory."""
    from safetensors.torch import save_file

    os.makedirs(directory, exist_ok=True)
    sd = adapter_state_dict(model)
    cfg = adapter_config(model, base_model_name_or_path, lora_dropout=lora_dropout)
    save_file(sd, os.path.join(directory, ADAPTER_WEIGHTS), metadata={"format": "pt"})
    with open(os.path.join(directory, ADAPTER_CONFIG), "w", encoding="utf-8") as fh:
        json.dump(cfg, fh, indent=2, sort_keys=True)
        fh.write("\n")
    return directory


def load_adapter(model, directory: str, strict: bool = True) -> dict:
    """Copy a PEFT LoRA adapter into the model's LoRA factors; returns its config.

    Checks that r and lora_alpha match the wrapped modules (the scale is baked
    into each module) and, with ``strict``, that the file and the model hold
    exactly the same set of LoRA tensors with the same shapes.
    """
    from safetensors.torch import load_file

    with open(os.path.join(directory, ADAPTER_CONFIG), encoding="utf-8") as fh:
        cfg = json.load(fh)
    if cfg.get("peft_type", "LORA") != "LORA":
        raise ValueError(f"not a LoRA adapter: peft_type={cfg.get('peft_type')}")
    if cfg.get("use_rslora") or cfg.get("use_dora"):
        raise ValueError("rsLoRA / DoRA adapters are not supported")
    tensors = load_file(os.path.join(directory, ADAPTER_WEIGHTS))
    mods = lora_modules(model)
    seen = set()
    for key, value in tensors.items():
        m = _KEY.match(key)
        if m is None:
            if strict:
                raise KeyError(f"unexpected tensor in adapter: {key}")
            continue
        path, which = m.group(1), m.group(2)
        mod = mods.get(path)
        if mod is None:
            if strict:
                raise KeyError(f"adapter tensor for a module the model does not wrap: {key}")
            continue
        param = mod.lora_A if which == "A" else mod.lora_B
        if tuple(param.shape) != tuple(value.shape):
            raise ValueError(f"{key}: shape {tuple(value.shape)} vs model {tuple(param.shape)}")
        with torch.no_grad():
            param.copy_(value.to(device=param.device, dtype=param.dtype))
        seen.add((path, which))
    if strict:
        missing = [f"{p}.lora_{w}" for p in mods for w in "AB" if (p, w) not in seen]
        if missing:
            raise KeyError(f"adapter lacks {len(missing)} LoRA tensors, e.g. {missing[:3]}")
    for path, mod in mods.items():
        r = mod.lora_A.shape[0]
        if int(cfg.get("r", r)) != r:
            raise ValueError(f"adapter r={cfg.get('r')} but {path} has rank {r}")
        alpha = float(cfg.get("lora_alpha", mod.scaling * r))
        if abs(alpha / r - mod.scaling) > 1e-12 * max(1.0, abs(mod.scaling)):
            raise ValueError(f"adapter scale {alpha}/{r} differs from {path}'s {mod.scaling}")
    return cfg


def header_listing(path: str) -> Dict[str, list]:
    """Names -> [dtype, shape] from a safetensors header (what the reference harness reads)."""
    import struct

    with open(path, "rb") as fh:
        n = struct.unpack("<Q", fh.read(8))[0]
        header = json.loads(fh.read(n))
    return {k: [v.get("dtype"), v.get("shape")] for k, v in sorted(header.items())
            if k != "__metadata__"}
