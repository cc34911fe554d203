"""Random weights for a configuration and a seed, written as a model folder.

The folder holds config.json and model.safetensors with the checkpoint's tensor names,
so it is read back exactly like a real model. Tensors are drawn in float32 from one CPU
generator seeded once, in the order of the model's tensor list, then stored in `dtype`.
The reference has no whole-model random weights; its tests seed tiny models per module
(tests/models/llama32_1b/test_hf_adaptor.py:178-190).
"""

from __future__ import annotations

import json
import os
from typing import Dict

import torch
from safetensors.torch import save_file

from ..parts.model import DecoderModel
from ..registry import architecture_of, get_architecture


def random_tensors(config_dict: dict, seed: int, std: float = 0.02, norm_std: float = 0.0,
                   dtype: torch.dtype = torch.bfloat16, device="cpu") -> Dict[str, torch.Tensor]:
    """Matrices ~ N(0, std); vectors (norm weights) 1 + N(0, norm_std). With a CUDA `device`
    the numbers are drawn there (other numbers than on the CPU for the same seed): large
    models for measurements are made in seconds that way."""
    arch = get_architecture(architecture_of(config_dict))
    model = DecoderModel(arch.model_spec(arch.load_config(config_dict)))
    gen = torch.Generator(device=device)
    gen.manual_seed(int(seed))
    out = {}
    for spec in model.tensor_specs():
        if spec.kind == "int":
            raise ValueError(f"{spec.name}: random integer tables are not defined")
        shape = tuple(spec.free_size if n is None else n for n in spec.shape)
        if len(shape) == 1:
            t = torch.ones(shape, dtype=torch.float32, device=device)
            if norm_std:
                t = t + torch.randn(shape, generator=gen, dtype=torch.float32, device=device) * norm_std
        else:
            t = torch.randn(shape, generator=gen, dtype=torch.float32, device=device) * std
        out[spec.name] = t.to(dtype).contiguous()
    return out


def write_model_folder(folder: str, config_dict: dict, seed: int, std: float = 0.02, norm_std: float = 0.0,
                       dtype: torch.dtype = torch.bfloat16) -> str:
    os.makedirs(folder, exist_ok=True)
    tensors = random_tensors(config_dict, seed, std, norm_std, dtype)
    config = dict(config_dict)
    config.setdefault("torch_dtype", str(dtype).replace("torch.", ""))
    with open(os.path.join(folder, "config.json"), "w") as f:
        json.dump(config, f, indent=1)
    save_file(tensors, os.path.join(folder, "model.safetensors"), metadata={"format": "pt"})
    return folder
