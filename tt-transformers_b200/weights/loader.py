"""Weights from safetensors files, by tensor name.

The reference walks a loaded model object attribute by attribute
(src/tt_transformers/models/llama32_1b/hf_generator.py:224-262); the attribute paths
are the checkpoint's tensor names, which is what is read here, straight from the files.
Floating-point tensors are kept in bfloat16 unless they are stored in 32-bit, which
stays 32-bit (float16, whose mantissa bfloat16 cannot hold, becomes float32 when the engine
computes in float32, so that the 32-bit path loses nothing); integer tables become int32. All problems of a checkpoint are reported
together, in one error.
"""

from __future__ import annotations

import json
import os
from typing import Callable, Dict, Iterable, List

import torch
from safetensors import safe_open

from ..parts.base import TensorSpec


class WeightError(ValueError):
    """The checkpoint does not fit the model: missing, unexpected or misshapen tensors."""


_FLOAT = (torch.float16, torch.bfloat16, torch.float32, torch.float64)


def _checkpoint_files(folder: str) -> List[str]:
    index = os.path.join(folder, "model.safetensors.index.json")
    if os.path.isfile(index):
        with open(index) as f:
            weight_map = json.load(f).get("weight_map", {})
        return sorted({os.path.join(folder, name) for name in weight_map.values()})
    single = os.path.join(folder, "model.safetensors")
    if os.path.isfile(single):
        return [single]
    files = sorted(os.path.join(folder, n) for n in os.listdir(folder) if n.endswith(".safetensors"))
    if not files:
        raise WeightError(f"{folder}: no .safetensors file")
    return files


def _normalise(tensor: torch.Tensor, widen_float16: bool = False) -> torch.Tensor:
    if tensor.dtype in (torch.float32, torch.float64) or (widen_float16 and tensor.dtype == torch.float16):
        return tensor.to(torch.float32)          # stored in 32-bit (or wider): stays 32-bit
    if tensor.dtype in _FLOAT or tensor.dtype.is_floating_point:
        return tensor.to(torch.bfloat16)
    return tensor.to(torch.int32)                 # integer tables


def read_safetensors(folder: str, wanted: Iterable[str] = None, widen_float16: bool = False) -> Dict[str, torch.Tensor]:
    """name -> tensor on the CPU. With `wanted`, tensors of other names are listed
    (as zero-size placeholders are not needed, only their names and shapes are kept
    under the key '__unread__') instead of being read. widen_float16: float16 tensors become
    float32 instead of bfloat16 (for an engine that computes in float32)."""
    wanted = set(wanted) if wanted is not None else None
    tensors: Dict[str, torch.Tensor] = {}
    unread: Dict[str, tuple] = {}
    for path in _checkpoint_files(folder):
        if not os.path.isfile(path):
            raise WeightError(f"{path}: listed in the index but not present")
        with safe_open(path, framework="pt", device="cpu") as f:
            for name in f.keys():
                if wanted is None or name in wanted:
                    tensors[name] = _normalise(f.get_tensor(name), widen_float16)
                else:
                    unread[name] = tuple(f.get_slice(name).get_shape())
    tensors["__unread__"] = unread
    return tensors


def check_tensors(tensors: Dict[str, torch.Tensor], specs: List[TensorSpec],
                  ignorable: Callable[[str], bool] = lambda name: False) -> None:
    """Raise one WeightError that lists every missing tensor, every unexpected one and
    every wrong shape or kind; return silently if the checkpoint fits."""
    unread = tensors.get("__unread__", {})
    present = {n for n in tensors if n != "__unread__"} | set(unread)
    missing, wrong = [], []
    needed = set()
    for spec in specs:
        needed.add(spec.name)
        if spec.name not in tensors or spec.name == "__unread__":
            if not spec.optional:
                missing.append(f"{spec.name} {list(spec.shape)}")
            continue
        t = tensors[spec.name]
        if len(t.shape) != len(spec.shape) or any(want is not None and have != want for have, want in zip(t.shape, spec.shape)):
            wrong.append(f"{spec.name}: shape {list(t.shape)}, expected {list(spec.shape)}")
        elif spec.kind == "float" and not t.dtype.is_floating_point:
            wrong.append(f"{spec.name}: holds {t.dtype}, expected floating-point values")
        elif spec.kind == "int" and t.dtype.is_floating_point:
            wrong.append(f"{spec.name}: holds {t.dtype}, expected integers")
    unexpected = sorted(n for n in present - needed if not ignorable(n))
    if missing or wrong or unexpected:
        lines = ["the checkpoint does not fit the model:"]
        if missing:
            lines.append(f"  missing tensors ({len(missing)}): " + "; ".join(missing))
        if unexpected:
            lines.append(f"  unexpected tensors ({len(unexpected)}): " + "; ".join(unexpected))
        if wrong:
            lines.append(f"  wrong shapes or kinds ({len(wrong)}): " + "; ".join(wrong))
        raise WeightError("\n".join(lines))
