"""One registry from the architecture's name (config.json `architectures[0]`, or `architecture`) to its model.

An architecture is three functions in one module: `load_config(dict)` gives the typed
configuration, `model_spec(config)` the ModelSpec, `ignorable(config, tensor_name)` says
which checkpoint tensors may go unused. The reference maps architecture names to model
packages in the same way, importing lazily and listing what it knows when a name is
unknown (src/tt_transformers/vllm_registry.py:84-111,170-177).
"""

from __future__ import annotations

import importlib
from dataclasses import dataclass
from typing import Callable, Dict, Union


class UnknownArchitecture(KeyError):
    pass


@dataclass(frozen=True)
class Architecture:
    load_config: Callable
    model_spec: Callable
    ignorable: Callable


_ARCHITECTURES: Dict[str, Union[str, Architecture]] = {
    "LlamaForCausalLM": "tt_transformers_b200.models.llama",
    "Bozavik": "tt_transformers_b200.models.bozavik",
    "Pedazen": "tt_transformers_b200.models.pedazen",
    "Sezanex": "tt_transformers_b200.models.sezanex",
    "Bufolorn": "tt_transformers_b200.models.bufolorn",
}


def register_architecture(name: str, load_config, model_spec, ignorable=lambda cfg, tensor: False) -> None:
    _ARCHITECTURES[name] = Architecture(load_config, model_spec, ignorable)


def known_architectures():
    return sorted(_ARCHITECTURES)


def get_architecture(name: str) -> Architecture:
    if name not in _ARCHITECTURES:
        raise UnknownArchitecture(f"architecture {name!r} is not registered; known: {known_architectures()}")
    entry = _ARCHITECTURES[name]
    if isinstance(entry, str):                         # imported on first use
        module = importlib.import_module(entry)
        entry = Architecture(module.load_config, module.model_spec, getattr(module, "ignorable", lambda c, t: False))
        _ARCHITECTURES[name] = entry
    return entry


def architecture_of(config_dict: dict) -> str:
    single = config_dict.get("architecture")
    if isinstance(single, str) and "architectures" not in config_dict:
        return single                                  # configurations that name their one class under 'architecture'
    archs = config_dict.get("architectures")
    if not isinstance(archs, list) or not archs or not isinstance(archs[0], str):
        from .config.base import ConfigError
        raise ConfigError("config.json: 'architectures' must be a list holding the model class name")
    return archs[0]
