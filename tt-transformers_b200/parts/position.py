"""Position encodings.

`rotary`: rotation frequencies theta^(-2i/d), optionally with Llama-3 per-frequency
scaling (src/tt_transformers/models/llama3_8b/hf_generator.py:88-120). The frequencies
are computed once, in float32, by the same sequence of float32 operations that the
reference uses; the angles position x frequency and their sines and cosines are
computed in the kernels, in float32, from the positions of each step.
Scaling {"type": "blend", factor, original, fast, slow} blends f and f / factor by the pair index and gives the
cosines and sines an amplitude (`Rotary.amplitude`).
`none`: nothing is rotated (for mixers that carry order by themselves).
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from .base import PositionEncoding, register_part


def rotary_inverse_frequencies(rotary_dim: int, theta: float, scaling: Optional[dict]) -> torch.Tensor:
    exponents = torch.arange(0, rotary_dim, 2, dtype=torch.float32) / rotary_dim
    inv_freq = 1.0 / (theta ** exponents)
    if scaling is None:
        return inv_freq
    if scaling.get("type") == "blend":
        return blended_inverse_frequencies(rotary_dim, theta, scaling)
    factor = float(scaling["factor"])
    low, high = float(scaling["low_freq_factor"]), float(scaling["high_freq_factor"])
    original = float(scaling["original_max_position_embeddings"])
    scaled = []
    for freq in inv_freq:                      # element by element, as float32 scalars
        wavelength = 2 * math.pi / freq
        if wavelength < original / high:       # short waves keep their frequency
            scaled.append(freq)
        elif wavelength > original / low:      # long waves are slowed down by the factor
            scaled.append(freq / factor)
        else:                                  # between the two: a linear blend
            blend = (original / wavelength - low) / (high - low)
            scaled.append((1 - blend) * freq / factor + blend * freq)
    return torch.stack([torch.as_tensor(s, dtype=torch.float32) for s in scaled])


def _turn_index(rotary_dim: int, theta: float, original: float, turns: float) -> float:
    """The (fractional) pair index whose wave turns `turns` times over `original` positions."""
    return rotary_dim * math.log(original / (2 * math.pi * turns)) / (2 * math.log(theta))


def blended_inverse_frequencies(rotary_dim: int, theta: float, scaling: dict) -> torch.Tensor:
    """Frequencies for contexts `factor` times longer than the `original` one (Peng et al., "YaRN: Efficient Context
    Window Extension of Large Language Models", 2023): pair i keeps f_i = theta^(-2i/d) below the pair that turns `fast`
    times over the original length, takes f_i / factor above the pair that turns `slow` times, and blends the two
    linearly in the pair index between them. Computed in float64, rounded to float32 once."""
    factor, original = float(scaling["factor"]), float(scaling["original"])
    low = max(math.floor(_turn_index(rotary_dim, theta, original, float(scaling["fast"]))), 0)
    high = min(math.ceil(_turn_index(rotary_dim, theta, original, float(scaling["slow"]))), rotary_dim - 1)
    out = []
    for i in range(rotary_dim // 2):
        freq = theta ** (-2.0 * i / rotary_dim)
        ramp = min(max((i - low) / max(high - low, 0.001), 0.0), 1.0)
        out.append(freq / factor * ramp + freq * (1.0 - ramp))
    return torch.tensor(out, dtype=torch.float64).to(torch.float32)


def blended_amplitude(scaling: dict) -> float:
    """What the cosines and sines of blended frequencies are multiplied by: 0.1 ln(factor) + 1."""
    return 0.1 * math.log(float(scaling["factor"])) + 1.0


class Rotary(PositionEncoding):
    """`interleaved` False pairs element i of a head with element i + rotary_dim/2 (the row order of the
    checkpoints this engine reads); True pairs 2i with 2i + 1, the order on which the reference rotates after
    permuting the checkpoint's rows (src/tt_transformers/models/llama32_1b/weight_utils.py:23-25)."""

    def __init__(self, rotary_dim: int, theta: float, scaling: Optional[dict] = None, interleaved: bool = False):
        if rotary_dim % 2:
            raise ValueError(f"rotary_dim must be even, got {rotary_dim}")
        self.rotary_dim, self.theta, self.scaling = int(rotary_dim), float(theta), scaling
        self.interleaved = bool(interleaved)
        self.inv_freq_host = rotary_inverse_frequencies(self.rotary_dim, self.theta, scaling)
        # cosines and sines are multiplied by this (1 unless the scaling says otherwise); mixers that rotate hand it
        # to their kernels
        self.amplitude = blended_amplitude(scaling) if scaling is not None and scaling.get("type") == "blend" else 1.0

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        self.inv_freq = self.inv_freq_host.to(runtime.device)

    def rotation(self):
        return self.inv_freq, self.rotary_dim


class NoPosition(PositionEncoding):
    def __init__(self):
        pass


register_part("position", "rotary", Rotary)
register_part("position", "none", NoPosition)
