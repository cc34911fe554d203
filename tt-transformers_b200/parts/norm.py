"""RMSNorm: y = x / sqrt(mean(x^2) + eps) * w, fused with the residual add before it.

Formula: src/tt_transformers/modules/rmsnorm/rmsnorm_1d.py:208-215 (no unit offset,
:68); statistics in float32 (:346-354). Here the sum of residual and delta is float32
as well and is written back to the residual stream.
"""

from __future__ import annotations

import torch

from .base import ADDED, DeferredNorm, Norm, SumDelta, TensorSpec, register_part


class RMSNorm(Norm):
    """`unit_offset` True: the weight is stored around zero and the row is scaled by 1 + w."""

    can_defer = True

    def __init__(self, width: int, eps: float, weight_name: str, unit_offset: bool = False):
        self.width, self.eps, self.weight_name = int(width), float(eps), weight_name
        self.unit_offset = bool(unit_offset)
        if self.unit_offset:
            self.can_defer = False          # the products' fused norm epilogues know the plain weight only

    def tensor_specs(self):
        return [TensorSpec(self.weight_name, (self.width,))]

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        self.weight = runtime.vector(tensors[self.weight_name])
        self._weight_f32 = None

    def fusion_args(self):
        """What a product needs to prepare this norm in its epilogue: the weight in float32 and eps."""
        if self._weight_f32 is None:
            self._weight_f32 = self.weight.float().contiguous()
        return self._weight_f32, self.eps

    def forward_add(self, residual, delta, defer=False):
        """defer: the caller's next step takes a DeferredNorm. If the sub-layer before has prepared this
        norm (delta is a DeferredNorm made for it), no kernel runs here."""
        k = self.runtime.kernels
        if isinstance(delta, DeferredNorm):
            if delta.made_for is self:
                return delta if defer else delta.materialize()
            delta = None                         # prepared for another norm: the stream itself is up to date
        if delta is ADDED:
            delta = None
        if isinstance(delta, SumDelta) and not delta.plain:
            delta.settle(residual)               # factors and a row term: added first, by the kernel that knows them
            delta = None
        if isinstance(delta, SumDelta) or self.unit_offset or (delta is not None and delta.dtype != self.runtime.dtype):
            # several outputs at once, outputs in another dtype than the compute dtype, or the 1 + w form
            deltas = delta.tensors if isinstance(delta, SumDelta) else ([delta] if delta is not None else [])
            return k.stream_add_norm(residual, deltas, weight=self.weight, eps=self.eps,
                                     offset=1.0 if self.unit_offset else 0.0, out_dtype=self.runtime.dtype)
        return k.add_rmsnorm(residual, delta, self.weight, self.eps, self.runtime.dtype)


register_part("norm", "rmsnorm", RMSNorm)


class LayerNorm(Norm):
    """y = (x - mean) / sqrt(var + eps) * w + b with the variance as the mean squared deviation; mean,
    variance and scaling in float32. `bias_name` None: no bias. Used before a sub-layer like RMSNorm
    (`forward_add`), and after one by blocks that norm a sub-layer's output before it joins the stream
    (`after`)."""

    def __init__(self, width: int, eps: float, weight_name: str, bias_name: str = None):
        self.width, self.eps, self.weight_name, self.bias_name = int(width), float(eps), weight_name, bias_name

    def tensor_specs(self):
        specs = [TensorSpec(self.weight_name, (self.width,))]
        if self.bias_name is not None:
            specs.append(TensorSpec(self.bias_name, (self.width,)))
        return specs

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        self.weight = tensors[self.weight_name].to(device=runtime.device, dtype=torch.float32).contiguous()
        self.bias = None
        if self.bias_name is not None:
            self.bias = tensors[self.bias_name].to(device=runtime.device, dtype=torch.float32).contiguous()

    def forward_add(self, residual, delta, after: "LayerNorm" = None, mult: float = 1.0):
        """residual += mult * (after(delta) if `after` else delta), then this norm of the residual. A SumDelta (several
        outputs with a factor each, and a row term) is added in the same kernel."""
        if delta is ADDED or isinstance(delta, DeferredNorm):
            delta = None
        if isinstance(delta, SumDelta):
            if after is not None:
                raise ValueError("a sum of sub-layer outputs joins the stream as it is, without a norm of its own")
            return self.runtime.kernels.add_layernorm_sum(residual, delta.tensors, delta.scales, delta.row_term, self,
                                                          self.runtime.dtype)
        return self.runtime.kernels.add_layernorm(residual, delta, after, mult, self, self.runtime.dtype)

    def join(self, residual, delta, mult: float = 1.0):
        """residual += mult * norm(delta): this norm applied to a sub-layer's output on its way into the stream."""
        self.runtime.kernels.add_layernorm(residual, delta, self, mult, None, self.runtime.dtype)


register_part("norm", "layernorm", LayerNorm)


class DynamicTanh(Norm):
    """y = tanh(alpha x) * w + b with one learned number alpha: no mean, no variance, every element by itself
    (Zhu et al., "Transformers without Normalization", 2025). Used before a sub-layer (`forward_add`) and after one by
    blocks that norm a sub-layer's output before it joins the stream (`after`, `join`). Float32 throughout."""

    def __init__(self, width: int, weight_name: str, bias_name: str, alpha_name: str):
        self.width, self.weight_name, self.bias_name, self.alpha_name = int(width), weight_name, bias_name, alpha_name

    def tensor_specs(self):
        return [TensorSpec(self.weight_name, (self.width,)), TensorSpec(self.bias_name, (self.width,)),
                TensorSpec(self.alpha_name, ())]

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        self.weight = tensors[self.weight_name].to(device=runtime.device, dtype=torch.float32).contiguous()
        self.bias = tensors[self.bias_name].to(device=runtime.device, dtype=torch.float32).contiguous()
        self.alpha = float(tensors[self.alpha_name].to(torch.float32))

    def forward_add(self, residual, delta, after: "DynamicTanh" = None, mult: float = 1.0):
        """residual += mult * (after(delta) if `after` else delta), then this norm of the residual."""
        if delta is ADDED or isinstance(delta, DeferredNorm):
            delta = None
        return self.runtime.kernels.add_dyntanh(residual, delta, after, mult, self, self.runtime.dtype)

    def join(self, residual, delta, mult: float = 1.0):
        """residual += mult * norm(delta): this norm applied to a sub-layer's output on its way into the stream."""
        self.runtime.kernels.add_dyntanh(residual, delta, self, mult, None, self.runtime.dtype)


register_part("norm", "dyntanh", DynamicTanh)
