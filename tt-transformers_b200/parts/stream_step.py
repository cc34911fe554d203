"""Steps on the residual stream between two entries of the layer order.

`pass_mix`: the stream becomes W [x ; x0] (below).
`pass_entry`: what happens at the start of a pass over looped layers. With `add_embedding` the embedding's
output joins the stream again (every pass but the first), and row `row` of a learned table [rows, width] is
added to every token's stream: x += (x0 if add_embedding) + table[row]. All in float32, in one kernel.
"""

from __future__ import annotations

import torch

from .base import StreamStep, TensorSpec, register_part


class PassEntry(StreamStep):
    def __init__(self, width: int, table_name: str, rows: int, row: int, add_embedding: bool = False):
        self.width, self.table_name, self.rows, self.row = int(width), table_name, int(rows), int(row)
        self.needs_embedding = bool(add_embedding)
        if not 0 <= self.row < self.rows:
            raise ValueError(f"row {row} is outside the table of {rows} rows")

    def tensor_specs(self):
        return [TensorSpec(self.table_name, (self.rows, self.width))]

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        self.vector = tensors[self.table_name][self.row].to(device=runtime.device, dtype=torch.float32).contiguous()

    def forward(self, x, embedded, batch):
        self.runtime.kernels.stream_add_norm(x, [embedded] if self.needs_embedding else [], row_vector=self.vector)


register_part("stream_step", "pass_entry", PassEntry)


class PassMix(StreamStep):
    """The start of a pass as a matrix on the stream and the embedding's output side by side:
    x <- W [x ; x0], W [width, 2 width] with the stream's columns first. The product's operands take the compute
    dtype, its sums and the new stream are float32."""

    needs_embedding = True
    settles_first = True

    def __init__(self, width: int, weight_name: str):
        self.width, self.weight_name = int(width), weight_name

    def tensor_specs(self):
        return [TensorSpec(self.weight_name, (self.width, 2 * self.width))]

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        self.weight = runtime.matrix(tensors[self.weight_name])

    def forward(self, x, embedded, batch):
        k = self.runtime.kernels
        return k.linear(k.concat_cast(x, embedded, self.runtime.dtype), self.weight, out_dtype=torch.float32)


register_part("stream_step", "pass_mix", PassMix)
