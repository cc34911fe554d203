"""The kernel table: Python entry points of the hand-written CUDA kernels.

`CudaKernels` loads the shared library that `build.py` compiles from csrc/ and calls
its C entry points with raw device pointers on torch's current stream. There is no
other implementation behind it: without a CUDA device, nvcc or the library, creating
it raises.

Library matrix products (cuBLAS through torch.mm) stand in for the large bfloat16
products of prefill, where the reference's engine calls its own library's linear op
(src/tt_transformers/modules/attention/attention_1d.py:507-514,
src/tt_transformers/modules/mlp/mlp_1d.py:240-294). Everything else is ours.
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional

import torch

from ..parts.base import ADDED, DeferredNorm
from .build import BuildError, build

_F32, _BF16 = 0, 1


class KernelError(RuntimeError):
    """A kernel refused its arguments or the launch failed."""


class EngineDeviceError(RuntimeError):
    """A kernel met an index outside its tables (token id, page id) and skipped the access."""


def _dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return _F32
    if dtype == torch.bfloat16:
        return _BF16
    raise KernelError(f"kernels take float32 or bfloat16 tensors, not {dtype}")


_raw_stream = torch._C._cuda_getCurrentRawStream      # device index -> handle of torch's current stream


_ERRORS = {-2: "unsupported size or option", -3: "bad argument (null pointer, alignment or contradiction)"}


class CudaKernels:
    """All kernels of the engine, on one CUDA device."""

    name = "cuda"
    # bfloat16 products with more rows than this go to the library; fewer rows stream the
    # weights through the hand-written skinny kernel.
    SKINNY_ROWS = 8
    # bfloat16 products with up to this many rows stream the weights through the tensor-core
    # skinny kernel (K a multiple of 8). The kernel takes up to 64 rows, but from 17 rows on the
    # activations' traffic through L1 holds it back and the library's product is faster (measured:
    # 13 us against 20 to 42 us for the down projection at 32 to 64 rows).
    TENSOR_SKINNY_ROWS = 16
    TCGEN05_SWIGLU_ROWS = 128
    SKINNY_TCGEN05_MIN_K = 8192
    # from this many rows on the weight-streaming tcgen05 kernel takes the products it is good at from the mma.sync
    # skinny kernel (measured at 9, 12 and 16 rows: down projection 10.8 to 11.1 us against 13.5 to 14.1, gate/up
    # with SwiGLU 14.5 to 15.5 against 17.3 to 18.6)
    SKINNY_TCGEN05_MIN_ROWS = 9
    RING_ROWS = 8
    # decode steps of up to this many tokens run projection, rotation and cache write as one kernel (at 9 to 16 rows
    # against the library's product and the rotation kernel: 1.560 -> 1.542 ms a step at batch 16, 1B sizes; 5.99 -> 5.90 at 8B)
    FUSED_QKV_ROWS = 16
    RING_SWIGLU_MIN_ROWS = 6
    RING_SWIGLU_ANY_ROWS_BYTES = 80 << 20

    def __init__(self, device: torch.device):
        if not torch.cuda.is_available():
            raise KernelError("no CUDA device is available; this engine has no CPU implementation")
        self.device = torch.device(device)
        self._device_index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        try:
            path = build()
        except BuildError as e:
            raise KernelError(f"the CUDA kernel library could not be built: {e}") from e
        try:
            self.lib = ctypes.CDLL(path)
        except OSError as e:
            raise KernelError(f"the CUDA kernel library {path} could not be loaded: {e}") from e
        self.library_path = path
        for name in ("ttb_embedding", "ttb_add_rmsnorm", "ttb_swiglu", "ttb_gather_rows", "ttb_rope_kv_write",
                     "ttb_paged_attention_generic", "ttb_gemm_simt", "ttb_gemv", "ttb_sample",
                     "ttb_paged_attention_mma", "ttb_attention_mma_tile_rows", "ttb_attention_mma_supports",
                     "ttb_gemv_mma", "ttb_gemv_mma_fused", "ttb_gemv_mma_parts", "ttb_argmax", "ttb_attention_decode_merges_in_kernel", "ttb_paged_attention_mma_checked", "ttb_attention_mma_blocks_per_sm",
                     "ttb_gemm_tcgen05", "ttb_paged_attention_tcgen05", "ttb_attention_tcgen05_supports",
                     "ttb_attention_tcgen05_tile_rows", "ttb_attention_merge", "ttb_gemv_qkv_rope",
                     "ttb_gemm_skinny_tcgen05", "ttb_gemm_skinny_tcgen05_rows", "ttb_softcap", "ttb_sample_scratch_bytes",
                     "ttb_gemv_ring", "ttb_gemm_skinny_tcgen05_qkv_rope", "ttb_add_layernorm", "ttb_latent_prepare",
                     "ttb_latent_attention_generic", "ttb_gate_heads", "ttb_gemm_simt_batched", "ttb_route_top",
                     "ttb_moe_align", "ttb_moe_group_gemm", "ttb_moe_combine", "ttb_glu_clamped",
                     "ttb_latent_attention_mma", "ttb_latent_attention_mma_supports", "ttb_moe_gemv", "ttb_moe_gemm_tcgen05", "ttb_latent_out",
                     "ttb_latent_attention_mma_tokens_per_tile", "ttb_stream_add_norm", "ttb_gated_rmsnorm",
                     "ttb_mean_rmsnorm_pair", "ttb_activation", "ttb_lightning_scan", "ttb_causal_conv", "ttb_gated_recurrence",
                     "ttb_paged_attention_generic_ext", "ttb_qk_norm_rope_write", "ttb_route_grouped", "ttb_moe_gemv_plain",
                     "ttb_paged_attention_mma_ext", "ttb_lightning_chunks", "ttb_lightning_chunks_supports",
                     "ttb_recurrent_token", "ttb_add_dyntanh", "ttb_concat_cast", "ttb_qk_whole_norm_rope_write",
                     "ttb_route_top_scored", "ttb_moe_gemv_scaled", "ttb_gather_rows_scaled", "ttb_conv_silu",
                     "ttb_state_space_scan", "ttb_state_space_supports", "ttb_gate_group_norm", "ttb_state_space_token",
                     "ttb_token_shift", "ttb_lowrank_expand", "ttb_add_row_vector", "ttb_shifted_state", "ttb_delta_rule",
                     "ttb_add_layernorm_sum", "ttb_qk_norm_rope_write_ext", "ttb_paged_attention_generic_bias",
                     "ttb_latent_prepare_ext", "ttb_latent_attention_generic_ext", "ttb_route_top_corrected",
                     "ttb_paged_attention_mma_bias", "ttb_latent_attention_mma_ext"):
            getattr(self.lib, name).restype = ctypes.c_int
        self.lib.ttb_sample_uniform.restype = ctypes.c_float
        self.lib.ttb_sample_uniform.argtypes = [ctypes.c_longlong, ctypes.c_int]
        self.lib.ttb_sample_max_top_k.restype = ctypes.c_int
        self.max_top_k = int(self.lib.ttb_sample_max_top_k())
        with torch.cuda.device(self.device):
            self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.launches = 0     # how many of our kernels were launched (counted for reports)
        self.sm_count = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.use_mma_attention = True
        # linear attention over prompt portions chunk by chunk on the tensor cores (False: token by token everywhere)
        self.use_lightning_chunks = os.environ.get("TTB200_LIGHTNING_CHUNKS", "1") == "1"
        # latent attention in bfloat16 on the tensor cores (False: the float32-arithmetic kernel everywhere)
        self.use_mma_latent_attention = os.environ.get("TTB200_MMA_LATENT", "1") == "1"
        # prompt portions at head size 64: the TMA + tcgen05 attention kernel (False: the mma.sync one)
        self.use_tcgen05_attention = os.environ.get("TTB200_TCGEN05_ATTENTION", "1") == "1"
        # decode steps (up to 16 query rows per segment and KV head): the transposed-product kernel with TMA
        # loads of attention_decode.cu (False: the decode shape of the mma.sync kernel)
        self.use_tma_decode = os.environ.get("TTB200_TMA_DECODE", "1") == "1"
        # skinny products take the residual add after them into their epilogue (fuse_add) and prepare the norm
        # that follows there, which the next skinny product finishes (fuse_norm)
        self.fuse_norm = os.environ.get("TTB200_FUSE_NORM", "0") == "1"
        self.fuse_add = os.environ.get("TTB200_FUSE_ADD", "0") == "1"
        # products of up to RING_ROWS rows by the persistent kernel of gemv_ring.cu, a bit for each kind:
        # 1 gate/up with SwiGLU (from RING_SWIGLU_MIN_ROWS rows on, or at any number of rows when the matrix has
        # RING_SWIGLU_ANY_ROWS_BYTES or more: at Llama 3.2 3B and 3.1 8B sizes it wins from one row on, 2.09 against
        # 2.17 ms and 3.54 against 3.62 ms a step at batch 1), 2 plain products with a long reduction (down),
        # 4 the other plain products with bfloat16 output (output projection), 8 products with float32 output (the
        # LM head). Measured inside the decode step at Llama 3.2 1B sizes, ms a step at batch 1 / 2 / 4 / 8 against
        # 0.793 / 0.842 / 0.928 / 1.106 without: bit 4 alone 0.774 / 0.824 / 0.907 / 1.076; bit 1 alone 0.814 /
        # 0.857 / 0.930 / 1.094; bit 8 alone 0.797 / 0.845 / 0.932 / 1.109; bits 1 and 2 1.101 at batch 8.
        self.ring_gemv = int(os.environ.get("TTB200_RING_GEMV", "5"))
        # decode steps of 17 to 64 tokens: QKV projection, rotation and cache write in the weight-streaming tcgen05
        # kernel (False: the library's product and the rotation kernel). One launch instead of two and no library on
        # the way, at the same speed: ms a step with / without, context 8,192 unless said: 1B sizes batch 32 2.261 /
        # 2.252, batch 64 3.543 / 3.552; 3B sizes batch 32 at 2,048 tokens 2.943 / 2.996; 8B sizes batch 64 at 4,096
        # tokens 8.922 / 8.890
        self.skinny_qkv_rope = os.environ.get("TTB200_SKINNY_QKV_ROPE", "1") == "1"
        # bfloat16 products with more rows than the skinny kernel takes: the TMA + tcgen05 kernel of
        # gemm_tcgen05.cu or the library's product. None (TTB200_TCGEN05 unset or "auto"): the feed-forward's
        # gate/up product with its fused SwiGLU goes to the tcgen05 kernel from TCGEN05_SWIGLU_ROWS rows on
        # (measured 1.1 to 1.35 times faster than the library's product followed by the SwiGLU kernel) and
        # plain products go to the library (the tcgen05 kernel reaches 0.75 to 0.95 of it). True ("1"):
        # every such product goes to the tcgen05 kernel. False ("0"): none does.
        self.use_tcgen05 = {"1": True, "0": False}.get(os.environ.get("TTB200_TCGEN05", "auto"))
        # bfloat16 products with more rows than the mma.sync skinny kernel takes and up to SKINNY_TCGEN05_ROWS
        # (decode steps of many requests): the weight-streaming tcgen05 kernel of gemm_skinny_tcgen05.cu
        # (False: the library's product)
        self.use_skinny_tcgen05 = os.environ.get("TTB200_SKINNY_TCGEN05", "1") == "1"
        self.SKINNY_TCGEN05_ROWS = int(self.lib.ttb_gemm_skinny_tcgen05_rows())
        with torch.cuda.device(self.device):
            self.tc_error = torch.zeros(1, dtype=torch.int32, device=self.device)

    # ------------------------------------------------------------------ helpers
    @staticmethod
    def _p(t: Optional[torch.Tensor]):
        return ctypes.c_void_p(0 if t is None else t.data_ptr())

    def _stream(self):
        # the handle of torch's current stream on this device, without building a Stream object for every launch
        return ctypes.c_void_p(_raw_stream(self._device_index))

    def _check(self, code: int, what: str):
        self.launches += 1
        if code != 0:
            reason = _ERRORS.get(code, f"CUDA error {code}")
            raise KernelError(f"{what}: {reason}")

    def check_status(self):
        """Raise if a kernel flagged an index outside its tables since the last check.
        Synchronises with the device."""
        tc = int(self.tc_error.item())
        if tc != 0:
            self.tc_error.zero_()
            role = {1: "the product's TMA producer", 2: "the product's MMA issuer", 3: "the product's epilogue",
                    11: "attention's TMA producer", 12: "attention's MMA issuer waiting for the queries",
                    13: "attention's MMA issuer waiting for keys", 14: "attention's MMA issuer waiting for P",
                    15: "attention's softmax warps", 16: "attention's epilogue",
                    17: "attention's shared memory, which is not aligned to 1,024 bytes",
                    21: "decode attention's TMA producer", 22: "decode attention's consumer warps",
                    31: "the skinny product's TMA producer", 32: "the skinny product's MMA issuer",
                    33: "the skinny product's epilogue"}.get(tc, f"role {tc}")
            raise EngineDeviceError(f"a tcgen05 kernel gave up waiting on a barrier ({role}); its result is invalid")
        value = int(self.status.item())
        if value != 0:
            self.status.zero_()
            kind = value >> 24
            where = value & 0xFFFFFF
            what = {0: f"token id out of range at token {where - 1}",
                    1: f"position beyond the block table at token {where}",
                    2: f"page id out of range at token {where}"}.get(kind, f"code {value}")
            raise EngineDeviceError(what)

    # ------------------------------------------------------------------ elementwise
    def embedding(self, table: torch.Tensor, token_ids: torch.Tensor, scale: float = 1.0) -> torch.Tensor:
        tokens, (vocab, width) = token_ids.shape[0], table.shape
        out = torch.empty(tokens, width, dtype=torch.float32, device=self.device)
        self._check(self.lib.ttb_embedding(self._p(table), _dtype_code(table.dtype), self._p(token_ids), self._p(out),
                                           tokens, width, vocab, ctypes.c_float(scale), self._p(self.status),
                                           self._stream()), "embedding")
        return out

    def softcap(self, logits: torch.Tensor, cap: float) -> torch.Tensor:
        """logits = cap * tanh(logits / cap), float32, in place."""
        if logits.dtype != torch.float32 or logits.dim() != 2 or logits.stride(1) != 1:
            raise KernelError("softcap: logits must be float32 [rows, columns], contiguous along the columns")
        self._check(self.lib.ttb_softcap(self._p(logits), logits.shape[0], logits.shape[1], logits.stride(0),
                                         ctypes.c_float(cap), self._stream()), "softcap")
        return logits

    def add_rmsnorm(self, residual: torch.Tensor, delta: Optional[torch.Tensor], weight: torch.Tensor, eps: float,
                    out_dtype: torch.dtype) -> torch.Tensor:
        rows, width = residual.shape
        if residual.dtype != torch.float32:
            raise KernelError("the residual stream is float32")
        if delta is not None and (delta.dtype != out_dtype or delta.shape != residual.shape):
            raise KernelError("add_rmsnorm: delta must have the compute dtype and the residual's shape")
        out = torch.empty(rows, width, dtype=out_dtype, device=self.device)
        self._check(self.lib.ttb_add_rmsnorm(self._p(residual), self._p(delta), self._p(weight),
                                             _dtype_code(weight.dtype), self._p(out), _dtype_code(out_dtype), rows,
                                             width, ctypes.c_float(eps), self._stream()), "add_rmsnorm")
        return out

    def swiglu(self, gate_up: torch.Tensor) -> torch.Tensor:
        rows, two_inter = gate_up.shape
        inter = two_inter // 2
        out = torch.empty(rows, inter, dtype=gate_up.dtype, device=self.device)
        self._check(self.lib.ttb_swiglu(self._p(gate_up), self._p(out), _dtype_code(gate_up.dtype), rows, inter,
                                        self._stream()), "swiglu")
        return out

    def gather_rows(self, x: torch.Tensor, rows: torch.Tensor) -> torch.Tensor:
        count = rows.shape[0]
        out = torch.empty(count, x.shape[1], dtype=x.dtype, device=self.device)
        self._check(self.lib.ttb_gather_rows(self._p(x), self._p(rows), self._p(out), count,
                                             x.shape[1] * x.element_size(), self._stream()), "gather_rows")
        return out

    # ------------------------------------------------------------------ matrix products
    def _skinny_fused(self, norm, x, w, out, out_dtype, M, N, K, pair_rows, accumulate, next_norm, what):
        """The tensor-core skinny product with a DeferredNorm as its input and/or the residual stream as its
        output. With next_norm (a norm part) it prepares that norm and returns the DeferredNorm for it."""
        src = norm.xg if norm is not None else x
        xg = ssq = None
        if next_norm is not None:
            weight, eps = next_norm.fusion_args()
            xg = torch.empty(M, N, dtype=w.dtype, device=self.device)
            ssq = torch.empty(int(self.lib.ttb_gemv_mma_parts(M, N)), 16, dtype=torch.float32, device=self.device)
        self._check(self.lib.ttb_gemv_mma_fused(
            self._p(src), self._p(norm.ssq if norm is not None else None), norm.ssq.shape[0] if norm is not None else 0,
            ctypes.c_float(norm.eps if norm is not None else 0.0), self._p(w), self._p(out), _dtype_code(out_dtype),
            M, N, K, src.stride(0), w.stride(0), N, pair_rows, self._p(accumulate),
            accumulate.stride(0) if accumulate is not None else 0, self._p(weight if next_norm is not None else None),
            self._p(xg), N, self._p(ssq), self._stream()), what)
        if next_norm is None:
            return None
        dtype = w.dtype
        return DeferredNorm(xg, ssq, eps, next_norm,
                            lambda: self.add_rmsnorm(accumulate, None, next_norm.weight, eps, dtype))

    def linear(self, x, w: torch.Tensor, out_dtype: Optional[torch.dtype] = None, accumulate: torch.Tensor = None,
               next_norm=None):
        """x [M, K] times w [N, K] transposed -> [M, N]. x may be a DeferredNorm. With `accumulate` (the float32
        residual stream [M, N]) the product may be added there instead of being returned: ADDED comes back then,
        or, with next_norm (the norm part that follows), a DeferredNorm made for it; else the product as usual
        (the caller adds it)."""
        norm = None
        if isinstance(x, DeferredNorm):
            if (self.fuse_norm and w.dtype == torch.bfloat16 and x.shape[0] <= self.TENSOR_SKINNY_ROWS
                    and w.stride(1) == 1 and w.stride(0) % 8 == 0 and w.shape[1] == x.shape[1]
                    and x.xg.dtype == torch.bfloat16 and x.xg.stride(1) == 1 and x.xg.stride(0) % 8 == 0):
                norm, x = x, x.xg
            else:
                x = x.materialize()
        M, K = x.shape
        N = w.shape[0]
        out_dtype = out_dtype or x.dtype
        if w.shape[1] != K or x.dtype != w.dtype:
            raise KernelError(f"linear: x {tuple(x.shape)} {x.dtype} does not match w {tuple(w.shape)} {w.dtype}")
        if x.stride(1) != 1 or w.stride(1) != 1:
            raise KernelError("linear: operands must be contiguous along K")
        streams = (x.dtype == torch.bfloat16 and self.use_skinny_tcgen05 and norm is None
                   and self.SKINNY_TCGEN05_MIN_ROWS <= M <= self.SKINNY_TCGEN05_ROWS and K >= self.SKINNY_TCGEN05_MIN_K
                   and K % 8 == 0 and x.stride(0) % 8 == 0 and w.stride(0) % 8 == 0
                   and x.data_ptr() % 16 == 0 and w.data_ptr() % 16 == 0
                   and not (self.fuse_add and accumulate is not None))
        if (not streams and x.dtype == torch.bfloat16 and M <= self.TENSOR_SKINNY_ROWS and K % 8 == 0
                and x.stride(0) % 8 == 0 and w.stride(0) % 8 == 0):
            fuse_add = (accumulate is not None and self.fuse_add and accumulate.dtype == torch.float32
                        and accumulate.shape == (M, N) and accumulate.stride(1) == 1)
            if norm is not None or fuse_add:
                out = None if fuse_add else torch.empty(M, N, dtype=out_dtype, device=self.device)
                prepared = self._skinny_fused(norm, x, w, out, out_dtype, M, N, K, 0, accumulate if fuse_add else None,
                                              next_norm if (fuse_add and self.fuse_norm) else None, "gemv_mma_fused")
                if not fuse_add:
                    return out
                return prepared if prepared is not None else ADDED
            kind = 8 if out_dtype != torch.bfloat16 else (2 if K >= self.SKINNY_TCGEN05_MIN_K else 4)
            if M <= self.RING_ROWS and (self.ring_gemv & kind):
                out = torch.empty(M, N, dtype=out_dtype, device=self.device)
                self._check(self.lib.ttb_gemv_ring(self._p(x), self._p(w), self._p(out), _dtype_code(out_dtype), M, N, K,
                                                   x.stride(0), w.stride(0), N, 0, self._stream()), "gemv_ring")
                return out
            # 9 to 16 rows, nothing fused, bfloat16 out (QKV and output projection): the library is as fast at
            # Llama 3.2 1B sizes and 1.1 to 1.3 times faster at 3B and 8B sizes (measured at 10 and 16 rows)
            if M <= self.SKINNY_ROWS or out_dtype != torch.bfloat16:
                out = torch.empty(M, N, dtype=out_dtype, device=self.device)
                self._check(self.lib.ttb_gemv_mma(self._p(x), self._p(w), self._p(out), _dtype_code(out_dtype), M, N, K,
                                                  x.stride(0), w.stride(0), N, 0, self._stream()), "gemv_mma")
                return out
        if norm is not None:
            x = norm.materialize()
        if M <= self.SKINNY_ROWS and not streams:
            out = torch.empty(M, N, dtype=out_dtype, device=self.device)
            self._check(self.lib.ttb_gemv(self._p(x), self._p(w), self._p(out), _dtype_code(x.dtype),
                                          _dtype_code(out_dtype), M, N, K, x.stride(0), w.stride(0), N,
                                          self._stream()), "gemv")
            return out
        # long reductions only (the down projection): measured against the library at 24 to 64 rows, 0.9 to 1.0 of
        # its time from K = 8,192 on and 1.1 to 1.4 for the QKV and output projections
        if streams:
            out = torch.empty(M, N, dtype=out_dtype, device=self.device)
            self._check(self.lib.ttb_gemm_skinny_tcgen05(self._p(x), self._p(w), self._p(out), _dtype_code(out_dtype),
                                                         M, N, K, x.stride(0), w.stride(0), N, 0, self._p(self.tc_error),
                                                         self._stream()), "gemm_skinny_tcgen05")
            return out
        if (x.dtype == torch.bfloat16 and self.use_tcgen05 and K % 8 == 0 and x.stride(0) % 8 == 0
                and w.stride(0) % 8 == 0):
            out = torch.empty(M, N, dtype=out_dtype, device=self.device)
            self._check(self.lib.ttb_gemm_tcgen05(self._p(x), self._p(w), self._p(out), _dtype_code(out_dtype), M, N, K,
                                                  x.stride(0), w.stride(0), N, 0, self._p(self.tc_error),
                                                  self._stream()), "gemm_tcgen05")
            return out
        if x.dtype == torch.bfloat16:
            # library product (cuBLAS), float32 accumulation
            if out_dtype == torch.bfloat16:
                return torch.mm(x, w.t())
            return torch.mm(x, w.t(), out_dtype=out_dtype)
        out = torch.empty(M, N, dtype=out_dtype, device=self.device)
        self._check(self.lib.ttb_gemm_simt(self._p(x), self._p(w), self._p(out), _dtype_code(x.dtype),
                                           _dtype_code(out_dtype), M, N, K, x.stride(0), w.stride(0), N,
                                           self._stream()), "gemm_simt")
        return out

    def linear_swiglu(self, x: torch.Tensor, w_gate_up: torch.Tensor) -> torch.Tensor:
        """silu(x Wg^T) * (x Wu^T) for w_gate_up = [Wg; Wu] stacked along the rows -> [M, rows / 2]."""
        if isinstance(x, DeferredNorm):
            M, K = x.shape
            inter = w_gate_up.shape[0] // 2
            if (self.fuse_norm and w_gate_up.dtype == torch.bfloat16 and M <= self.TENSOR_SKINNY_ROWS
                    and w_gate_up.shape[1] == K and w_gate_up.stride(1) == 1 and w_gate_up.stride(0) % 8 == 0
                    and x.xg.dtype == torch.bfloat16 and x.xg.stride(1) == 1 and x.xg.stride(0) % 8 == 0):
                out = torch.empty(M, inter, dtype=w_gate_up.dtype, device=self.device)
                self._skinny_fused(x, None, w_gate_up, out, w_gate_up.dtype, M, inter, K, inter, None, None,
                                   "gemv_mma_norm_swiglu")
                return out
            x = x.materialize()
        M, K = x.shape
        inter = w_gate_up.shape[0] // 2
        streams = (x.dtype == torch.bfloat16 and self.use_skinny_tcgen05
                   and self.SKINNY_TCGEN05_MIN_ROWS <= M <= self.SKINNY_TCGEN05_ROWS and K % 8 == 0
                   and x.stride(0) % 8 == 0 and w_gate_up.stride(0) % 8 == 0 and x.stride(1) == 1
                   and w_gate_up.stride(1) == 1 and x.data_ptr() % 16 == 0 and w_gate_up.data_ptr() % 16 == 0)
        if (not streams and x.dtype == torch.bfloat16 and M <= self.TENSOR_SKINNY_ROWS and K % 8 == 0
                and x.stride(0) % 8 == 0 and w_gate_up.stride(0) % 8 == 0 and x.stride(1) == 1
                and w_gate_up.stride(1) == 1):
            out = torch.empty(M, inter, dtype=x.dtype, device=self.device)
            ring = ((self.ring_gemv & 1) and M <= self.RING_ROWS
                    and (M >= self.RING_SWIGLU_MIN_ROWS or 2 * inter * K * 2 >= self.RING_SWIGLU_ANY_ROWS_BYTES))
            entry = self.lib.ttb_gemv_ring if ring else self.lib.ttb_gemv_mma
            self._check(entry(self._p(x), self._p(w_gate_up), self._p(out), _dtype_code(x.dtype), M,
                              inter, K, x.stride(0), w_gate_up.stride(0), inter, inter,
                              self._stream()), "gemv_swiglu")
            return out
        if streams:
            out = torch.empty(M, inter, dtype=x.dtype, device=self.device)
            self._check(self.lib.ttb_gemm_skinny_tcgen05(self._p(x), self._p(w_gate_up), self._p(out), _dtype_code(x.dtype),
                                                         M, inter, K, x.stride(0), w_gate_up.stride(0), inter, inter,
                                                         self._p(self.tc_error), self._stream()), "gemm_skinny_tcgen05_swiglu")
            return out
        fused = self.use_tcgen05 if self.use_tcgen05 is not None else M >= self.TCGEN05_SWIGLU_ROWS
        if (x.dtype == torch.bfloat16 and fused and K % 8 == 0 and x.stride(0) % 8 == 0
                and w_gate_up.stride(0) % 8 == 0 and x.stride(1) == 1 and w_gate_up.stride(1) == 1):
            out = torch.empty(M, inter, dtype=x.dtype, device=self.device)
            self._check(self.lib.ttb_gemm_tcgen05(self._p(x), self._p(w_gate_up), self._p(out), _dtype_code(x.dtype), M,
                                                  inter, K, x.stride(0), w_gate_up.stride(0), inter, inter,
                                                  self._p(self.tc_error), self._stream()), "gemm_tcgen05_swiglu")
            return out
        return self.swiglu(self.linear(x, w_gate_up))

    def fused_qkv_rope(self, x, w_qkv, batch, inv_freq, rotary_dim, heads, kv_heads, head_dim, view, write_kv=True,
                       interleaved=False):
        """The QKV projection, the rotation and the cache write of a decode step in one kernel.
        Returns the rotated queries [M, heads * head_dim], or None where the fused kernel does not
        apply (then the caller runs the three steps one by one)."""
        M, K = x.shape
        norm = x if isinstance(x, DeferredNorm) else None
        if (norm is not None and not self.fuse_norm) or interleaved:
            return None
        if (norm is None and self.skinny_qkv_rope and self.FUSED_QKV_ROWS < M <= self.SKINNY_TCGEN05_ROWS
                and w_qkv.dtype == torch.bfloat16 and x.dtype == torch.bfloat16 and K % 8 == 0 and x.stride(1) == 1
                and x.stride(0) % 8 == 0 and w_qkv.stride(1) == 1 and w_qkv.stride(0) % 8 == 0 and inv_freq is not None
                and rotary_dim == head_dim and head_dim in (16, 32, 64, 128) and view is not None
                and view.keys.dtype == torch.bfloat16 and view.keys.is_contiguous() and view.values.is_contiguous()
                and x.data_ptr() % 16 == 0 and w_qkv.data_ptr() % 16 == 0):
            q = torch.empty(M, heads * head_dim, dtype=w_qkv.dtype, device=self.device)
            self._check(self.lib.ttb_gemm_skinny_tcgen05_qkv_rope(
                self._p(x), self._p(w_qkv), self._p(q), M, K, x.stride(0), w_qkv.stride(0), self._p(batch.positions),
                self._p(batch.seg_of_token), self._p(inv_freq), heads, kv_heads, head_dim, self._p(view.keys),
                self._p(view.values), self._p(view.block_table), view.block_table.shape[1], view.page_size,
                view.keys.shape[0], 1 if write_kv else 0, self._p(self.status), self._p(self.tc_error), self._stream()),
                "gemm_skinny_tcgen05_qkv_rope")
            return q
        src = norm.xg if norm is not None else x
        if not (w_qkv.dtype == torch.bfloat16 and M <= self.FUSED_QKV_ROWS and K % 8 == 0 and src.stride(1) == 1
                and src.dtype == torch.bfloat16 and src.stride(0) % 8 == 0
                and w_qkv.stride(1) == 1 and w_qkv.stride(0) % 8 == 0 and inv_freq is not None
                and rotary_dim == head_dim and head_dim % 16 == 0 and view is not None
                and view.keys.dtype == torch.bfloat16 and view.keys.is_contiguous() and view.values.is_contiguous()):
            return None
        q = torch.empty(M, heads * head_dim, dtype=w_qkv.dtype, device=self.device)
        self._check(self.lib.ttb_gemv_qkv_rope(
            self._p(src), self._p(norm.ssq if norm is not None else None), norm.ssq.shape[0] if norm is not None else 0,
            ctypes.c_float(norm.eps if norm is not None else 0.0), self._p(w_qkv), self._p(q), M, K, src.stride(0),
            w_qkv.stride(0), self._p(batch.positions),
            self._p(batch.seg_of_token), self._p(inv_freq), heads, kv_heads, head_dim, self._p(view.keys),
            self._p(view.values), self._p(view.block_table), view.block_table.shape[1], view.page_size,
            view.keys.shape[0], 1 if write_kv else 0, self._p(self.status), self._stream()), "gemv_qkv_rope")
        return q

    # ------------------------------------------------------------------ attention
    def rope_kv_write(self, qkv, batch, inv_freq, rotary_dim, heads, kv_heads, head_dim, view, write_kv=True,
                      interleaved=False):
        """Rotate the queries and keys of qkv in place and write keys and values into their pages. Pairs are
        (i, i + rotary_dim/2), or (2i, 2i + 1) with `interleaved`."""
        tokens = qkv.shape[0]
        if qkv.shape[1] != (heads + 2 * kv_heads) * head_dim or not qkv.is_contiguous():
            raise KernelError("rope_kv_write: qkv must be contiguous [tokens, (heads + 2 kv_heads) * head_dim]")
        num_pages = view.keys.shape[0] if view is not None else 0
        self._check(self.lib.ttb_rope_kv_write(
            self._p(qkv), _dtype_code(qkv.dtype), self._p(batch.positions), self._p(batch.seg_of_token),
            self._p(inv_freq), int(rotary_dim), tokens, heads, kv_heads, head_dim,
            self._p(view.keys if view is not None else None), self._p(view.values if view is not None else None),
            self._p(view.block_table if view is not None else None),
            view.block_table.shape[1] if view is not None else 0, view.page_size if view is not None else 1,
            num_pages, 1 if (write_kv and view is not None) else 0, 1 if interleaved else 0, self._p(self.status),
            self._stream()), "rope_kv_write")

    def paged_attention(self, qkv, batch, heads, kv_heads, head_dim, scale, view) -> torch.Tensor:
        tokens = qkv.shape[0]
        out = torch.empty(tokens, heads * head_dim, dtype=qkv.dtype, device=self.device)
        if view.keys.dtype != qkv.dtype:
            raise KernelError("paged_attention: cache pages and queries differ in dtype")
        if (self.use_mma_attention and qkv.dtype == torch.bfloat16
                and self.lib.ttb_attention_mma_supports(heads, kv_heads, head_dim)):
            self._attention_mma(qkv, out, batch, heads, kv_heads, head_dim, scale, view)
            return out
        self._check(self.lib.ttb_paged_attention_generic(
            self._p(qkv), qkv.stride(0), self._p(out), _dtype_code(qkv.dtype), self._p(batch.positions),
            self._p(batch.seg_of_token), self._p(view.keys), self._p(view.values), self._p(view.block_table),
            view.block_table.shape[1], view.page_size, tokens, heads, kv_heads, head_dim, ctypes.c_float(scale),
            int(view.window or 0), view.keys.shape[0], self._p(self.status), self._stream()), "paged_attention")
        return out

    def attention_tables(self, seg_lens, seg_pos0, rep: int, fixed_tokens: int = 0):
        """The query-tile lists of a step as host tables, for the step's one metadata copy: {key: int32 array
        [2, tiles]} with the segment and the first token of every tile, the tile that sees most keys first (the
        longest blocks start first). One table per tile height a kernel may use; none for a step that the decode
        shape takes. fixed_tokens: the step always holds this many tokens in at most two segments (a captured
        prompt step): the table gets the length that any such step fits in, filled up with repeats of its last
        tile (a tile computed twice writes the same values twice)."""
        import numpy as np

        if max(seg_lens) * rep <= 16:
            return {}
        out = {}
        for rows in {int(self.lib.ttb_attention_tcgen05_tile_rows()), int(self.lib.ttb_attention_mma_tile_rows(0))}:
            per_tile = max(1, rows // rep)
            tiles = []
            for r, (n, pos0) in enumerate(zip(seg_lens, seg_pos0)):
                for t in range(0, n, per_tile):
                    tiles.append((-(pos0 + min(n, t + per_tile)), r, t))
            tiles.sort()
            if fixed_tokens:
                tiles += [tiles[-1]] * (fixed_tokens // per_tile + 2 - len(tiles))
            out[("attention_tiles", per_tile)] = np.array([[t[1] for t in tiles], [t[2] for t in tiles]], dtype=np.int32)
        return out

    def _attention_plan(self, batch, rep: int, kv_heads: int, head_dim: int, big_tiles: bool = False):
        """How the step's segments are cut into query tiles, and into how many key splits:
        derived once per step and geometry, reused by every layer. big_tiles: the 128-row
        tiles of the tcgen05 kernel."""
        key = ("attention_plan", rep, kv_heads, head_dim, big_tiles)
        plan = batch.extras.get(key)
        if plan is not None:
            return plan
        decode_shape = batch.max_seg_len * rep <= 16 and not big_tiles
        if big_tiles:
            rows = int(self.lib.ttb_attention_tcgen05_tile_rows())
        else:
            rows = int(self.lib.ttb_attention_mma_tile_rows(1 if decode_shape else 0))
        tokens_per_tile = max(1, rows // rep)
        if decode_shape:
            seg, tok0, n_tiles = None, None, batch.num_segments
        else:
            both = batch.extras.get(("attention_tiles", tokens_per_tile))      # came with the step's metadata
            if both is None:                  # a batch put together by hand: a copy of its own
                table = self.attention_tables(batch.seg_lens, batch.seg_pos0_list, rep)[("attention_tiles", tokens_per_tile)]
                both = torch.from_numpy(table).pin_memory().to(self.device, non_blocking=True)
                batch.extras[("attention_tiles", tokens_per_tile)] = both
            seg, tok0, n_tiles = both[0], both[1], both.shape[1]
        # Key splits: with fewer blocks than fit the GPU at once, as many splits as fill it in one
        # wave (chunks of at least 256 keys); with more, a few waves of chunks of at least 2,048 keys.
        blocks = n_tiles * kv_heads
        slots = self.sm_count * (2 if big_tiles else
                                 int(self.lib.ttb_attention_mma_blocks_per_sm(1 if decode_shape else 0, head_dim)))
        if blocks < slots and decode_shape and self.use_tma_decode:
            # The TMA decode kernel streams faster and pays relatively more for a split: chunks of at least 512
            # keys, and about 2.2 blocks an SM rather than all that fit (measured at 8,192 keys of context and
            # head size 64: 320 blocks are 2.6 % faster than 384 at batch 8, and 6 % faster than 416 at batch 4;
            # 256 are as slow as 384).
            splits = max(1, int(min(slots, 2.2 * self.sm_count) / blocks + 0.5))
            if splits * blocks > slots:
                splits -= 1
            # (with so few blocks that even 32 splits leave room, chunks of 256 keys: batch 1 at 8,192 keys is
            # 1.5 % faster with 32 splits and the merge kernel than with 16 merged by a cluster; batch 2 is not)
            least = 256 if blocks * 32 <= slots else 512
            splits = max(1, min(splits, batch.max_context // least))
        elif blocks < slots:
            splits = max(1, min(slots // blocks, batch.max_context // 256))
        else:
            splits = max(1, min(batch.max_context // 2048, -(-4 * slots // blocks)))
        plan = (decode_shape, seg, tok0, n_tiles, splits)
        batch.extras[key] = plan
        return plan

    def _attention_tcgen05(self, qkv, out, batch, heads, kv_heads, head_dim, scale, view):
        tokens = qkv.shape[0]
        _, seg, tok0, n_tiles, splits = self._attention_plan(batch, heads // kv_heads, kv_heads, head_dim, big_tiles=True)
        partial_o = partial_ml = None
        if splits > 1:
            partial_o = torch.empty(tokens * heads * splits * head_dim, dtype=torch.float32, device=self.device)
            partial_ml = torch.empty(tokens * heads * splits * 2, dtype=torch.float32, device=self.device)
        self._check(self.lib.ttb_paged_attention_tcgen05(
            self._p(qkv), qkv.stride(0), self._p(out), self._p(batch.cu_seqlens), self._p(batch.seg_pos0),
            self._p(view.keys), self._p(view.values), self._p(view.block_table), view.block_table.shape[1],
            view.page_size, self._p(seg), self._p(tok0), n_tiles, tokens, heads, kv_heads, head_dim,
            ctypes.c_float(scale), splits, self._p(partial_o), self._p(partial_ml), view.keys.shape[0],
            self._p(self.status), self._p(self.tc_error), self._stream()), "paged_attention_tcgen05")
        if splits > 1:
            self._check(self.lib.ttb_attention_merge(self._p(partial_o), self._p(partial_ml), self._p(out),
                                                     tokens * heads, splits, head_dim, self._stream()), "attention_merge")

    def _attention_mma(self, qkv, out, batch, heads, kv_heads, head_dim, scale, view):
        tokens = qkv.shape[0]
        if (self.use_tcgen05_attention and batch.max_seg_len * (heads // kv_heads) > 16 and view.keys.is_contiguous()
                and view.values.is_contiguous() and qkv.stride(0) % head_dim == 0
                and self.lib.ttb_attention_tcgen05_supports(heads, kv_heads, head_dim, view.page_size, int(view.window or 0))):
            return self._attention_tcgen05(qkv, out, batch, heads, kv_heads, head_dim, scale, view)
        decode_shape, seg, tok0, n_tiles, splits = self._attention_plan(batch, heads // kv_heads, kv_heads, head_dim)
        partial_o = partial_ml = None
        max_rows = batch.max_seg_len * (heads // kv_heads)
        if (decode_shape and self.use_tma_decode and view.keys.is_contiguous() and view.values.is_contiguous()
                and self.lib.ttb_attention_decode_supports(heads, kv_heads, head_dim, view.page_size, max_rows)):
            in_kernel = bool(self.lib.ttb_attention_decode_merges_in_kernel(splits, batch.num_segments * kv_heads * splits))  # a cluster merges the key splits
            if splits > 1 and not in_kernel:
                partial_o = torch.empty(tokens * heads * splits * head_dim, dtype=torch.float32, device=self.device)
                partial_ml = torch.empty(tokens * heads * splits * 2, dtype=torch.float32, device=self.device)
            self._check(self.lib.ttb_paged_attention_decode(
                self._p(qkv), qkv.stride(0), self._p(out), self._p(batch.cu_seqlens), self._p(batch.seg_pos0),
                self._p(view.keys), self._p(view.values), self._p(view.block_table), view.block_table.shape[1],
                view.page_size, batch.num_segments, tokens, max_rows, heads, kv_heads, head_dim, ctypes.c_float(scale),
                int(view.window or 0), splits, self._p(partial_o), self._p(partial_ml), view.keys.shape[0],
                self._p(self.status), self._p(self.tc_error), self._stream()), "paged_attention_decode")
            if splits > 1 and not in_kernel:
                self.launches += 1
            return
        if splits > 1:
            partial_o = torch.empty(tokens * heads * splits * head_dim, dtype=torch.float32, device=self.device)
            partial_ml = torch.empty(tokens * heads * splits * 2, dtype=torch.float32, device=self.device)
        self._check(self.lib.ttb_paged_attention_mma_checked(
            self._p(qkv), qkv.stride(0), self._p(out), self._p(batch.cu_seqlens), self._p(batch.seg_pos0),
            self._p(view.keys), self._p(view.values), self._p(view.block_table), view.block_table.shape[1],
            view.page_size, self._p(seg), self._p(tok0), n_tiles, tokens, heads, kv_heads, head_dim,
            ctypes.c_float(scale), int(view.window or 0), 1 if decode_shape else 0, splits,
            self._p(partial_o), self._p(partial_ml), view.keys.shape[0], self._p(self.status), self._stream()),
            "paged_attention_mma")
        if splits > 1:
            self.launches += 1

    # ------------------------------------------------------------------ layer norm around sub-layers
    def add_layernorm(self, residual, delta, after, mult, norm, out_dtype):
        """residual += mult * (after(delta) if after else delta), in place and in float32; then norm(residual) in
        out_dtype (None when norm is None). `after` and `norm` are layer-norm parts (weight, bias or None, eps)."""
        rows, width = residual.shape
        if residual.dtype != torch.float32 or not residual.is_contiguous():
            raise KernelError("the residual stream is float32 and contiguous")
        if delta is not None and (delta.shape != residual.shape or delta.stride(1) != 1):
            raise KernelError("add_layernorm: delta must have the residual's shape")
        out = torch.empty(rows, width, dtype=out_dtype, device=self.device) if norm is not None else None
        self._check(self.lib.ttb_add_layernorm(
            self._p(residual), self._p(delta), _dtype_code(delta.dtype) if delta is not None else 0,
            delta.stride(0) if delta is not None else 0,
            self._p(after.weight if after is not None else None), self._p(after.bias if after is not None else None),
            ctypes.c_float(after.eps if after is not None else 0.0), ctypes.c_float(mult),
            self._p(norm.weight if norm is not None else None), self._p(norm.bias if norm is not None else None),
            ctypes.c_float(norm.eps if norm is not None else 0.0), self._p(out), _dtype_code(out_dtype), rows, width,
            self._stream()), "add_layernorm")
        return out

    LN_SUM_TERMS = 4

    def add_layernorm_sum(self, residual, tensors, scales, row_term, norm, out_dtype):
        """residual += sum_i scales[i] * tensors[i] + row_term[1] * row_term[0], in place and in float32 (each tensor
        [rows, width], float32 or bfloat16, contiguous; scales None: all one; row_term (float32 vector [width], factor) or
        None); then norm(residual) in out_dtype (None when norm is None). `norm` is a layer-norm part (weight, bias or
        None, eps)."""
        rows, width = residual.shape
        if residual.dtype != torch.float32 or not residual.is_contiguous():
            raise KernelError("the residual stream is float32 and contiguous")
        tensors = list(tensors)
        scales = [1.0] * len(tensors) if scales is None else [float(s) for s in scales]
        for t in tensors:
            if t.shape != residual.shape or not t.is_contiguous():
                raise KernelError("add_layernorm_sum: every term must be contiguous and have the stream's shape")
        out = None
        while True:
            now, tensors = tensors[:self.LN_SUM_TERMS], tensors[self.LN_SUM_TERMS:]
            now_scales, scales = scales[:self.LN_SUM_TERMS], scales[self.LN_SUM_TERMS:]
            last = not tensors
            n = len(now)
            ptrs = (ctypes.c_void_p * max(n, 1))(*[t.data_ptr() for t in now])
            dtypes = (ctypes.c_int * max(n, 1))(*[_dtype_code(t.dtype) for t in now])
            factors = (ctypes.c_float * max(n, 1))(*now_scales)
            normed = last and norm is not None
            if normed:
                out = torch.empty(rows, width, dtype=out_dtype, device=self.device)
            row = row_term if last else None
            if n or row is not None or normed:
                self._check(self.lib.ttb_add_layernorm_sum(
                    self._p(residual), ptrs, dtypes, factors, n, self._p(row[0] if row is not None else None),
                    ctypes.c_float(row[1] if row is not None else 0.0), self._p(norm.weight if normed else None),
                    self._p(norm.bias if normed else None), ctypes.c_float(norm.eps if normed else 0.0), self._p(out),
                    _dtype_code(out_dtype) if normed else 0, rows, width, self._stream()), "add_layernorm_sum")
            if last:
                return out

    def add_row_vector(self, x, vector):
        """x [rows, width] += vector (float32 [width]), in place."""
        rows, width = x.shape
        if x.stride(1) != 1 or vector.dtype != torch.float32 or vector.shape != (width,):
            raise KernelError("add_row_vector: contiguous columns and a float32 vector of the row's width")
        self._check(self.lib.ttb_add_row_vector(self._p(x), _dtype_code(x.dtype), x.stride(0), self._p(vector), rows, width,
                                                self._stream()), "add_row_vector")
        return x

    # ------------------------------------------------------------------ latent attention
    def latent_prepare(self, down, batch, q_rank, kv_rank, rot_dim, q_norm, kv_norm, eps, inv_freq, rotary_dim, view,
                       write, out_dtype, amplitude=1.0):
        """down: float32 [T, >= q_rank + kv_rank + rot_dim]. Returns the RMS-normed query latent [T, q_rank] (None with
        q_rank 0); writes the RMS-normed key/value latent and the rotated shared key part (cosines and sines times
        `amplitude`) into the tokens' page rows."""
        tokens = down.shape[0]
        if down.dtype != torch.float32 or down.stride(1) != 1:
            raise KernelError("latent_prepare: the down projection must be float32, contiguous along its columns")
        write = bool(write and view is not None)
        if write and (view.rows.dtype != out_dtype or not view.rows.is_contiguous()):
            raise KernelError("latent_prepare: the cache rows must be contiguous and of the compute dtype")
        cq = torch.empty(tokens, q_rank, dtype=out_dtype, device=self.device) if q_rank else None
        self._check(self.lib.ttb_latent_prepare_ext(
            self._p(down), down.stride(0), q_rank, kv_rank, rot_dim, self._p(q_norm), self._p(kv_norm),
            ctypes.c_float(eps), self._p(inv_freq), int(rotary_dim), self._p(batch.positions), self._p(batch.seg_of_token),
            self._p(cq), self._p(view.rows if write else None), _dtype_code(out_dtype),
            self._p(view.block_table if write else None), view.block_table.shape[1] if write else 0,
            view.page_size if write else 1, view.rows.shape[0] if write else 0, 1 if write else 0, tokens,
            self._p(self.status), ctypes.c_float(amplitude), self._stream()), "latent_prepare")
        return cq

    MOE_TCGEN05_PAIRS = 1024     # from this many pairs on the experts' products run on the grouped tcgen05 kernel
    MOE_GEMV_PAIRS = 64          # up to this many (token, choice) pairs the experts run as matrix-vector products
    HEADS_LIBRARY_ROWS = 32      # per-head bfloat16 products with at least this many rows go to the library's batched product

    def heads_linear(self, x, w, out_dtype=None):
        """x [T, H, K] (any token and head strides) times w [H, N, K], head by head -> [T, H, N] (a view that may
        be strided; its last axis is contiguous). out_dtype: float32 keeps the float32 sums of a bfloat16 product."""
        T, H, K = x.shape
        N = w.shape[1]
        out_dtype = out_dtype or x.dtype
        if w.shape[0] != H or w.shape[2] != K or x.dtype != w.dtype or x.stride(2) != 1 or not w.is_contiguous():
            raise KernelError(f"heads_linear: x {tuple(x.shape)} does not match w {tuple(w.shape)}")
        if x.dtype == torch.bfloat16 and T >= self.HEADS_LIBRARY_ROWS:
            if out_dtype == torch.bfloat16:
                return torch.bmm(x.transpose(0, 1), w.transpose(1, 2)).transpose(0, 1)       # library product (cuBLAS)
            return torch.bmm(x.transpose(0, 1), w.transpose(1, 2), out_dtype=out_dtype).transpose(0, 1)
        out = torch.empty(T, H, N, dtype=out_dtype, device=self.device)
        self._check(self.lib.ttb_gemm_simt_batched(
            self._p(x), self._p(w), self._p(out), _dtype_code(x.dtype), _dtype_code(out_dtype), H, T, N, K, x.stride(0), K,
            H * N, ctypes.c_longlong(x.stride(1)), ctypes.c_longlong(N * K), ctypes.c_longlong(N), self._stream()),
            "heads_linear")
        return out

    LATENT_OUT_ROWS = 64         # up to this many tokens the end of the mixer (merge, W_uv, gate) is one kernel

    def latent_attention(self, q_latent, q_rot, batch, view, scale, sinks, inv_freq, rotary_dim, amplitude=1.0, window="view"):
        """q_latent [T, H, latent], q_rot [T, H, extra] or None (rotated here by the tokens' positions, cosines and sines
        times `amplitude`); the cache rows hold [latent | extra] per token. `window`: what a query sees ("view": what the
        cache keeps). Returns the weighted sums of the latents [T, H, latent]."""
        return self._latent_attention(q_latent, q_rot, batch, view, scale, sinks, inv_freq, rotary_dim, True, amplitude, window)[0]

    def latent_attention_out(self, q_latent, q_rot, batch, view, scale, sinks, inv_freq, rotary_dim, w_uv, gate, amplitude=1.0,
                             window="view"):
        """Attention over the latents, then per head W_uv [H, vdim, latent] and the gate (float32 logits [T, H] or
        [T, H * vdim], or None) -> [T, H * vdim]. For a handful of tokens the key splits' merge, the per-head
        product and the gate are one kernel."""
        T, H, R = q_latent.shape
        V = w_uv.shape[1]
        if T > self.LATENT_OUT_ROWS or R * 4 > 48 * 1024:
            mixed = self.latent_attention(q_latent, q_rot, batch, view, scale, sinks, inv_freq, rotary_dim, amplitude, window)
            return self.gate_heads(self.heads_linear(mixed, w_uv), gate)
        mixed, partial_o, partial_ml, splits = self._latent_attention(q_latent, q_rot, batch, view, scale, sinks, inv_freq,
                                                                      rotary_dim, False, amplitude, window)
        return self.latent_out(mixed if splits == 1 else None, partial_o, partial_ml, splits, w_uv, gate, T, H, R)

    def latent_out(self, mixed, partial_o, partial_ml, splits, w_uv, gate, T, H, R):
        """The mixer's end for a handful of tokens in one kernel: the key splits' partial sums merged (or `mixed`
        [T, H, latent] read), W_uv [H, vdim, latent] per head, the gate -> [T, H * vdim]."""
        V = w_uv.shape[1]
        if w_uv.shape != (H, V, R) or not w_uv.is_contiguous():
            raise KernelError("latent_out: W_uv must be contiguous [heads, vdim, latent]")
        per_head = 0
        if gate is not None:
            if gate.dtype != torch.float32 or gate.stride(1) != 1 or gate.shape[1] not in (H, H * V):
                raise KernelError("latent_out: gate must be float32 [T, heads] or [T, heads * vdim]")
            per_head = 1 if gate.shape[1] == H and V != 1 else 0
        res = torch.empty(T, H * V, dtype=w_uv.dtype, device=self.device)
        self._check(self.lib.ttb_latent_out(
            self._p(mixed), ctypes.c_longlong(mixed.stride(0) if mixed is not None else 0),
            ctypes.c_longlong(mixed.stride(1) if mixed is not None else 0), self._p(partial_o), self._p(partial_ml), splits,
            self._p(w_uv),
            self._p(gate), gate.stride(0) if gate is not None else 0, per_head, self._p(res), _dtype_code(res.dtype), T, H, R,
            V, self._stream()), "latent_out")
        return res

    def _latent_attention(self, q_latent, q_rot, batch, view, scale, sinks, inv_freq, rotary_dim, merge, amplitude=1.0,
                          window="view"):
        """-> (weighted sums [T, H, latent], partial sums, their maxima and sums, number of key splits); with merge
        False and more than one split the first is not filled in and the partial results are the caller's to merge."""
        T, H, R = q_latent.shape
        window = view.window if window == "view" else window
        if R != view.latent or q_latent.dtype != view.rows.dtype or q_latent.stride(2) != 1:
            raise KernelError("latent_attention: the queries do not fit the cache rows")
        if (q_rot is None) != (view.extra == 0) or (q_rot is not None and (q_rot.shape[2] != view.extra or q_rot.stride(2) != 1)):
            raise KernelError("latent_attention: the rotated query part does not fit the cache rows")
        out = torch.empty(T, H, R, dtype=q_latent.dtype, device=self.device)
        if (self.use_mma_latent_attention and q_latent.dtype == torch.bfloat16 and view.rows.is_contiguous() and scale > 0
                and q_latent.stride(0) % 8 == 0 and q_latent.stride(1) % 8 == 0 and q_latent.data_ptr() % 16 == 0
                and self.lib.ttb_latent_attention_mma_supports(R, view.extra, int(rotary_dim), int(window or 0))):
            # tensor cores; few blocks (decode): the keys are split over blocks and merged afterwards
            per_tile = int(self.lib.ttb_latent_attention_mma_tokens_per_tile(H))
            blocks = batch.num_segments * -(-batch.max_seg_len // per_tile) * -(-H // 64) * -(-R // (256 if R > 128 else 128))
            splits = 1
            if blocks < self.sm_count:
                reach = min(batch.max_context, window + batch.max_seg_len) if window else batch.max_context
                splits = max(1, min(-(-2 * self.sm_count // blocks), reach // 128, 64))
            partial_o = partial_ml = None
            if splits > 1:
                partial_o = torch.empty(T * H * splits * R, dtype=torch.float32, device=self.device)
                partial_ml = torch.empty(T * H * splits * 2, dtype=torch.float32, device=self.device)
            self._check(self.lib.ttb_latent_attention_mma_ext(
                self._p(q_latent), ctypes.c_longlong(q_latent.stride(0)), ctypes.c_longlong(q_latent.stride(1)),
                self._p(q_rot), ctypes.c_longlong(q_rot.stride(0) if q_rot is not None else 0),
                ctypes.c_longlong(q_rot.stride(1) if q_rot is not None else 0), self._p(out), self._p(batch.cu_seqlens),
                self._p(batch.seg_pos0), self._p(view.rows), self._p(view.block_table), view.block_table.shape[1],
                view.page_size, view.rows.shape[0], batch.num_segments, batch.max_seg_len, T, H, R, view.extra,
                ctypes.c_float(scale), self._p(sinks), self._p(inv_freq), int(rotary_dim), splits, self._p(partial_o),
                self._p(partial_ml), 1 if merge else 0, self._p(self.status), int(window or 0), ctypes.c_float(amplitude),
                self._stream()), "latent_attention_mma")
            if splits > 1 and merge:
                self.launches += 1
            return out, partial_o, partial_ml, splits
        self._check(self.lib.ttb_latent_attention_generic_ext(
            self._p(q_latent), ctypes.c_longlong(q_latent.stride(0)), ctypes.c_longlong(q_latent.stride(1)),
            self._p(q_rot), ctypes.c_longlong(q_rot.stride(0) if q_rot is not None else 0),
            ctypes.c_longlong(q_rot.stride(1) if q_rot is not None else 0), self._p(out), _dtype_code(q_latent.dtype),
            self._p(batch.positions), self._p(batch.seg_of_token), self._p(view.rows), self._p(view.block_table),
            view.block_table.shape[1], view.page_size, T, H, R, view.extra, ctypes.c_float(scale), self._p(sinks),
            self._p(inv_freq), int(rotary_dim), int(window or 0), view.rows.shape[0], self._p(self.status),
            ctypes.c_float(amplitude), self._stream()), "latent_attention")
        return out, None, None, 1

    def gate_heads(self, out, gate):
        """out [T, H, V] (any token and head strides) times sigmoid(gate), gate float32 [T, H] or [T, H * V] or
        None -> contiguous [T, H * V]."""
        T, H, V = out.shape
        if out.stride(2) != 1:
            raise KernelError("gate_heads: the last axis must be contiguous")
        per_head = 0
        if gate is not None:
            if gate.dtype != torch.float32 or gate.stride(1) != 1 or gate.shape[1] not in (H, H * V):
                raise KernelError("gate_heads: gate must be float32 [T, heads] or [T, heads * vdim]")
            per_head = 1 if gate.shape[1] == H and V != 1 else 0
        res = torch.empty(T, H * V, dtype=out.dtype, device=self.device)
        self._check(self.lib.ttb_gate_heads(
            self._p(out), ctypes.c_longlong(out.stride(0)), ctypes.c_longlong(out.stride(1)), self._p(gate),
            gate.stride(0) if gate is not None else 0, per_head, self._p(res), _dtype_code(out.dtype), T, H, V,
            self._stream()), "gate_heads")
        return res

    # ------------------------------------------------------------------ routed experts
    _ROUTER_SCORES = {"softmax": 0, "sigmoid": 1}

    def route_top(self, x, w_router, experts, top, shared, scores="softmax"):
        """Float32 router: the `top` experts with the largest logits per token and the softmax over their logits
        (`scores` "sigmoid": each chosen expert's own sigmoid(logit) instead, not renormalised);
        with `shared`, row `experts` of w_router gives sigmoid(w . x) per token. -> (int32 [T, top], float32 [T, top],
        float32 [T] or None)."""
        if scores not in self._ROUTER_SCORES:
            raise KernelError(f"route_top: scores {scores!r} is not known; known: {sorted(self._ROUTER_SCORES)}")
        T, width = x.shape
        if w_router.dtype != torch.float32 or w_router.shape != (experts + (1 if shared else 0), width) or x.stride(1) != 1:
            raise KernelError("route_top: the router's matrix must be float32 [experts (+ 1), width]")
        choice = torch.empty(T, top, dtype=torch.int32, device=self.device)
        weight = torch.empty(T, top, dtype=torch.float32, device=self.device)
        gate = torch.empty(T, dtype=torch.float32, device=self.device) if shared else None
        self._check(self.lib.ttb_route_top_scored(self._p(x), _dtype_code(x.dtype), x.stride(0), self._p(w_router), T, width,
                                                  experts, top, 1 if shared else 0, self._p(choice), self._p(weight),
                                                  self._p(gate), self._ROUTER_SCORES[scores], self._stream()), "route_top")
        return choice, weight, gate

    def route_corrected(self, x, w_router, correction, experts, top, scale, floor):
        """Float32 router with a score per expert, s = sigmoid(W_r x): the `top` experts with the largest s + correction
        are chosen (the lower index among equals), their weights are s / (sum of the chosen s + floor) * scale.
        -> (int32 [T, top], float32 [T, top])."""
        T, width = x.shape
        if (w_router.dtype != torch.float32 or w_router.shape != (experts, width) or x.stride(1) != 1
                or correction.dtype != torch.float32 or correction.shape != (experts,)):
            raise KernelError("route_corrected: the router's matrix must be float32 [experts, width], the corrections float32 [experts]")
        choice = torch.empty(T, top, dtype=torch.int32, device=self.device)
        weight = torch.empty(T, top, dtype=torch.float32, device=self.device)
        self._check(self.lib.ttb_route_top_corrected(self._p(x), _dtype_code(x.dtype), x.stride(0), self._p(w_router), T, width,
                                                     experts, top, 0, self._p(choice), self._p(weight), None, 2,
                                                     self._p(correction), ctypes.c_float(scale), ctypes.c_float(floor),
                                                     self._stream()), "route_corrected")
        return choice, weight

    def _ones(self, count):
        """`count` float32 ones on the device; made once and sliced."""
        have = getattr(self, "_ones_buffer", None)
        if have is None or have.numel() < count:
            have = torch.ones(max(count, 1 << 16), dtype=torch.float32, device=self.device)
            self._ones_buffer = have
        return have[:count]

    def glu_clamped(self, gate_up, limit, alpha):
        rows, two = gate_up.shape
        out = torch.empty(rows, two // 2, dtype=gate_up.dtype, device=self.device)
        if not gate_up.is_contiguous():
            raise KernelError("glu_clamped: the product must be contiguous")
        self._check(self.lib.ttb_glu_clamped(self._p(gate_up), self._p(out), _dtype_code(gate_up.dtype), rows, two // 2,
                                             ctypes.c_float(limit), ctypes.c_float(alpha), self._stream()), "glu_clamped")
        return out

    def linear_glu_clamped(self, x, w_gate_up, limit, alpha):
        """g' * sigmoid(alpha g') * (u' + 1) with g' = min(x Wg^T, limit), u' = clamp(x Wu^T, -limit, limit), for
        w_gate_up = [Wg; Wu] stacked along the rows."""
        return self.glu_clamped(self.linear(x, w_gate_up), limit, alpha)

    def routed_experts(self, x, choice, weight, w_gate_up, w_down, limit, alpha, shared=None, shared_gate=None):
        """x [T, width]; choice, weight [T, top]; w_gate_up [E, 2 inter, width]; w_down [E, width, inter] ->
        float32 [T, width]: sum_j weight[t, j] * expert_choice[t, j](x[t]) + shared_gate[t] * shared_expert(x[t]).
        shared: None or (w_gate_up [2 s, width], w_down [width, s], limit) of the expert every token uses."""
        T, width = x.shape
        E, two_inter, _ = w_gate_up.shape
        inter, top = two_inter // 2, choice.shape[1]
        pairs = T * top
        if x.dtype != w_gate_up.dtype or x.stride(1) != 1 or not w_gate_up.is_contiguous() or not w_down.is_contiguous():
            raise KernelError("routed_experts: operands must share a dtype and be contiguous")
        if shared is not None and shared_gate is None:
            shared_gate = self._ones(T)                    # a shared expert without a gate of its own
        if shared is not None and (shared_gate is None or not shared[0].is_contiguous() or not shared[1].is_contiguous()):
            raise KernelError("routed_experts: the shared expert needs contiguous weights and a gate per token")
        out = torch.empty(T, width, dtype=torch.float32, device=self.device)
        hidden = torch.empty(pairs, inter, dtype=x.dtype, device=self.device)
        shared_inter = shared[0].shape[0] // 2 if shared is not None else 0
        if pairs <= self.MOE_GEMV_PAIRS and width * 4 <= 48 * 1024 and (top * inter + shared_inter) * 4 <= 48 * 1024:
            # a handful of pairs (decode): every pair streams its expert's rows, no grouping; the shared expert runs
            # inside the same two kernels as one more expert per token
            shared_hidden = torch.empty(T, shared_inter, dtype=x.dtype, device=self.device) if shared is not None else None
            self._check(self.lib.ttb_moe_gemv(
                self._p(x), x.stride(0), self._p(w_gate_up), self._p(w_down), self._p(choice), self._p(weight),
                self._p(hidden), None, self._p(shared_gate), self._p(out), _dtype_code(x.dtype), T, E, top,
                inter, width, ctypes.c_float(limit), ctypes.c_float(alpha),
                self._p(shared[0] if shared is not None else None), self._p(shared[1] if shared is not None else None),
                self._p(shared_hidden), shared_inter, ctypes.c_float(shared[2] if shared is not None else 0.0),
                self._stream()), "moe_gemv")
            self.launches += 1
            return out
        shared_out = None
        if shared is not None:
            shared_out = self.linear(self.linear_glu_clamped(x, shared[0], shared[2], alpha), shared[1])
        offsets = torch.empty(E + 1, dtype=torch.int32, device=self.device)
        order = torch.empty(pairs, dtype=torch.int32, device=self.device)
        code = _dtype_code(x.dtype)
        pair_out = torch.empty(pairs, width, dtype=torch.float32, device=self.device)
        grouped_tc = (x.dtype == torch.bfloat16 and self.use_tcgen05 is not False and pairs >= self.MOE_TCGEN05_PAIRS
                      and width % 8 == 0 and inter % 8 == 0 and x.stride(0) % 8 == 0 and x.data_ptr() % 16 == 0)
        if grouped_tc:
            # many pairs (prompt portions): the tokens' rows are laid out expert by expert and both products run on
            # the fifth-generation tensor cores over those groups; no size is read back by the host
            max_tiles = -(-pairs // 128) + E
            tokens_of = torch.empty(pairs, dtype=torch.int32, device=self.device)
            tile_info = torch.empty(2 * max_tiles + 1, dtype=torch.int32, device=self.device)
            self._check(self.lib.ttb_moe_align(self._p(choice), pairs, E, top, self._p(offsets), self._p(order),
                                               self._p(tokens_of), self._p(tile_info[1:]), self._p(tile_info), 128,
                                               self._stream()), "moe_align")
            grouped = self.gather_rows(x, tokens_of)
            self._check(self.lib.ttb_moe_gemm_tcgen05(
                self._p(grouped), width, self._p(w_gate_up), width, self._p(hidden), inter, 1, self._p(offsets),
                self._p(order), self._p(tile_info[1:]), self._p(tile_info), pairs, E, max_tiles, inter, width,
                ctypes.c_float(limit), ctypes.c_float(alpha), self._p(self.tc_error), self._stream()), "moe_gate_up_tcgen05")
            self._check(self.lib.ttb_moe_gemm_tcgen05(
                self._p(hidden), inter, self._p(w_down), inter, self._p(pair_out), width, 0, self._p(offsets),
                self._p(order), self._p(tile_info[1:]), self._p(tile_info), pairs, E, max_tiles, width, inter,
                ctypes.c_float(limit), ctypes.c_float(alpha), self._p(self.tc_error), self._stream()), "moe_down_tcgen05")
        else:
            self._check(self.lib.ttb_moe_align(self._p(choice), pairs, E, top, self._p(offsets), self._p(order), None, None,
                                               None, 0, self._stream()), "moe_align")
            self._check(self.lib.ttb_moe_group_gemm(
                self._p(x), x.stride(0), self._p(w_gate_up), ctypes.c_longlong(two_inter * width), width, self._p(hidden), inter,
                code, 1, self._p(offsets), self._p(order), pairs, E, top, inter, width, ctypes.c_float(limit),
                ctypes.c_float(alpha), self._stream()), "moe_gate_up")
            self._check(self.lib.ttb_moe_group_gemm(
                self._p(hidden), inter, self._p(w_down), ctypes.c_longlong(width * inter), inter, self._p(pair_out), width,
                code, 0, self._p(offsets), self._p(order), pairs, E, top, width, inter, ctypes.c_float(limit),
                ctypes.c_float(alpha), self._stream()), "moe_down")
        self._check(self.lib.ttb_moe_combine(
            self._p(pair_out), self._p(weight), top, self._p(shared_out),
            _dtype_code(shared_out.dtype) if shared_out is not None else 0, self._p(shared_gate), self._p(out), T, width,
            self._stream()), "moe_combine")
        return out

    # ------------------------------------------------------------------ the float32 stream, several outputs at once
    def stream_add_norm(self, residual, deltas, row_vector=None, weight=None, eps=0.0, offset=0.0, out_dtype=None):
        """residual += sum(deltas) + row_vector, in place and in float32 (each delta [rows, width], float32 or
        bfloat16; row_vector float32 [width], the same for every row); then, with a weight,
        residual / sqrt(mean(residual^2) + eps) * (offset + weight) in out_dtype comes back (None without)."""
        rows, width = residual.shape
        if residual.dtype != torch.float32 or not residual.is_contiguous():
            raise KernelError("the residual stream is float32 and contiguous")
        deltas = [d for d in deltas if d is not None]
        for d in deltas:
            if d.shape != residual.shape or not d.is_contiguous():
                raise KernelError("stream_add_norm: every delta must be contiguous and have the stream's shape")
        out = None
        while True:
            now, deltas = deltas[:2], deltas[2:]
            last = not deltas
            d1 = now[0] if len(now) > 0 else None
            d2 = now[1] if len(now) > 1 else None
            if last and weight is not None:
                out = torch.empty(rows, width, dtype=out_dtype, device=self.device)
            if not last or d1 is not None or row_vector is not None or out is not None:
                self._check(self.lib.ttb_stream_add_norm(
                    self._p(residual), self._p(d1), _dtype_code(d1.dtype) if d1 is not None else 0, self._p(d2),
                    _dtype_code(d2.dtype) if d2 is not None else 0, self._p(row_vector if last else None),
                    self._p(weight if last else None), _dtype_code(weight.dtype) if weight is not None else 0,
                    ctypes.c_float(offset), ctypes.c_float(eps), self._p(out), _dtype_code(out_dtype) if out is not None else 0,
                    rows, width, self._stream()), "stream_add_norm")
            if last:
                return out

    def gated_rmsnorm(self, x, weight, eps, gate, out_dtype):
        """x float32 [rows, width] / sqrt(mean(x^2) + eps) * weight * sigmoid(gate) -> out_dtype; gate [rows, width] may be
        a slice of a wider tensor (its columns contiguous)."""
        rows, width = x.shape
        if x.dtype != torch.float32 or not x.is_contiguous() or gate.shape != x.shape or gate.stride(1) != 1:
            raise KernelError("gated_rmsnorm: x must be float32 and contiguous, the gate of its shape")
        out = torch.empty(rows, width, dtype=out_dtype, device=self.device)
        self._check(self.lib.ttb_gated_rmsnorm(self._p(x), self._p(gate), _dtype_code(gate.dtype), gate.stride(0),
                                               self._p(weight), ctypes.c_float(eps), self._p(out), _dtype_code(out_dtype),
                                               rows, width, self._stream()), "gated_rmsnorm")
        return out

    def mean_rmsnorm_pair(self, a, wa, b, wb, eps):
        """(rms(a) * wa + rms(b) * wb) / 2 -> float32 [rows, width]."""
        if a.shape != b.shape or a.dtype != b.dtype or not a.is_contiguous() or not b.is_contiguous():
            raise KernelError("mean_rmsnorm_pair: both inputs must be contiguous and alike")
        rows, width = a.shape
        out = torch.empty(rows, width, dtype=torch.float32, device=self.device)
        self._check(self.lib.ttb_mean_rmsnorm_pair(self._p(a), self._p(b), _dtype_code(a.dtype), self._p(wa), self._p(wb),
                                                   ctypes.c_float(eps), self._p(out), rows, width, self._stream()),
                    "mean_rmsnorm_pair")
        return out

    _ACTIVATIONS = {"silu": 0, "gelu_tanh": 1, "relu2": 2, "gelu_erf": 3, "relu": 4}

    def glu_activation(self, gate_up, activation):
        """act(gate) * up over [rows, gate | up] -> [rows, columns / 2]; activation "silu", "relu" or "gelu_tanh"."""
        rows, two = gate_up.shape
        if gate_up.stride(1) != 1 or activation not in ("silu", "gelu_tanh", "relu"):
            raise KernelError("glu_activation: the product must be contiguous along its columns; silu, relu or gelu_tanh")
        out = torch.empty(rows, two // 2, dtype=gate_up.dtype, device=self.device)
        self._check(self.lib.ttb_activation(self._p(gate_up), _dtype_code(gate_up.dtype), gate_up.stride(0), self._p(out),
                                            _dtype_code(out.dtype), rows, two // 2, self._ACTIVATIONS[activation],
                                            self._stream()), "glu_activation")
        return out

    def activation(self, x, activation, out_dtype):
        """An activation element by element ("relu2": relu(z)^2; "gelu_erf": 0.5 z (1 + erf(z / sqrt 2))), computed in
        float32 -> out_dtype."""
        rows, cols = x.shape
        if x.stride(1) != 1 or activation not in ("relu2", "gelu_erf"):
            raise KernelError("activation: contiguous columns; relu2 or gelu_erf")
        out = torch.empty(rows, cols, dtype=out_dtype, device=self.device)
        self._check(self.lib.ttb_activation(self._p(x), _dtype_code(x.dtype), x.stride(0), self._p(out), _dtype_code(out_dtype),
                                            rows, cols, self._ACTIVATIONS[activation], self._stream()), "activation")
        return out

    # ------------------------------------------------------------------ recurrent mixers
    RECURRENCE_PART = 16            # tokens of one part of a long segment in the gated recurrence
    LIGHTNING_PART = 128            # tokens of one part of a long segment in chunked lightning attention (two chunks)
    LIGHTNING_SCRATCH_BYTES = 256 << 20     # most memory for the parts' states; longer parts beyond it
    LIGHTNING_SCAN_TOKENS = 16      # steps whose longest segment is at most this long walk token by token

    def lightning_attention(self, proj, batch, view, heads, dim, vdim, decays, write_state=True):
        """proj [T, q | k | v | ...] before their silu; the state float32 [slots, heads, dim, vdim] of view continues
        per segment: S = decay S + k v^T, o = S^T q. -> float32 [T, heads * vdim]."""
        tokens = proj.shape[0]
        if proj.stride(1) != 1 or proj.shape[1] < heads * (2 * dim + vdim):
            raise KernelError("lightning_attention: the projection must hold q, k and v, contiguous along its columns")
        if view.state.dtype != torch.float32 or tuple(view.state.shape[1:]) != (heads, dim, vdim) or not view.state.is_contiguous():
            raise KernelError("lightning_attention: the state must be float32 [slots, heads, dim, vdim]")
        out = torch.empty(tokens, heads * vdim, dtype=torch.float32, device=self.device)
        if (self.use_lightning_chunks and proj.dtype == torch.bfloat16 and batch.max_seg_len > self.LIGHTNING_SCAN_TOKENS
                and proj.stride(0) % 8 == 0 and proj.data_ptr() % 16 == 0 and self.lib.ttb_lightning_chunks_supports(dim, vdim)):
            # prompt portions: chunk by chunk on the tensor cores (decoded tokens and float32 walk token by token);
            # long segments as parts side by side (two launches), as many as their scratch states may take room for
            part_len, parts, scratch = self.LIGHTNING_PART, 1, None
            if batch.max_seg_len >= 2 * part_len:
                per_part = batch.num_segments * heads * dim * vdim * 4
                while -(-batch.max_seg_len // part_len) * per_part > self.LIGHTNING_SCRATCH_BYTES and part_len < batch.max_seg_len:
                    part_len *= 2
                parts = -(-batch.max_seg_len // part_len)
            if parts > 1:
                scratch = torch.empty(batch.num_segments * heads * (parts + 1) * dim * vdim, dtype=torch.float32, device=self.device)
                self.launches += 1
            self._check(self.lib.ttb_lightning_chunks(
                self._p(proj), proj.stride(0), self._p(batch.cu_seqlens), self._p(view.slots), self._p(view.state),
                self._p(decays), self._p(out), batch.num_segments, heads, dim, vdim, 1 if write_state else 0,
                self._p(scratch), parts, part_len, self._stream()), "lightning_chunks")
            return out
        self._check(self.lib.ttb_lightning_scan(
            self._p(proj), _dtype_code(proj.dtype), proj.stride(0), self._p(batch.cu_seqlens), self._p(view.slots),
            self._p(view.state), self._p(decays), self._p(out), batch.num_segments, heads, dim, vdim, 1 if write_state else 0,
            self._stream()), "lightning_scan")
        return out

    def causal_conv(self, x, bias_x, conv_w, conv_b, batch, view):
        """u[t] = conv_b + sum_j conv_w[:, j] * (x + bias_x)[t - taps + 1 + j] per channel, reading the request's kept
        inputs (view.tail) before the step's first token. x [T, channels] may be a slice of a wider product."""
        tokens, channels = x.shape
        taps = conv_w.shape[1]
        if x.stride(1) != 1 or view.tail.dtype != x.dtype or not view.tail.is_contiguous():
            raise KernelError("causal_conv: contiguous columns, and kept inputs of the compute dtype")
        u = torch.empty(tokens, channels, dtype=x.dtype, device=self.device)
        self._check(self.lib.ttb_causal_conv(
            self._p(x), _dtype_code(x.dtype), x.stride(0), self._p(bias_x), self._p(conv_w), self._p(conv_b),
            self._p(batch.seg_of_token), self._p(batch.cu_seqlens), self._p(view.slots), self._p(view.tail), self._p(u),
            tokens, channels, taps, self._stream()), "causal_conv")
        return u

    def gated_recurrence(self, u, gates, gate_bias, rate, yx, bias_yx, batch, view, write_state=True):
        """a = exp(-rate * sigmoid(gates_r + b)); S = a S + sqrt(1 - a^2) * sigmoid(gates_i + b) * u;
        out = S * gelu_tanh(yx[:, :C] + bias_yx[:C]). Leaves S and the convolution's last inputs (yx[:, C:] + bias) in
        the request's slot. gates float32 [T, blocks, 2 s]."""
        tokens, channels = u.shape
        blocks = gates.shape[1]
        if gates.dtype != torch.float32 or gates.stride(2) != 1 or not u.is_contiguous() or yx.stride(1) != 1:
            raise KernelError("gated_recurrence: float32 gates contiguous along their last axis, contiguous u")
        out = torch.empty(tokens, channels, dtype=u.dtype, device=self.device)
        # long segments run as parts of RECURRENCE_PART tokens side by side (two launches: the parts' own products
        # and end states, then the walk that writes out from each part's folded start state)
        parts = -(-batch.max_seg_len // self.RECURRENCE_PART) if batch.max_seg_len >= 4 * self.RECURRENCE_PART else 1
        scratch = torch.empty(batch.num_segments * (parts + 1) * channels * 2, dtype=torch.float32, device=self.device) if parts > 1 else None
        if parts > 1:
            self.launches += 1
        self._check(self.lib.ttb_gated_recurrence(
            self._p(u), _dtype_code(u.dtype), self._p(gates), ctypes.c_longlong(gates.stride(0)),
            ctypes.c_longlong(gates.stride(1)), self._p(gate_bias), self._p(rate), self._p(yx), yx.stride(0),
            self._p(bias_yx), self._p(batch.cu_seqlens), self._p(view.slots), self._p(view.state), self._p(view.tail),
            self._p(out), batch.num_segments, channels, blocks, view.taps, 1 if write_state else 0, self._p(scratch), parts,
            self.RECURRENCE_PART, self._stream()), "gated_recurrence")
        return out

    def recurrent_token(self, yx, bias_yx, conv_w, conv_b, w_gates, gate_bias, rate, batch, view, write_state=True):
        """causal_conv, the gates' block products and gated_recurrence for a step in which every segment holds one
        token, in one kernel. yx [T, y | x'] before their biases; w_gates [blocks, 2 s, s]. -> [T, channels]."""
        tokens, two = yx.shape
        channels, blocks = two // 2, w_gates.shape[0]
        if (yx.stride(1) != 1 or w_gates.dtype != yx.dtype or not w_gates.is_contiguous() or view.tail.dtype != yx.dtype
                or batch.max_seg_len != 1):
            raise KernelError("recurrent_token: one token per segment, weights and kept inputs of the compute dtype")
        out = torch.empty(tokens, channels, dtype=yx.dtype, device=self.device)
        self._check(self.lib.ttb_recurrent_token(
            self._p(yx), _dtype_code(yx.dtype), yx.stride(0), self._p(bias_yx), self._p(conv_w), self._p(conv_b),
            self._p(w_gates), self._p(gate_bias), self._p(rate), self._p(batch.cu_seqlens), self._p(view.slots),
            self._p(view.state), self._p(view.tail), self._p(out), batch.num_segments, channels, blocks, view.taps,
            1 if write_state else 0, self._stream()), "recurrent_token")
        return out

    # ------------------------------------------------------------------ attention with a sink, a cap, chunks
    def qk_norm_rope_write(self, qkv, batch, q_norm, k_norm, eps, inv_freq, rotary_dim, heads, kv_heads, dim, vdim, view,
                           write_kv=True, whole=False, amplitude=1.0, bias=None, q_temp=None):
        """In place on qkv [T, heads * dim | kv_heads * dim | kv_heads * vdim]: RMS norm per head of q and k (weights
        float32 [dim] or None), rotation of their first rotary_dim elements; keys and values go into their pages.
        whole: one RMS norm over all of a token's query elements and one over all of its key elements (weights float32
        [heads * dim] and [kv_heads * dim]); amplitude: what the rotation's cosines and sines are multiplied by."""
        tokens = qkv.shape[0]
        if (bias is not None or q_temp is not None) and (whole or amplitude != 1.0):
            raise KernelError("qk_norm_rope_write: biases and a query temperature come with the per-head norm and amplitude 1")
        if whole or amplitude != 1.0:
            if q_norm is not None and not whole:
                raise KernelError("qk_norm_rope_write: a rotation amplitude comes with the norm over the whole projection, or none")
            if q_norm is not None and (q_norm.shape[0] != heads * dim or k_norm.shape[0] != kv_heads * dim):
                raise KernelError("qk_norm_rope_write: whole-projection norms need a weight per element of q and of k")
            if qkv.shape[1] != (heads + kv_heads) * dim + kv_heads * vdim or qkv.stride(1) != 1:
                raise KernelError("qk_norm_rope_write: qkv must be [tokens, heads * dim + kv_heads * (dim + vdim)], contiguous along its columns")
            write = bool(write_kv and view is not None)
            if write and (view.keys.dtype != qkv.dtype or not view.keys.is_contiguous() or not view.values.is_contiguous()):
                raise KernelError("qk_norm_rope_write: cache pages must be contiguous and of the compute dtype")
            self._check(self.lib.ttb_qk_whole_norm_rope_write(
                self._p(qkv), _dtype_code(qkv.dtype), qkv.stride(0), self._p(batch.positions), self._p(batch.seg_of_token),
                self._p(q_norm), self._p(k_norm), ctypes.c_float(eps), self._p(inv_freq), int(rotary_dim),
                ctypes.c_float(amplitude), tokens, heads, kv_heads, dim, vdim, self._p(view.keys if write else None),
                self._p(view.values if write else None), self._p(view.block_table if write else None),
                view.block_table.shape[1] if write else 0, view.page_size if write else 1,
                view.keys.shape[0] if write else 0, 1 if write else 0, self._p(self.status), self._stream()),
                "qk_whole_norm_rope_write")
            return
        if qkv.shape[1] != (heads + kv_heads) * dim + kv_heads * vdim or qkv.stride(1) != 1:
            raise KernelError("qk_norm_rope_write: qkv must be [tokens, heads * dim + kv_heads * (dim + vdim)], contiguous along its columns")
        if (q_norm is None) != (k_norm is None):
            raise KernelError("qk_norm_rope_write: both norms or none")
        write = bool(write_kv and view is not None)
        if write and (view.keys.dtype != qkv.dtype or not view.keys.is_contiguous() or not view.values.is_contiguous()):
            raise KernelError("qk_norm_rope_write: cache pages must be contiguous and of the compute dtype")
        if bias is not None and (bias.dtype != torch.float32 or bias.shape != (qkv.shape[1],) or not bias.is_contiguous()):
            raise KernelError("qk_norm_rope_write: the bias must be float32, one number per column of qkv")
        coef, every = (float(q_temp[0]), int(q_temp[1])) if q_temp is not None else (0.0, 1)
        self._check(self.lib.ttb_qk_norm_rope_write_ext(
            self._p(qkv), _dtype_code(qkv.dtype), qkv.stride(0), self._p(batch.positions), self._p(batch.seg_of_token),
            self._p(q_norm), self._p(k_norm), ctypes.c_float(eps), self._p(inv_freq), int(rotary_dim), tokens, heads, kv_heads,
            dim, vdim, self._p(view.keys if write else None), self._p(view.values if write else None),
            self._p(view.block_table if write else None), view.block_table.shape[1] if write else 0,
            view.page_size if write else 1, view.keys.shape[0] if write else 0, 1 if write else 0, self._p(self.status),
            self._p(bias), ctypes.c_float(coef), every, self._stream()), "qk_norm_rope_write")

    def sink_attention(self, qkv, batch, heads, kv_heads, dim, vdim, scale, softcap, sinks, view, distance_bias=None):
        """Causal attention of the queries in qkv over the paged keys and values, with a cap on the scores, chunks or
        a window (from the view), a sink per head (float32 [heads] or None) and a bias by distance (float32
        [heads, far + 1], added to the capped score; distances beyond `far` take the last column). -> [T, heads * vdim]."""
        tokens = qkv.shape[0]
        if view.keys.dtype != qkv.dtype:
            raise KernelError("sink_attention: cache pages and queries differ in dtype")
        out = torch.empty(tokens, heads * vdim, dtype=qkv.dtype, device=self.device)
        if distance_bias is not None and (distance_bias.dtype != torch.float32 or distance_bias.dim() != 2
                                          or distance_bias.shape[0] != heads or not distance_bias.is_contiguous()):
            raise KernelError("sink_attention: the bias by distance must be float32 [heads, far + 1]")
        if (self.use_mma_attention and qkv.dtype == torch.bfloat16 and dim == vdim and qkv.stride(0) % 8 == 0
                and qkv.data_ptr() % 16 == 0 and view.keys.is_contiguous() and view.values.is_contiguous()
                and (distance_bias is None or scale > 0)
                and self.lib.ttb_attention_mma_supports(heads, kv_heads, dim)):
            # keys and values of one size that the tensor-core kernel takes: 64-row tiles for prompt portions, the
            # decode shape for single tokens; key splits sized by what a query can see at most
            decode_shape, seg, tok0, n_tiles, splits = self._attention_plan(batch, heads // kv_heads, kv_heads, dim)
            reach = min(x for x in (batch.max_context, view.chunk, view.window) if x)
            splits = max(1, min(splits, reach // 256))
            partial_o = partial_ml = None
            if splits > 1:
                partial_o = torch.empty(tokens * heads * splits * dim, dtype=torch.float32, device=self.device)
                partial_ml = torch.empty(tokens * heads * splits * 2, dtype=torch.float32, device=self.device)
            self._check(self.lib.ttb_paged_attention_mma_bias(
                self._p(qkv), qkv.stride(0), self._p(out), self._p(batch.cu_seqlens), self._p(batch.seg_pos0),
                self._p(view.keys), self._p(view.values), self._p(view.block_table), view.block_table.shape[1],
                view.page_size, self._p(seg), self._p(tok0), n_tiles, tokens, heads, kv_heads, dim, ctypes.c_float(scale),
                int(view.window or 0), 1 if decode_shape else 0, splits, self._p(partial_o), self._p(partial_ml),
                view.keys.shape[0], self._p(self.status), ctypes.c_float(softcap or 0.0), int(view.chunk or 0),
                self._p(sinks), self._p(distance_bias), distance_bias.shape[1] - 1 if distance_bias is not None else 0,
                self._stream()), "sink_attention_mma")
            if splits > 1:
                self.launches += 1
            return out
        self._check(self.lib.ttb_paged_attention_generic_bias(
            self._p(qkv), qkv.stride(0), self._p(out), _dtype_code(qkv.dtype), self._p(batch.positions),
            self._p(batch.seg_of_token), self._p(view.keys), self._p(view.values), self._p(view.block_table),
            view.block_table.shape[1], view.page_size, tokens, heads, kv_heads, dim, ctypes.c_float(scale),
            int(view.window or 0), view.keys.shape[0], self._p(self.status), vdim, ctypes.c_float(softcap or 0.0),
            int(view.chunk or 0), self._p(sinks), self._p(distance_bias),
            distance_bias.shape[1] - 1 if distance_bias is not None else 0, self._stream()), "sink_attention")
        return out

    # ------------------------------------------------------------------ token shift, low-rank maps, matrix states
    def token_shift(self, x, mu, batch, view):
        """The mixes of every token with the token before it: out[t, s] = x[t] + (before[t] - x[t]) * mu[s], mu float32
        [mixes, width]; before a segment's first token stands the request's kept input (view.tail), which the walk
        refreshes afterwards. -> [T, mixes, width] in x's dtype."""
        T, width = x.shape
        if x.stride(1) != 1 or mu.dtype != torch.float32 or mu.shape[1] != width or not mu.is_contiguous():
            raise KernelError("token_shift: contiguous columns, and float32 mixing weights [mixes, width]")
        if view.tail.dtype != x.dtype or not view.tail.is_contiguous() or tuple(view.tail.shape[1:]) != (1, width):
            raise KernelError("token_shift: one kept input of the model's width per request, of the compute dtype")
        out = torch.empty(T, mu.shape[0], width, dtype=x.dtype, device=self.device)
        self._check(self.lib.ttb_token_shift(self._p(x), _dtype_code(x.dtype), x.stride(0), self._p(mu), mu.shape[0],
                                             self._p(batch.seg_of_token), self._p(batch.cu_seqlens), self._p(view.slots),
                                             self._p(view.tail), self._p(out), T, width, self._stream()), "token_shift")
        return out

    _LOWRANK_OUT = {"none": 0, "neg_exp": 1, "neg_rate_softplus": 2}

    def lowrank_expand(self, x, w, bias, in_act, out_kind, rate=None):
        """The second half of a low-rank map, in float32 arithmetic: f(act(x) W^T + bias). x float32 [T, rank] (a slice
        of a wider product); W [N, rank] of the compute dtype; bias float32 [N] or None. in_act None or "tanh"; out_kind
        "none", "neg_exp" (-exp(z)) or "neg_rate_softplus" (-rate[head] * softplus(z), rate float32 [heads], N = heads *
        per_head). -> float32 [T, N]."""
        T, rank = x.shape
        N = w.shape[0]
        if x.dtype != torch.float32 or x.stride(1) != 1 or w.shape[1] != rank or not w.is_contiguous():
            raise KernelError("lowrank_expand: float32 input contiguous along its columns, and W [N, rank]")
        if in_act not in (None, "tanh") or out_kind not in self._LOWRANK_OUT:
            raise KernelError(f"lowrank_expand: in_act {in_act!r} or out_kind {out_kind!r} is not known")
        out = torch.empty(T, N, dtype=torch.float32, device=self.device)
        self._check(self.lib.ttb_lowrank_expand(
            self._p(x), x.stride(0), self._p(w), _dtype_code(w.dtype), self._p(bias), self._p(rate),
            rate.shape[0] if rate is not None else 1, 1 if in_act == "tanh" else 0, self._LOWRANK_OUT[out_kind], self._p(out),
            T, N, rank, self._stream()), "lowrank_expand")
        return out

    MATRIX_STATE_PART = 64                  # tokens of one part of a long segment in the matrix-state walks
    MATRIX_STATE_PARTS_FROM = 256           # segments from this many tokens on run as parts side by side
    MATRIX_STATE_SCRATCH_BYTES = 512 << 20  # most memory for the parts' states; longer parts beyond it

    def _matrix_state_parts(self, batch, heads, rows, cols, cols_end):
        """How a step's long segments are cut into parts: (parts, part_len, end states, start states) with scratch
        tensors, or (1, 0, None, None) for steps whose segments are walked whole."""
        if batch.max_seg_len < self.MATRIX_STATE_PARTS_FROM:
            return 1, 0, None, None
        part_len = self.MATRIX_STATE_PART
        per_part = batch.num_segments * heads * rows * (cols + cols_end) * 4
        while -(-batch.max_seg_len // part_len) * per_part > self.MATRIX_STATE_SCRATCH_BYTES and part_len < batch.max_seg_len:
            part_len *= 2
        parts = -(-batch.max_seg_len // part_len)
        if parts < 2:
            return 1, 0, None, None
        ends = torch.empty(batch.num_segments * heads * parts * rows * cols_end, dtype=torch.float32, device=self.device)
        starts = torch.empty(batch.num_segments * heads * parts * rows * cols, dtype=torch.float32, device=self.device)
        self.launches += 2
        return parts, part_len, ends, starts

    def shifted_state(self, rkvg, log_decay, bonus, norm_w, eps, heads, dim, x, batch, view, write_state=True):
        """rkvg [T, 4, heads * dim] (r, k, v and the gate before its silu; any token stride), or those four as separate
        tensors [T, heads * dim] with one row stride; log_decay float32 [T, heads * dim]
        (ln w, never positive); per head o = (S + diag(bonus) k v^T)^T r, S = diag(w) S + k v^T on the float32 state of
        view.state; then o / rms(o) per head, times norm_w, times silu(gate) -> [T, heads * dim]. Leaves the state and the
        request's last input (x's last row of the segment) in the request's slot."""
        inner = heads * dim
        four = [rkvg[:, i] for i in range(4)] if torch.is_tensor(rkvg) else list(rkvg)
        T, dtype, ld = four[0].shape[0], four[0].dtype, four[0].stride(0)
        if (len(four) != 4 or any(t.shape != (T, inner) or t.stride(1) != 1 or t.stride(0) != ld or t.dtype != dtype for t in four)
                or log_decay.dtype != torch.float32 or not log_decay.is_contiguous()):
            raise KernelError("shifted_state: r, k, v and the gate [T, heads * dim] with one row stride, float32 decays")
        if (view.state.dtype != torch.float32 or tuple(view.state.shape[1:]) != (heads, dim, dim) or not view.state.is_contiguous()
                or view.tail.dtype != x.dtype or not view.tail.is_contiguous() or x.dtype != dtype or x.stride(1) != 1):
            raise KernelError("shifted_state: the state must be float32 [slots, heads, dim, dim], the kept input of the compute dtype")
        out = torch.empty(T, inner, dtype=dtype, device=self.device)
        parts, part_len, ends, starts = self._matrix_state_parts(batch, heads, dim, dim, dim)
        logs = torch.empty(batch.num_segments * heads * parts * dim, dtype=torch.float32, device=self.device) if parts > 1 else None
        self._check(self.lib.ttb_shifted_state(
            self._p(four[0]), self._p(four[1]), self._p(four[2]), self._p(four[3]), _dtype_code(dtype), ctypes.c_longlong(ld),
            self._p(log_decay), self._p(bonus), self._p(norm_w), ctypes.c_float(eps), self._p(x), ctypes.c_longlong(x.stride(0)),
            x.shape[1], self._p(batch.cu_seqlens), self._p(view.slots), self._p(view.state), self._p(view.tail), self._p(out),
            batch.num_segments, heads, dim, 1 if write_state else 0, parts, part_len, self._p(ends), self._p(starts),
            self._p(logs), self._stream()), "shifted_state")
        return out

    def short_conv_silu(self, x, conv_w, batch, view):
        """silu of a causal convolution per channel without a bias: sum_j conv_w[:, j] * x[t - taps + 1 + j], reading the
        request's kept inputs (view.tail) before the step's first token; they are refreshed by the mixer's walk. x [T, channels]."""
        T, C = x.shape
        taps = conv_w.shape[1]
        if x.stride(1) != 1 or conv_w.dtype != torch.float32 or conv_w.shape[0] != C or not conv_w.is_contiguous():
            raise KernelError("short_conv_silu: contiguous columns, float32 taps [channels, taps]")
        if view.tail.dtype != x.dtype or not view.tail.is_contiguous() or view.tail.shape[2] != C:
            raise KernelError("short_conv_silu: kept inputs of the compute dtype over the same channels")
        zeros = getattr(self, "_conv_zero_bias", None)
        if zeros is None or zeros.numel() < C:
            zeros = torch.zeros(max(C, 1 << 14), dtype=torch.float32, device=self.device)
            self._conv_zero_bias = zeros
        u = torch.empty(T, C, dtype=x.dtype, device=self.device)
        self._check(self.lib.ttb_conv_silu(self._p(x), _dtype_code(x.dtype), x.stride(0), self._p(conv_w), self._p(zeros),
                                           self._p(batch.seg_of_token), self._p(batch.cu_seqlens), self._p(view.slots),
                                           self._p(view.tail), self._p(u), T, C, taps, self._stream()), "short_conv_silu")
        return u

    def delta_rule(self, u, raw, beta, log_decay, gate, norm_w, eps, heads, kv_heads, dim, vdim, batch, view, write_state=True):
        """u [T, q | k | v] behind the convolutions (q, k: kv_heads * dim; v: heads * vdim), raw their inputs; beta float32
        logits [T, heads] (a slice); log_decay float32 [T, heads * dim] (ln g); gate float32 logits [T, heads * vdim]. Per head,
        with q and k made unit vectors (q also times dim^-1/2): S = diag(g) S; d = sigmoid(beta) (v - S^T k); S += k d^T;
        o = S^T q; then o / rms(o), times norm_w [vdim], times sigmoid(gate) -> [T, heads * vdim]. Leaves the state and the
        convolutions' last inputs in the request's slot."""
        T, C = u.shape
        if C != 2 * kv_heads * dim + heads * vdim or raw.shape != u.shape or u.stride(1) != 1 or raw.stride(1) != 1 or raw.dtype != u.dtype:
            raise KernelError("delta_rule: u and raw must be [T, 2 kv_heads dim + heads vdim], contiguous along their columns")
        if (beta.dtype != torch.float32 or beta.shape != (T, heads) or beta.stride(1) != 1 or log_decay.dtype != torch.float32
                or not log_decay.is_contiguous() or gate.dtype != torch.float32 or not gate.is_contiguous()):
            raise KernelError("delta_rule: float32 beta logits, decays and gate logits")
        if (view.state.dtype != torch.float32 or tuple(view.state.shape[1:]) != (heads, dim, vdim) or not view.state.is_contiguous()
                or view.tail.dtype != u.dtype or not view.tail.is_contiguous() or view.tail.shape[2] != C):
            raise KernelError("delta_rule: the state must be float32 [slots, heads, dim, vdim], the kept inputs of the compute dtype")
        out = torch.empty(T, heads * vdim, dtype=u.dtype, device=self.device)
        parts, part_len, ends, starts = self._matrix_state_parts(batch, heads, dim, vdim, vdim + dim)
        self._check(self.lib.ttb_delta_rule(
            self._p(u), _dtype_code(u.dtype), ctypes.c_longlong(u.stride(0)), self._p(raw), ctypes.c_longlong(raw.stride(0)),
            self._p(beta), beta.stride(0), self._p(log_decay), self._p(gate), self._p(norm_w), ctypes.c_float(eps),
            self._p(batch.cu_seqlens), self._p(view.slots), self._p(view.state), self._p(view.tail), self._p(out),
            batch.num_segments, heads, kv_heads, dim, vdim, view.taps, 1 if write_state else 0, parts, part_len,
            self._p(ends), self._p(starts), self._stream()), "delta_rule")
        return out

    # ------------------------------------------------------------------ experts chosen from the best groups
    def route_grouped(self, x, w_router, experts, top, groups, keep, floor):
        """Float32 router over all experts' softmax scores, restricted to the `keep` best of `groups` groups:
        -> (int32 [T, top], float32 [T, top] = chosen scores / (their sum + floor))."""
        T, width = x.shape
        if w_router.dtype != torch.float32 or w_router.shape != (experts, width) or x.stride(1) != 1 or not w_router.is_contiguous():
            raise KernelError("route_grouped: the router's matrix must be float32 [experts, width]")
        choice = torch.empty(T, top, dtype=torch.int32, device=self.device)
        weight = torch.empty(T, top, dtype=torch.float32, device=self.device)
        self._check(self.lib.ttb_route_grouped(self._p(x), _dtype_code(x.dtype), x.stride(0), self._p(w_router), T, width,
                                               experts, top, groups, keep, ctypes.c_float(floor), self._p(choice),
                                               self._p(weight), self._stream()), "route_grouped")
        return choice, weight

    def plain_experts(self, x, choice, weight, w_up, w_down, activation="relu2"):
        """x [T, width]; choice, weight [T, top]; w_up [E, inter, width]; w_down [E, width, inter] -> float32 [T, width]:
        sum_j weight[t, j] * W_down,e act(W_up,e x[t]), e = choice[t, j], summed in the order of j."""
        T, width = x.shape
        E, inter, _ = w_up.shape
        top = choice.shape[1]
        pairs = T * top
        if x.dtype != w_up.dtype or x.stride(1) != 1 or not w_up.is_contiguous() or not w_down.is_contiguous():
            raise KernelError("plain_experts: operands must share a dtype and be contiguous")
        if activation != "relu2":
            raise KernelError("plain_experts: relu2 is the activation that is built")
        out = torch.empty(T, width, dtype=torch.float32, device=self.device)
        code = _dtype_code(x.dtype)
        if pairs <= self.MOE_GEMV_PAIRS and width * 4 <= 48 * 1024 and top * inter * 4 <= 48 * 1024:
            hidden = torch.empty(pairs, inter, dtype=x.dtype, device=self.device)
            self._check(self.lib.ttb_moe_gemv_plain(
                self._p(x), x.stride(0), self._p(w_up), self._p(w_down), self._p(choice), self._p(weight), self._p(hidden),
                self._p(out), code, T, E, top, inter, width, self._stream()), "moe_gemv_plain")
            self.launches += 1
            return out
        # many pairs: the tokens' rows are laid out expert by expert; the first product leaves the activated hidden rows
        # in that order (on the fifth-generation tensor cores in its epilogue; on the other paths as float32 rows,
        # written through the index 0, 1, 2, ..., that an activation kernel rounds to the compute dtype), the second
        # product scatters to the pairs' own rows
        offsets = torch.empty(E + 1, dtype=torch.int32, device=self.device)
        order = torch.empty(pairs, dtype=torch.int32, device=self.device)
        tokens_of = torch.empty(pairs, dtype=torch.int32, device=self.device)
        pair_out = torch.empty(pairs, width, dtype=torch.float32, device=self.device)
        grouped_tc = (x.dtype == torch.bfloat16 and self.use_tcgen05 is not False and pairs >= self.MOE_TCGEN05_PAIRS
                      and width % 8 == 0 and inter % 8 == 0)
        if grouped_tc:
            max_tiles = -(-pairs // 128) + E
            tile_info = torch.empty(2 * max_tiles + 1, dtype=torch.int32, device=self.device)
            self._check(self.lib.ttb_moe_align(self._p(choice), pairs, E, top, self._p(offsets), self._p(order),
                                               self._p(tokens_of), self._p(tile_info[1:]), self._p(tile_info), 128,
                                               self._stream()), "moe_align")
            grouped = self.gather_rows(x, tokens_of)
            hidden = torch.empty(pairs, inter, dtype=x.dtype, device=self.device)      # the activation in the product's epilogue
            self._check(self.lib.ttb_moe_gemm_tcgen05(
                self._p(grouped), width, self._p(w_up), width, self._p(hidden), inter, 2, self._p(offsets), self._p(order),
                self._p(tile_info[1:]), self._p(tile_info), pairs, E, max_tiles, inter, width, ctypes.c_float(0.0),
                ctypes.c_float(0.0), self._p(self.tc_error), self._stream()), "moe_up_tcgen05")
            self._check(self.lib.ttb_moe_gemm_tcgen05(
                self._p(hidden), inter, self._p(w_down), inter, self._p(pair_out), width, 0, self._p(offsets), self._p(order),
                self._p(tile_info[1:]), self._p(tile_info), pairs, E, max_tiles, width, inter, ctypes.c_float(0.0),
                ctypes.c_float(0.0), self._p(self.tc_error), self._stream()), "moe_down_tcgen05")
        else:
            self._check(self.lib.ttb_moe_align(self._p(choice), pairs, E, top, self._p(offsets), self._p(order),
                                               self._p(tokens_of), None, None, 0, self._stream()), "moe_align")
            grouped = self.gather_rows(x, tokens_of)
            straight = self._iota(pairs)
            pre = torch.empty(pairs, inter, dtype=torch.float32, device=self.device)
            self._check(self.lib.ttb_moe_group_gemm(
                self._p(grouped), grouped.stride(0), self._p(w_up), ctypes.c_longlong(inter * width), width, self._p(pre), inter,
                code, 0, self._p(offsets), self._p(straight), pairs, E, top, inter, width, ctypes.c_float(0.0),
                ctypes.c_float(0.0), self._stream()), "moe_up")
            hidden = self.activation(pre, activation, x.dtype)
            self._check(self.lib.ttb_moe_group_gemm(
                self._p(hidden), inter, self._p(w_down), ctypes.c_longlong(width * inter), inter, self._p(pair_out), width,
                code, 0, self._p(offsets), self._p(order), pairs, E, top, width, inter, ctypes.c_float(0.0),
                ctypes.c_float(0.0), self._stream()), "moe_down")
        self._check(self.lib.ttb_moe_combine(self._p(pair_out), self._p(weight), top, None, 0, None, self._p(out), T, width,
                                             self._stream()), "moe_combine")
        return out

    # ------------------------------------------------------------------ Dynamic Tanh around sub-layers, pass mixing
    def add_dyntanh(self, residual, delta, after, mult, norm, out_dtype):
        """residual += mult * (after(delta) if after else delta), in place and in float32; then norm(residual) in
        out_dtype (None when norm is None). `after` and `norm` are Dynamic Tanh parts (weight, bias, alpha):
        tanh(alpha x) * weight + bias."""
        rows, width = residual.shape
        if residual.dtype != torch.float32 or not residual.is_contiguous():
            raise KernelError("the residual stream is float32 and contiguous")
        if delta is not None and (delta.shape != residual.shape or delta.stride(1) != 1):
            raise KernelError("add_dyntanh: delta must have the residual's shape")
        out = torch.empty(rows, width, dtype=out_dtype, device=self.device) if norm is not None else None
        self._check(self.lib.ttb_add_dyntanh(
            self._p(residual), self._p(delta), _dtype_code(delta.dtype) if delta is not None else 0,
            delta.stride(0) if delta is not None else 0,
            self._p(after.weight if after is not None else None), self._p(after.bias if after is not None else None),
            ctypes.c_float(after.alpha if after is not None else 0.0), ctypes.c_float(mult),
            self._p(norm.weight if norm is not None else None), self._p(norm.bias if norm is not None else None),
            ctypes.c_float(norm.alpha if norm is not None else 0.0), self._p(out),
            _dtype_code(out_dtype) if norm is not None else 0, rows, width, self._stream()), "add_dyntanh")
        return out

    def concat_cast(self, a, b, out_dtype):
        """[a | b] row by row for two float32 [rows, width] tensors -> [rows, 2 width] in out_dtype."""
        rows, width = a.shape
        if a.dtype != torch.float32 or b.dtype != torch.float32 or a.shape != b.shape or not a.is_contiguous() or not b.is_contiguous():
            raise KernelError("concat_cast: two contiguous float32 tensors of one shape")
        out = torch.empty(rows, 2 * width, dtype=out_dtype, device=self.device)
        self._check(self.lib.ttb_concat_cast(self._p(a), self._p(b), self._p(out), _dtype_code(out_dtype), rows, width,
                                             self._stream()), "concat_cast")
        return out

    # ------------------------------------------------------------------ experts whose weight multiplies their input
    def input_weighted_experts(self, x, choice, weight, w_gate_up, w_down):
        """x [T, width]; choice, weight [T, top]; w_gate_up [E, 2 inter, width]; w_down [E, width, inter] -> float32
        [T, width]: sum_j expert_e(weight[t, j] * x[t]), e = choice[t, j], expert(u) = W_down (silu(W_gate u) * (W_up u)),
        summed in the order of j. The weighted input is rounded to the compute dtype like any stored row."""
        T, width = x.shape
        E, two_inter, _ = w_gate_up.shape
        inter, top = two_inter // 2, choice.shape[1]
        pairs = T * top
        if x.dtype != w_gate_up.dtype or x.stride(1) != 1 or not w_gate_up.is_contiguous() or not w_down.is_contiguous():
            raise KernelError("input_weighted_experts: operands must share a dtype and be contiguous")
        if weight.dtype != torch.float32 or not weight.is_contiguous() or not choice.is_contiguous():
            raise KernelError("input_weighted_experts: contiguous choices and float32 weights")
        out = torch.empty(T, width, dtype=torch.float32, device=self.device)
        hidden = torch.empty(pairs, inter, dtype=x.dtype, device=self.device)
        code = _dtype_code(x.dtype)
        no_limit, alpha = ctypes.c_float(0.0), ctypes.c_float(1.0)       # the plain gated unit silu(g) * u
        if pairs <= self.MOE_GEMV_PAIRS and width * 4 <= 48 * 1024 and top * inter * 4 <= 48 * 1024:
            # a handful of pairs (decode): every pair streams its expert's rows; the second kernel sums a token's pairs
            self._check(self.lib.ttb_moe_gemv_scaled(
                self._p(x), x.stride(0), self._p(w_gate_up), self._p(w_down), self._p(choice), self._p(weight),
                self._p(hidden), self._p(out), code, T, E, top, inter, width, no_limit, alpha, self._stream()), "moe_gemv_scaled")
            self.launches += 1
            return out
        offsets = torch.empty(E + 1, dtype=torch.int32, device=self.device)
        order = torch.empty(pairs, dtype=torch.int32, device=self.device)
        tokens_of = torch.empty(pairs, dtype=torch.int32, device=self.device)
        pair_out = torch.empty(pairs, width, dtype=torch.float32, device=self.device)
        grouped = torch.empty(pairs, width, dtype=x.dtype, device=self.device)
        grouped_tc = (x.dtype == torch.bfloat16 and self.use_tcgen05 is not False and pairs >= self.MOE_TCGEN05_PAIRS
                      and width % 8 == 0 and inter % 8 == 0)
        max_tiles = -(-pairs // 128) + E
        tile_info = torch.empty(2 * max_tiles + 1, dtype=torch.int32, device=self.device) if grouped_tc else None
        self._check(self.lib.ttb_moe_align(self._p(choice), pairs, E, top, self._p(offsets), self._p(order),
                                           self._p(tokens_of), self._p(tile_info[1:] if grouped_tc else None),
                                           self._p(tile_info), 128 if grouped_tc else 0, self._stream()), "moe_align")
        # the tokens' rows in the grouped order, each times its pair's weight
        self._check(self.lib.ttb_gather_rows_scaled(self._p(x), code, x.stride(0), self._p(tokens_of), self._p(order),
                                                    self._p(weight), self._p(grouped), pairs, width, self._stream()),
                    "gather_rows_scaled")
        if grouped_tc:
            self._check(self.lib.ttb_moe_gemm_tcgen05(
                self._p(grouped), width, self._p(w_gate_up), width, self._p(hidden), inter, 1, self._p(offsets),
                self._p(order), self._p(tile_info[1:]), self._p(tile_info), pairs, E, max_tiles, inter, width,
                no_limit, alpha, self._p(self.tc_error), self._stream()), "moe_gate_up_tcgen05")
            self._check(self.lib.ttb_moe_gemm_tcgen05(
                self._p(hidden), inter, self._p(w_down), inter, self._p(pair_out), width, 0, self._p(offsets),
                self._p(order), self._p(tile_info[1:]), self._p(tile_info), pairs, E, max_tiles, width, inter,
                no_limit, alpha, self._p(self.tc_error), self._stream()), "moe_down_tcgen05")
        else:
            straight = self._iota(pairs)          # the gathered rows are in the grouped order already
            self._check(self.lib.ttb_moe_group_gemm(
                self._p(grouped), width, self._p(w_gate_up), ctypes.c_longlong(two_inter * width), width, self._p(hidden), inter,
                code, 1, self._p(offsets), self._p(straight), pairs, E, 1, inter, width, no_limit, alpha, self._stream()),
                "moe_gate_up")
            self._check(self.lib.ttb_moe_group_gemm(
                self._p(hidden), inter, self._p(w_down), ctypes.c_longlong(width * inter), inter, self._p(pair_out), width,
                code, 0, self._p(offsets), self._p(order), pairs, E, top, width, inter, no_limit, alpha, self._stream()),
                "moe_down")
        self._check(self.lib.ttb_moe_combine(self._p(pair_out), None, top, None, 0, None, self._p(out), T, width,
                                             self._stream()), "moe_combine")
        return out

    # ------------------------------------------------------------------ state-space mixer
    STATE_SPACE_PART = 64                   # tokens of one part of a long segment in the state-space recurrence
    STATE_SPACE_SCRATCH_BYTES = 256 << 20   # most memory for the parts' states; longer parts beyond it

    def state_space(self, proj, conv_w, conv_b, dt_bias, rate, skip, norm_w, eps, heads, vdim, state, groups, norm_groups,
                    batch, view, write_state=True):
        """proj [T, z | x B C | dt] (z, x: heads * vdim; B, C: groups * state; dt: heads) -> [T, heads * vdim]:
        u = silu(conv(x B C) + b) from the request's kept inputs on; dt = softplus(dt + dt_bias); per head
        S = exp(-rate dt) S + dt B x^T (float32 [state, vdim] in view.state), y = S^T C + skip x; then y * silu(z),
        RMS-normed in norm_groups equal parts, times norm_w. Leaves the state and the convolution's last inputs in the
        request's slot."""
        T = proj.shape[0]
        inner, GN = heads * vdim, groups * state
        C, taps = inner + 2 * GN, conv_w.shape[1]
        if proj.stride(1) != 1 or proj.shape[1] != 2 * inner + 2 * GN + heads:
            raise KernelError("state_space: the projection must hold z, x, B, C and dt, contiguous along its columns")
        if (view.state.dtype != torch.float32 or tuple(view.state.shape[1:]) != (heads, state, vdim)
                or not view.state.is_contiguous() or view.tail.dtype != proj.dtype or not view.tail.is_contiguous()
                or view.tail.shape[2] != C or conv_w.shape[0] != C):
            raise KernelError("state_space: the state must be float32 [slots, heads, state, vdim], the kept inputs of the compute dtype")
        if not self.lib.ttb_state_space_supports(vdim, state):
            raise KernelError(f"state_space: a state of {state} x {vdim} per head is more than the kernel holds")
        code = _dtype_code(proj.dtype)
        xin = proj[:, inner:inner + C]
        u = torch.empty(T, C, dtype=proj.dtype, device=self.device)
        self._check(self.lib.ttb_conv_silu(self._p(xin), code, proj.stride(0), self._p(conv_w), self._p(conv_b),
                                           self._p(batch.seg_of_token), self._p(batch.cu_seqlens), self._p(view.slots),
                                           self._p(view.tail), self._p(u), T, C, taps, self._stream()), "conv_silu")
        if (batch.max_seg_len == 1 and T == batch.num_segments and heads % norm_groups == 0 and vdim % 4 == 0 and vdim <= 1024
                and (vdim + 2 * state + 3 + min(256 // max(vdim // 4, 1), state) * vdim) * 4 <= 48 * 1024):
            # one token a segment: the walk, the gate and the group norm in one launch
            counter = getattr(self, "_ss_counter", None)
            if counter is None or counter.numel() < T * norm_groups:
                counter = torch.zeros(max(T * norm_groups, 1 << 14), dtype=torch.int32, device=self.device)
                self._ss_counter = counter                              # the kernel leaves it at zero
            gated = torch.empty(T, inner, dtype=torch.float32, device=self.device)
            partial = torch.empty(T, heads, dtype=torch.float32, device=self.device)
            out = torch.empty(T, inner, dtype=proj.dtype, device=self.device)
            self._check(self.lib.ttb_state_space_token(
                self._p(u), self._p(proj), code, proj.stride(0), inner, inner + C, self._p(dt_bias), self._p(rate), self._p(skip),
                self._p(batch.cu_seqlens), self._p(view.slots), self._p(view.state), self._p(view.tail), self._p(gated),
                self._p(norm_w), ctypes.c_float(eps), self._p(out), self._p(partial), self._p(counter), batch.num_segments, heads,
                vdim, state, groups, norm_groups, taps, 1 if write_state else 0, self._stream()), "state_space_token")
            return out
        # long segments run as parts side by side (three launches: the parts' end states from zero, their start states,
        # the walk that writes out)
        part_len, parts, part_state, part_log = self.STATE_SPACE_PART, 1, None, None
        if batch.max_seg_len >= 3 * part_len:
            per_part = batch.num_segments * heads * state * vdim * 4
            while -(-batch.max_seg_len // part_len) * per_part > self.STATE_SPACE_SCRATCH_BYTES and part_len < batch.max_seg_len:
                part_len *= 2
            parts = -(-batch.max_seg_len // part_len)
        if parts > 1:
            # the parts' end states and, behind them, room for their start states
            part_state = torch.empty(2 * batch.num_segments * heads * parts * state * vdim, dtype=torch.float32, device=self.device)
            part_log = torch.empty(batch.num_segments * heads * parts, dtype=torch.float32, device=self.device)
            self.launches += 2
        y = torch.empty(T, inner, dtype=torch.float32, device=self.device)
        self._check(self.lib.ttb_state_space_scan(
            self._p(u), self._p(proj), code, proj.stride(0), inner, inner + C, self._p(dt_bias), self._p(rate), self._p(skip),
            self._p(batch.cu_seqlens), self._p(view.slots), self._p(view.state), self._p(view.tail), self._p(y),
            batch.num_segments, heads, vdim, state, groups, taps, 1 if write_state else 0, self._p(part_state),
            self._p(part_log), parts, part_len, self._stream()), "state_space_scan")
        out = torch.empty(T, inner, dtype=proj.dtype, device=self.device)
        self._check(self.lib.ttb_gate_group_norm(self._p(y), self._p(proj), code, proj.stride(0), self._p(norm_w),
                                                 ctypes.c_float(eps), self._p(out), code, T, inner, norm_groups,
                                                 self._stream()), "gate_group_norm")
        return out

    def _iota(self, count):
        """0, 1, .. count-1 as int32 on the device; made once and sliced (steps of a captured size never grow it)."""
        have = getattr(self, "_iota_buffer", None)
        if have is None or have.numel() < count:
            have = torch.arange(max(count, 1 << 16), dtype=torch.int32, device=self.device)
            self._iota_buffer = have
        return have[:count]

    # ------------------------------------------------------------------ sampling
    def sample(self, logits, temperature=None, top_k=None, top_p=None, seeds=None, counters=None) -> torch.Tensor:
        """One token per row of float32 logits. temperature None: argmax everywhere."""
        rows, vocab = logits.shape
        if logits.dtype != torch.float32 or logits.stride(1) != 1:
            raise KernelError("sample: logits must be float32, contiguous along the vocabulary")
        out = torch.empty(rows, dtype=torch.int32, device=self.device)
        if temperature is None and rows <= 65535:
            # greedy everywhere: the vocabulary in slices over many blocks, then one warp per row
            scratch = torch.empty(int(self.lib.ttb_argmax_scratch_bytes(rows)), dtype=torch.uint8, device=self.device)
            self._check(self.lib.ttb_argmax(self._p(logits), logits.stride(0), rows, vocab, self._p(scratch),
                                            self._p(out), self._stream()), "argmax")
            self.launches += 1
            return out
        # rows with a top_k up to the kernel's candidate list: candidates per slice of the vocabulary, then per row
        scratch = None
        if temperature is not None and top_k is not None:
            scratch = torch.empty(int(self.lib.ttb_sample_scratch_bytes(rows)), dtype=torch.uint8, device=self.device)
        self._check(self.lib.ttb_sample(self._p(logits), logits.stride(0), rows, vocab, self._p(temperature),
                                        self._p(top_k), self._p(top_p), self._p(seeds), self._p(counters),
                                        self._p(out), self._p(scratch), self._stream()), "sample")
        if scratch is not None:
            self.launches += 2
        return out

    def uniform(self, seed: int, counter: int) -> float:
        """The number in [0, 1) that the sampler draws for (seed, counter); host copy of the device function."""
        return float(self.lib.ttb_sample_uniform(ctypes.c_longlong(seed), int(counter)))


_CACHE = {}


def load_kernels(device) -> CudaKernels:
    """The kernel table of `device`, built and loaded on first use."""
    device = torch.device(device)
    if device.type != "cuda":
        raise KernelError(f"this engine runs on CUDA devices only, not on {device}")
    key = str(device)
    if key not in _CACHE:
        _CACHE[key] = CudaKernels(device)
    return _CACHE[key]
