"""Parts that layers are put together from, and the generic decoder that runs them."""

from . import (attention, block, corrected_experts, delta_rule, embedding, feed_forward, gated_recurrence, grouped_experts, latent_attention, lightning_attention,  # noqa: F401
               mixer_pair, norm, position, routed_experts, scored_experts, shifted_state, sink_attention, state_space, stream_step)  # noqa: F401  (they register themselves)
from .base import (Block, CacheRequest, FeedForward, LatentPages, LatentPagesView, PendingDelta, Mixer, Norm, OutputHead, PagedKV, PagedKVView, Part, PartSpec, PositionEncoding, Runtime,
                   SlotState, SlotStateView, StepBatch, TensorSpec, TokenEmbedding, build_part, register_part)
from .model import DecoderModel, LayerCall, LayerSpec, ModelSpec

__all__ = ["Block", "LatentPages", "LatentPagesView", "PendingDelta", "CacheRequest", "OutputHead", "TokenEmbedding", "FeedForward", "Mixer", "Norm", "PagedKV", "PagedKVView", "Part", "PartSpec", "PositionEncoding",
           "Runtime", "SlotState", "SlotStateView", "StepBatch", "TensorSpec", "build_part", "register_part",
           "DecoderModel", "LayerCall", "LayerSpec", "ModelSpec"]
