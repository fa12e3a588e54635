"""Sparse-MoE serving engine (Qwen3-MoE / Kimi-K2 shapes).

The B200 counterpart of the reference's sparse-MoE engines
(crates/cascadia-engine-sparse-moe/src/engine.rs, glm/model.rs): the same
continuous-batching ``LLMEngine`` drives a :class:`~cascadia_b200.models.moe.MoEModel`
whose FFN is the routed-expert block (fused router/top-k kernel, counting-sort
permute, grouped INT4 expert GEMMs, weighted combine).  Everything above the
model (scheduler, paged KV, CUDA-graph decode, sampling, chunk protocol) is
shared with the dense engine.
"""
from __future__ import annotations

from .llm import LLMBuilder


class MoEBuilder(LLMBuilder):
    """LLMBuilder that always builds the MoE model (rejects dense presets)."""

    def model_class(self, cfg):
        from .base import InvalidConfig

        if not cfg.is_moe:
            raise InvalidConfig(f"{self.model_name}: not a sparse-MoE config")
        return super().model_class(cfg)
