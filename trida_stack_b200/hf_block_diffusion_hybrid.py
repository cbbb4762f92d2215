"""Compatibility import name for the hybrid two-stream model (the reference's
``train.hf_block_diffusion_hybrid``, deprecated there); use ``trida_stack_b200.models.hybrid``."""
import warnings

from .models.hybrid import HybridBlockDiffusionLM, doc_positions, doc_starts  # noqa: F401

HFBlockDiffusionHybrid = HybridBlockDiffusionLM
warnings.warn("trida_stack_b200.hf_block_diffusion_hybrid is a compatibility name; use trida_stack_b200.models",
              DeprecationWarning, stacklevel=2)
