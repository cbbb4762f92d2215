"""Compatibility import name for the dense block-diffusion model (the reference's
``train.hf_block_diffusion``, deprecated there); use ``trida_stack_b200.models.block_diffusion``."""
import warnings

from .models.block_diffusion import BlockDiffusionLM, bucketed_clean_len  # noqa: F401

HFBlockDiffusion = BlockDiffusionLM
warnings.warn("trida_stack_b200.hf_block_diffusion is a compatibility name; use trida_stack_b200.models",
              DeprecationWarning, stacklevel=2)
