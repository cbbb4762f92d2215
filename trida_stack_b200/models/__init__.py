"""Native decoders and training objectives."""
from .block_diffusion import BlockDiffusionLM, bucketed_clean_len
from .config import ModelConfig, qwen3_config
from .decoder import Decoder

__all__ = ["BlockDiffusionLM", "bucketed_clean_len", "ModelConfig", "qwen3_config", "Decoder"]
