"""Hot ops: sm_100a CUDA kernels on GPU tensors, plain PyTorch statements on CPU tensors."""
from . import reference
from ._ext import available as extension_available
from .blocks import AttnContext, attn_block, embedding, mlp_block, rmsnorm, rope_tables
from .ce import fused_linear_ce

__all__ = ["reference", "extension_available", "AttnContext", "attn_block", "embedding", "mlp_block",
           "rmsnorm", "rope_tables", "fused_linear_ce"]
