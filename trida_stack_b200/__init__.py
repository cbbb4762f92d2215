"""trida_stack_b200: a Blackwell-native (sm_100a) block-diffusion training and serving framework.

Subpackages: ``models`` (native Qwen3 / Qwen3.5 decoders, block-diffusion objectives, decision
head), ``ops`` (sm_100a CUDA kernels behind autograd functions, plus their PyTorch statements),
``parallel`` (sharded data parallel with fused peer-memory collectives), ``data`` (SFT / decision
data pipelines), ``serving`` (self-speculative engine and OpenAI-compatible server), ``utils``.
"""
__version__ = "0.1.0"
