"""glm53: a B200-native (sm_100a) serving engine for the GLM-5.3-Flash hybrid MoE architecture.

Layout:
  config.py        model / engine configuration (full architecture and the tiny CPU proxy)
  models/          fp32 CPU reference model (the oracle), random-init checkpoint writer, the GPU model runtime,
                   the block drafter
  ops/             Python bindings of the hand-written sm_100a CUDA kernels (csrc/), EXL3 codec
  parallel/        process groups, symmetric peer memory, NCCL baseline collectives and fused comm kernels
  engine/          paged fp8 KV, scheduler with chunked prefill, prefix cache, speculative decoding, CUDA graphs
  api/             OpenAI-compatible generate / serve entry points
  utils/           env flags, tracing, metrics, timing
"""

from .config import ModelConfig, full_config, tiny_config  # noqa: F401

__version__ = "0.1.0"
