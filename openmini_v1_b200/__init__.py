"""openmini_v1_b200: a B200-native LLM serving and RL framework.

Layers: ``ops`` (sm_100a kernels + fp32 oracle), ``models`` (decoder, MoE,
DSA, GGUF loading), ``engine`` (paged KV, continuous batching, CUDA graphs),
``parallel`` (process groups, NCCL baseline, fused NVLink kernels), ``serve``
(HTTP, gRPC, metrics, worker pool, gateway), ``rl`` / ``train`` (GRPO with
Keep-Routing and sampling-mask replay), ``config`` (server.toml semantics).
"""
__version__ = "0.1.0"
