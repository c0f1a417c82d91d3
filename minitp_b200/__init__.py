"""minitp_b200: B200-native (sm_100a) tensor-parallel decode for Qwen2 models.

A drop-in for the mini-TP Python API (ColumnParallelLinear / RowParallelLinear,
VocabParallelEmbedding / VocabParallelLMHead, GenerationState,
generate_greedy, the sharded KV cache) whose hot path runs on hand-written
CUDA kernels (``minitp_b200/csrc``) behind the C ABI of
``libminitp_b200.so`` (``include/minitp_b200.h``).
"""

__version__ = "0.1.0"
