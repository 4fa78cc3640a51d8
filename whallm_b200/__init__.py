"""whallm_b200: B200-native routed-expert MoE path and quantized KV formats.

A drop-in for the hot path of baha2046/Whallm's MLX runtime: router top-k,
permute-by-expert, the fused MXFP4 / affine-4 SwiGLU expert FFN with the
top-k weighted combine, and the FP8/FP4 KV-cache row formats.  All arithmetic
runs in ``libwhallm_b200.so`` (hand-written sm_100a CUDA behind a C ABI,
``include/whallm_b200.h``); this package is the Python host side that keeps
the reference's call signatures.
"""
from . import _lib  # noqa: F401
from .experts import (Affine4BatchedExperts, BatchedExperts, ClampedSwiGLU, ExpertWeights,  # noqa: F401
                      QwenBatchedExperts, QwenExpertWeights, ResidentExpertStore, StreamingExperts,
                      StreamingSwitchGLU, experts_forward, permute)
from .formats import (affine4_dequantize, affine4_quantize, kv_dequantize, kv_gather_dequantize,  # noqa: F401
                      kv_quantize, kv_scores, mxfp4_dequantize, mxfp4_quantize, split_e4m3)
from .moe import MoE, SparseMoE, TinyMoE, moe_layer, route_reduce, streaming_moe  # noqa: F401
from .router import Gate, qwen_route, route, stable_topk_indices, topk_scores  # noqa: F401

from .linear import MXFP8Linear, expand_block_scales, mx_linear  # noqa: F401
from .loader import load_expert_layer, load_installed_experts, read_layout  # noqa: F401
from .kvcache import MXFP8PoolingCache, PackedRows, QSAQuantizedCache  # noqa: F401

__version__ = "0.1.0"
