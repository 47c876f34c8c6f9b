"""hllm_b200 -- a B200-native stage executor for hLLM.

The per-step hot path of one hLLM stage (ragged packing, paged-KV GQA
attention with RoPE and q/k-norm, RMSNorm, SwiGLU, tcgen05 projection GEMMs,
sampling) as hand-written sm_100a CUDA in libhllm_b200.so, behind the C ABI in
include/hllm_b200.h.  ``B200Stage`` mirrors hLLM's runtime::StageBackend.
"""
from .backend import (B200Stage, BoundaryActivation, DecodeBatchItem, ModelConfig,  # noqa: F401
                      PrefillProgress, SampledToken, SamplingOptions, SequenceState, StageError,
                      TokenInput)

__all__ = ["B200Stage", "BoundaryActivation", "DecodeBatchItem", "ModelConfig", "PrefillProgress",
           "SampledToken", "SamplingOptions", "SequenceState", "StageError", "TokenInput"]
