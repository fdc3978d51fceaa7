"""B200-native HOFA attention hot path (prefill + decode).

Drop-in for the Hybrid Outlier-Factorized Attention layer of
LotanGutman/OutlierNeuronAttention: the module
``HybridOutlierFactorizedAttention`` and the operators ``fused_hofa_decode``,
``chunk_gla_inlier_fwd`` and ``exact_attention_triton`` keep the reference's
names, signatures and cache layouts, and run hand-written sm_100a CUDA kernels
through the C ABI of ``libhofa_b200.so`` (include/hofa.h).  There is no CPU
fallback: the ops raise when the library is missing or a tensor is not on a
CUDA device.
"""
from .config import InferenceConfig, ModelConfig
from .modules import RotaryEmbedding, apply_rotary_pos_emb, rotate_half

__all__ = ["ModelConfig", "InferenceConfig", "RotaryEmbedding", "apply_rotary_pos_emb", "rotate_half",
           "HybridOutlierFactorizedAttention", "fused_hofa_decode", "fused_hofa_decode_step", "chunk_gla_inlier_fwd",
           "exact_attention_triton", "prep"]


def __getattr__(name):
    # the operator modules are imported lazily so that `import outlierneuronattention_b200`
    # works on machines without the built library (e.g. to read the config)
    if name == "HybridOutlierFactorizedAttention":
        from .layer import HybridOutlierFactorizedAttention
        return HybridOutlierFactorizedAttention
    if name == "fused_hofa_decode":
        from .hofa_decode import fused_hofa_decode
        return fused_hofa_decode
    if name == "fused_hofa_decode_step":
        from .hofa_decode import fused_hofa_decode_step
        return fused_hofa_decode_step
    if name == "chunk_gla_inlier_fwd":
        from .chunk_gla_inlier import chunk_gla_inlier_fwd
        return chunk_gla_inlier_fwd
    if name == "exact_attention_triton":
        from .exact_attention import exact_attention_triton
        return exact_attention_triton
    if name == "prep":
        from .prep import prep
        return prep
    raise AttributeError(name)
