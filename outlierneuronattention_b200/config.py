"""Layer configuration, field for field the reference's ``ModelConfig`` and
``InferenceConfig`` (src/config.py:5-42 of LotanGutman/OutlierNeuronAttention)."""
from dataclasses import dataclass
from typing import List, Tuple, Union


@dataclass
class ModelConfig:
    d_model: int = 384
    num_heads: int = 6
    num_layers: int = 6
    r: Union[int, List[int], Tuple[int, ...]] = 8
    block_size: int = 1024
    tokenizer_name: str = "gpt2"
    seed: int = 42
    chunk_size: int = 32
    device: str = "cuda"
    use_rope: bool = True
    mix_gate_bias_init: float = 0.0
    initializer_range: float = 0.02
    scale_residual_proj: bool = True
    mha_heads_for_width_split: int = 0
    fixed_blend_weight: bool = False
    pure_mha_low_rank_k: bool = False
    attention_scale: float = 1.0
    rope_base: float = 10000.0
    learnable_alpha: bool = False

    @property
    def d_head(self) -> int:
        return self.d_model // self.num_heads


@dataclass
class InferenceConfig:
    max_new_tokens: int = 100
    temperature: float = 0.8
    top_k: int = 50
    repetition_penalty: float = 1.15
    stream: bool = True
    seed: int = 42
