"""Host-side checks of the decoder LM harness (no GPU)."""
import torch

from outlierneuronattention_b200.lm import HofaLM, LMConfig


def test_350m_shape_parameter_count():
    """24 layers, d_model 1024, 16 heads, MLP 4096, vocabulary 32000, tied
    embedding: 435.4M matrix parameters plus 0.2M of gates, norms and
    gla_scale (built on the meta device, no memory)."""
    with torch.device("meta"):
        m = HofaLM(LMConfig())
    n = m.num_parameters()
    assert abs(n - 435.6e6) < 0.1e6, n
    assert m.blocks[0].attn.r == 16 and m.blocks[0].attn.d_head == 64
