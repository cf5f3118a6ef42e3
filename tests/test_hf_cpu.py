"""The transformers attention registration (host side; no GPU needed)."""
import pytest
import torch


def test_register_and_refuse_cpu_tensors():
    transformers = pytest.importorskip("transformers")
    from bytes_b200 import hf_attention
    name = hf_attention.register()
    cfg = transformers.LlamaConfig(vocab_size=64, hidden_size=256, intermediate_size=256, num_hidden_layers=1,
                                   num_attention_heads=2, num_key_value_heads=1, head_dim=128,
                                   max_position_embeddings=64)
    model = transformers.LlamaForCausalLM(cfg).eval()
    model.set_attn_implementation(name)
    assert model.config._attn_implementation == name
    with pytest.raises(RuntimeError, match="CUDA"):
        model(torch.randint(0, 64, (1, 4)))
