"""A transformers Llama (random weights, bf16) decoding through the bytes_b200 attention.

Teacher-forced decode steps after a prefill: the logits of every step with the bytes_b200
attention implementation must match those with transformers' SDPA attention, and the
kernel path must have served each layer of each step.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _model(cuda):
    transformers = pytest.importorskip("transformers")
    cfg = transformers.LlamaConfig(vocab_size=512, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, head_dim=128,
                                   max_position_embeddings=1024)
    torch.manual_seed(0)
    return transformers.LlamaForCausalLM(cfg).to(device=cuda, dtype=torch.bfloat16).eval()


def _decode_logits(model, impl, prompt, forced):
    model.set_attn_implementation(impl)
    steps = []
    with torch.no_grad():
        out = model(prompt, use_cache=True)
        past = out.past_key_values
        for t in range(forced.shape[1]):
            out = model(forced[:, t:t + 1], past_key_values=past, use_cache=True)
            past = out.past_key_values
            steps.append(out.logits[:, -1].float())
    return torch.stack(steps)


def test_llama_decode_steps_match_sdpa(cuda):
    from bytes_b200 import hf_attention
    name = hf_attention.register()
    model = _model(cuda)
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, 512, (2, 300), generator=g).to(cuda)
    forced = torch.randint(0, 512, (2, 8), generator=g).to(cuda)
    ref = _decode_logits(model, "sdpa", prompt, forced)
    before = hf_attention.calls
    got = _decode_logits(model, name, prompt, forced)
    assert hf_attention.calls - before == 8 * 2  # every decode step of both layers on the kernel
    d = (got - ref).abs()
    scale = ref.abs().max().item()
    assert torch.isfinite(got).all()
    # bf16 model: attention outputs rounded to bf16 on both paths, two layers deep
    assert d.max().item() <= 2e-2 * max(scale, 1.0), (d.max().item(), scale)
    assert d.mean().item() <= 2e-3 * max(scale, 1.0), (d.mean().item(), scale)


def _decode_logits_kivi(model, impl, prompt, forced, bits):
    from bytes_b200 import hf_attention
    model.set_attn_implementation(impl)
    cache = hf_attention.KiviCache(model.config, bits=bits, residual=128, max_tokens=1024)
    steps = []
    with torch.no_grad():
        model(prompt, past_key_values=cache, use_cache=True)
        for t in range(forced.shape[1]):
            out = model(forced[:, t:t + 1], past_key_values=cache, use_cache=True)
            steps.append(out.logits[:, -1].float())
    return torch.stack(steps), cache


def _oracle_kivi_attention(module, query, key, value, attention_mask, dropout=0.0, scaling=None, **kwargs):
    """The same KIVI cache state attended by the CPU oracle (test checker only)."""
    import oracle
    from transformers.integrations.sdpa_attention import sdpa_attention_forward
    layer = getattr(key, "_bytes_kivi", None)
    if layer is not None and query.shape[2] == 1:
        kq, ks, km, vq, vs, vm = (t.cpu() for t in layer.packed_views())
        out = oracle.kivi_decode_attn(query.cpu(), kq, ks, km, key.cpu(), vq, vs, vm, value.cpu(), layer.bits)
        return out.to(query.device).transpose(1, 2), None
    return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout, scaling=scaling,
                                  **kwargs)


@pytest.mark.parametrize("bits", [2, 4])
def test_llama_kivi_cache_decode_matches_oracle(cuda, bits):
    """Prefill packs the prompt (300 tokens: 160 packed, 140 in the window), 40 decode steps
    cross one flush of 32 window tokens into the packed caches; every step of both layers
    runs kivi_decode_attn, and the logits match the oracle attending the same cache state."""
    from transformers import AttentionInterface
    from transformers.masking_utils import AttentionMaskInterface, sdpa_mask
    from bytes_b200 import hf_attention
    name = hf_attention.register()
    AttentionInterface.register("kivi_oracle", _oracle_kivi_attention)
    AttentionMaskInterface.register("kivi_oracle", sdpa_mask)
    model = _model(cuda)
    g = torch.Generator().manual_seed(2)
    prompt = torch.randint(0, 512, (2, 300), generator=g).to(cuda)
    forced = torch.randint(0, 512, (2, 40), generator=g).to(cuda)
    before = hf_attention.calls
    got, cache = _decode_logits_kivi(model, name, prompt, forced, bits)
    assert hf_attention.calls - before == 40 * 2
    assert cache.layers[0].n_packed == 192 and cache.layers[0].n_res == 148
    ref, _ = _decode_logits_kivi(model, "kivi_oracle", prompt, forced, bits)
    d = (got - ref).abs()
    scale = ref.abs().max().item()
    assert torch.isfinite(got).all()
    assert d.max().item() <= 2e-2 * max(scale, 1.0), (d.max().item(), scale)
    assert d.mean().item() <= 2e-3 * max(scale, 1.0), (d.mean().item(), scale)


def test_kivi_cache_reorder_follows_the_batch(cuda):
    """Beam-search reordering moves packed codes, scales, minima and window together: a
    reordered cache decodes exactly like the original one with the batch rows swapped."""
    from bytes_b200 import hf_attention
    name = hf_attention.register()
    model = _model(cuda)
    model.set_attn_implementation(name)
    g = torch.Generator().manual_seed(3)
    prompt = torch.randint(0, 512, (2, 260), generator=g).to(cuda)
    nxt = torch.randint(0, 512, (2, 1), generator=g).to(cuda)
    with torch.no_grad():
        a = hf_attention.KiviCache(model.config, bits=2, residual=128, max_tokens=512)
        model(prompt, past_key_values=a, use_cache=True)
        la = model(nxt, past_key_values=a, use_cache=True).logits[:, -1].float()
        b = hf_attention.KiviCache(model.config, bits=2, residual=128, max_tokens=512)
        model(prompt, past_key_values=b, use_cache=True)
        b.reorder_cache(torch.tensor([1, 0], device=cuda))
        lb = model(nxt.flip(0), past_key_values=b, use_cache=True).logits[:, -1].float()
    d = (la - lb.flip(0)).abs().max().item()
    assert d <= 1e-3 * max(la.abs().max().item(), 1.0), d
