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


def test_kivi_cache_window_bookkeeping(monkeypatch):
    """Host logic of the KIVI cache layer, with the packing kernel replaced by a recorder:
    the prompt's oldest whole groups go to the packed caches, the window then fills to
    residual + 32 and flushes its oldest 32 tokens, in order."""
    pytest.importorskip("transformers")
    from bytes_b200 import hf_attention, kivi
    flushed = []
    monkeypatch.setattr(kivi, "kivi_append",
                        lambda k, v, bits, off, *caches: flushed.append((off, k[0, 0, :, 0].tolist())))

    class Cfg:
        def get_text_config(self, decoder=True):
            return self
        num_hidden_layers = 1

    layer = hf_attention.KiviCache(Cfg(), bits=2, residual=8, max_tokens=128).layers[0]
    tok = lambda t0, n: torch.arange(t0, t0 + n, dtype=torch.float32).view(1, 1, n, 1).expand(1, 1, n, 128)
    k, v = layer.update(tok(0, 45), tok(0, 45))  # prefill: 45 tokens, residual 8
    assert k.shape[2] == 45  # prefill attends at full precision
    assert flushed == [(0, [float(x) for x in range(32)])] and layer.n_packed == 32 and layer.n_res == 13
    for t in range(45, 72):  # window 14 .. 40 = residual + 32: flush at token 71
        k, v = layer.update(tok(t, 1), tok(t, 1))
    assert layer.cumulative_length == 72
    assert flushed[1] == (32, [float(x) for x in range(32, 64)])
    assert layer.n_packed == 64 and layer.n_res == 8
    assert k.shape[2] == 8 and k[0, 0, :, 0].tolist() == [float(x) for x in range(64, 72)]
    assert getattr(k, "_bytes_kivi", None) is layer


def test_kivi_cache_reset_restarts_packed_range(monkeypatch):
    """After Cache.reset() the next prompt packs from token 0 again: no packed tokens of the
    previous sequence stay visible to decode."""
    pytest.importorskip("transformers")
    from bytes_b200 import hf_attention, kivi
    flushed = []
    monkeypatch.setattr(kivi, "kivi_append", lambda k, v, bits, off, *caches: flushed.append((off, k.shape[2])))

    class Cfg:
        def get_text_config(self, decoder=True):
            return self
        num_hidden_layers = 1

    cache = hf_attention.KiviCache(Cfg(), bits=2, residual=8, max_tokens=256)
    layer = cache.layers[0]
    tok = lambda n: torch.ones(1, 1, n, 128)
    layer.update(tok(80), tok(80))  # 64 packed, 16 in the window
    for _ in range(30):  # the window reaches residual + 32 at the 24th step and flushes
        layer.update(tok(1), tok(1))
    assert layer.n_packed == 96 and layer.n_res == 14 and layer.cumulative_length == 110
    layer.Kq.fill_(7)
    cache.reset()
    assert layer.n_packed == 0 and layer.n_res == 0 and layer.cumulative_length == 0
    assert int(layer.Kq.abs().sum()) == 0 and layer.packed_views()[0].shape[-1] == 0
    flushed.clear()
    layer.update(tok(45), tok(45))  # a new prompt: its first 32 tokens pack at offset 0
    assert flushed == [(0, 32)] and layer.n_packed == 32 and layer.n_res == 13
