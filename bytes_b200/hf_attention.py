"""Decode-time attention for Hugging Face ``transformers`` models through the bytes_b200 kernels.

The reference evaluates its KV-cache methods by patching the attention forward of HF models
(benchmarks/eval_ppl.py:95-375). This module is the serving-side counterpart for the dense
path: ``register()`` adds an attention implementation to transformers' registry, and a model
loaded or switched with ``attn_implementation="bytes_b200"`` then runs every decode step
(one query token per sequence, no padding mask) of every layer on the split-KV bf16 / fp8
decode kernel over the layer's own KV cache. Prefill and masked (padded) batches are not
decode steps; they keep transformers' SDPA attention, the model's usual path.

    from bytes_b200 import hf_attention
    hf_attention.register()
    model.set_attn_implementation("bytes_b200")   # or from_pretrained(..., attn_implementation=...)

The mask function registered alongside is transformers' SDPA one, which drops the mask of a
pure causal pattern; a decode step with a mask left (padding) goes to SDPA.

``KiviCache`` keeps a model's KV cache in the KIVI form instead (2- or 4-bit packed codes
with fp16 scales and minima, plus a bf16 window of the newest tokens): the prompt is packed
at prefill, every 32 tokens that leave the window are appended to the packed caches in place
(``kivi_append``), and each decode step runs ``kivi_decode_attn`` over packed caches and
window. Prefill attention stays full precision (SDPA over the prompt).

    cache = hf_attention.KiviCache(model.config, bits=2, residual=128, max_tokens=4096)
    model(prompt, past_key_values=cache, use_cache=True)        # then decode steps as usual
"""
import functools

import torch

from . import _ops
from . import kivi as _kivi

NAME = "bytes_b200"

# decode steps served by the kernel since import (tests read it to see the path was taken)
calls = 0


def _kernel_ok(query, key, value, attention_mask):
    return (query.dim() == 4 and query.shape[2] == 1 and attention_mask is None
            and key.dtype == value.dtype and key.dtype in (torch.bfloat16, torch.float8_e4m3fn)
            and query.shape[-1] in (64, 128) and query.shape[1] % key.shape[1] == 0)


def attention_forward(module, query, key, value, attention_mask, dropout=0.0, scaling=None, **kwargs):
    """transformers attention interface: query [B,H_q,q_len,D], key/value [B,H_k,S,D] (the
    cache, GQA not expanded) -> (output [B,q_len,H_q,D], None)."""
    global calls
    if not query.is_cuda:
        raise RuntimeError("bytes_b200 attention serves CUDA tensors only (there is no CPU path)")
    layer = getattr(key, "_bytes_kivi", None)
    if layer is not None and query.shape[2] == 1:
        if attention_mask is not None:
            raise ValueError("KiviCache decode steps take unpadded batches (no attention mask)")
        if scaling is not None and abs(float(scaling) - query.shape[-1] ** -0.5) > 1e-6:
            raise ValueError("KIVI decode applies softmax scaling 1/sqrt(head_dim)")
        kq, ks, km, vq, vs, vm = layer.packed_views()
        out = _kivi.kivi_decode_attn(query, kq, ks, km, key, vq, vs, vm, value, layer.bits)
        calls += 1
        return out.transpose(1, 2), None
    if _kernel_ok(query, key, value, attention_mask):
        q3 = query[:, :, 0, :]
        if key.dtype == torch.bfloat16 and q3.dtype != torch.bfloat16:
            q3 = q3.to(torch.bfloat16)
        out = torch.empty(q3.shape, dtype=query.dtype, device=query.device)
        scale = float(scaling) if scaling is not None else query.shape[-1] ** -0.5
        _ops.decode_attn(q3, key, value, scale, out)
        calls += 1
        return out.unsqueeze(1), None
    from transformers.integrations.sdpa_attention import sdpa_attention_forward
    return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout, scaling=scaling,
                                  **kwargs)


def register(name=NAME):
    """Add ``name`` to transformers' attention and attention-mask registries."""
    from transformers import AttentionInterface
    from transformers.masking_utils import AttentionMaskInterface, sdpa_mask
    AttentionInterface.register(name, attention_forward)
    AttentionMaskInterface.register(name, sdpa_mask)
    return name


@functools.lru_cache(maxsize=None)
def _kivi_layer_class():
    # built on first use, so importing this module does not import transformers
    from transformers.cache_utils import CacheLayerMixin

    class KiviLayer(CacheLayerMixin):
        """One layer's KIVI cache: packed codes for tokens [0, n_packed), the bf16 window
        for the newest n_res tokens (between residual and residual + 31 after prefill)."""

        is_sliding = False

        def __init__(self, bits=2, residual=128, max_tokens=4096):
            super().__init__()
            if bits not in (2, 4):
                raise ValueError("bits must be 2 or 4")
            self.bits, self.R = bits, int(residual)
            self.cap = (int(max_tokens) + 63) // 64 * 64
            self.cumulative_length = 0
            self.n_packed = 0
            self.n_res = 0

        def lazy_initialization(self, key_states, value_states):
            B, Hk, _, D = key_states.shape
            dev, fpi = key_states.device, 32 // self.bits
            self.dtype, self.device = key_states.dtype, dev
            i32, f16 = torch.int32, torch.float16
            self.Kq = torch.zeros(B, Hk, D, self.cap // fpi, dtype=i32, device=dev)
            self.Ks = torch.zeros(B, Hk, D, self.cap // 32, dtype=f16, device=dev)
            self.Km = torch.zeros_like(self.Ks)
            self.Vq = torch.zeros(B, Hk, self.cap, D // fpi, dtype=i32, device=dev)
            self.Vs = torch.zeros(B, Hk, self.cap, D // 32, dtype=f16, device=dev)
            self.Vm = torch.zeros_like(self.Vs)
            self.res_k = torch.zeros(B, Hk, self.R + 32, D, dtype=torch.bfloat16, device=dev)
            self.res_v = torch.zeros_like(self.res_k)
            self.keys, self.values = self.res_k, self.res_v
            self.is_initialized = True

        def packed_views(self):
            """(Kq, K_scale, K_mn, Vq, V_scale, V_mn) of the packed tokens, views into the
            capacity buffers (rows keep the buffer pitch)."""
            n, fpi = self.n_packed, 32 // self.bits
            return (self.Kq[..., :n // fpi], self.Ks[..., :n // 32], self.Km[..., :n // 32],
                    self.Vq[:, :, :n], self.Vs[:, :, :n], self.Vm[:, :, :n])

        def _flush(self, k, v):
            if self.n_packed + k.shape[2] > self.cap:
                raise ValueError("KiviCache: max_tokens exceeded")
            _kivi.kivi_append(k.to(torch.float16), v.to(torch.float16), self.bits, self.n_packed, self.Kq,
                              self.Ks, self.Km, self.Vq, self.Vs, self.Vm)
            self.n_packed += k.shape[2]

        def update(self, key_states, value_states, *args, **kwargs):
            if not self.is_initialized:
                self.lazy_initialization(key_states, value_states)
            T = key_states.shape[2]
            if T > 1:
                if self.cumulative_length:
                    raise ValueError("KiviCache: multi-token updates only as the first (prefill) update")
                self.cumulative_length = T
                n_flush = max(0, (T - self.R) // 32 * 32)
                if n_flush:
                    self._flush(key_states[:, :, :n_flush], value_states[:, :, :n_flush])
                self.n_res = T - n_flush
                self.res_k[:, :, :self.n_res] = key_states[:, :, n_flush:]
                self.res_v[:, :, :self.n_res] = value_states[:, :, n_flush:]
                return key_states, value_states  # prefill attends at full precision
            self.cumulative_length += 1
            self.res_k[:, :, self.n_res] = key_states[:, :, 0]
            self.res_v[:, :, self.n_res] = value_states[:, :, 0]
            self.n_res += 1
            if self.n_res == self.R + 32:  # the oldest 32 window tokens join the packed caches
                self._flush(self.res_k[:, :, :32], self.res_v[:, :, :32])
                self.res_k[:, :, :self.R] = self.res_k[:, :, 32:].clone()
                self.res_v[:, :, :self.R] = self.res_v[:, :, 32:].clone()
                self.n_res = self.R
            k, v = self.res_k[:, :, :self.n_res], self.res_v[:, :, :self.n_res]
            k._bytes_kivi = self
            return k, v

        def _batch_apply(self, fn):
            # every buffer has batch first: packed codes, scales, minima and the window
            for name in ("Kq", "Ks", "Km", "Vq", "Vs", "Vm", "res_k", "res_v"):
                setattr(self, name, fn(getattr(self, name)).contiguous())
            self.keys, self.values = self.res_k, self.res_v

        def reorder_cache(self, beam_idx):
            if self.is_initialized:
                self._batch_apply(lambda t: t.index_select(0, beam_idx.to(t.device)))

        def batch_repeat_interleave(self, repeats):
            if self.is_initialized:
                self._batch_apply(lambda t: t.repeat_interleave(repeats, dim=0))

        def batch_select_indices(self, indices):
            if self.is_initialized:
                self._batch_apply(lambda t: t[indices])

        def reset(self):
            # the base reset clears the window and the token count; the packed range and
            # the window length must restart too, or the next prompt would be appended after
            # (and attend over) the previous sequence's packed tokens
            super().reset()
            self.n_packed = 0
            self.n_res = 0
            if self.is_initialized:
                for name in ("Kq", "Ks", "Km", "Vq", "Vs", "Vm"):
                    getattr(self, name).zero_()

        def crop(self, max_length):
            raise NotImplementedError("KiviCache: packed tokens cannot be cropped")

        def get_mask_sizes(self, query_length):
            return self.cumulative_length + query_length, 0

        def get_seq_length(self):
            return self.cumulative_length

        def get_max_cache_shape(self):
            return -1

    return KiviLayer


def KiviCache(config, bits=2, residual=128, max_tokens=4096):
    """A transformers ``Cache`` whose layers hold KIVI-compressed keys and values (see the
    module docstring); decode steps need the "bytes_b200" attention implementation."""
    from transformers.cache_utils import Cache
    layer_cls = _kivi_layer_class()
    n = config.get_text_config(decoder=True).num_hidden_layers
    return Cache(layers=[layer_cls(bits, residual, max_tokens) for _ in range(n)])
