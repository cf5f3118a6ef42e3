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
"""
import torch

from . import _ops

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
