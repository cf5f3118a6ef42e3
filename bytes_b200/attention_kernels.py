"""Drop-in for ``src/attention_kernels.py`` of saifmb0/bytes, backed by sm_100a CUDA kernels.

Same function names, argument meaning and output shapes/dtypes as the reference
module; the ``BLOCK_*`` keyword arguments are accepted and ignored (the kernels
pick their own tiling). All inputs must be CUDA tensors; there is no CPU path.
"""
import math

import torch

from . import _ops


def _squeeze_q(q):
    if q.dim() != 4 or q.shape[2] != 1:
        raise ValueError("q must be [B, H_q, 1, D]")
    return q[:, :, 0, :]


def decode_attn_bf16(q, k, v):
    """softmax(q.k) . v per query head, GQA by h_q // (H_q/H_k); NO scale is applied.

    ref: src/attention_kernels.py:65-92. q [B,H_q,1,D]; k,v [B,H_k,S,D] bf16
    -> [B,H_q,1,D] in q.dtype. A non-bf16 query is rounded to bf16 for the
    tensor-core contraction.
    """
    q3 = _squeeze_q(q)
    if q3.dtype != torch.bfloat16:
        q3 = q3.to(torch.bfloat16)
    out = torch.empty(q3.shape, dtype=q.dtype, device=q.device)
    _ops.decode_attn(q3, k, v, 1.0, out)
    return out.unsqueeze(2)


def decode_attn_fp8(q, k, v):
    """decode_attn_bf16 over an fp8 e4m3 KV cache. ref: src/attention_kernels.py:156-182."""
    q3 = _squeeze_q(q)
    out = torch.empty(q3.shape, dtype=q.dtype, device=q.device)
    _ops.decode_attn(q3, k, v, 1.0, out)
    return out.unsqueeze(2)
