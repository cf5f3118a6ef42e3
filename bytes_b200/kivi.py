"""KIVI decode step, pack and GEMV, drop-in for the entry points used by
``benchmarks/kivi_latency.py`` of saifmb0/bytes (and the external KIVI package it wraps).
"""
import math

import torch

from . import _ops


def kivi_decode_attn(Q, Kq, K_scale, K_mn, K_residual, Vq, V_scale, V_mn, V_residual, bits, group_size=32):
    """One fused KIVI decode step: softmax(Q.[K;K_res]^T/sqrt(D)).[V;V_res].

    ref: benchmarks/kivi_latency.py:59-90 (kivi_decode_attn). Q [B,H_q,1,D];
    Kq int32 [B,H_k,D,Sq*bits/32]; K_scale/K_mn f16 [B,H_k,D,Sq/32];
    K_residual bf16 [B,H_k,R,D]; Vq int32 [B,H_k,Sq,D*bits/32];
    V_scale/V_mn f16 [B,H_k,Sq,D/32]; V_residual bf16 [B,H_k,R,D].
    Returns [B,H_q,1,D] in Q.dtype. Two launches: a split-KV kernel over the packed
    cache, then one over the residual window that also merges the split partials (the
    reference issues 6+ launches and materialises the scores).
    """
    if Q.is_cuda:
        rc, out = _ops.N.glue().kivi_decode_attn(Q, Kq, K_scale, K_mn, K_residual, Vq, V_scale, V_mn, V_residual,
                                                 int(bits), int(group_size))
        if rc == 0:
            return out
    if Q.dim() != 4 or Q.shape[2] != 1:
        raise ValueError("Q must be [B, H_q, 1, D]")
    Q3 = Q[:, :, 0, :]
    D = Q.shape[-1]
    if K_residual.dtype != torch.bfloat16:
        K_residual = K_residual.to(torch.bfloat16)
    if V_residual.dtype != torch.bfloat16:
        V_residual = V_residual.to(torch.bfloat16)
    if Q3.dtype != torch.bfloat16 and K_residual.shape[2] > 0:
        Q3 = Q3.to(torch.bfloat16)
    K_scale, K_mn, V_scale, V_mn = (t if t.dtype == torch.float16 else t.to(torch.float16)
                                    for t in (K_scale, K_mn, V_scale, V_mn))
    out = torch.empty(Q3.shape, dtype=Q.dtype, device=Q.device)
    _ops.kivi_decode(Q3, Kq, K_scale, K_mn, K_residual, Vq, V_scale, V_mn, V_residual, bits, group_size,
                     1.0 / math.sqrt(D), out)
    return out.unsqueeze(2)


def kivi_append(k_new, v_new, bits, token_offset, Kq, K_scale, K_mn, Vq, V_scale, V_mn, group_size=32):
    """Streaming cache write: quantize whole 32-token groups of new keys and values into
    the packed caches in place, starting at token ``token_offset`` (a multiple of 32).

    k_new, v_new [B,H_k,Tn,D] (Tn a multiple of 32); Kq int32 [B,H_k,D,cap*bits/32],
    K_scale/K_mn f16 [B,H_k,D,cap/32], Vq int32 [B,H_k,cap,D*bits/32], V_scale/V_mn f16
    [B,H_k,cap,D/32]. After any sequence of appends the caches hold exactly what
    ``triton_quantize_and_pack_along_last_dim`` of the whole sequence gives (keys passed
    transposed, as benchmarks/kivi_latency.py:123,127 does), so a serving loop flushes
    the oldest 32 tokens of the bf16 residual window once it exceeds R and keeps decoding
    with kivi_decode_attn. The reference has no incremental form; it packs whole tensors
    and keeps the newest R tokens exact (KIVIQuantizer, src/quantization.py:468-501).
    """
    _ops.kivi_append(k_new, v_new, bits, group_size, token_offset, Kq, K_scale, K_mn, Vq, V_scale, V_mn)


def triton_quantize_and_pack_along_last_dim(data, group_size, bit):
    """Group-wise asymmetric quantize + pack along the last dim (KIVI packer contract).

    Call sites in the reference: benchmarks/kivi_latency.py:123,127,208,210.
    Per group of ``group_size`` elements: fp32 min/max, scale = max(max-min, 1e-8) /
    (2^bit-1), code = clamp(round_half_even((x-min)/scale)); element e lands in int32
    word e // (32/bit) at bit offset (e % (32/bit))*bit. Returns (code int32
    [...,N*bit/32], scale [...,N/gs], mn [...,N/gs]) with scale/mn in data.dtype.
    """
    return _ops.kivi_pack(data, group_size, bit)


def cuda_bmm_fA_qB_outer(group_size, fA, qB, scales, zeros, bits):
    """fA [B,H_q,M,K] @ dequant(qB [B,H_k,K,N*bits/32]) -> f16 [B,H_q,M,N], GQA-aware.

    Contract of the external KIVI GEMV as used at benchmarks/kivi_latency.py:67-69,83-85.
    """
    return _ops.kivi_gemv(group_size, fA, qB, scales, zeros, bits)


def repeat_kv(x, G):
    """[B,H_k,S,D] -> [B,H_k*G,S,D]. ref: benchmarks/kivi_latency.py:20-24."""
    if G == 1:
        return x
    B, H_k, S, D = x.shape
    return x[:, :, None, :, :].expand(B, H_k, G, S, D).reshape(B, H_k * G, S, D)
