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


def _decode_all_positions(q3, k, v, out_dtype):
    """Exact attention of each query head over every cached position through the gather
    kernel (fp32 arithmetic on the unrounded query), for queries the tensor-core decode
    tiles would have to round. The position list is one [S] ramp viewed with zero batch /
    head strides."""
    B, Hq, D = q3.shape
    S = k.shape[2]
    idx = torch.arange(S, dtype=torch.int32, device=q3.device).expand(B, Hq, S)
    out = torch.empty(q3.shape, dtype=out_dtype, device=q3.device)
    _ops.gather_attn(q3, k, v, idx, 1.0, out)
    return out.unsqueeze(2)


def decode_attn_bf16(q, k, v):
    """softmax(q.k) . v per query head, GQA by h_q // (H_q/H_k); NO scale is applied.

    ref: src/attention_kernels.py:65-92. q [B,H_q,1,D]; k,v [B,H_k,S,D] bf16
    -> [B,H_q,1,D] in q.dtype. A bf16 query takes the tensor-core decode tiles (every
    product exact in fp32); an f16 or fp32 query, which they would round, and an f16 or
    fp32 cache are computed in fp32 over every position by the gather kernel, as the
    reference widens them.
    """
    if q.is_cuda and q.dtype == torch.bfloat16 and k.dtype == torch.bfloat16:
        rc, out = _ops.N.glue().decode_attn_nq(q, k, v)
        if rc == 0:
            return out
    q3 = _squeeze_q(q)
    if k.dtype in (torch.float16, torch.float32) and v.dtype == k.dtype:
        # an f16 / fp32 cache (off the function's name, as the reference allows): fp32
        # attention over every position by the gather kernel
        if q3.dtype not in (torch.bfloat16, torch.float16, torch.float32):
            q3 = q3.float()
        out_dt = q.dtype if q.dtype in (torch.bfloat16, torch.float16, torch.float32) else torch.float32
        return _decode_all_positions(q3, k, v, out_dt).to(q.dtype)
    if q3.dtype in (torch.float16, torch.float32):
        return _decode_all_positions(q3, k, v, q.dtype)
    if q3.dtype != torch.bfloat16:
        q3 = q3.float()
        return _decode_all_positions(q3, k, v, torch.float32).to(q.dtype)
    out = torch.empty(q3.shape, dtype=q.dtype, device=q.device)
    _ops.decode_attn(q3, k, v, 1.0, out)
    return out.unsqueeze(2)


def decode_attn_fp8(q, k, v):
    """decode_attn_bf16 over an fp8 e4m3 KV cache. ref: src/attention_kernels.py:156-182.

    bf16 and f16 queries meet the keys as exact f16 operands on the tensor cores; an fp32
    query, which that would round, is computed in fp32 over every position by the gather
    kernel.
    """
    if q.is_cuda and q.dtype in (torch.bfloat16, torch.float16):
        rc, out = _ops.N.glue().decode_attn_nq(q, k, v)
        if rc == 0:
            return out
    q3 = _squeeze_q(q)
    if q3.dtype not in (torch.bfloat16, torch.float16):
        out = _decode_all_positions(q3.float(), k, v, torch.float32)
        return out.to(q.dtype)
    out = torch.empty(q3.shape, dtype=q.dtype, device=q.device)
    _ops.decode_attn(q3, k, v, 1.0, out)
    return out.unsqueeze(2)


def sparse_score_scalar(q, k_score, scaling, *, score_bits=16, BLOCK_N=128):
    """Pass-1 exact scores [B,H_q,S] fp32 = scaling * q.k.

    ref: src/attention_kernels.py:1113-1133. Like the reference, the key dtype decides the
    arithmetic and ``score_bits`` is a label: fp8 e4m3 keys, or bf16 / f16 / fp32 keys
    (bf16 query and keys on the tensor cores, where every product is exact in fp32; other
    combinations in fp32 on the CUDA cores, unrounded). Other float dtypes are read as fp32.
    """
    q3 = _squeeze_q(q)
    if q3.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        q3 = q3.float()
    if k_score.dtype == torch.float8_e4m3fn:
        bits = 8
    else:
        bits = 16
        if k_score.dtype not in (torch.bfloat16, torch.float16, torch.float32):
            k_score = k_score.float()
    return _ops.sparse_score(q3, k_score, None, None, scaling, bits, 32)


def sparse_score_packed(q, k_packed, scale, zero, scaling, *, score_bits=4, group_size=32, BLOCK_N=128):
    """Pass-1 scores [B,H_q,S] fp32 from uint8-packed 2/4-bit keys (k = code*scale + zero).

    ref: src/attention_kernels.py:1136-1222.
    """
    if score_bits not in (2, 4):
        raise ValueError("Unsupported score_bits")
    return _ops.sparse_score(_squeeze_q(q), k_packed, scale, zero, scaling, score_bits, group_size)


def quantize_and_pack_score_keys(k, score_bits, group_size):
    """Per-token groups of `group_size` channels -> (packed uint8, scale, zero) in k.dtype.

    ref: src/attention_kernels.py:1225-1249, bit-exact with the reference run on a CUDA
    device: fp32 min/max, scale = range times the fp32 reciprocal of levels-1 (PyTorch's
    CUDA division by a number), codes by IEEE division, round-half-even, low bits first.
    """
    if score_bits not in (2, 4):
        raise ValueError("Unsupported score_bits")
    return _ops.pack_score_keys(k, score_bits, group_size)


def sparse_gather_attn(q, k, v, idx, scaling, BLOCK_K=64):
    """Exact softmax attention over gathered key positions idx [B,H_q,kb].

    ref: src/attention_kernels.py:1037-1059. Output bf16 for fp8 V, else v.dtype.
    Positions outside [0, S) are skipped (the reference kernel reads them unchecked).
    """
    q3 = _squeeze_q(q)
    out_dtype = torch.bfloat16 if v.dtype == torch.float8_e4m3fn else v.dtype
    if k.dtype not in (torch.bfloat16, torch.float16, torch.float32, torch.float8_e4m3fn) or k.dtype != v.dtype:
        k, v = k.float(), v.float()
    if q3.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        q3 = q3.float()
    out = torch.empty(q3.shape, dtype=out_dtype if out_dtype in (torch.bfloat16, torch.float16, torch.float32)
                      else torch.float32, device=q.device)
    _ops.gather_attn(q3, k, v, idx, scaling, out)
    return out.to(out_dtype).unsqueeze(2)


def _budget(frac, S):
    return max(1, int(round(frac * S)))


def sparse_decode_scalar(q, k_score_or_packed, scale, zero, k_val, v_val, frac, scaling, *, score_bits,
                         group_size=32, BLOCK_N=128, BLOCK_K=64):
    """Two-pass sparse decode: score all keys -> top-kb (lower index wins ties) -> gather.

    ref: src/attention_kernels.py:1252-1263. kb = max(1, round(frac*S)).
    """
    if score_bits in (16, 8):
        scores = sparse_score_scalar(q, k_score_or_packed, scaling, score_bits=score_bits)
    else:
        scores = sparse_score_packed(q, k_score_or_packed, scale, zero, scaling, score_bits=score_bits,
                                     group_size=group_size)
    kb = _budget(frac, scores.shape[-1])
    _, idx = _ops.topk(scores, kb, sorted=False, want_values=False, idx_dtype=torch.int32)
    return sparse_gather_attn(q, k_val, v_val, idx, scaling)


def topk(scores, k, sorted=True):
    """Top-k along the last dim; equal values keep the lower index first.

    Replaces ``scores.topk(k)`` (src/attention_kernels.py:1069,1262). Returns
    (values fp32, indices int64).
    """
    return _ops.topk(scores, k, sorted=sorted)


def _v_for_pq(v):
    """Values as the PQ kernels take them: bf16, f16, fp8 e4m3 or int8 as given; other
    dtypes (fp32) as bf16, which keeps their range."""
    return v if v.dtype in (torch.bfloat16, torch.float16, torch.float8_e4m3fn, torch.int8) else v.to(torch.bfloat16)


def decode_attn_dequant(q, k_idx, centroids, v, d_sub=8):
    """Dense decode over PQ-reconstructed keys, no scale. ref: src/attention_kernels.py:267-296.

    Served as LUT[b,h,j,c] = q_j . centroids[j,c] followed by the LUT path (the same sum
    over channels, grouped by subspace). Output dtype q.dtype.
    """
    q3 = _squeeze_q(q)
    lut = _ops.pq_build_lut(q3, centroids)
    out = _ops.pq_decode(lut, k_idx, v=_v_for_pq(v), out_dtype=q.dtype)
    return out.unsqueeze(2)


def decode_attn_pq_lut(lut, k_idx, v):
    """LUT-scored decode (scale folded into the LUT by the caller). ref: src/attention_kernels.py:365-392.

    lut [B,H_q,M,K] fp32; k_idx uint8 [B,H_k,S,M]; v [B,H_k,S,D] -> [B,H_q,1,D] in v.dtype.
    """
    out = _ops.pq_decode(lut, k_idx, v=_v_for_pq(v), out_dtype=v.dtype)
    return out.unsqueeze(2)


def decode_attn_pq_lut_kv(lut, k_idx, v_idx, v_centroids, d_sub_v=8):
    """LUT scores + PQ-reconstructed values. ref: src/attention_kernels.py:471-500.

    Output dtype v_centroids.dtype.
    """
    out = _ops.pq_decode(lut, k_idx, v_idx=v_idx, v_cent=v_centroids, out_dtype=v_centroids.dtype)
    return out.unsqueeze(2)


def paged_attn_pq_lut_kv(lut, k_idx_paged, v_idx_paged, v_centroids, block_table, context_lens, block_size=16):
    """Paged LUT-KV decode. ref: src/attention_kernels.py:588-619 (context_lens per sequence,
    token t at block_table[b, t // block_size], offset t % block_size)."""
    out = _ops.pq_decode(lut, k_idx_paged, v_idx=v_idx_paged, v_cent=v_centroids, block_table=block_table,
                         context_lens=context_lens, block_size=block_size, out_dtype=v_centroids.dtype)
    return out.unsqueeze(2)


def _asym_out(v):
    return torch.bfloat16 if v.dtype == torch.float8_e4m3fn else v.dtype


def decode_attn_pq_lut_asym(lut, k_idx, k_out, q_out, v, BLOCK_N=256):
    """LUT scores + exact outlier channels q_out.k_out; fp8/bf16 V. ref: src/attention_kernels.py:713-750."""
    out = _ops.pq_decode(lut, k_idx, v=_v_for_pq(v), k_out=k_out, q_out=q_out, out_dtype=_asym_out(v))
    return out.unsqueeze(2)


def paged_attn_pq_lut_asym(lut, k_idx_paged, k_out_paged, q_out, v_paged, block_table, context_lens,
                           block_size=16, BLOCK_N=256):
    """Paged asymmetric PQ-LUT decode. ref: src/attention_kernels.py:858-898."""
    out = _ops.pq_decode(lut, k_idx_paged, v=_v_for_pq(v_paged), k_out=k_out_paged, q_out=q_out,
                         block_table=block_table, context_lens=context_lens, block_size=block_size,
                         out_dtype=_asym_out(v_paged))
    return out.unsqueeze(2)


def sparse_score_pq_lut_asym(lut, k_idx, k_out, q_out, BLOCK_N=256):
    """Pass-1 LUT + outlier scores [B,H_q,S] fp32. ref: src/attention_kernels.py:960-984."""
    return _ops.pq_scores(lut, k_idx, k_out, q_out)


def sparse_decode_pq_lut(lut, k_idx, k_out, q_out, q, k, v, frac, scaling, BLOCK_N=256, BLOCK_K=64):
    """LUT-score all keys -> top-kb (lower index wins ties) -> exact gather attention.

    ref: src/attention_kernels.py:1062-1070.
    """
    scores = sparse_score_pq_lut_asym(lut, k_idx, k_out, q_out)
    kb = _budget(frac, scores.shape[-1])
    _, idx = _ops.topk(scores, kb, sorted=False, want_values=False, idx_dtype=torch.int32)
    return sparse_gather_attn(q, k, v, idx, scaling)


def decode_attn_pq_lut_int8v(lut, k_idx, v_int8, v_scale):
    """Config-2 extension (no counterpart in the reference): LUT-scored keys with int8
    values and a per-token f16 scale (V = v_int8 * v_scale). lut [B,H_q,M,K];
    k_idx uint8 [B,H_k,S,M]; v_int8 [B,H_k,S,D]; v_scale f16 [B,H_k,S] -> bf16 [B,H_q,1,D].
    """
    if v_scale.dtype != torch.float16:
        v_scale = v_scale.to(torch.float16)
    out = _ops.pq_decode(lut, k_idx, v=v_int8, v_scale=v_scale, out_dtype=torch.bfloat16)
    return out.unsqueeze(2)
