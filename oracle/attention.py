"""fp32 CPU restatement of the reference's decode-attention kernels (test oracle only).

Reference: ``src/attention_kernels.py`` of saifmb0/bytes. Each Triton kernel there
runs one program per (batch, query head) and streams the context with an online
softmax in fp32; the restatements below compute the same quantities in one shot
(max-subtracted softmax over the whole context), which differs from the kernels
only in fp32 summation order.
"""
import math

import torch

NEG_INF = float("-inf")


def repeat_kv(x, n_rep):
    """[B,H_k,S,D] -> [B,H_k*n_rep,S,D]. Follows benchmarks/sparse_attention.py:85-90."""
    if n_rep == 1:
        return x
    B, H, S, D = x.shape
    return x[:, :, None, :, :].expand(B, H, n_rep, S, D).reshape(B, H * n_rep, S, D)


def _softmax_pv(scores, vf):
    """scores [B,Hk,G,S] fp32, vf [B,Hk,S,D] fp32 -> [B,Hk,G,D] fp32.

    An all-masked (or empty) row yields NaN, like the reference kernels' final
    ``acc / sum_val`` with sum_val == 0 (src/attention_kernels.py:61).
    """
    if scores.shape[-1] == 0:
        return torch.full(scores.shape[:-1] + (vf.shape[-1],), float("nan"))
    m = scores.amax(dim=-1, keepdim=True)
    p = torch.exp(scores - m)
    l = p.sum(dim=-1, keepdim=True)
    return torch.einsum("bkgs,bksd->bkgd", p, vf) / l


def decode_attn_dense(q, k, v, scaling=1.0, out_dtype=None):
    """softmax(q.k * scaling) . v per query head, GQA by h_k = h_q // G.

    Follows ``_decode_attn_bf16_kernel`` / ``_decode_attn_fp8_kernel``
    (src/attention_kernels.py:8-63, 97-154) and the loop reference of
    benchmarks/test_correctness.py:64-75. The reference wrappers apply NO scale
    (scaling=1.0, src/attention_kernels.py:42); ``scaling`` exists for reuse.
    q [B,H_q,1,D]; k,v [B,H_k,S,D] (bf16 or fp8 e4m3) -> [B,H_q,1,D] in q.dtype.
    """
    B, Hq, _, D = q.shape
    Hk = k.shape[1]
    G = Hq // Hk
    qf = q[:, :, 0, :].float().reshape(B, Hk, G, D)
    scores = torch.einsum("bkgd,bksd->bkgs", qf, k.float()) * scaling
    o = _softmax_pv(scores, v.float())
    return o.reshape(B, Hq, 1, D).to(out_dtype or q.dtype)


def _pq_reconstruct(idx, centroids, D):
    """codes [B,H,S,M] + centroids [M,K,d_sub] -> [B,H,S,D] fp32 (columns beyond M*d_sub are 0).

    Follows the in-register reconstruction of src/attention_kernels.py:220-241 and
    ProductQuantizer.dequantize (src/quantization.py:213-226).
    """
    M, _, d_sub = centroids.shape
    c = centroids.float()
    parts = [c[j][idx[..., j].long()] for j in range(M)]  # each [B,H,S,d_sub]
    rec = torch.cat(parts, dim=-1)
    if rec.shape[-1] < D:
        rec = torch.cat([rec, rec.new_zeros(rec.shape[:-1] + (D - rec.shape[-1],))], dim=-1)
    return rec[..., :D]


def decode_attn_dequant(q, k_idx, centroids, v, d_sub=8):
    """PQ-reconstructed keys, dense decode, no scale. src/attention_kernels.py:187-296."""
    D = q.shape[-1]
    k_hat = _pq_reconstruct(k_idx, centroids, D)
    return decode_attn_dense(q, k_hat, v, 1.0, out_dtype=q.dtype)


def _lut_scores(lut, k_idx, Hk):
    """scores[b,h_q,s] = sum_j lut[b,h_q,j,k_idx[b,h_k,s,j]] (fp32) -> [B,Hk,G,S].

    Follows src/attention_kernels.py:329-341 (and :674-680 for the asym kernels).
    """
    B, Hq, M, K = lut.shape
    G = Hq // Hk
    S = k_idx.shape[2]
    lutf = lut.float().reshape(B, Hk, G, M, K)
    idx = k_idx.long()[:, :, None, :, :M].expand(B, Hk, G, S, M)  # [B,Hk,G,S,M]
    gath = torch.gather(lutf[:, :, :, None, :, :].expand(B, Hk, G, S, M, K), 5,
                        idx.unsqueeze(-1)).squeeze(-1)
    return gath.sum(dim=-1)


def decode_attn_pq_lut(lut, k_idx, v):
    """LUT-scored keys (scale folded into the LUT by the caller), dense V.

    src/attention_kernels.py:301-392. Output dtype is v.dtype (:376).
    """
    B, Hq = lut.shape[:2]
    Hk, S, D = v.shape[1], v.shape[2], v.shape[3]
    scores = _lut_scores(lut, k_idx, Hk)
    o = _softmax_pv(scores, v.float())
    return o.reshape(B, Hq, 1, D).to(v.dtype)


def decode_attn_pq_lut_kv(lut, k_idx, v_idx, v_centroids, d_sub_v=8):
    """LUT-scored keys and PQ-reconstructed values. src/attention_kernels.py:397-500.

    Output dtype is v_centroids.dtype (:484).
    """
    B, Hq = lut.shape[:2]
    Hk = v_idx.shape[1]
    M_v, _, dsv = v_centroids.shape
    D = M_v * dsv
    scores = _lut_scores(lut, k_idx, Hk)
    v_hat = _pq_reconstruct(v_idx, v_centroids, D)
    o = _softmax_pv(scores, v_hat)
    return o.reshape(B, Hq, 1, D).to(v_centroids.dtype)


def _gather_paged(paged, block_table, b, L, block_size):
    """Rebuild the first L tokens of sequence b from a paged [NB,H,bs,X] tensor."""
    t = torch.arange(L)
    phys = block_table[b, t // block_size].long()
    return paged[phys, :, t % block_size, :].permute(1, 0, 2)  # [H, L, X]


def paged_attn_pq_lut_kv(lut, k_idx_paged, v_idx_paged, v_centroids, block_table,
                         context_lens, block_size=16):
    """Paged K5: tokens t < context_lens[b] live at block_table[b, t//bs], offset t%bs.

    src/attention_kernels.py:505-619. An empty sequence yields NaN (0/0, :584).
    """
    B, Hq = lut.shape[:2]
    Hk = v_idx_paged.shape[1]
    M_v, _, dsv = v_centroids.shape
    D = M_v * dsv
    out = torch.empty(B, Hq, 1, D, dtype=v_centroids.dtype)
    for b in range(B):
        L = int(context_lens[b])
        ki = _gather_paged(k_idx_paged, block_table, b, L, block_size)[None]
        vi = _gather_paged(v_idx_paged, block_table, b, L, block_size)[None]
        scores = _lut_scores(lut[b:b + 1], ki, Hk)
        o = _softmax_pv(scores, _pq_reconstruct(vi, v_centroids, D))
        out[b] = o.reshape(Hq, 1, D).to(v_centroids.dtype)
    return out


def _asym_out_dtype(v):
    return torch.bfloat16 if v.dtype == torch.float8_e4m3fn else v.dtype


def _outlier_scores(q_out, k_out, Hk):
    """sum_c q_out[b,h_q,c] * k_out[b,h_k,s,c] in fp32 -> [B,Hk,G,S]. src/attention_kernels.py:683-690."""
    B, Hq, C = q_out.shape
    G = Hq // Hk
    if C == 0:
        return torch.zeros(B, Hk, G, k_out.shape[2])
    qo = q_out.float().reshape(B, Hk, G, C)
    return torch.einsum("bkgc,bksc->bkgs", qo, k_out.float())


def decode_attn_pq_lut_asym(lut, k_idx, k_out, q_out, v, BLOCK_N=256):
    """LUT scores + exact outlier channels, fp8/bf16 V. src/attention_kernels.py:625-750."""
    B, Hq = lut.shape[:2]
    Hk, S, D = v.shape[1], v.shape[2], v.shape[3]
    scores = _lut_scores(lut, k_idx, Hk) + _outlier_scores(q_out, k_out, Hk)
    o = _softmax_pv(scores, v.float())
    return o.reshape(B, Hq, 1, D).to(_asym_out_dtype(v))


def paged_attn_pq_lut_asym(lut, k_idx_paged, k_out_paged, q_out, v_paged, block_table,
                           context_lens, block_size=16, BLOCK_N=256):
    """Paged K7. src/attention_kernels.py:756-898."""
    B, Hq = lut.shape[:2]
    Hk, D = v_paged.shape[1], v_paged.shape[3]
    out = torch.empty(B, Hq, 1, D, dtype=_asym_out_dtype(v_paged))
    for b in range(B):
        L = int(context_lens[b])
        ki = _gather_paged(k_idx_paged, block_table, b, L, block_size)[None]
        ko = _gather_paged(k_out_paged, block_table, b, L, block_size)[None]
        vv = _gather_paged(v_paged, block_table, b, L, block_size)[None]
        scores = _lut_scores(lut[b:b + 1], ki, Hk) + _outlier_scores(q_out[b:b + 1], ko, Hk)
        o = _softmax_pv(scores, vv.float())
        out[b] = o.reshape(Hq, 1, D).to(out.dtype)
    return out


def decode_attn_pq_lut_int8v(lut, k_idx, v_int8, v_scale):
    """Config-2 extension (not in the reference): LUT-scored keys, int8 V with a per-token
    fp16 scale. Oracle by composition: V = v_int8.float() * v_scale.float() then the
    decode_attn_pq_lut math (src/attention_kernels.py:301-363). Output bf16.
    """
    B, Hq = lut.shape[:2]
    Hk, S, D = v_int8.shape[1], v_int8.shape[2], v_int8.shape[3]
    vf = v_int8.float() * v_scale.float().unsqueeze(-1)
    scores = _lut_scores(lut, k_idx, Hk)
    o = _softmax_pv(scores, vf)
    return o.reshape(B, Hq, 1, D).to(torch.bfloat16)


def sparse_score_pq_lut_asym(lut, k_idx, k_out, q_out, BLOCK_N=256):
    """Pass-1 LUT+outlier scores [B,H_q,S] fp32. src/attention_kernels.py:909-984."""
    B, Hq = lut.shape[:2]
    Hk, S = k_idx.shape[1], k_idx.shape[2]
    s = _lut_scores(lut, k_idx, Hk) + _outlier_scores(q_out, k_out, Hk)
    return s.reshape(B, Hq, S)


def sparse_score_scalar(q, k_score, scaling, score_bits=16):
    """Pass-1 exact scores q.k*scaling [B,H_q,S] fp32 over bf16/fp8 keys.

    src/attention_kernels.py:1077-1133.
    """
    B, Hq, _, D = q.shape
    Hk, S = k_score.shape[1], k_score.shape[2]
    G = Hq // Hk
    qf = q[:, :, 0, :].float().reshape(B, Hk, G, D)
    s = torch.einsum("bkgd,bksd->bkgs", qf, k_score.float()) * scaling
    return s.reshape(B, Hq, S)


def sparse_score_packed(q, k_packed, scale, zero, scaling, score_bits=4, group_size=32):
    """Pass-1 scores from uint8-packed 2/4-bit keys: k = code*scale + zero (fp32).

    src/attention_kernels.py:1136-1222 (byte c//epb, shift (c%epb)*bits, group c//gs).
    """
    from .quant import unpack_score_keys
    B, Hq, _, D = q.shape
    Hk, S = k_packed.shape[1], k_packed.shape[2]
    codes = unpack_score_keys(k_packed, score_bits).float()  # [B,Hk,S,D]
    gi = torch.arange(D) // group_size
    kf = codes * scale.float()[..., gi] + zero.float()[..., gi]
    return sparse_score_scalar(q, kf, scaling)


def sparse_gather_attn(q, k, v, idx, scaling, BLOCK_K=64):
    """Exact softmax(q.k_sel*scaling).v_sel over gathered key positions idx [B,H_q,kb].

    src/attention_kernels.py:987-1059. Positions outside [0,S) are excluded (the
    reference kernel would read out of bounds there; attend_topk,
    benchmarks/sparse_attention.py:378, masks idx >= S). Output bf16 for fp8 V.
    """
    B, Hq, _, D = q.shape
    Hk, S = k.shape[1], k.shape[2]
    G = Hq // Hk
    kb = idx.shape[-1]
    out_dtype = torch.bfloat16 if v.dtype == torch.float8_e4m3fn else v.dtype
    ii = idx.long()
    valid = (ii >= 0) & (ii < S)
    gi = ii.clamp(0, max(S - 1, 0))
    # rows of query head h come from KV head h // G (repeat_kv's mapping); indexing the
    # cache directly keeps the check affordable at 32K-token caches
    bi = torch.arange(B)[:, None, None]
    hi = (torch.arange(Hq) // G)[None, :, None]

    def rows(t):
        if t.dtype == torch.float8_e4m3fn:
            return t.view(torch.uint8)[bi, hi, gi].view(torch.float8_e4m3fn).float()
        return t[bi, hi, gi].float()

    ks, vs = rows(k), rows(v)
    sc = (q.float()[:, :, 0, None, :] * ks).sum(-1) * scaling
    sc = torch.where(valid, sc, torch.full_like(sc, NEG_INF))
    m = sc.amax(-1, keepdim=True)
    p = torch.exp(sc - m)
    o = (p.unsqueeze(-1) * vs).sum(2) / p.sum(-1, keepdim=True)
    return o.unsqueeze(2).to(out_dtype)


def budget(frac, S):
    """kb = max(1, int(round(frac*S))) with Python's round-half-even.

    src/attention_kernels.py:1068,1261.
    """
    return max(1, int(round(frac * S)))


def sparse_decode_scalar(q, k_score_or_packed, scale, zero, k_val, v_val, frac, scaling,
                         score_bits, group_size=32):
    """Two-pass sparse decode: score -> top-kb (lower index wins ties) -> gather-attend.

    src/attention_kernels.py:1252-1263.
    """
    from .select import topk_lower_index
    if score_bits in (16, 8):
        scores = sparse_score_scalar(q, k_score_or_packed, scaling, score_bits)
    else:
        scores = sparse_score_packed(q, k_score_or_packed, scale, zero, scaling,
                                     score_bits, group_size)
    kb = budget(frac, scores.shape[-1])
    _, idx = topk_lower_index(scores, kb)
    return sparse_gather_attn(q, k_val, v_val, idx, scaling)


def sparse_decode_pq_lut(lut, k_idx, k_out, q_out, q, k, v, frac, scaling):
    """LUT-score all keys -> top-kb -> exact gather. src/attention_kernels.py:1062-1070."""
    from .select import topk_lower_index
    scores = sparse_score_pq_lut_asym(lut, k_idx, k_out, q_out)
    kb = budget(frac, scores.shape[-1])
    _, idx = topk_lower_index(scores, kb)
    return sparse_gather_attn(q, k, v, idx, scaling)


def split_partials(q, k, v, scaling, n_splits):
    """Per-shard (m, l, o) of dense decode over n_splits contiguous key ranges.

    Used to check the split-KV combine (within a GPU and across GPUs): shard i covers
    keys [i*S/n, (i+1)*S/n). m, l: [n,B,H_q] fp32; o: [n,B,H_q,D] fp32 (normalised).
    """
    B, Hq, _, D = q.shape
    Hk, S = k.shape[1], k.shape[2]
    G = Hq // Hk
    qf = q[:, :, 0, :].float().reshape(B, Hk, G, D)
    bounds = [S * i // n_splits for i in range(n_splits + 1)]
    ms, ls, os_ = [], [], []
    for i in range(n_splits):
        s0, s1 = bounds[i], bounds[i + 1]
        sc = torch.einsum("bkgd,bksd->bkgs", qf, k[:, :, s0:s1].float()) * scaling
        m = sc.amax(-1)
        p = torch.exp(sc - m.unsqueeze(-1))
        l = p.sum(-1)
        o = torch.einsum("bkgs,bksd->bkgd", p, v[:, :, s0:s1].float()) / l.unsqueeze(-1)
        ms.append(m.reshape(B, Hq)); ls.append(l.reshape(B, Hq)); os_.append(o.reshape(B, Hq, D))
    return torch.stack(ms), torch.stack(ls), torch.stack(os_)


def lse_combine(m, l, o):
    """Log-sum-exp merge of shard partials: O = sum_i o_i l_i e^(m_i-M) / sum_i l_i e^(m_i-M)."""
    M = m.amax(0)
    w = l * torch.exp(m - M)
    return (o * w.unsqueeze(-1)).sum(0) / w.sum(0).unsqueeze(-1)
