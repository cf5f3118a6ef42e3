"""fp32 CPU restatement of the reference's quantize / pack / encode steps (test oracle only).

References: ``src/quantization.py`` and ``src/attention_kernels.py`` of saifmb0/bytes,
``benchmarks/kivi_latency.py`` (in-tree KIVI unpack / dequant / reference decode).

Two device rules. The reference's quantizers are PyTorch expressions, and PyTorch
evaluates ``tensor / python_number`` differently by device: on the CPU as a true
division, on a CUDA device as a multiplication by the fp32 reciprocal of the number
(computed once on the host; for bf16 / f16 tensors the product is formed in fp32 and
rounded to the tensor's type). The two differ in the last bit of about half of all
fp32 quotients, which moves a few percent of the quantised codes. ``rule="cuda"`` (the
default) restates what the reference computes on a GPU, the device its decode path runs
on; ``rule="cpu"`` restates its CPU run. ``ProductQuantizer.quantize`` is a different
algorithm on each device (a Triton f16-dot-product kernel on CUDA, cdist + argmin on the
CPU); ``pq_encode`` restates both.
"""
import math

import numpy as np
import torch


def div_scalar(t, n, rule="cuda"):
    """``t / n`` for a tensor t and a Python number n, as PyTorch evaluates it on ``rule``'s
    device: CPU = true division; CUDA = t * fp32(1/n), formed in fp32 and rounded to t's type."""
    if rule == "cpu":
        return t / n
    if rule != "cuda":
        raise ValueError(f"unknown rule {rule!r}")
    rcp = torch.tensor(np.float32(1.0) / np.float32(n), dtype=torch.float32)
    return (t.float() * rcp).to(t.dtype)


def asym_uniform_fakequant(x, levels, dim, rule="cuda"):
    """Quantize-then-dequantize with the [min,max] range taken over ``dim``.

    src/quantization.py:432-442: scale = clamp(max-min, 1e-8)/(levels-1);
    q = clamp(round((x-min)/scale), 0, levels-1); return q*scale + min. The division by
    levels-1 follows ``rule`` (see ``div_scalar``); (x-min)/scale is a true division on
    both devices.
    """
    xmin = x.amin(dim=dim, keepdim=True)
    xmax = x.amax(dim=dim, keepdim=True)
    scale = div_scalar((xmax - xmin).clamp(min=1e-8), levels - 1, rule)
    q = torch.clamp(torch.round((x - xmin) / scale), 0, levels - 1)
    return q * scale + xmin


def kivi_quantize_key(k, bits=4, group_size=32, residual_length=32, rule="cuda"):
    """KIVIQuantizer.quantize_key (src/quantization.py:468-489): per-channel scales over
    groups of ``group_size`` tokens; a ragged token tail forms one group; the last
    ``residual_length`` tokens stay exact."""
    levels = 2 ** bits
    B, H, S, D = k.shape
    R = min(residual_length, S)
    S_q = S - R
    if S_q <= 0:
        return k
    k_q = k[:, :, :S_q, :].float()
    k_res = k[:, :, S_q:, :]
    G = group_size
    n_full = S_q // G
    parts = []
    if n_full > 0:
        main = k_q[:, :, :n_full * G, :].reshape(B, H, n_full, G, D)
        parts.append(asym_uniform_fakequant(main, levels, 3, rule).reshape(B, H, n_full * G, D))
    if n_full * G < S_q:
        parts.append(asym_uniform_fakequant(k_q[:, :, n_full * G:, :], levels, 2, rule))
    k_dq = torch.cat(parts, dim=2) if len(parts) > 1 else parts[0]
    return torch.cat([k_dq.to(k.dtype), k_res], dim=2)


def kivi_quantize_value(v, bits=4, group_size=32, residual_length=32, rule="cuda"):
    """KIVIQuantizer.quantize_value (src/quantization.py:491-501): per-token range over
    all channels, last ``residual_length`` tokens exact."""
    levels = 2 ** bits
    S = v.shape[2]
    R = min(residual_length, S)
    S_q = S - R
    if S_q <= 0:
        return v
    v_dq = asym_uniform_fakequant(v[:, :, :S_q, :].float(), levels, 3, rule)
    return torch.cat([v_dq.to(v.dtype), v[:, :, S_q:, :]], dim=2)


def quantize_and_pack_score_keys(k, score_bits, group_size, rule="cuda"):
    """Per-token groups of ``group_size`` channels, fp32 min/max/scale, round-half-even,
    2 codes (4-bit) or 4 codes (2-bit) per byte, low bits first.

    src/attention_kernels.py:1225-1249. Returns (packed uint8 [B,H,S,D*bits/8],
    scale [B,H,S,D/gs] in k.dtype, zero=min [B,H,S,D/gs] in k.dtype).
    """
    if score_bits not in (2, 4):
        raise ValueError("Unsupported score_bits")
    B, H, S, D = k.shape
    ng = D // group_size
    levels = 2 ** score_bits
    kr = k.reshape(B, H, S, ng, group_size).float()
    xmin = kr.amin(dim=-1, keepdim=True)
    xmax = kr.amax(dim=-1, keepdim=True)
    scale = div_scalar((xmax - xmin).clamp(min=1e-8), levels - 1, rule)
    q = torch.clamp(torch.round((kr - xmin) / scale), 0, levels - 1).to(torch.uint8)
    qf = q.reshape(B, H, S, D)
    epb = 8 // score_bits
    packed = torch.zeros(B, H, S, D // epb, dtype=torch.uint8)
    for i in range(epb):
        packed |= (qf[..., i::epb] & (levels - 1)) << (i * score_bits)
    return packed, scale.reshape(B, H, S, ng).to(k.dtype), xmin.reshape(B, H, S, ng).to(k.dtype)


def unpack_score_keys(packed, score_bits):
    """Inverse of the byte packing: channel c at byte c//epb, shift (c%epb)*bits.

    src/attention_kernels.py:1160-1178.
    """
    epb = 8 // score_bits
    mask = (1 << score_bits) - 1
    p = packed.to(torch.int32)
    cols = [(p >> (i * score_bits)) & mask for i in range(epb)]
    return torch.stack(cols, dim=-1).reshape(packed.shape[:-1] + (packed.shape[-1] * epb,)).to(torch.uint8)


def kivi_pack_last_dim(x, group_size, bits, rule="cuda"):
    """Group-wise asymmetric quantize + pack along the last dim (KIVI packer contract).

    The packer lives in the un-vendored external KIVI checkout (call sites
    benchmarks/kivi_latency.py:123,127,208,210). Layout follows the reference's
    in-tree unpacker (benchmarks/kivi_latency.py:26-35): element e -> int32 word
    e // (32/bits), bit offset (e % (32/bits)) * bits. Quantisation follows
    src/quantization.py:438-442 in fp32 (scale clamped at 1e-8; the division by 2^bits-1
    follows ``rule``, as PyTorch evaluates the packer's scale on the device it runs on);
    scale and mn are stored in x.dtype. Returns (code int32 [...,N*bits/32], scale [...,N/gs], mn [...,N/gs]).
    """
    N = x.shape[-1]
    fpi = 32 // bits
    lead = x.shape[:-1]
    xf = x.float().reshape(lead + (N // group_size, group_size))
    mn = xf.amin(dim=-1, keepdim=True)
    mx = xf.amax(dim=-1, keepdim=True)
    scale = div_scalar((mx - mn).clamp(min=1e-8), 2 ** bits - 1, rule)
    q = torch.clamp(torch.round((xf - mn) / scale), 0, 2 ** bits - 1).to(torch.int64)
    q = q.reshape(lead + (N // fpi, fpi))
    shifts = torch.arange(fpi, dtype=torch.int64) * bits
    words = (q << shifts).sum(dim=-1)  # disjoint bit fields: sum == OR
    words = torch.where(words >= 2 ** 31, words - 2 ** 32, words).to(torch.int32)
    return words, scale.squeeze(-1).to(x.dtype), mn.squeeze(-1).to(x.dtype)


def kivi_unpack_last_dim(code, bits):
    """int32 words -> integer codes, element i of each word at bits [i*bits,(i+1)*bits).

    benchmarks/kivi_latency.py:26-35 (returns int64 codes instead of fp16 values).
    """
    fpi = 32 // bits
    c = code.to(torch.int64) & 0xFFFFFFFF
    vals = [(c >> (i * bits)) & ((1 << bits) - 1) for i in range(fpi)]
    return torch.stack(vals, dim=-1).reshape(code.shape[:-1] + (code.shape[-1] * fpi,))


def kivi_dequant_k(Kq, K_scale, K_mn, group_size, bits):
    """Kq [B,H,D,Sq/fpi] (channel-major, tokens packed) -> K [B,H,Sq,D] fp32.

    benchmarks/kivi_latency.py:37-46 (fp32 arithmetic here; the reference runs fp16).
    """
    codes = kivi_unpack_last_dim(Kq, bits).float()  # [B,H,D,Sq]
    gi = torch.arange(codes.shape[-1]) // group_size
    k = codes * K_scale.float()[..., gi] + K_mn.float()[..., gi]
    return k.transpose(2, 3).contiguous()


def kivi_dequant_v(Vq, V_scale, V_mn, group_size, bits):
    """Vq [B,H,Sq,D/fpi] (token-major, channels packed) -> V [B,H,Sq,D] fp32.

    benchmarks/kivi_latency.py:48-57.
    """
    codes = kivi_unpack_last_dim(Vq, bits).float()
    gi = torch.arange(codes.shape[-1]) // group_size
    return codes * V_scale.float()[..., gi] + V_mn.float()[..., gi]


def kivi_decode_attn(Q, Kq, K_scale, K_mn, K_residual, Vq, V_scale, V_mn, V_residual,
                     bits, group_size=32):
    """One KIVI decode step: softmax(Q.[K_dq;K_res]^T/sqrt(D)).[V_dq;V_res], fp32.

    benchmarks/kivi_latency.py:59-100 (kivi_decode_attn / kivi_decode_attn_ref).
    Output [B,H_q,1,D] in Q.dtype.
    """
    from .attention import decode_attn_dense
    D = Q.shape[-1]
    K = torch.cat([kivi_dequant_k(Kq, K_scale, K_mn, group_size, bits), K_residual.float()], 2)
    V = torch.cat([kivi_dequant_v(Vq, V_scale, V_mn, group_size, bits), V_residual.float()], 2)
    return decode_attn_dense(Q, K, V, 1.0 / math.sqrt(D), out_dtype=Q.dtype)


def kivi_gemv_outer(group_size, fA, qB, scales, zeros, bits):
    """fA [B,Hq,M,K] @ dequant(qB) where qB [B,Hk,K,N/fpi] packs along its last dim and
    scales/zeros [B,Hk,K,N/gs] group along it; GQA h_k = h_q // (Hq/Hk); fp16 output.

    Contract of the external cuda_bmm_fA_qB_outer as used at
    benchmarks/kivi_latency.py:67-69,83-85.
    """
    codes = kivi_unpack_last_dim(qB, bits).float()  # [B,Hk,K,N]
    gi = torch.arange(codes.shape[-1]) // group_size
    deq = codes * scales.float()[..., gi] + zeros.float()[..., gi]
    B, Hq = fA.shape[:2]
    Hk = qB.shape[1]
    deq = deq.repeat_interleave(Hq // Hk, dim=1)
    return torch.matmul(fA.float(), deq).to(torch.float16)


def pq_encode(X, centroids, rule="cuda"):
    """Nearest centroid per subspace. X [...,D], centroids [M,K,d_sub] -> int64 [...,M].

    rule="cuda": ProductQuantizer.quantize on a CUDA device (src/quantization.py:167-199,
    Triton kernel :8-60): score_k = f16(x) . f16(dtype_x(c_k)) summed in fp32, minus
    dtype_x(0.5*||c_k||^2); argmax, first index on ties. (The reference's kernel reads the
    first 16 elements of a sub-vector; this restatement, like the engine, uses all d_sub.)
    The products of f16 values are exact in fp32 and are summed in element order.

    rule="cpu": the CPU path (src/quantization.py:203-211), argmin of the fp32 squared
    distance, first index on ties.
    """
    M, K, d_sub = centroids.shape
    lead = X.shape[:-1]
    if rule == "cpu":
        Xs = X.float().reshape(-1, M, d_sub)
        c = centroids.float()
        d2 = ((Xs[:, :, None, :] - c[None, :, :, :]) ** 2).sum(-1)  # [N,M,K]
        return d2.argmin(dim=-1).reshape(lead + (M,))
    if rule != "cuda":
        raise ValueError(f"unknown rule {rule!r}")
    return pq_encode_scores(X, centroids).argmax(dim=-1).reshape(lead + (M,))


def pq_encode_scores(X, centroids):
    """The CUDA-rule scores [N,M,K] of ``pq_encode`` (higher is nearer)."""
    M, K, d_sub = centroids.shape
    xs = X.reshape(-1, M, d_sub).to(torch.float16).float()
    c = centroids.to(X.dtype).to(torch.float16).float()
    c2 = centroids.float() * centroids.float()
    s2 = torch.zeros(M, K)
    for e in range(d_sub):
        s2 = s2 + c2[:, :, e]
    norms = (0.5 * s2).to(X.dtype).float()
    dot = torch.zeros(xs.shape[0], M, K)
    for e in range(d_sub):
        dot = dot + xs[:, :, None, e] * c[None, :, :, e]
    return dot - norms[None]


def pq_distances(X, centroids):
    """Squared distances [N,M,K] used by the margin rule of the PQ-encode parity test."""
    M, K, d_sub = centroids.shape
    Xs = X.float().reshape(-1, M, d_sub)
    return ((Xs[:, :, None, :] - centroids.float()[None]) ** 2).sum(-1)


def pq_dequantize(codes, centroids):
    """ProductQuantizer.dequantize (src/quantization.py:213-226)."""
    M, K, d_sub = centroids.shape
    parts = [centroids[j][codes[..., j].long()] for j in range(M)]
    return torch.cat(parts, dim=-1)


def pq_lut(q_rot, centroids):
    """LUT[b,h,j,c] = q_rot[b,h,j*d_sub:(j+1)*d_sub] . centroids[j,c] (fp32).

    benchmarks/test_correctness.py:181-182 (einsum "bhmd,mkd->bhmk").
    """
    B, H, D = q_rot.shape
    M, K, d_sub = centroids.shape
    return torch.einsum("bhmd,mkd->bhmk", q_rot.float().reshape(B, H, M, d_sub), centroids.float())
