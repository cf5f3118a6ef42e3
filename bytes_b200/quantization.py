"""Drop-in for the hot-path parts of ``src/quantization.py`` of saifmb0/bytes.

``ProductQuantizer.quantize`` (PQ encode), ``KIVIQuantizer.quantize_key/quantize_value``
and ``_asym_uniform_fakequant`` run on sm_100a kernels. ``fit`` (offline k-means
calibration) and ``dequantize`` (a table lookup) keep the reference's torch formulation;
the other calibration utilities of the reference module are out of scope.
"""
import torch

from . import _ops


def _asym_uniform_fakequant(x, levels, dim):
    """Quantize-then-dequantize with the range taken over `dim` (bit-identical to the reference).

    ref: src/quantization.py:432-442.
    """
    xt = x.movedim(dim, -1)
    lead = xt.shape[:-1]
    g = xt.shape[-1]
    y = _ops.asym_fakequant_5d(xt.reshape(-1, 1, 1, g, 1), levels)
    return y.reshape(tuple(lead) + (g,)).movedim(-1, dim)


class KIVIQuantizer:
    """KIVI fake-quant of the KV cache (ref: src/quantization.py:445-507).

    Keys: per channel over groups of `group_size` tokens (a ragged tail is one group);
    values: per token over all channels; the last `residual_length` tokens stay exact.
    """

    def __init__(self, bits=4, group_size=32, residual_length=32):
        self.bits = bits
        self.levels = 2 ** bits
        self.group_size = group_size
        self.residual_length = residual_length

    def quantize_key(self, k):
        B, H, S, D = k.shape
        R = min(self.residual_length, S)
        S_q = S - R
        if S_q <= 0:
            return k
        k_q = k[:, :, :S_q, :].float()
        G = self.group_size
        n_full = S_q // G
        parts = []
        if n_full > 0:
            main = k_q[:, :, :n_full * G, :].reshape(B, H, n_full, G, D)
            parts.append(_ops.asym_fakequant_5d(main, self.levels).reshape(B, H, n_full * G, D))
        if n_full * G < S_q:
            tail = k_q[:, :, n_full * G:, :].unsqueeze(2)  # (B, H, 1, r, D)
            parts.append(_ops.asym_fakequant_5d(tail, self.levels).reshape(B, H, S_q - n_full * G, D))
        k_dq = torch.cat(parts, dim=2) if len(parts) > 1 else parts[0]
        return torch.cat([k_dq.to(k.dtype), k[:, :, S_q:, :]], dim=2)

    def quantize_value(self, v):
        B, H, S, D = v.shape
        R = min(self.residual_length, S)
        S_q = S - R
        if S_q <= 0:
            return v
        v_q = v[:, :, :S_q, :].float().unsqueeze(-1)  # (B, H, S_q, D, 1): group axis D
        v_dq = _ops.asym_fakequant_5d(v_q, self.levels).reshape(B, H, S_q, D)
        return torch.cat([v_dq.to(v.dtype), v[:, :, S_q:, :]], dim=2)

    def bpw(self, seq_len):
        """Effective key bits per weight (ref: src/quantization.py:503-507)."""
        R = min(self.residual_length, seq_len)
        return self.bits * (seq_len - R) / seq_len + 16.0 * (R / seq_len)


class ProductQuantizer:
    """Product quantizer with a GPU nearest-centroid encoder (ref: src/quantization.py:134-226).

    ``quantize`` returns int64 codes [..., M] like the reference and follows the reference's
    CUDA encoder: score = f16(x) . f16(centroid) - 0.5*||centroid||^2, argmax, first index
    on ties (the centroids are rounded to x's dtype before f16, the norms to x's dtype).
    Only scores equal to within fp32 summation order may pick another centroid than the
    reference's tensor-core kernel. (The reference's CPU fallback, cdist + argmin, differs
    from its CUDA kernel wherever f16 rounding reorders two centroids.)
    """

    def __init__(self, d, d_sub, bits=3, device="cuda"):
        assert d % d_sub == 0, f"d ({d}) must be divisible by d_sub ({d_sub})"
        self.d, self.d_sub, self.bits = d, d_sub, bits
        self.k = 2 ** bits
        self.M = d // d_sub
        self.device = device
        self.centroids = torch.zeros((self.M, self.k, self.d_sub), device=device)

    def fit(self, X, num_iters=20, generator=None):
        """Per-subspace k-means (offline calibration, torch ops)."""
        X = X.to(self.device).float()
        N = X.shape[0]
        Xs = X.view(N, self.M, self.d_sub)
        for j in range(self.M):
            xj = Xs[:, j, :]
            if N <= self.k:
                c = torch.zeros(self.k, self.d_sub, device=X.device)
                c[:N] = xj
                self.centroids[j] = c
                continue
            c = xj[torch.randperm(N, device=X.device, generator=generator)[:self.k]].clone()
            for _ in range(num_iters):
                lab = torch.cdist(xj, c).argmin(1)
                cnt = torch.bincount(lab, minlength=self.k).float()
                s = torch.zeros_like(c).index_add_(0, lab, xj)
                empty = cnt == 0
                c = torch.where(empty[:, None], xj[torch.randint(0, N, (self.k,), device=X.device)],
                                s / cnt.clamp(min=1)[:, None])
            self.centroids[j] = c

    def quantize(self, X):
        """Nearest-centroid codes [..., M] (int64) on the GPU."""
        lead = list(X.shape[:-1])
        codes = _ops.pq_encode(X.reshape(-1, self.d), self.centroids.to(X.device))
        return codes.view(*(lead + [self.M]))

    def dequantize(self, indices):
        lead = list(indices.shape[:-1])
        ind = indices.reshape(-1, self.M).long()
        parts = [self.centroids[j][ind[:, j]] for j in range(self.M)]
        return torch.stack(parts, dim=1).view(*(lead + [self.d]))
