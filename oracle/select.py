"""fp32 CPU restatement of the reference's selection primitives (test oracle only).

References: ``benchmarks/sparse_attention.py`` (select_topk, _quest_select,
attend_topk) and the ``scores.topk`` calls of ``src/attention_kernels.py``.
Decode-shaped: one query row per (batch, head) at position S-1, so every cached key
is causally valid.
"""
import torch

NEG_INF = float("-inf")


def topk_lower_index(scores, k):
    """Top-k along the last dim, descending by value; equal values keep the lower index first.

    Replaces ``scores.topk(k)`` (src/attention_kernels.py:1069,1262), whose tie order
    is unspecified, with a stable descending sort. Returns (values, int64 indices).
    """
    vals, idx = torch.sort(scores, dim=-1, descending=True, stable=True)
    return vals[..., :k], idx[..., :k]


def select_topk_exact(q, sel_keys, S, kb, scaling):
    """Decode-shaped ``select_topk('exact', ...)``: top-kb keys by q.k*scaling (fp32).

    benchmarks/sparse_attention.py:287-309. The streaming merge over key chunks keeps
    the earlier (lower-index) candidate first on equal values, so the result equals a
    global stable top-kb. Slots beyond S hold the sentinel S (:292-293).
    q [B,Hq,1,D], sel_keys [B,Hq,S,D] -> idx [B,Hq,1,kb] int64.
    """
    sc = torch.einsum("bhqd,bhsd->bhqs", q.float(), sel_keys[:, :, :S].float()) * scaling
    kk = min(kb, S)
    _, idx = topk_lower_index(sc, kk)
    if kb > kk:
        pad = torch.full(idx.shape[:-1] + (kb - kk,), S, dtype=torch.long)
        idx = torch.cat([idx, pad], dim=-1)
    return idx


def quest_page_minmax(k, page):
    """Per-page elementwise key min/max [B,H,np,D]; a ragged last page covers only real keys.

    benchmarks/sparse_attention.py:334-341 (the reference pads by repeating the last
    key, which leaves min/max unchanged).
    """
    B, H, S, D = k.shape
    np_ = (S + page - 1) // page
    padS = np_ * page
    kp = k
    if padS > S:
        kp = torch.cat([k, k[:, :, -1:, :].expand(B, H, padS - S, D)], dim=2)
    kp = kp.reshape(B, H, np_, page, D)
    return kp.amin(dim=3), kp.amax(dim=3)


def quest_page_bounds(q, kmin, kmax, scaling):
    """bound[b,h_q,p] = scaling * sum_d max(q_d*kmin_pd, q_d*kmax_pd) in fp32.

    benchmarks/sparse_attention.py:342-345; kmin/kmax are per KV head [B,Hk,np,D].
    """
    B, Hq, _, D = q.shape
    Hk = kmin.shape[1]
    G = Hq // Hk
    qf = q[:, :, 0, :].float().reshape(B, Hk, G, 1, D)
    lo = qf * kmin.float()[:, :, None]
    hi = qf * kmax.float()[:, :, None]
    return (torch.maximum(lo, hi).sum(-1) * scaling).reshape(B, Hq, -1)


def _expand_pages(pidx, page, S):
    off = torch.arange(page)
    idx = (pidx[..., None] * page + off).reshape(pidx.shape[:-1] + (pidx.shape[-1] * page,))
    return idx.clamp(max=S - 1)


def quest_select(q, k_r, S, kb, page, scaling):
    """Decode-shaped ``_quest_select`` (benchmarks/sparse_attention.py:328-364).

    q [B,Hq,1,D], k_r [B,Hq,S,D] (GQA-expanded) -> idx [B,Hq,1,npick*page], npick =
    min(max(1, ceil(kb/page)), np); pages ranked by bound, lower page index first on
    ties; indices clamped to S-1.
    """
    kmin, kmax = quest_page_minmax(k_r[:, :, :S], page)
    return quest_select_from_meta(q, kmin, kmax, S, kb, page, scaling)


def quest_select_from_meta(q, kmin, kmax, S, kb, page, scaling):
    """Same as quest_select from precomputed per-KV-head page metadata [B,Hk,np,D]."""
    bound = quest_page_bounds(q, kmin, kmax, scaling)  # [B,Hq,np]
    np_ = bound.shape[-1]
    npick = min(max(1, (kb + page - 1) // page), np_)
    _, pidx = topk_lower_index(bound, npick)
    return _expand_pages(pidx, page, S).unsqueeze(2)


def attend_topk(q, k_r, v, idx, q_pos, scaling):
    """Exact softmax attention over selected keys, fp32 throughout.

    benchmarks/sparse_attention.py:367-387: valid = idx <= q_pos & idx < S; duplicate
    indices count once per occurrence. q [B,Hq,Qc,D], k_r/v [B,Hq,S,D] (expanded),
    idx [B,Hq,Qc,ksel] -> [B,Hq,Qc,D] in v.dtype.
    """
    B, Hq, Qc, D = q.shape
    S = k_r.shape[2]
    ksel = idx.shape[-1]
    valid = (idx <= q_pos[None, None, :, None]) & (idx < S) & (idx >= 0)
    gi = idx.clamp(0, S - 1)
    g = gi.unsqueeze(-1).expand(B, Hq, Qc, ksel, D)
    ks = torch.gather(k_r.float().unsqueeze(2).expand(B, Hq, Qc, S, D), 3, g)
    vs = torch.gather(v.float().unsqueeze(2).expand(B, Hq, Qc, S, D), 3, g)
    sc = (q.float().unsqueeze(3) * ks).sum(-1) * scaling
    sc = torch.where(valid, sc, torch.full_like(sc, NEG_INF))
    w = torch.softmax(sc, dim=-1)
    return (w.unsqueeze(-1) * vs).sum(3).to(v.dtype)
