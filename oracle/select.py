"""fp32 CPU restatement of the reference's selection primitives (test oracle only).

References: ``benchmarks/sparse_attention.py`` (select_topk, _quest_select,
attend_topk, sparse_attention_chunked) and the ``scores.topk`` calls of
``src/attention_kernels.py``. The decode-shaped functions take one query row per
(batch, head) at position S-1 (every cached key causally valid); the ``*_window`` forms take
a block of query rows at positions q_pos with per-row causal limits, as the reference's
prefill loop does.
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


def select_topk_exact_window(q, sel_keys, q_pos, S, kb, scaling, local_w=0):
    """``select_topk('exact', ...)`` over a block of query rows.

    benchmarks/sparse_attention.py:287-309: fp32 scores q.k*scaling of the causal keys
    (position <= the row's q_pos), the most recent local_w causal keys forced in (:253-262),
    top-kb with the lower index first on equal scores (the streaming merge keeps earlier
    candidates first); slots no causal key fills hold the sentinel S (:292-293).
    q [B,Hq,Qc,D], sel_keys [B,Hq,S,D], q_pos [Qc] -> [B,Hq,Qc,kb] int64.
    """
    sc = torch.einsum("bhqd,bhsd->bhqs", q.float(), sel_keys[:, :, :S].float()) * scaling
    kpos = torch.arange(S)
    pos = q_pos.reshape(-1)
    sc = sc.masked_fill(kpos[None, None, None, :] > pos[None, None, :, None], NEG_INF)
    if local_w > 0:
        rec = (kpos[None, :] > (pos[:, None] - local_w)) & (kpos[None, :] <= pos[:, None])
        sc = sc.masked_fill(rec[None, None], float("inf"))
    kk = min(kb, S)
    vals, idx = topk_lower_index(sc, kk)
    idx = torch.where(vals == NEG_INF, torch.full_like(idx, S), idx)
    if kb > kk:
        idx = torch.cat([idx, torch.full(idx.shape[:-1] + (kb - kk,), S, dtype=torch.long)], dim=-1)
    return idx


def quest_bounds_window(q, k_r, q_pos, S, page, scaling, local_w=0):
    """Page bounds of _quest_select over a block of query rows (benchmarks/sparse_attention.py:
    334-355): pages starting after a row's position -inf, pages overlapping the row's recent
    window (p-local_w, p] +inf. q [B,Hq,Qc,D], k_r [B,Hq,S,D] -> [B,Hq,Qc,np] fp32."""
    kmin, kmax = quest_page_minmax(k_r[:, :, :S], page)
    qf = q.float()[:, :, :, None, :]
    bound = torch.maximum(qf * kmin.float()[:, :, None], qf * kmax.float()[:, :, None]).sum(-1) * scaling
    np_ = bound.shape[-1]
    pos = q_pos.reshape(-1)
    pstart = torch.arange(np_) * page
    bound = bound.masked_fill(pstart[None, None, None, :] > pos[None, None, :, None], NEG_INF)
    if local_w > 0:
        pg = torch.arange(np_)
        lo = (pos - local_w + 1).clamp(min=0) // page
        hi = pos // page
        rec = (pg[None, :] >= lo[:, None]) & (pg[None, :] <= hi[:, None])
        bound = bound.masked_fill(rec[None, None], float("inf"))
    return bound


def quest_select_window(q, k_r, q_pos, S, kb, page, scaling, local_w=0):
    """_quest_select over a block of query rows (benchmarks/sparse_attention.py:328-364):
    top npick = min(max(1, ceil(kb/page)), np) pages by bound (lower page first on ties),
    expanded to token indices clamped to S-1. -> [B,Hq,Qc,npick*page] int64."""
    bound = quest_bounds_window(q, k_r, q_pos, S, page, scaling, local_w)
    np_ = bound.shape[-1]
    npick = min(max(1, (kb + page - 1) // page), np_)
    _, pidx = topk_lower_index(bound, npick)
    return _expand_pages(pidx, page, S)


SOFT_SELECTORS = ("approx", "int4", "int2", "fp8", "signvq")


def select_topk_window(selector, q, sel_keys, q_pos, S, kb, scaling, page=16, local_w=0, sparq_r=16):
    """``select_topk`` over a block of query rows for the deterministic selectors
    (benchmarks/sparse_attention.py:226-309): 'exact' and the soft selectors (exact top-k over
    the keys given), 'sparq' (the query cut to its sparq_r largest-magnitude channels, lower
    channel first on equal magnitudes, then exact), 'recent' ([p-kb+1 .. p] clamped at 0)
    and 'quest'."""
    B, Hq, Qc, D = q.shape
    if selector == "recent":
        idx = (q_pos.reshape(-1)[:, None] - torch.arange(kb)[None, :]).clamp(min=0)
        return idx[None, None].expand(B, Hq, Qc, kb).contiguous()
    if selector == "quest":
        return quest_select_window(q, sel_keys, q_pos, S, kb, page, scaling, local_w)
    if selector == "sparq":
        r = min(sparq_r, D)
        _, topr = topk_lower_index(q.float().abs(), r)
        q = q * torch.zeros_like(q).scatter_(-1, topr, 1.0)
    elif selector != "exact" and selector not in SOFT_SELECTORS:
        raise ValueError(selector)
    return select_topk_exact_window(q, sel_keys, q_pos, S, kb, scaling, local_w)


def sparse_attention_chunked(q_r, k_r, v, selector, frac, n_kv_groups, scaling, page=16, q_chunk=256, local_w=0,
                             sel_override=None):
    """The reference's chunked prefill loop (benchmarks/sparse_attention.py:463-497) for the
    deterministic selectors of ``select_topk_window``, in fp32; the soft selectors rank by
    ``sel_override`` [B,Hk,S,D] when it is given."""
    B, Hq, S, D = q_r.shape
    kb = max(1, int(round(frac * S)))
    kfull = k_r.repeat_interleave(n_kv_groups, dim=1)
    vfull = v.repeat_interleave(n_kv_groups, dim=1)
    sel = sel_override.repeat_interleave(n_kv_groups, dim=1) \
        if selector in SOFT_SELECTORS and sel_override is not None else kfull
    out = torch.empty(q_r.shape, dtype=v.dtype)
    for q0 in range(0, S, q_chunk):
        q1 = min(q0 + q_chunk, S)
        q_blk = q_r[:, :, q0:q1]
        pos = torch.arange(q0, q1)
        idx = select_topk_window(selector, q_blk, sel, pos, S, kb, scaling, page, local_w)
        out[:, :, q0:q1] = attend_topk(q_blk, kfull, vfull, idx, pos, scaling)
    return out
