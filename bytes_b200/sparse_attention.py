"""Drop-in for the selection primitives of ``benchmarks/sparse_attention.py``.

The hot path is decode: one query row per (batch, head) at position S-1, where every cached
key is causally valid; those calls take the fused kernels directly (Quest's bound + page
top-k + expansion in one entry point, exact selection as score pass + top-k). The
reference's functions also run over prefill windows (a block of Qc query rows at
positions q_pos, keys causal per row); those calls fold the Qc rows of each head into the
head axis (row (h, r) -> head h*Qc + r, so every kernel sees Qc "query heads" per key
head), run the same kernels, and apply the per-row causal limits on the way: masked scores
and page bounds, invalid gather positions. ``sparse_attention_chunked`` is the reference's
chunked prefill loop over these, for the 'exact' and 'quest' selectors.
"""
import torch

from . import _ops

NEG_INF = float("-inf")

# Selectors that rank keys by an approximate key tensor the caller supplies (as
# ``sel_keys``, or as ``sel_override`` of ``sparse_attention_chunked``); the ranking itself
# is the exact top-k over those keys (benchmarks/sparse_attention.py:32-35, 287-309).
SOFT_SELECTORS = ("approx", "int4", "int2", "fp8", "signvq")
# SparQ: query channels kept for scoring, the top-r by magnitude (reference default 16)
SPARQ_R = 16


def repeat_kv(x, n_rep):
    """[B,H_k,S,D] -> [B,H_k*n_rep,S,D]. ref: benchmarks/sparse_attention.py:85-90."""
    if n_rep == 1:
        return x
    B, H, S, D = x.shape
    return x[:, :, None, :, :].expand(B, H, n_rep, S, D).reshape(B, H * n_rep, S, D)


def _positions(q_pos, Qc, device):
    if q_pos is None:
        raise ValueError("q_pos is required")
    pos = torch.as_tensor(q_pos).reshape(-1).to(device=device, dtype=torch.long)
    if pos.numel() != Qc:
        raise ValueError("q_pos must hold one position per query row")
    return pos


def _is_decode_row(q_blk, q_pos, S):
    if q_blk.shape[2] != 1 or q_pos is None:
        return False
    p = torch.as_tensor(q_pos).reshape(-1)
    return p.numel() == 1 and int(p[0]) == S - 1


def _fold(q_blk):
    """[B,H,Qc,D] -> [B,H*Qc,D] (row r of head h at h*Qc + r)."""
    B, H, Qc, D = q_blk.shape
    q3 = q_blk.reshape(B, H * Qc, D)
    if q3.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        q3 = q3.float()
    return q3


def _full_precision(t):
    return t if t.dtype in (torch.bfloat16, torch.float16, torch.float32) else t.float()


def select_topk(selector, q_blk, sel_keys, q_pos, S, kb, k_chunk, scaling, page=16, generator=None, local_w=0):
    """Top-kb causal key indices per query row.

    Selectors: 'exact' (q.k scores), the soft selectors (the same exact top-k over the
    approximate keys passed as ``sel_keys``), 'sparq' (the query cut to its SPARQ_R
    largest-magnitude channels), 'quest' (page bounds), 'recent' and 'random'.

    ref: benchmarks/sparse_attention.py:226-325. q_blk [B,Hq,Qc,D]; sel_keys [B,Hq,S,D];
    q_pos [Qc] -> [B,Hq,Qc,kb] int64. Exact selection breaks ties by lower index (the
    reference's streaming merge keeps the earlier candidate first as well); slots that no
    causal key fills hold the sentinel S like the reference's placeholders; with local_w the
    most recent local_w causal keys of each row are forced in (:253-262). ``k_chunk`` is the
    reference's streaming granularity; the exact top-k here is global (same selection).
    """
    if selector == "quest":
        return _quest_select(q_blk, sel_keys, q_pos, S, kb, page, scaling, local_w)
    B, Hq, Qc, D = q_blk.shape
    if selector == "recent":
        # the kb most recent causal positions [p-kb+1 .. p] (clamped at 0), :265-269
        pos = _positions(q_pos, Qc, q_blk.device)
        idx = (pos[:, None] - torch.arange(kb, device=q_blk.device)[None, :]).clamp(min=0)
        return idx[None, None].expand(B, Hq, Qc, kb).contiguous()
    if selector == "random":
        # kb uniform draws over [0, p] per row from the caller's generator, :271-276
        pos = _positions(q_pos, Qc, q_blk.device)
        rnd = torch.rand(B, Hq, Qc, kb, device=q_blk.device, generator=generator)
        return (rnd * (pos[None, None, :, None].float() + 1)).long().clamp(min=0)
    if selector == "sparq":
        # score with the query cut to its SPARQ_R largest-magnitude channels, :281-285
        r = min(SPARQ_R, D)
        mag = _fold(q_blk).abs().float()
        _, topr = _ops.topk(mag, r, sorted=False, want_values=False)
        m = torch.zeros(mag.shape, dtype=q_blk.dtype, device=q_blk.device).scatter_(-1, topr, 1.0)
        q_blk = q_blk * m.view(B, Hq, Qc, D)
    elif selector != "exact" and selector not in SOFT_SELECTORS:
        raise ValueError(f"selector {selector!r} is not on the decode hot path")
    keys = _full_precision(sel_keys[:, :, :S])
    q3 = _fold(q_blk)
    # scores in fp32 from the unrounded inputs, like the reference's fp32 score tiles
    # (bf16 query and keys on the tensor cores, where every product is exact)
    scores = _ops.sparse_score(q3, keys, None, None, scaling, 16, 32)  # [B, Hq*Qc, S]
    kk = min(kb, S)
    if _is_decode_row(q_blk, q_pos, S) and local_w <= 0:
        _, idx = _ops.topk(scores, kk, sorted=True, want_values=False)
    else:
        pos = _positions(q_pos, Qc, scores.device)
        kpos = torch.arange(S, device=scores.device)
        sc = scores.view(B, Hq, Qc, S)
        sc.masked_fill_(kpos[None, None, None, :] > pos[None, None, :, None], NEG_INF)
        if local_w > 0:
            rec = (kpos[None, :] > (pos[:, None] - local_w)) & (kpos[None, :] <= pos[:, None])
            sc.masked_fill_(rec[None, None], float("inf"))
        vals, idx = _ops.topk(scores, kk, sorted=True)
        idx = torch.where(vals == NEG_INF, torch.full_like(idx, S), idx)
    if kb > kk:
        idx = torch.cat([idx, torch.full((B, Hq * Qc, kb - kk), S, dtype=idx.dtype, device=idx.device)], -1)
    return idx.view(B, Hq, Qc, kb)


def _quest_select(q_blk, k_r, pos, S, kb, page, scaling, local_w=0):
    """Quest page selection per query row (per-query-head keys k_r [B,Hq,S,D]).

    ref: benchmarks/sparse_attention.py:328-364. Returns [B,Hq,Qc,npick*page] int64, pages
    ordered by bound (lower page wins ties), indices clamped to S-1; pages that start after
    a row's position are excluded, and with local_w the pages overlapping the row's recent
    window (p-local_w, p] are forced in.
    """
    B, Hq, Qc, D = q_blk.shape
    kmin, kmax = _ops.quest_page_minmax(_full_precision(k_r[:, :, :S]), page)
    np_ = kmin.shape[2]
    q3 = _fold(q_blk)
    if _is_decode_row(q_blk, pos, S):
        force = None
        if local_w > 0:
            force = max(0, S - local_w) // page
        idx = _ops.quest_select(q3, kmin, kmax, S, kb, page, scaling, force)
        return idx.unsqueeze(2)
    p = _positions(pos, Qc, q3.device)
    bounds = _ops.quest_page_bounds(q3, kmin, kmax, scaling).view(B, Hq, Qc, np_)
    pstart = torch.arange(np_, device=q3.device) * page
    bounds.masked_fill_(pstart[None, None, None, :] > p[None, None, :, None], NEG_INF)
    if local_w > 0:
        pg = torch.arange(np_, device=q3.device)
        lo = (p - local_w + 1).clamp(min=0) // page
        hi = p // page
        rec = (pg[None, :] >= lo[:, None]) & (pg[None, :] <= hi[:, None])
        bounds.masked_fill_(rec[None, None], float("inf"))
    npick = min(max(1, (kb + page - 1) // page), np_)
    _, pidx = _ops.topk(bounds.view(B, Hq * Qc, np_), npick, sorted=True, want_values=False)
    off = torch.arange(page, device=q3.device)
    idx = (pidx[..., None] * page + off).reshape(B, Hq, Qc, npick * page)
    return idx.clamp(max=S - 1)


def quest_page_metadata(k, page):
    """Per-KV-head page min/max [B,H_k,np,D] for the decode Quest path (cache-side step)."""
    return _ops.quest_page_minmax(k, page)


def quest_page_metadata_update(k, kmin, kmax, page, first_page, last_page):
    """Refresh pages [first_page, last_page) of an existing metadata cache in place.

    k [B,H_k,S,D] is the key cache holding S valid tokens; kmin/kmax [B,H_k,>=last_page,D].
    A serving loop calls this for the page the new token fell into (its min/max grows
    until the page fills) -- the cache-side maintenance the reference recomputes from
    scratch on every call (benchmarks/sparse_attention.py:334-341).
    """
    S = k.shape[2]
    t0, t1 = first_page * page, min(S, last_page * page)
    if first_page < 0 or last_page * page - page >= S or t0 >= t1:
        raise ValueError("page range must cover valid tokens")
    _ops.quest_page_minmax_into(k[:, :, t0:t1], page, kmin[:, :, first_page:last_page],
                                kmax[:, :, first_page:last_page])


def quest_select_decode(q, kmin, kmax, S, kb, page, scaling):
    """Quest selection from per-KV-head metadata: q [B,H_q,1,D] -> idx [B,H_q,npick*page]."""
    return _ops.quest_select(q[:, :, 0, :], kmin, kmax, S, kb, page, scaling)


def attend_topk(q_blk, k_r, v, idx, q_pos, scaling):
    """Exact softmax attention over the selected keys of each query row.

    ref: benchmarks/sparse_attention.py:367-387: a position is used when it is causal for its
    row (idx <= q_pos) and inside [0, S); duplicate indices count once per occurrence; a row
    with no usable position gives NaN, like the reference's softmax over -inf. q_blk
    [B,Hq,Qc,D]; k_r, v [B,Hq,S,D] (per query head); idx [B,Hq,Qc,ksel] -> [B,Hq,Qc,D] in
    v.dtype.
    """
    B, Hq, Qc, D = q_blk.shape
    S = k_r.shape[2]
    q3 = _fold(q_blk)
    ksel = idx.shape[-1]
    if _is_decode_row(q_blk, q_pos, S):
        idx3 = idx.reshape(B, Hq * Qc, ksel)
    else:
        pos = _positions(q_pos, Qc, idx.device)
        ok = (idx <= pos[None, None, :, None]) & (idx < S) & (idx >= 0)
        idx3 = torch.where(ok, idx, torch.full_like(idx, -1)).reshape(B, Hq * Qc, ksel)
    odt = v.dtype if v.dtype in (torch.bfloat16, torch.float16, torch.float32) else torch.float32
    out = torch.empty(B, Hq * Qc, D, dtype=odt, device=q3.device)
    kk, vv = k_r, v
    if kk.dtype not in (torch.bfloat16, torch.float16, torch.float32, torch.float8_e4m3fn) or kk.dtype != vv.dtype:
        kk, vv = kk.float(), vv.float()
    _ops.gather_attn(q3, kk, vv, idx3, scaling, out)
    return out.to(v.dtype).view(B, Hq, Qc, D)


def sparse_attention_chunked(q_r, k_r, v, sel_override, selector, frac, n_kv_groups, scaling, page=16, q_chunk=256,
                             k_chunk=2048, generator=None, local_w=0):
    """Chunked sparse attention over a prefill window (every position is a query): per chunk
    of q_chunk query rows, select the top-kb causal keys (kb = max(1, round(frac*S))) and
    attend over them exactly.

    ref: benchmarks/sparse_attention.py:463-497. q_r [B,Hq,S,D]; k_r, v [B,Hk,S,D] ->
    [B,Hq,S,D]. Selectors as ``select_topk``; the soft selectors rank by ``sel_override``
    [B,Hk,S,D] (approximate keys) when it is given, otherwise by the exact keys. The
    global keep-set selectors ('h2o', 'snapkv') and the SDPA 'dense' route are not built.
    """
    if selector not in ("exact", "quest", "sparq", "recent", "random") + SOFT_SELECTORS:
        raise ValueError(f"selector {selector!r} is not on the decode hot path")
    B, Hq, S, D = q_r.shape
    kb = max(1, int(round(frac * S)))
    kfull = repeat_kv(k_r, n_kv_groups)
    vfull = repeat_kv(v, n_kv_groups)
    sel_keys = repeat_kv(sel_override, n_kv_groups) if selector in SOFT_SELECTORS and sel_override is not None \
        else kfull
    out = torch.empty_like(q_r)
    for q0 in range(0, S, q_chunk):
        q1 = min(q0 + q_chunk, S)
        q_blk = q_r[:, :, q0:q1, :]
        q_pos = torch.arange(q0, q1, device=q_r.device)
        idx = select_topk(selector, q_blk, sel_keys, q_pos, S, kb, k_chunk, scaling, page=page, generator=generator,
                          local_w=local_w)
        out[:, :, q0:q1, :] = attend_topk(q_blk, kfull, vfull, idx, q_pos, scaling)
    return out
