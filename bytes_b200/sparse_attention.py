"""Decode-shaped drop-in for the selection primitives of ``benchmarks/sparse_attention.py``.

The reference functions run over prefill windows (every position is a query); the hot
path here is decode: one query row per (batch, head) at position S-1, so every cached key
is causally valid. The functions accept the reference's arguments and raise if a call is
not decode-shaped.
"""
import torch

from . import _ops


def repeat_kv(x, n_rep):
    """[B,H_k,S,D] -> [B,H_k*n_rep,S,D]. ref: benchmarks/sparse_attention.py:85-90."""
    if n_rep == 1:
        return x
    B, H, S, D = x.shape
    return x[:, :, None, :, :].expand(B, H, n_rep, S, D).reshape(B, H * n_rep, S, D)


def _decode_row(q_blk, q_pos, S):
    if q_blk.shape[2] != 1:
        raise ValueError("decode-shaped: q_blk must hold one query row")
    if q_pos is not None and int(torch.as_tensor(q_pos).reshape(-1)[-1]) != S - 1:
        raise ValueError("decode-shaped: the query must sit at position S-1")


def select_topk(selector, q_blk, sel_keys, q_pos, S, kb, k_chunk, scaling, page=16, generator=None, local_w=0):
    """Top-kb key indices of one decode row: 'exact' (q.k scores) or 'quest' (page bounds).

    ref: benchmarks/sparse_attention.py:226-325. Returns [B,Hq,1,kb] int64; slots beyond
    S hold the sentinel S like the reference. Exact selection breaks ties by lower index
    (the reference's streaming merge keeps the earlier candidate first as well).
    """
    _decode_row(q_blk, q_pos, S)
    if selector == "quest":
        return _quest_select(q_blk, sel_keys, q_pos, S, kb, page, scaling, local_w)
    if selector != "exact":
        raise ValueError(f"selector {selector!r} is not on the decode hot path")
    if local_w:
        raise ValueError("local_w is not supported for exact decode selection")
    B, Hq, _, D = q_blk.shape
    keys = sel_keys[:, :, :S]
    q3 = q_blk[:, :, 0, :]
    # scores in fp32 from the unrounded inputs, like the reference's fp32 score tiles
    # (bf16 query and keys on the tensor cores, where every product is exact)
    if keys.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        keys = keys.float()
    if q3.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        q3 = q3.float()
    scores = _ops.sparse_score(q3, keys, None, None, scaling, 16, 32)
    kk = min(kb, S)
    _, idx = _ops.topk(scores, kk, sorted=True, want_values=False)
    if kb > kk:
        idx = torch.cat([idx, torch.full((B, Hq, kb - kk), S, dtype=idx.dtype, device=idx.device)], -1)
    return idx.unsqueeze(2)


def _quest_select(q_blk, k_r, pos, S, kb, page, scaling, local_w=0):
    """Quest page selection for one decode row (per-query-head keys k_r [B,Hq,S,D]).

    ref: benchmarks/sparse_attention.py:328-364. Returns [B,Hq,1,npick*page] int64,
    pages ordered by bound (lower page wins ties), indices clamped to S-1.
    """
    _decode_row(q_blk, pos, S)
    kmin, kmax = _ops.quest_page_minmax(k_r[:, :, :S], page)
    force = None
    if local_w > 0:
        force = max(0, S - local_w) // page
    idx = _ops.quest_select(q_blk[:, :, 0, :], kmin, kmax, S, kb, page, scaling, force)
    return idx.unsqueeze(2)


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
    """Exact softmax attention over selected keys of one decode row.

    ref: benchmarks/sparse_attention.py:367-387: indices >= S are masked; duplicate
    indices count once per occurrence. q_blk [B,Hq,1,D]; k_r, v [B,Hq,S,D] (per query
    head); idx [B,Hq,1,ksel] -> [B,Hq,1,D] in v.dtype.
    """
    S = k_r.shape[2]
    _decode_row(q_blk, q_pos, S)
    q3 = q_blk[:, :, 0, :]
    odt = v.dtype if v.dtype in (torch.bfloat16, torch.float16, torch.float32) else torch.float32
    out = torch.empty(q3.shape, dtype=odt, device=q3.device)
    kk, vv = k_r, v
    if kk.dtype not in (torch.bfloat16, torch.float16, torch.float32, torch.float8_e4m3fn) or kk.dtype != vv.dtype:
        kk, vv = kk.float(), vv.float()
    if q3.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        q3 = q3.float()
    _ops.gather_attn(q3, kk, vv, idx[:, :, 0, :], scaling, out)
    return out.to(v.dtype).unsqueeze(2)
