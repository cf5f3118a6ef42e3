"""Multi-GPU decode: batch sharding and split-KV of one long sequence across ranks.

One process per GPU (torch.distributed, NCCL over NVLink/NVSwitch).

* Batch sharding needs no collective: rank r owns sequences [r*B/n, (r+1)*B/n) and their
  whole KV cache; ``shard_range`` gives the slice.
* Split-KV for a context too long for one GPU: rank r holds keys/values of tokens
  [r*S/n, (r+1)*S/n). Each rank computes its shard's per-head (max, sum, numerator)
  partials with one split-KV kernel, the ranks all-gather those partials (B*Hq*(D+2)
  floats per rank, ~14.6 KB for 28 heads x 128 dims), and every rank merges them with a
  log-sum-exp combine kernel, so all ranks end with the full attention output. The
  all-gather is NCCL's, or (``PeerExchange``) peer stores over NVLink done by the same
  kernel that merges this rank's splits and combines the ranks' partials.
* Exact top-k sparse decode over such a sharded sequence: each rank scores its shard and
  keeps its own top-kb (value, global position) pairs; one all-gather of those pairs lets
  every rank pick the same global top-kb (value descending, lower position first on
  ties — the single-GPU rule, since the union of the shard top-kb sets holds the global
  top-kb); each rank gather-attends over the winners inside its shard and one more
  all-gather of (max, sum, numerator) partials feeds the same combine.

The reference is single-GPU; this module has no counterpart there. The merge is the same
online-softmax identity its kernels apply across key blocks
(src/attention_kernels.py:45-59 of saifmb0/bytes).
"""
import torch

from . import _ops


def shard_range(n_items, rank, world):
    """Contiguous [start, stop) of n_items owned by `rank` (sizes differ by at most one)."""
    base, extra = divmod(n_items, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def split_kv_partials(q, k_shard, v_shard, scaling):
    """(m, l, o) of this rank's key shard: m,l [B,Hq] and o [B,Hq,D] fp32 (o un-normalised)."""
    if q.dim() == 4:
        q = q[:, :, 0, :]
    return _ops.decode_attn_partial(q, k_shard, v_shard, scaling)


def merge_partials(m_all, l_all, o_all, out_dtype=torch.bfloat16):
    """m_all,l_all [n,B,Hq], o_all [n,B,Hq,D] -> [B,Hq,1,D] (log-sum-exp combine kernel)."""
    return _ops.lse_combine(m_all, l_all, o_all, out_dtype).unsqueeze(2)


class PeerExchange:
    """Split-KV across the ranks of `group` over NVLink peer memory, for a fixed (B, Hq, D).

    ``decode(q, k_shard, v_shard, scaling)`` is the whole step in two launches: the dense
    split pass over this rank's shard, then one kernel that merges its splits, stores the
    merged (max, sum, numerator) into every rank's buffer, raises a per-step flag on each,
    waits (bounded) for all ranks and writes the log-sum-exp combine
    (``bd_split_kv_decode_peer``). ``__call__(m, l, o)`` runs the exchange kernel alone on
    partials the caller computed (``bd_peer_exchange_combine``). The buffers are one
    symmetric allocation (``torch.distributed._symmetric_memory``) mapped on every GPU of the
    group; building the object is collective. Every rank must make the same calls, one per
    step, on the current stream; the step counters live in the buffer, so the calls can be
    captured in a CUDA graph. Raises if symmetric memory is unavailable (use the NCCL
    all-gather of ``split_kv_decode`` then).
    """

    def __init__(self, B, Hq, D, device, group=None):
        import ctypes
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem
        from . import _native as N
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.B, self.Hq, self.D = B, Hq, D
        f = N.lib().bd_peer_exchange_buffer_bytes
        f.restype = ctypes.c_size_t
        f.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int]
        nbytes = int(f(B * Hq, D, self.world))
        if nbytes == 0:
            raise ValueError("peer exchange needs a non-empty problem")
        self.buf = symm_mem.empty(nbytes // 4, dtype=torch.float32, device=device)
        self.buf.zero_()
        grp = group if group is not None else dist.group.WORLD
        self.hdl = symm_mem.rendezvous(self.buf, grp)
        self.peers_dev = int(self.hdl.buffer_ptrs_dev)
        torch.cuda.synchronize(device)
        dist.barrier(group=group)  # every rank's buffer is zero before any rank writes

    def _check(self, B, Hq, D):
        if (B, Hq, D) != (self.B, self.Hq, self.D):
            raise ValueError(f"PeerExchange built for {(self.B, self.Hq, self.D)}, called with {(B, Hq, D)}")

    def __call__(self, m, l, o, out_dtype=torch.bfloat16):
        """m, l [B, Hq], o [B, Hq, D] fp32 (this rank's shard) -> [B, Hq, D] combined."""
        self._check(*o.shape)
        return _ops.peer_exchange_combine(m, l, o, self.peers_dev, self.rank, self.world, out_dtype)

    def decode(self, q, k_shard, v_shard, scaling, out_dtype=torch.bfloat16):
        """q [B, Hq, 1, D] or [B, Hq, D]; k, v [B, Hk, S_r, D] this rank's shard -> [B, Hq, D]."""
        q3 = q[:, :, 0, :] if q.dim() == 4 else q
        self._check(*q3.shape)
        return _ops.split_kv_decode_peer(q3, k_shard, v_shard, scaling, self.peers_dev, self.rank, self.world,
                                         out_dtype)


def split_kv_decode(q, k_shard, v_shard, scaling, group=None, partial_fn=None, merge_fn=None,
                    out_dtype=torch.bfloat16, exchange=None):
    """Attention of q over a sequence sharded along its tokens across the ranks of `group`.

    Every rank passes its own contiguous token shard; every rank returns the full output
    [B,Hq,1,D]. One all-gather of the partials is the only communication: NCCL, or, with
    ``exchange`` (a PeerExchange for these shapes), NVLink peer stores fused with the split
    merge and the combine in one kernel behind the split pass.
    `partial_fn` / `merge_fn` default to the CUDA kernels; they are parameters so the
    host-side exchange can be exercised on CPU ranks.
    """
    import torch.distributed as dist
    if exchange is not None and partial_fn is None:
        return exchange.decode(q, k_shard, v_shard, scaling, out_dtype).unsqueeze(2)
    partial_fn = partial_fn or split_kv_partials
    merge_fn = merge_fn or merge_partials
    m, l, o = partial_fn(q, k_shard, v_shard, scaling)
    if exchange is not None:
        return exchange(m, l, o, out_dtype).unsqueeze(2)
    world = dist.get_world_size(group)
    B, Hq, D = o.shape
    packed = torch.cat([m.reshape(-1), l.reshape(-1), o.reshape(-1)]).contiguous()
    parts = [torch.empty_like(packed) for _ in range(world)]
    dist.all_gather(parts, packed, group=group)
    g = torch.stack(parts)
    n_ml = B * Hq
    m_all = g[:, :n_ml].reshape(world, B, Hq)
    l_all = g[:, n_ml:2 * n_ml].reshape(world, B, Hq)
    o_all = g[:, 2 * n_ml:].reshape(world, B, Hq, D)
    return merge_fn(m_all, l_all, o_all, out_dtype)


def _shard_scores(q, k_shard, scaling):
    from . import attention_kernels as ak
    return ak.sparse_score_scalar(q if q.dim() == 4 else q.unsqueeze(2), k_shard, scaling, score_bits=16)


def _shard_topk(scores, k):
    return _ops.topk(scores, k, sorted=True, want_values=True, idx_dtype=torch.int64)


def _shard_gather_partial(q, k_shard, v_shard, idx_local, scaling):
    if q.dim() == 4:
        q = q[:, :, 0, :]
    return _ops.gather_attn_partial(q, k_shard, v_shard, idx_local, scaling)


def global_topk_merge(vals_all, pos_all, kb):
    """Top-kb of per-shard candidates: vals_all, pos_all [n, B, Hq, kc] (pos global) ->
    pos [B, Hq, kb], ordered by value descending, lower position first among equals."""
    n, B, Hq, kc = vals_all.shape
    v = vals_all.permute(1, 2, 0, 3).reshape(B, Hq, n * kc)
    p = pos_all.permute(1, 2, 0, 3).reshape(B, Hq, n * kc)
    # stable two-key order: sort by position, then stably by value descending
    order = torch.argsort(p, dim=-1, stable=True)
    v, p = torch.gather(v, -1, order), torch.gather(p, -1, order)
    order = torch.argsort(v, dim=-1, descending=True, stable=True)
    return torch.gather(p, -1, order)[..., :kb]


def split_kv_sparse_decode(q, k_shard, v_shard, kb, scaling, shard_start, seq_len, group=None, score_fn=None,
                           topk_fn=None, partial_fn=None, merge_fn=None, out_dtype=torch.bfloat16):
    """Exact top-kb sparse decode of q over a sequence sharded along its tokens.

    Every rank passes its own contiguous token shard starting at global position
    `shard_start` (of `seq_len`); every rank returns the full output [B,Hq,1,D], equal to
    the single-GPU pipeline (scores -> top-kb -> gather-attend) over the whole sequence.
    Two all-gathers: B*Hq*kb (value, position) pairs, then B*Hq*(D+2) partial floats.
    The four kernel steps are parameters so the exchange runs on CPU ranks too.
    """
    import torch.distributed as dist
    score_fn = score_fn or _shard_scores
    topk_fn = topk_fn or _shard_topk
    partial_fn = partial_fn or _shard_gather_partial
    merge_fn = merge_fn or merge_partials
    world = dist.get_world_size(group)
    S_loc = k_shard.shape[2]
    kc = min(kb, S_loc)
    scores = score_fn(q, k_shard, scaling)  # [B, Hq, S_loc] fp32
    vals, idx = topk_fn(scores, kc)
    pos = idx.long() + shard_start
    B, Hq = vals.shape[:2]
    # shards shorter than kb pad with -inf / sentinel positions that never win
    if kc < kb:
        pad = kb - kc
        vals = torch.cat([vals.float(), vals.new_full((B, Hq, pad), float("-inf"), dtype=torch.float32)], -1)
        pos = torch.cat([pos, pos.new_full((B, Hq, pad), seq_len)], -1)
    vals_all = [torch.empty_like(vals, dtype=torch.float32) for _ in range(world)]
    pos_all = [torch.empty_like(pos) for _ in range(world)]
    dist.all_gather(vals_all, vals.float().contiguous(), group=group)
    dist.all_gather(pos_all, pos.contiguous(), group=group)
    win = global_topk_merge(torch.stack(vals_all), torch.stack(pos_all), kb)  # [B, Hq, kb] global
    local = win - shard_start
    local = torch.where((local >= 0) & (local < S_loc), local, torch.full_like(local, -1))
    m, l, o = partial_fn(q, k_shard, v_shard, local, scaling)
    D = o.shape[-1]
    flat = torch.cat([m.reshape(-1), l.reshape(-1), o.reshape(-1)]).contiguous()
    parts = [torch.empty_like(flat) for _ in range(world)]
    dist.all_gather(parts, flat, group=group)
    g = torch.stack(parts)
    n_ml = B * Hq
    return merge_fn(g[:, :n_ml].reshape(world, B, Hq), g[:, n_ml:2 * n_ml].reshape(world, B, Hq),
                    g[:, 2 * n_ml:].reshape(world, B, Hq, D), out_dtype)
