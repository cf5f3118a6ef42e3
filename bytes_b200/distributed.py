"""Multi-GPU decode: batch sharding and split-KV of one long sequence across ranks.

One process per GPU (torch.distributed, NCCL over NVLink/NVSwitch).

* Batch sharding needs no collective: rank r owns sequences [r*B/n, (r+1)*B/n) and their
  whole KV cache; ``shard_range`` gives the slice.
* Split-KV for a context too long for one GPU: rank r holds keys/values of tokens
  [r*S/n, (r+1)*S/n). Each rank computes its shard's per-head (max, sum, numerator)
  partials with one split-KV kernel, the ranks all-gather those partials (B*Hq*(D+2)
  floats per rank, ~14.6 KB for 28 heads x 128 dims), and every rank merges them with a
  log-sum-exp combine kernel, so all ranks end with the full attention output.

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


def split_kv_decode(q, k_shard, v_shard, scaling, group=None, partial_fn=None, merge_fn=None,
                    out_dtype=torch.bfloat16):
    """Attention of q over a sequence sharded along its tokens across the ranks of `group`.

    Every rank passes its own contiguous token shard; every rank returns the full output
    [B,Hq,1,D]. One all-gather of the partials is the only communication.
    `partial_fn` / `merge_fn` default to the CUDA kernels; they are parameters so the
    host-side exchange can be exercised on CPU ranks.
    """
    import torch.distributed as dist
    partial_fn = partial_fn or split_kv_partials
    merge_fn = merge_fn or merge_partials
    m, l, o = partial_fn(q, k_shard, v_shard, scaling)
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
