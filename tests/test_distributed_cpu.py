"""Host-side logic of the multi-GPU paths on CPU ranks (gloo, world_size 2).

The split-KV exchange (pack partials, all-gather, merge) runs exactly as on GPUs; the
per-shard partials and the merge come from the CPU oracle because the CUDA kernels need
a device. The batch-shard ranges are checked for coverage and balance.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from bytes_b200 import distributed as bdist


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _oracle_partial(q, k, v, scaling):
    m, l, o = oracle.split_partials(q, k, v, scaling, 1)
    return m[0], l[0], o[0] * l[0].unsqueeze(-1)  # un-normalised numerator


def _oracle_merge(m_all, l_all, o_all, out_dtype):
    o_norm = o_all / l_all.unsqueeze(-1)
    return oracle.lse_combine(m_all, l_all, o_norm).to(out_dtype).unsqueeze(2)


def _worker(rank, world, port, q, k, v, ref, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        S = k.shape[2]
        s0, s1 = bdist.shard_range(S, rank, world)
        out = bdist.split_kv_decode(q, k[:, :, s0:s1], v[:, :, s0:s1], 0.125, partial_fn=_oracle_partial,
                                    merge_fn=_oracle_merge, out_dtype=torch.float32)
        result_q.put((rank, (out - ref).abs().max().item()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_split_kv_exchange_gloo(world):
    g = torch.Generator().manual_seed(0)
    q = torch.randn(2, 8, 1, 64, generator=g)
    k = torch.randn(2, 2, 301, 64, generator=g)
    v = torch.randn(2, 2, 301, 64, generator=g)
    ref = oracle.decode_attn_dense(q, k, v, 0.125, out_dtype=torch.float32)
    ctx = mp.get_context("spawn")
    rq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, k, v, ref, rq)) for r in range(world)]
    for p in procs:
        p.start()
    res = [rq.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err in res:
        assert err < 1e-5, (rank, err)


def test_shard_range_covers_everything():
    for n in (1, 7, 64, 1000003):
        for world in (1, 2, 3, 8):
            spans = [bdist.shard_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


def _oracle_gather_partial(q, k_shard, v_shard, idx_local, scaling):
    """(m, l, o) of gather-attend over this shard's positions (-1 skipped), o un-normalised."""
    B, Hq, _, D = q.shape
    Hk, S = k_shard.shape[1], k_shard.shape[2]
    G = Hq // Hk
    ii = idx_local.long()
    valid = (ii >= 0) & (ii < S)
    gi = ii.clamp(0, max(S - 1, 0))
    kr = k_shard.float().repeat_interleave(G, dim=1)
    vr = v_shard.float().repeat_interleave(G, dim=1)
    ks = torch.gather(kr, 2, gi.unsqueeze(-1).expand(*gi.shape, D))
    vs = torch.gather(vr, 2, gi.unsqueeze(-1).expand(*gi.shape, D))
    sc = (q.float()[:, :, 0, None, :] * ks).sum(-1) * scaling
    sc = torch.where(valid, sc, torch.full_like(sc, float("-inf")))
    m = sc.amax(-1)
    msafe = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    p = torch.exp(sc - msafe.unsqueeze(-1))
    return m, p.sum(-1), (p.unsqueeze(-1) * vs).sum(2)


def _oracle_merge_raw(m_all, l_all, o_all, out_dtype):
    M = m_all.amax(0)
    w = torch.where(torch.isfinite(m_all), torch.exp(m_all - M), torch.zeros_like(m_all))
    return ((o_all * w.unsqueeze(-1)).sum(0) / (l_all * w).sum(0).unsqueeze(-1)).to(out_dtype).unsqueeze(2)


def _sparse_worker(rank, world, port, q, k, v, kb, ref, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        S = k.shape[2]
        s0, s1 = bdist.shard_range(S, rank, world)
        out = bdist.split_kv_sparse_decode(
            q, k[:, :, s0:s1], v[:, :, s0:s1], kb, 0.125, s0, S,
            score_fn=lambda qq, kk, sc: oracle.sparse_score_scalar(qq, kk, sc),
            topk_fn=oracle.topk_lower_index, partial_fn=_oracle_gather_partial, merge_fn=_oracle_merge_raw,
            out_dtype=torch.float32)
        result_q.put((rank, (out - ref).abs().max().item()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,kb", [(2, 37), (3, 200)])
def test_split_kv_sparse_topk_exchange_gloo(world, kb):
    """Cross-shard exact top-kb: per-shard top-kb, all-gather of (value, position), the
    same global pick on every rank (ties: lower position), gather partials merged. Equal
    to the single-device pipeline, including ties that straddle shard boundaries."""
    g = torch.Generator().manual_seed(1)
    q = torch.randn(2, 8, 1, 64, generator=g)
    k = torch.randn(2, 2, 301, 64, generator=g)
    v = torch.randn(2, 2, 301, 64, generator=g)
    k[:, :, 250] = k[:, :, 10]  # equal scores in different shards
    k[:, :, 140] = k[:, :, 160]
    scores = oracle.sparse_score_scalar(q, k, 0.125)
    _, idx = oracle.topk_lower_index(scores, kb)
    ref = oracle.sparse_gather_attn(q, k, v, idx, 0.125).float()
    ctx = mp.get_context("spawn")
    rq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sparse_worker, args=(r, world, port, q, k, v, kb, ref, rq)) for r in range(world)]
    for p in procs:
        p.start()
    res = [rq.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err in res:
        assert err < 1e-5, (rank, err)


def test_global_topk_merge_tie_order():
    vals = torch.tensor([[[[3., 2., 2.]]], [[[3., 2., 1.]]]])  # [n=2, B=1, Hq=1, kc=3]
    pos = torch.tensor([[[[40, 7, 9]]], [[[5, 3, 80]]]])
    assert bdist.global_topk_merge(vals, pos, 4).tolist() == [[[5, 40, 3, 7]]]
