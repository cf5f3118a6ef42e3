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
