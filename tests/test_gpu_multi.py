"""Multi-GPU split-KV decode over NCCL and NVLink peer memory (one process per GPU, world size 2).

Skipped on boxes with fewer than two GPUs. Each rank holds a contiguous token shard of one
long sequence; the dense split-KV exchange (NCCL all-gather, and peer stores fused with the
combine) and the exact top-k sparse exchange must give every rank the single-GPU result. Ranks use a short process-group timeout so a failure
ends with an error instead of a wait.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs():
    g = torch.Generator().manual_seed(3)
    B, Hq, Hk, S, D = 2, 8, 2, 3000, 128
    q = torch.randn(B, Hq, 1, D, generator=g).bfloat16()
    k = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    v = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    return q, k, v


def _steps_done(ex):
    """Fewest steps any row's counter recorded (counters [rows] u32 follow the records
    [2][world][rows][D+4] f32 and flags [2][world][rows] u32 in the exchange buffer)."""
    rows = ex.B * ex.Hq
    at = 2 * ex.world * rows * (ex.D + 4) + 2 * ex.world * rows
    return int(ex.buf[at:at + rows].view(torch.int32).min().item())


def _worker(rank, world, port, result_q):
    import torch.distributed as dist
    import oracle
    from bytes_b200 import attention_kernels as ak
    from bytes_b200 import distributed as bdist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        dev = torch.device("cuda", rank)
        q, k, v = (t.to(dev) for t in _inputs())
        S, sc, kb = k.shape[2], 0.088, 150
        s0, s1 = bdist.shard_range(S, rank, world)
        ks, vs = k[:, :, s0:s1].contiguous(), v[:, :, s0:s1].contiguous()
        dense = bdist.split_kv_decode(q, ks, vs, sc)
        # the NVLink peer-memory exchange: four steps cover both buffer parities
        ex = bdist.PeerExchange(q.shape[0], q.shape[1], q.shape[3], dev)
        peer = [bdist.split_kv_decode(q, ks, vs, sc, exchange=ex) for _ in range(3)]
        peer.append(ex(*bdist.split_kv_partials(q, ks, vs, sc)).unsqueeze(2))  # exchange of given partials
        sparse = bdist.split_kv_sparse_decode(q, ks, vs, kb, sc, s0, S)
        ref_dense = oracle.decode_attn_dense(q.cpu(), k.cpu(), v.cpu(), sc, out_dtype=torch.float32).to(dev)
        _, idx = ak.topk(ak.sparse_score_scalar(q, k, sc, score_bits=16), kb, sorted=True)
        ref_sparse = ak.sparse_gather_attn(q, k, v, idx, sc)
        torch.cuda.synchronize()
        result_q.put((rank, (dense.float() - ref_dense.float()).abs().max().item(),
                      (sparse.float() - ref_sparse.float()).abs().max().item(),
                      max((p.float() - dense.float()).abs().max().item() for p in peer),
                      _steps_done(ex)))
        ex.buf = None
    finally:
        dist.destroy_process_group()


def test_split_kv_dense_and_sparse_over_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    rq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, rq)) for r in range(world)]
    for p in procs:
        p.start()
    res = [rq.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, e_dense, e_sparse, e_peer, steps in res:
        # both exchanges combine the same partials; bf16 outputs may differ by one rounding
        assert e_peer < 1e-2, (rank, e_peer)
        assert steps == 4
        # bf16 outputs against an fp32 oracle (dense) and the single-GPU kernels (sparse)
        assert e_dense < 2e-2, (rank, e_dense)
        assert e_sparse < 1e-2, (rank, e_sparse)
