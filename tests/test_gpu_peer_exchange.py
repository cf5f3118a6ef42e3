"""The NVLink peer-memory split-KV exchange kernel (bd_peer_exchange_combine) on one GPU.

The kernel is one rank's side of the exchange: it stores this rank's (max, sum, numerator)
partials into every rank's buffer, raises its step flag there and waits for the other
ranks' flags in its own buffer. On one GPU the other rank is emulated by the test: its
partials and flag are written into rank 0's buffer before the call, so the kernel never
waits on another kernel. Checked: the combine equals the log-sum-exp combine kernel over
the same partials, rank 0's partials and flag land in the peer's buffer, the step counter
advances through both buffer parities (also when replayed from a CUDA graph), and a flag
that nothing raises ends the wait after its time limit with a NaN output and a counted
timeout (in a child process, so this session's timeout count stays zero).
"""
import ctypes
import math

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _layout(rows, D, world):
    """Buffer bytes; records [2][world][rows][D+4] f32, flags [2][world][rows] u32, counters [rows] u32."""
    from bytes_b200 import _native as N
    f = N.lib().bd_peer_exchange_buffer_bytes
    f.restype = ctypes.c_size_t
    f.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int]
    nbytes = int(f(rows, D, world))
    words = 2 * world * rows * (D + 4) + 2 * world * rows + rows
    assert nbytes == (words * 4 + 15) // 16 * 16
    return nbytes


def _partials(B, Hq, D, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    m = torch.randn(B, Hq, device=dev, generator=g) * 3
    l = torch.rand(B, Hq, device=dev, generator=g) * 50 + 1
    o = torch.randn(B, Hq, D, device=dev, generator=g) * 10
    return m, l, o


class _Emulated:
    """Rank 0 of a world-2 exchange on one GPU; the test plays rank 1."""

    def __init__(self, B, Hq, D, dev, world=2):
        self.B, self.Hq, self.D, self.world = B, Hq, D, world
        self.rows = B * Hq
        nbytes = _layout(self.rows, D, world)
        self.bufs = [torch.zeros(nbytes // 4, dtype=torch.float32, device=dev) for _ in range(world)]
        self.peers = torch.tensor([b.data_ptr() for b in self.bufs], dtype=torch.int64, device=dev)

    def records(self, buf, par, r):
        """[B, Hq, D + 4] view of slot [par][r] of buffer `buf`: o[D], m, l, 0, 0 per row."""
        n = self.rows * (self.D + 4)
        base = (par * self.world + r) * n
        return self.bufs[buf][base:base + n].view(self.B, self.Hq, self.D + 4)

    def words(self, buf):
        return self.bufs[buf][2 * self.world * self.rows * (self.D + 4):].view(torch.int32)

    def flags(self, buf, par, r):
        base = (par * self.world + r) * self.rows
        return self.words(buf)[base:base + self.rows]

    def counters(self, buf=0):
        base = 2 * self.world * self.rows
        return self.words(buf)[base:base + self.rows]

    def play_rank(self, r, step, m, l, o):
        rec = self.records(0, step & 1, r)
        rec[..., :self.D].copy_(o)
        rec[..., self.D].copy_(m)
        rec[..., self.D + 1].copy_(l)
        self.flags(0, step & 1, r).fill_(step)

    def call(self, m, l, o, dtype=torch.float32):
        from bytes_b200 import _ops
        return _ops.peer_exchange_combine(m, l, o, self.peers.data_ptr(), 0, self.world, dtype)


def _expected(parts, dtype=torch.float32):
    from bytes_b200 import _ops
    m = torch.stack([p[0] for p in parts])
    l = torch.stack([p[1] for p in parts])
    o = torch.stack([p[2] for p in parts])
    return _ops.lse_combine(m, l, o, dtype)


def test_world1_self_exchange(cuda):
    """One rank: the combine is o / l."""
    B, Hq, D = 2, 8, 128
    ex = _Emulated(B, Hq, D, cuda, world=1)
    for step in (1, 2, 3):
        m, l, o = _partials(B, Hq, D, step, cuda)
        got = ex.call(m, l, o)
        torch.testing.assert_close(got, o / l.unsqueeze(-1), rtol=1e-5, atol=1e-5)
        assert bool((ex.counters() == step).all())


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_emulated_two_ranks_matches_lse_combine(cuda, dtype):
    B, Hq, D = 1, 28, 128
    ex = _Emulated(B, Hq, D, cuda)
    for step in (1, 2, 3, 4):
        mine = _partials(B, Hq, D, 100 + step, cuda)
        other = _partials(B, Hq, D, 200 + step, cuda)
        ex.play_rank(1, step, *other)
        got = ex.call(*mine, dtype=dtype)
        want = _expected([mine, other], dtype)
        tol = dict(rtol=1e-5, atol=1e-5) if dtype == torch.float32 else dict(rtol=1e-2, atol=1e-2)
        torch.testing.assert_close(got, want, **tol)
        # rank 0's partials and flag were stored into rank 1's buffer, in this step's parity
        par = step & 1
        rec = ex.records(1, par, 0)
        assert torch.equal(rec[..., ex.D], mine[0]) and torch.equal(rec[..., ex.D + 1], mine[1])
        assert torch.equal(rec[..., :ex.D], mine[2])
        assert bool((ex.flags(1, par, 0) == step).all()) and bool((ex.flags(0, par, 0) == step).all())
        assert bool((ex.counters() == step).all())


def test_emulated_two_ranks_with_masked_shard(cuda):
    """A shard with no keys (max -inf, sum 0) contributes nothing."""
    B, Hq, D = 2, 4, 64
    ex = _Emulated(B, Hq, D, cuda)
    mine = _partials(B, Hq, D, 7, cuda)
    empty = (torch.full((B, Hq), -math.inf, device=cuda), torch.zeros(B, Hq, device=cuda),
             torch.zeros(B, Hq, D, device=cuda))
    ex.play_rank(1, 1, *empty)
    got = ex.call(*mine)
    torch.testing.assert_close(got, mine[2] / mine[1].unsqueeze(-1), rtol=1e-5, atol=1e-5)


def test_emulated_two_ranks_graph_replay(cuda):
    """The step counter lives in device memory: a captured call advances it on every replay."""
    B, Hq, D = 1, 28, 128
    ex = _Emulated(B, Hq, D, cuda)
    mine_in = [torch.empty(B, Hq, device=cuda), torch.empty(B, Hq, device=cuda), torch.empty(B, Hq, D, device=cuda)]
    # warm-up call outside the graph (step 1), then capture
    first = _partials(B, Hq, D, 1, cuda)
    for t, x in zip(mine_in, first):
        t.copy_(x)
    ex.play_rank(1, 1, *_partials(B, Hq, D, 2, cuda))
    ex.call(*mine_in)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = ex.call(*mine_in)
    for step in (2, 3, 4, 5):
        mine = _partials(B, Hq, D, 10 * step, cuda)
        other = _partials(B, Hq, D, 10 * step + 1, cuda)
        for t, x in zip(mine_in, mine):
            t.copy_(x)
        ex.play_rank(1, step, *other)
        g.replay()
        torch.testing.assert_close(out, _expected([mine, other]), rtol=1e-5, atol=1e-5)
        assert bool((ex.counters() == step).all())
    del g


def _split_case(seed, S0, S1, dev, kv_dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    B, Hq, Hk, D = 2, 28, 4, 128
    q = torch.randn(B, Hq, D, generator=g).bfloat16()
    k = torch.randn(B, Hk, S0 + S1, D, generator=g)
    v = torch.randn(B, Hk, S0 + S1, D, generator=g)
    k, v = k.to(kv_dtype), v.to(kv_dtype)
    return q.to(dev), k.to(dev), v.to(dev)


@pytest.mark.parametrize("S0,S1", [(1700, 1300), (0, 2048), (4096, 64)])
def test_split_kv_decode_peer_emulated(cuda, S0, S1):
    """The whole step (dense split pass + fused exchange) on rank 0's shard, rank 1's merged
    partials written by the test: equals decode over the whole sequence."""
    import oracle
    from bytes_b200 import _ops
    q, k, v = _split_case(S0 + 7 * S1, S0, S1, cuda)
    B, Hq, D = q.shape
    sc = 1.0 / math.sqrt(D)
    ex = _Emulated(B, Hq, D, cuda)
    k0, v0 = k[:, :, :S0].contiguous(), v[:, :, :S0].contiguous()
    k1, v1 = k[:, :, S0:].contiguous(), v[:, :, S0:].contiguous()
    ref = oracle.decode_attn_dense(q.cpu().unsqueeze(2), k.cpu(), v.cpu(), sc, out_dtype=torch.float32)[:, :, 0]
    for step in (1, 2, 3):
        ex.play_rank(1, step, *_ops.decode_attn_partial(q, k1, v1, sc))
        got = _ops.split_kv_decode_peer(q, k0, v0, sc, ex.peers.data_ptr(), 0, 2, torch.float32)
        torch.testing.assert_close(got.cpu(), ref, rtol=2e-3, atol=2e-3)
        # rank 0's merged record, as stored into rank 1's buffer, is its shard partial
        rec = ex.records(1, step & 1, 0)
        m0, l0, o0 = _ops.decode_attn_partial(q, k0, v0, sc)
        if S0:
            torch.testing.assert_close(rec[..., ex.D], m0, rtol=1e-5, atol=1e-5)
            torch.testing.assert_close(rec[..., :ex.D] / rec[..., ex.D + 1:ex.D + 2], o0 / l0.unsqueeze(-1),
                                       rtol=1e-4, atol=1e-4)
        else:
            assert bool(torch.isneginf(rec[..., ex.D]).all()) and bool((rec[..., ex.D + 1] == 0).all())
        assert bool((ex.counters() == step).all())


def test_split_kv_decode_peer_fp8_graph(cuda):
    """fp8 e4m3 shards; the two launches captured once and replayed."""
    from bytes_b200 import _ops
    q, k, v = _split_case(5, 2048, 2048, cuda)
    k8, v8 = k.to(torch.float8_e4m3fn), v.to(torch.float8_e4m3fn)
    B, Hq, D = q.shape
    sc = 1.0 / math.sqrt(D)
    ex = _Emulated(B, Hq, D, cuda)
    k0, v0 = k8[:, :, :2048].contiguous(), v8[:, :, :2048].contiguous()
    k1, v1 = k8[:, :, 2048:].contiguous(), v8[:, :, 2048:].contiguous()
    part1 = _ops.decode_attn_partial(q, k1, v1, sc)
    whole = _ops.decode_attn(q, k8, v8, sc, torch.empty(B, Hq, D, device=cuda))  # one GPU, whole sequence
    ex.play_rank(1, 1, *part1)
    first = _ops.split_kv_decode_peer(q, k0, v0, sc, ex.peers.data_ptr(), 0, 2, torch.float32)
    torch.testing.assert_close(first, whole, rtol=1e-3, atol=1e-3)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = _ops.split_kv_decode_peer(q, k0, v0, sc, ex.peers.data_ptr(), 0, 2, torch.float32)
    for step in (2, 3):
        ex.play_rank(1, step, *part1)
        g.replay()
        torch.testing.assert_close(out, first, rtol=1e-6, atol=1e-6)
        assert bool((ex.counters() == step).all())
    del g


def test_rejects_bad_arguments(cuda):
    from bytes_b200 import _ops
    m, l, o = _partials(1, 6, 128, 0, cuda)
    peers = torch.zeros(2, dtype=torch.int64, device=cuda)
    with pytest.raises((ValueError, RuntimeError)):
        _ops.peer_exchange_combine(m, l, o[..., :126].contiguous(), peers.data_ptr(), 0, 2)  # D % 4
    with pytest.raises((ValueError, RuntimeError)):
        _ops.peer_exchange_combine(m, l, o, peers.data_ptr(), 2, 2)  # rank >= world
    with pytest.raises((ValueError, RuntimeError)):
        _ops.peer_exchange_combine(m, l, o, 0, 0, 2)  # no peer table


def _late_peer_child(q):
    """Rank 1 never raises its flag: the wait gives up after its limit (NaN output, one
    counted timeout); a later step whose flag is raised combines normally."""
    import time
    from bytes_b200 import _native as N
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = N.lib()
    f = lib.bd_wait_timeouts
    f.restype = ctypes.c_longlong
    B, Hq, D = 1, 8, 128
    ex = _Emulated(B, Hq, D, dev)
    mine = _partials(B, Hq, D, 1, dev)
    before = f()
    t0 = time.perf_counter()
    out = ex.call(*mine)
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    all_nan = bool(torch.isnan(out).all().item())
    after = f()
    other = _partials(B, Hq, D, 2, dev)
    ex.play_rank(1, 2, *other)
    out2 = ex.call(*mine)
    err = (out2 - _expected([mine, other])).abs().max().item()
    q.put((before, after, all_nan, waited, int(ex.counters().min().item()), err))


def test_wait_for_missing_peer_times_out(cuda):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_late_peer_child, args=(q,))
    p.start()
    before, after, all_nan, waited, counter, err = q.get(timeout=300)
    p.join(timeout=120)
    assert p.exitcode == 0
    assert before == 0 and after == 8  # one per row: B*Hq = 8 rows wait on their own
    assert all_nan
    assert 0.9 < waited < 10.0  # the wait limit is 1 s
    assert counter == 2
    assert err < 1e-4
