"""GPU parity for the sparse path: score-key packing (bit-exact), pass-1 scores, top-k
(bit-exact on identical scores, lower index wins ties), gather-attention, Quest page
selection and the end-to-end two-pass decode."""
import math

import pytest
import torch

import oracle
from bytes_b200 import _ops
from bytes_b200 import attention_kernels as ak
from bytes_b200 import sparse_attention as sa

pytestmark = pytest.mark.gpu


def gen(seed):
    return torch.Generator().manual_seed(seed)


def close(out, ref, max_abs=2e-2, mean_abs=1e-3):
    d = (out.float().cpu() - ref.float().cpu()).abs()
    assert torch.isfinite(out.float()).all()
    assert d.max().item() <= max_abs, f"max abs diff {d.max().item()}"
    assert d.mean().item() <= mean_abs, f"mean abs diff {d.mean().item()}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("bits", [2, 4])
def test_pack_score_keys_bit_exact(cuda, dtype, bits):
    g = gen(1)
    k = torch.randn(2, 3, 257, 128, generator=g).to(dtype)
    k[0, 0, 3, 32:64] = 0.75
    k[1, 2, 5, :] *= 40
    p, s, z = ak.quantize_and_pack_score_keys(k.to(cuda), bits, 32)
    rp, rs, rz = oracle.quantize_and_pack_score_keys(k, bits, 32)
    assert torch.equal(p.cpu(), rp) and torch.equal(s.cpu(), rs) and torch.equal(z.cpu(), rz)


def test_pack_score_keys_golden(cuda, golden_cuda):
    """Against the reference's packer run on a CUDA device (bit-exact)."""
    for c in golden_cuda["pack_score_keys"]:
        p, s, z = ak.quantize_and_pack_score_keys(c["k"].to(cuda), c["bits"], c["group_size"])
        assert torch.equal(p.cpu(), c["packed"])
        assert torch.equal(s.cpu(), c["scale"])
        assert torch.equal(z.cpu(), c["zero"])


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("bits", [16, 8, 4, 2])
def test_sparse_scores_match_oracle(cuda, D, bits):
    """Shapes of the reference test (test_correctness.py:673-723) plus a long ragged one."""
    for (B, Hq, Hk, S) in ((2, 8, 2, 128), (1, 28, 4, 3001)):
        g = gen(D * 100 + bits + S)
        q = torch.randn(B, Hq, 1, D, generator=g).bfloat16()
        k = torch.randn(B, Hk, S, D, generator=g).bfloat16()
        if bits == 16:
            out = ak.sparse_score_scalar(q.to(cuda), k.to(cuda), 0.125, score_bits=16)
            ref = oracle.sparse_score_scalar(q, k, 0.125)
        elif bits == 8:
            k8 = k.to(torch.float8_e4m3fn)
            out = ak.sparse_score_scalar(q.to(cuda), k8.to(cuda), 0.125, score_bits=8)
            ref = oracle.sparse_score_scalar(q, k8, 0.125)
        else:
            kp, sc, zr = oracle.quantize_and_pack_score_keys(k, bits, 32)
            out = ak.sparse_score_packed(q.to(cuda), kp.to(cuda), sc.to(cuda), zr.to(cuda), 0.125,
                                         score_bits=bits, group_size=32)
            ref = oracle.sparse_score_packed(q, kp, sc, zr, 0.125, bits, 32)
        assert out.shape == (B, Hq, S) and out.dtype == torch.float32
        assert torch.allclose(out.cpu(), ref, rtol=1e-4, atol=2e-4), (out.cpu() - ref).abs().max()


def _topk_check(scores, k, sorted_):
    dev = scores.cuda()
    v, i = ak.topk(dev, k, sorted=sorted_)
    rv, ri = oracle.topk_lower_index(scores, k)
    if sorted_:
        assert torch.equal(i.cpu(), ri)
        assert torch.equal(v.cpu(), rv)
    else:
        assert torch.equal(i.cpu(), ri.sort(-1).values)


@pytest.mark.parametrize("sorted_", [True, False])
def test_topk_bit_exact_with_ties(cuda, sorted_):
    g = gen(7)
    s = torch.randint(-50, 50, (64, 2048), generator=g).float()  # heavy ties
    s[0, :] = 3.0  # all equal
    s[1, ::3] = -0.0
    s[1, 1::3] = 0.0
    for k in (1, 7, 33, 64, 100, 1000, 2048):
        _topk_check(s, k, sorted_)
    assert oracle.topk_lower_index(torch.tensor([[1., 3., 3., 2., 3., 0.]]), 2)[1].tolist() == [[1, 2]]
    v, i = ak.topk(torch.tensor([[1., 3., 3., 2., 3., 0.]], device=cuda), 2)
    assert i.tolist() == [[1, 2]]


@pytest.mark.parametrize("n,k", [(32768, 1024), (65536, 655), (100, 100), (5, 3)])
def test_topk_random_rows(cuda, n, k):
    g = gen(n + k)
    s = torch.randn(16, n, generator=g)
    _topk_check(s, k, True)
    _topk_check(s, k, False)


@pytest.mark.parametrize("sorted_", [True, False])
def test_topk_threshold_bucket_overflow(cuda, sorted_):
    # three distinct values over 32768 keys: the threshold's first digit holds ~11K keys,
    # more than the candidate buffer, so the remaining digits are resolved on the whole row
    g = gen(5)
    s = torch.randint(0, 3, (4, 32768), generator=g).float()
    for k in ((1000, 4000) if sorted_ else (1000, 20000)):  # sorted output must fit shared memory
        _topk_check(s, k, sorted_)


@pytest.mark.parametrize("n", [1, 2047, 4096, 4097])
def test_topk_short_rows(cuda, n):
    """Row lengths around the short-row kernel's limit (4096 keys held in registers), odd
    lengths (element loads) and rows that start off a 16-byte boundary."""
    g = gen(n)
    full = torch.randint(-20, 20, (33, n + 1), generator=g).float()
    dev = full.to(cuda)[:, 1:]  # rows start 4 bytes past a 16-byte boundary
    s = full[:, 1:].contiguous()
    for k in sorted({1, min(n, 64), min(n, 1024), n}):
        rv, ri = oracle.topk_lower_index(s, k)
        v, i = ak.topk(dev, k, sorted=True)
        assert torch.equal(i.cpu(), ri) and torch.equal(v.cpu(), rv)
        _, i = ak.topk(dev, k, sorted=False)
        assert torch.equal(i.cpu(), ri.sort(-1).values)


@pytest.mark.parametrize("n", [4100, 8192, 32768])
def test_topk_unsorted_long_rows(cuda, n):
    """Unsorted selection of rows past the short-row kernel (the streaming kernel): heavy
    ties, all-equal rows, signed zeros, infinities, candidate-list overflow, a sample that
    misleads the bracket, sorted rows, k = n - 1 and n; indices in ascending order, values
    read back from the scores."""
    from bytes_b200 import _ops
    g = gen(n)
    s = torch.randint(-30, 30, (12, n), generator=g).float()
    s[0] = 2.5
    s[1, ::2] = -0.0
    s[1, 1::2] = 0.0
    s[2] = torch.randn(n, generator=g)
    s[2, 100:200] = float("inf")
    s[3] = float("-inf")
    s[3, n // 2:] = -1.0
    s[4] = torch.randn(n, generator=g) * 1e-30
    s[5] = torch.randint(0, 2, (n,), generator=g).float()  # two values: a threshold digit of ~n/2 keys
    s[6] = torch.randn(n, generator=g) + 100.0
    s[6, ::16] = 0.0  # every sampled position is small: the sample's bracket misses, radix fallback
    s[7] = torch.randn(n, generator=g)
    s[7, ::16] += 1000.0  # only the sampled positions are large
    s[8] = torch.arange(n).float()  # ascending
    s[9] = -torch.arange(n).float()  # descending
    dev = s.to(cuda)
    for k in sorted({1, 5, 1000, 2047, 2048, 2049, n // 2, n - 1, n}):
        v, i = _ops.topk(dev, k, sorted=False, want_values=True, idx_dtype=torch.int64)
        _, ri = oracle.topk_lower_index(s, k)
        assert torch.equal(i.cpu(), ri.sort(-1).values), k
        assert torch.equal(v.cpu(), torch.gather(s, -1, i.cpu())), k
        _, i32 = _ops.topk(dev, k, sorted=False, want_values=False, idx_dtype=torch.int32)
        assert torch.equal(i32.cpu().long(), i.cpu())


def test_topk_unsorted_strided_rows(cuda):
    """Rows of a [B, H, n] view whose rows sit 8200 floats apart (16-byte aligned)."""
    from bytes_b200 import _ops
    g = gen(99)
    big = torch.randn(2, 8, 8200, generator=g)
    view = big.to(cuda)[..., :8192]
    assert view.stride(1) == 8200
    _, i = _ops.topk(view, 300, sorted=False, want_values=False, idx_dtype=torch.int64)
    _, ri = oracle.topk_lower_index(big[..., :8192].contiguous(), 300)
    assert torch.equal(i.cpu(), ri.sort(-1).values)


def test_topk_3d_rows(cuda):
    g = gen(3)
    s = torch.randn(2, 8, 3000, generator=g)
    _topk_check(s, 150, True)


@pytest.mark.parametrize("kv_dtype", [torch.bfloat16, torch.float8_e4m3fn])
def test_gather_attn_matches_oracle(cuda, kv_dtype):
    g = gen(11)
    B, Hq, Hk, S, D, kb = 2, 8, 2, 500, 128, 77
    q = torch.randn(B, Hq, 1, D, generator=g).bfloat16()
    k = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    v = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    if kv_dtype == torch.float8_e4m3fn:
        k, v = k.to(kv_dtype), v.to(kv_dtype)
    idx = torch.randint(0, S, (B, Hq, kb), generator=g)
    idx[0, 0, :5] = 3  # duplicates count once per occurrence
    out = ak.sparse_gather_attn(q.to(cuda), k.to(cuda), v.to(cuda), idx.to(cuda), 0.088)
    ref = oracle.sparse_gather_attn(q, k, v, idx, 0.088)
    assert out.dtype == torch.bfloat16
    close(out, ref)


def test_gather_attn_skips_out_of_range(cuda):
    g = gen(12)
    q = torch.randn(1, 4, 1, 64, generator=g).bfloat16()
    k = torch.randn(1, 1, 50, 64, generator=g).bfloat16()
    v = torch.randn(1, 1, 50, 64, generator=g).bfloat16()
    idx = torch.tensor([[[0, 5, 50, 7, -1, 60]] * 4])
    out = ak.sparse_gather_attn(q.to(cuda), k.to(cuda), v.to(cuda), idx.to(cuda), 0.125)
    close(out, oracle.sparse_gather_attn(q, k, v, idx, 0.125))


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("bits", [16, 8, 4, 2])
def test_sparse_decode_pipeline(cuda, D, bits):
    """Reference pipeline test shapes (test_correctness.py:726-810): the kernel's index
    set must equal the exact (lower-index) top-k of its own scores, and the output must
    match exact attention over that set."""
    g = gen(D + bits)
    B, Hq, Hk, S, frac, scaling = 2, 8, 2, 256, 0.05, 0.125
    q = torch.randn(B, Hq, 1, D, generator=g).bfloat16()
    k = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    v = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    if bits == 16:
        ks, sc, zr = k, None, None
    elif bits == 8:
        ks, sc, zr = k.to(torch.float8_e4m3fn), None, None
    else:
        ks, sc, zr = oracle.quantize_and_pack_score_keys(k, bits, 32)
    dv = lambda t: None if t is None else t.to(cuda)
    out = ak.sparse_decode_scalar(q.to(cuda), ks.to(cuda), dv(sc), dv(zr), k.to(cuda), v.to(cuda), frac, scaling,
                                  score_bits=bits, group_size=32)
    # recompute the kernel's scores and its index set
    if bits in (16, 8):
        sc_gpu = ak.sparse_score_scalar(q.to(cuda), ks.to(cuda), scaling, score_bits=bits)
    else:
        sc_gpu = ak.sparse_score_packed(q.to(cuda), ks.to(cuda), sc.to(cuda), zr.to(cuda), scaling,
                                        score_bits=bits, group_size=32)
    kb = max(1, int(round(frac * S)))
    _, idx = oracle.topk_lower_index(sc_gpu.cpu(), kb)
    ref = oracle.sparse_gather_attn(q, k, v, idx, scaling)
    close(out, ref, max_abs=2e-2)


def test_quest_minmax_bounds_select(cuda):
    g = gen(21)
    B, Hq, Hk, S, D, page, kb = 2, 8, 2, 1000, 128, 16, 100
    q = torch.randn(B, Hq, 1, D, generator=g).bfloat16()
    k = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    kmin, kmax = sa.quest_page_metadata(k.to(cuda), page)
    rmin, rmax = oracle.quest_page_minmax(k, page)
    assert torch.equal(kmin.cpu(), rmin) and torch.equal(kmax.cpu(), rmax)
    from bytes_b200 import _ops
    bounds = _ops.quest_page_bounds(q[:, :, 0].to(cuda), kmin, kmax, 0.125)
    rb = oracle.quest_page_bounds(q, rmin, rmax, 0.125)
    assert torch.allclose(bounds.cpu(), rb, rtol=1e-5, atol=1e-4)
    idx = sa.quest_select_decode(q.to(cuda), kmin, kmax, S, kb, page, 0.125)
    # page set = exact top-npick of the kernel's own bounds, ordered by bound, lower page first
    npick = min(max(1, (kb + page - 1) // page), rb.shape[-1])
    _, pidx = oracle.topk_lower_index(bounds.cpu(), npick)
    ref = oracle.select._expand_pages(pidx, page, S)
    assert torch.equal(idx.cpu(), ref)


def test_quest_golden_reference(cuda, golden):
    for c in golden["quest"]:
        q, k, v = c["q"], c["k"], c["v"]
        G = q.shape[1] // k.shape[1]
        kr = oracle.repeat_kv(k, G)
        idx = sa._quest_select(q.to(cuda), kr.to(cuda), torch.tensor([c["S"] - 1]), c["S"], c["kb"], c["page"],
                               c["scaling"])
        assert torch.equal(idx.cpu(), c["idx"])
        out = sa.attend_topk(q.to(cuda), kr.to(cuda), oracle.repeat_kv(v, G).to(cuda), idx,
                             torch.tensor([c["S"] - 1]), c["scaling"])
        close(out, c["out"])


def test_select_topk_exact_matches_oracle(cuda):
    g = gen(31)
    B, Hq, S, D, kb = 2, 4, 700, 64, 40
    q = torch.randn(B, Hq, 1, D, generator=g).bfloat16()
    keys = torch.randn(B, Hq, S, D, generator=g).bfloat16()
    idx = sa.select_topk("exact", q.to(cuda), keys.to(cuda), torch.tensor([S - 1]), S, kb, 2048, 0.17)
    sc = ak.sparse_score_scalar(q.to(cuda), keys.to(cuda), 0.17, score_bits=16)
    _, ref = oracle.topk_lower_index(sc.cpu(), kb)
    assert torch.equal(idx.cpu(), ref.unsqueeze(2))
    # also agrees with the fp32 oracle selection outside near-ties
    idx_o = oracle.select_topk_exact(q, keys, S, kb, 0.17)
    agree = (idx.cpu().sort(-1).values == idx_o.sort(-1).values).float().mean().item()
    assert agree > 0.97


def test_sharded_sparse_decode_matches_single_device(cuda):
    """The kernels of the cross-GPU sparse decode, with two shards emulated on one device:
    per-shard scores and top-kb, the global pick, per-shard gather partials
    (bd_sparse_gather_attn_partial) and the combine equal the single-device pipeline."""
    from bytes_b200 import _ops
    from bytes_b200 import distributed as bdist
    g = gen(21)
    B, Hq, Hk, S, D, kb, sc = 2, 8, 2, 1500, 128, 100, 0.088
    q = torch.randn(B, Hq, 1, D, generator=g).bfloat16().to(cuda)
    k = torch.randn(B, Hk, S, D, generator=g).bfloat16().to(cuda)
    v = torch.randn(B, Hk, S, D, generator=g).bfloat16().to(cuda)
    k[:, :, 1200] = k[:, :, 30]  # a tie across the shard boundary
    full_scores = ak.sparse_score_scalar(q, k, sc, score_bits=16)
    _, idx = ak.topk(full_scores, kb, sorted=True)
    ref = ak.sparse_gather_attn(q, k, v, idx, sc)
    cut = 700
    vals, poss, shards = [], [], [(0, cut), (cut, S)]
    for s0, s1 in shards:
        s_ = ak.sparse_score_scalar(q, k[:, :, s0:s1], sc, score_bits=16)
        v_, i_ = ak.topk(s_, kb, sorted=True)
        vals.append(v_.float()); poss.append(i_.long() + s0)
    win = bdist.global_topk_merge(torch.stack(vals), torch.stack(poss), kb)
    assert torch.equal(win.sort(-1).values, idx.long().sort(-1).values)
    ms, ls, os_ = [], [], []
    for s0, s1 in shards:
        loc = win - s0
        loc = torch.where((loc >= 0) & (loc < s1 - s0), loc, torch.full_like(loc, -1))
        m, l, o = _ops.gather_attn_partial(q[:, :, 0], k[:, :, s0:s1], v[:, :, s0:s1], loc, sc)
        ms.append(m); ls.append(l); os_.append(o)
    out = _ops.lse_combine(torch.stack(ms), torch.stack(ls), torch.stack(os_), torch.bfloat16)
    close(out.unsqueeze(2), ref, max_abs=1e-2, mean_abs=1e-4)


def test_quest_bounds_every_head_dim_in_one_process(cuda):
    """The tensor-core bound kernel has one instance per head_dim, each with its own shared
    memory size: calls at 32, 128 and 64 in a row must each launch (and match the oracle)."""
    g = gen(31)
    for D in (32, 128, 64):
        B, Hq, Hk, S, page = 2, 8, 2, 640, 16
        q = torch.randn(B, Hq, 1, D, generator=g).bfloat16()
        k = torch.randn(B, Hk, S, D, generator=g).bfloat16()
        kmin, kmax = oracle.quest_page_minmax(k, page)
        bounds = _ops.quest_page_bounds(q[:, :, 0].to(cuda), kmin.to(cuda), kmax.to(cuda), 0.125)
        ref = oracle.quest_page_bounds(q, kmin, kmax, 0.125)
        assert torch.allclose(bounds.cpu(), ref, rtol=1e-5, atol=1e-4), (D, (bounds.cpu() - ref).abs().max())
