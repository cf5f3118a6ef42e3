"""This engine's drop-in functions beside the reference's own GPU code, on the same inputs.

``baseline/_ref`` holds the installed reference project, unmodified. Its kernel and
quantizer modules (src/attention_kernels.py, src/quantization.py: Triton kernels and
PyTorch expressions) are loaded under private module names, and every public function of
them that this engine replaces is called on the same seeded device tensors as this
engine's function of the same name; the two outputs are compared directly. This pins
parity on the reference itself run on the same GPU, independently of the CPU oracle.

Tolerances (the reference accumulates in fp32 Triton blocks, this engine in tensor-core
tiles with fp32 accumulators; only the summation order and the rounding of the softmax
weights differ): attention outputs within 4e-3 max-abs / 2e-4 mean-abs, fp32 scores within
1e-4 relative + 1e-4 absolute, the quantizers (score-key packer, fake-quant, KIVI) bit-exact,
PQ codes equal except between centroids whose scores tie to fp32 summation order, and the
top-k index set equal to ``scores.topk`` on tie-free scores. Every index handed to the
reference's gather kernel is in range (that kernel does not bounds-check its key
positions). Skipped when the install is absent.
"""
import importlib.util
import math
import os
import sys

import pytest
import torch

import oracle
from bytes_b200 import attention_kernels as ak
from bytes_b200 import quantization as qz

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_ROOT = os.path.join(ROOT, "baseline", "_ref")
REF_SRC = os.path.join(REF_ROOT, "src")


def _load(name, fname):
    if not os.path.isfile(os.path.join(REF_SRC, fname)):
        pytest.skip("reference install (baseline/_ref) not present")
    pytest.importorskip("triton")
    spec = importlib.util.spec_from_file_location(name, os.path.join(REF_SRC, fname))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def ref(cuda):
    return _load("_reference_attention_kernels", "attention_kernels.py")


@pytest.fixture(scope="module")
def ref_q(cuda):
    return _load("_reference_quantization", "quantization.py")


@pytest.fixture(scope="module")
def ref_sa(cuda):
    """benchmarks/sparse_attention.py of the reference (it imports src.quantization; the
    reference's own ``src`` package is importable only while the module loads)."""
    path = os.path.join(REF_ROOT, "benchmarks", "sparse_attention.py")
    if not os.path.isfile(path):
        pytest.skip("reference install (baseline/_ref) not present")
    owned = lambda k: k == "src" or k.startswith("src.")
    saved = {k: v for k, v in sys.modules.items() if owned(k)}
    for k in saved:
        del sys.modules[k]
    sys.path.insert(0, REF_ROOT)
    try:
        spec = importlib.util.spec_from_file_location("_reference_sparse_attention", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    finally:
        sys.path.remove(REF_ROOT)
        for k in [k for k in sys.modules if owned(k)]:
            del sys.modules[k]
        sys.modules.update(saved)
    return mod


def gen(seed):
    return torch.Generator().manual_seed(seed)


def same(ours, theirs, max_abs=4e-3, mean_abs=2e-4):
    assert ours.shape == theirs.shape, (ours.shape, theirs.shape)
    assert ours.dtype == theirs.dtype, (ours.dtype, theirs.dtype)
    a, b = ours.float(), theirs.float()
    assert torch.isfinite(a).all() and torch.isfinite(b).all()
    d = (a - b).abs()
    assert d.max().item() <= max_abs, f"max abs diff {d.max().item()}"
    assert d.mean().item() <= mean_abs, f"mean abs diff {d.mean().item()}"


def same_scores(ours, theirs):
    assert ours.shape == theirs.shape and ours.dtype == theirs.dtype == torch.float32
    assert torch.allclose(ours, theirs, rtol=1e-4, atol=1e-4), (ours - theirs).abs().max().item()


def to(dev, *ts):
    return [t.to(dev) for t in ts]


DENSE_SHAPES = [
    (2, 8, 2, 128, 64),      # the reference test's shape
    (1, 28, 4, 4097, 128),   # config 0 heads, ragged tail past 4096
    (2, 16, 1, 300, 128),    # G=16
    (3, 4, 4, 1000, 128),    # G=1
]


@pytest.mark.parametrize("B,Hq,Hk,S,D", DENSE_SHAPES)
@pytest.mark.parametrize("kv", ["bf16", "fp8"])
def test_dense_decode(ref, cuda, B, Hq, Hk, S, D, kv):
    g = gen(B * 7 + S + D)
    q = (torch.randn(B, Hq, 1, D, generator=g) / math.sqrt(D)).bfloat16()
    k = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    v = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    q, k, v = to(cuda, q, k, v)
    if kv == "fp8":
        k, v = k.to(torch.float8_e4m3fn), v.to(torch.float8_e4m3fn)
        same(ak.decode_attn_fp8(q, k, v), ref.decode_attn_fp8(q, k, v))
    else:
        same(ak.decode_attn_bf16(q, k, v), ref.decode_attn_bf16(q, k, v))


def _pq(g, B, Hq, Hk, S, D, K, d_sub=8):
    M = D // d_sub
    cent = torch.randn(M, K, d_sub, generator=g)
    codes = torch.randint(0, K, (B, Hk, S, M), generator=g).to(torch.uint8)
    q_rot = torch.randn(B, Hq, D, generator=g) / math.sqrt(D)
    lut = torch.einsum("bhmd,mkd->bhmk", q_rot.view(B, Hq, M, d_sub), cent).contiguous()
    return cent, codes, lut


@pytest.mark.parametrize("D", [64, 128])
def test_decode_attn_dequant(ref, cuda, D):
    g = gen(10 + D)
    B, Hq, Hk, S = 2, 8, 2, 700
    cent, codes, _ = _pq(g, B, Hq, Hk, S, D, 16)
    q = (torch.randn(B, Hq, 1, D, generator=g) / math.sqrt(D)).bfloat16()
    v = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    q, codes, cent, v = to(cuda, q, codes, cent, v)
    same(ak.decode_attn_dequant(q, codes, cent, v, d_sub=8), ref.decode_attn_dequant(q, codes, cent, v, d_sub=8))


@pytest.mark.parametrize("B,Hq,Hk,S,D,K", [(2, 8, 2, 128, 64, 8), (1, 28, 4, 1000, 128, 256),
                                           (4, 32, 8, 2051, 128, 256)])
def test_decode_attn_pq_lut(ref, cuda, B, Hq, Hk, S, D, K):
    g = gen(20 + S)
    _, codes, lut = _pq(g, B, Hq, Hk, S, D, K)
    v = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    lut, codes, v = to(cuda, lut, codes, v)
    same(ak.decode_attn_pq_lut(lut, codes, v), ref.decode_attn_pq_lut(lut, codes, v))


def test_decode_attn_pq_lut_kv(ref, cuda):
    g = gen(30)
    B, Hq, Hk, S, D = 2, 8, 2, 333, 64
    _, codes, lut = _pq(g, B, Hq, Hk, S, D, 16)
    vcent = torch.randn(D // 8, 16, 8, generator=g)
    vidx = torch.randint(0, 16, (B, Hk, S, D // 8), generator=g).to(torch.uint8)
    lut, codes, vidx, vcent = to(cuda, lut, codes, vidx, vcent)
    same(ak.decode_attn_pq_lut_kv(lut, codes, vidx, vcent, d_sub_v=8),
         ref.decode_attn_pq_lut_kv(lut, codes, vidx, vcent, d_sub_v=8))


def _paged(x, lens, bs, perm_seed):
    """[B,H,S,X] -> pages [NB,H,bs,X] in a shuffled physical order, with the block table."""
    B, H, S, X = x.shape
    nb = [math.ceil(int(l) / bs) for l in lens]
    order = torch.randperm(sum(nb), generator=gen(perm_seed))
    table = torch.full((B, max(nb)), -1, dtype=torch.int32)
    paged = torch.zeros(sum(nb), H, bs, X, dtype=x.dtype)
    c = 0
    for b in range(B):
        for i in range(nb[b]):
            p = int(order[c])
            c += 1
            table[b, i] = p
            n = min(bs, int(lens[b]) - i * bs)
            paged[p, :, :n] = x[b, :, i * bs:i * bs + n]
    return paged, table


def test_paged_attn_pq_lut_kv(ref, cuda):
    g = gen(40)
    B, Hq, Hk, D, bs = 3, 8, 2, 64, 16
    lens = torch.tensor([45, 78, 16], dtype=torch.int32)
    S = int(lens.max())
    _, codes, lut = _pq(g, B, Hq, Hk, S, D, 16)
    vcent = torch.randn(D // 8, 16, 8, generator=g)
    vidx = torch.randint(0, 16, (B, Hk, S, D // 8), generator=g).to(torch.uint8)
    kp, table = _paged(codes, lens, bs, 1)
    vp, _ = _paged(vidx, lens, bs, 1)
    lut, kp, vp, vcent, table, lens = to(cuda, lut, kp, vp, vcent, table, lens)
    same(ak.paged_attn_pq_lut_kv(lut, kp, vp, vcent, table, lens, block_size=bs),
         ref.paged_attn_pq_lut_kv(lut, kp, vp, vcent, table, lens, block_size=bs))


def _asym(g, B, Hq, Hk, S, D, C_out, K=16):
    _, codes, lut = _pq(g, B, Hq, Hk, S, D, K)
    k_raw = torch.randn(B, Hk, S, D, generator=g)
    for ch in [12, 45][:C_out]:
        k_raw[..., ch] = (torch.randn(B, Hk, S, generator=g) + 3.0) * 50.0
    oi = torch.tensor([12, 45][:C_out])
    q = (torch.randn(B, Hq, 1, D, generator=g) / math.sqrt(D)).bfloat16()
    k_out = k_raw[..., oi].bfloat16()
    q_out = q[:, :, 0][..., oi].contiguous()
    return lut, codes, k_out, q_out


@pytest.mark.parametrize("v_dtype", [torch.bfloat16, torch.float8_e4m3fn])
@pytest.mark.parametrize("B,Hq,Hk,S,D,C_out", [(2, 8, 2, 300, 64, 2), (1, 16, 2, 1029, 128, 1)])
def test_decode_attn_pq_lut_asym(ref, cuda, B, Hq, Hk, S, D, C_out, v_dtype):
    g = gen(50 + S + C_out)
    lut, codes, k_out, q_out = _asym(g, B, Hq, Hk, S, D, C_out)
    v = torch.randn(B, Hk, S, D, generator=g).to(v_dtype)
    lut, codes, k_out, q_out, v = to(cuda, lut, codes, k_out, q_out, v)
    same(ak.decode_attn_pq_lut_asym(lut, codes, k_out, q_out, v),
         ref.decode_attn_pq_lut_asym(lut, codes, k_out, q_out, v))


@pytest.mark.parametrize("v_dtype", [torch.bfloat16, torch.float8_e4m3fn])
def test_paged_attn_pq_lut_asym(ref, cuda, v_dtype):
    g = gen(60)
    B, Hq, Hk, D, C_out, bs = 2, 8, 2, 128, 2, 16
    lens = torch.tensor([45, 300], dtype=torch.int32)
    S = int(lens.max())
    lut, codes, k_out, q_out = _asym(g, B, Hq, Hk, S, D, C_out)
    v = torch.randn(B, Hk, S, D, generator=g).to(v_dtype)
    kp, table = _paged(codes, lens, bs, 2)
    kop, _ = _paged(k_out, lens, bs, 2)
    vp, _ = _paged(v.view(torch.uint8) if v_dtype == torch.float8_e4m3fn else v, lens, bs, 2)
    vp = vp.view(v_dtype)
    lut, kp, kop, q_out, vp, table, lens = to(cuda, lut, kp, kop, q_out, vp, table, lens)
    same(ak.paged_attn_pq_lut_asym(lut, kp, kop, q_out, vp, table, lens, block_size=bs),
         ref.paged_attn_pq_lut_asym(lut, kp, kop, q_out, vp, table, lens, block_size=bs))


def test_sparse_pq_lut_scores_and_chain(ref, cuda):
    g = gen(70)
    B, Hq, Hk, S, D = 2, 8, 2, 4096, 128
    lut, codes, k_out, q_out = _asym(g, B, Hq, Hk, S, D, 2, K=256)
    q = torch.randn(B, Hq, 1, D, generator=g).bfloat16()
    k = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    v = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    lut, codes, k_out, q_out, q, k, v = to(cuda, lut, codes, k_out, q_out, q, k, v)
    same_scores(ak.sparse_score_pq_lut_asym(lut, codes, k_out, q_out),
                ref.sparse_score_pq_lut_asym(lut, codes, k_out, q_out))
    # kb = 205 of 4096: a boundary swap between near-tied scores moves the output by well
    # under the tolerance
    same(ak.sparse_decode_pq_lut(lut, codes, k_out, q_out, q, k, v, 0.05, 0.088),
         ref.sparse_decode_pq_lut(lut, codes, k_out, q_out, q, k, v, 0.05, 0.088), max_abs=2e-2, mean_abs=1e-3)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("bits", [4, 2])
@pytest.mark.parametrize("D", [64, 128])
def test_pack_score_keys_bit_exact(ref, cuda, dtype, bits, D):
    k = (torch.randn(2, 4, 777, D, generator=gen(80 + bits + D)) * 3).to(dtype).to(cuda)
    ours = ak.quantize_and_pack_score_keys(k, bits, 32)
    theirs = ref.quantize_and_pack_score_keys(k, bits, 32)
    for a, b in zip(ours, theirs):
        assert a.dtype == b.dtype and a.shape == b.shape
        assert torch.equal(a, b), int((a != b).sum())


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("levels", [4, 16])
def test_fakequant_bit_exact(ref_q, cuda, dtype, levels):
    x = (torch.randn(64, 33, 128, generator=gen(levels)) * 2).to(dtype).to(cuda)
    for dim in (1, 2):
        a = qz._asym_uniform_fakequant(x, levels, dim)
        b = ref_q._asym_uniform_fakequant(x, levels, dim)
        assert a.dtype == b.dtype and torch.equal(a, b), int((a != b).sum())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("bits", [2, 4])
def test_kivi_quantizer_bit_exact(ref_q, cuda, dtype, bits):
    x = (torch.randn(2, 4, 1000, 128, generator=gen(bits)) * 2).to(dtype).to(cuda)
    for S in (1000, 77, 20):
        xs = x[:, :, :S]
        ours, theirs = qz.KIVIQuantizer(bits, 32, 32), ref_q.KIVIQuantizer(bits, 32, 32)
        assert torch.equal(ours.quantize_key(xs), theirs.quantize_key(xs))
        assert torch.equal(ours.quantize_value(xs), theirs.quantize_value(xs))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("d,d_sub,bits", [(128, 8, 3), (128, 8, 8), (64, 4, 4), (128, 16, 4)])
def test_pq_encode(ref_q, cuda, dtype, d, d_sub, bits):
    """Codes equal the reference's CUDA encoder except where the two centroids' scores agree
    to fp32 summation order (its tensor-core dot sums in another order)."""
    g = gen(d + d_sub + bits)
    X = torch.randn(5000, d, generator=g).to(dtype)
    C = torch.randn(d // d_sub, 2 ** bits, d_sub, generator=g)
    pr = ref_q.ProductQuantizer(d, d_sub, bits, device="cuda")
    pr.centroids = C.to(cuda)
    po = qz.ProductQuantizer(d, d_sub, bits, device="cuda")
    po.centroids = C.to(cuda)
    rc = pr.quantize(X.to(cuda)).cpu()
    oc = po.quantize(X.to(cuda)).cpu()
    assert oc.dtype == rc.dtype == torch.int64 and oc.shape == rc.shape
    assert torch.equal(oc, oracle.pq_encode(X, C))
    diff = oc != rc
    if diff.any():
        sc = oracle.quant.pq_encode_scores(X, C)
        a = sc.gather(-1, oc.unsqueeze(-1)).squeeze(-1)[diff]
        b = sc.gather(-1, rc.unsqueeze(-1)).squeeze(-1)[diff]
        assert torch.allclose(a, b, rtol=1e-5, atol=1e-5), (a - b).abs().max().item()
    assert diff.float().mean().item() < 1e-3


@pytest.mark.parametrize("bits", [16, 8, 4, 2])
@pytest.mark.parametrize("B,Hq,Hk,S,D", [(2, 8, 2, 128, 64), (1, 28, 4, 3001, 128), (2, 32, 8, 4100, 128)])
def test_sparse_scores(ref, cuda, bits, B, Hq, Hk, S, D):
    g = gen(90 + bits + S)
    q = torch.randn(B, Hq, 1, D, generator=g).bfloat16().to(cuda)
    k = torch.randn(B, Hk, S, D, generator=g).bfloat16().to(cuda)
    sc = 1.0 / math.sqrt(D)
    if bits in (16, 8):
        ks = k if bits == 16 else k.to(torch.float8_e4m3fn)
        same_scores(ak.sparse_score_scalar(q, ks, sc, score_bits=bits),
                    ref.sparse_score_scalar(q, ks, sc, score_bits=bits))
    else:
        kp, s_, z_ = ref.quantize_and_pack_score_keys(k, bits, 32)
        same_scores(ak.sparse_score_packed(q, kp, s_, z_, sc, score_bits=bits, group_size=32),
                    ref.sparse_score_packed(q, kp, s_, z_, sc, score_bits=bits, group_size=32))


@pytest.mark.parametrize("kv", ["bf16", "fp8"])
@pytest.mark.parametrize("kb", [1, 77, 1024])
def test_sparse_gather_attn(ref, cuda, kv, kb):
    g = gen(100 + kb)
    B, Hq, Hk, S, D = 2, 8, 2, 3000, 128
    q = torch.randn(B, Hq, 1, D, generator=g).bfloat16()
    k = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    v = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    idx = torch.randint(0, S, (B, Hq, kb), generator=g)
    idx[0, 0, : min(kb, 5)] = 3  # a repeated position counts once per occurrence
    q, k, v, idx = to(cuda, q, k, v, idx)
    if kv == "fp8":
        k, v = k.to(torch.float8_e4m3fn), v.to(torch.float8_e4m3fn)
    same(ak.sparse_gather_attn(q, k, v, idx, 0.088), ref.sparse_gather_attn(q, k, v, idx, 0.088))


@pytest.mark.parametrize("n,k", [(4096, 205), (32768, 1638), (1000, 1)])
def test_topk_matches_torch_topk(cuda, n, k):
    """The reference's selection step is ``scores.topk(kb)`` (src/attention_kernels.py:1069,
    1262). On scores with no repeated value the indices and the sorted values agree exactly."""
    g = gen(n + k)
    rows = torch.randperm(64 * n, generator=g).view(64, n).float() / 7.0 - 1000.0
    scores = rows.to(cuda)
    tv, ti = scores.topk(k, dim=-1)
    ov, oi = ak.topk(scores, k, sorted=True)
    assert torch.equal(ov, tv) and torch.equal(oi, ti)
    _, ui = ak.topk(scores, k, sorted=False)
    assert torch.equal(ui.sort(-1).values, ti.sort(-1).values)


@pytest.mark.parametrize("bits", [16, 8, 4, 2])
def test_sparse_decode_chain(ref, cuda, bits):
    g = gen(110 + bits)
    B, Hq, Hk, S, D, frac, scaling = 2, 16, 4, 4096, 128, 0.05, 1.0 / math.sqrt(128)
    q = torch.randn(B, Hq, 1, D, generator=g).bfloat16()
    k = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    v = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    q, k, v = to(cuda, q, k, v)
    if bits == 16:
        ks, s_, z_ = k, None, None
    elif bits == 8:
        ks, s_, z_ = k.to(torch.float8_e4m3fn), None, None
    else:
        ks, s_, z_ = ref.quantize_and_pack_score_keys(k, bits, 32)
    ours = ak.sparse_decode_scalar(q, ks, s_, z_, k, v, frac, scaling, score_bits=bits, group_size=32)
    theirs = ref.sparse_decode_scalar(q, ks, s_, z_, k, v, frac, scaling, score_bits=bits, group_size=32)
    same(ours, theirs, max_abs=2e-2, mean_abs=1e-3)


def _clear_rows(scores, k, margin=1e-4):
    v = scores.sort(-1, descending=True).values
    return (v[..., k - 1] - v[..., k]) > margin


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_select_topk_exact_vs_reference(ref_sa, cuda, dt):
    """select_topk('exact') of benchmarks/sparse_attention.py:226-325 on the GPU: the same
    key set on every row whose cut-off is not a near-tie."""
    from bytes_b200 import sparse_attention as sa
    g = gen(120)
    B, Hq, S, D, kb = 2, 8, 3000, 128, 150
    q = torch.randn(B, Hq, 1, D, generator=g).to(dt)
    keys = torch.randn(B, Hq, S, D, generator=g).to(dt)
    pos = torch.tensor([S - 1])
    theirs = ref_sa.select_topk("exact", q.to(cuda), keys.to(cuda), pos.to(cuda), S, kb, 512, 0.088)
    ours = sa.select_topk("exact", q.to(cuda), keys.to(cuda), pos, S, kb, 512, 0.088)
    assert ours.shape == theirs.shape
    sc = torch.einsum("bhqd,bhsd->bhqs", q.float(), keys.float()) * 0.088
    ok = _clear_rows(sc, kb)
    assert ok.float().mean() > 0.5
    a, b = ours.cpu().sort(-1).values, theirs.cpu().sort(-1).values
    assert torch.equal(a[ok], b[ok])


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_quest_select_vs_reference(ref_sa, cuda, dt):
    """_quest_select (benchmarks/sparse_attention.py:328-364) on the GPU: the same pages on
    every row whose page cut-off is not a near-tie."""
    from bytes_b200 import sparse_attention as sa
    g = gen(121)
    B, Hq, S, D, page, kb = 2, 8, 1000, 128, 16, 160
    q = torch.randn(B, Hq, 1, D, generator=g).to(dt)
    kr = (torch.randn(B, Hq, S, D, generator=g) * 2).to(dt)
    pos = torch.tensor([S - 1])
    theirs = ref_sa._quest_select(q.to(cuda), kr.to(cuda), pos.to(cuda), S, kb, page, 0.088)
    ours = sa._quest_select(q.to(cuda), kr.to(cuda), pos, S, kb, page, 0.088)
    assert ours.shape == theirs.shape
    kmin, kmax = oracle.quest_page_minmax(kr, page)
    rb = oracle.quest_page_bounds(q, kmin, kmax, 0.088)
    ok = _clear_rows(rb, kb // page)
    assert ok.float().mean() > 0.5
    a, b = ours.cpu()[:, :, 0].sort(-1).values, theirs.cpu()[:, :, 0].sort(-1).values
    assert torch.equal(a[ok], b[ok])


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_attend_topk_vs_reference(ref_sa, cuda, dt):
    """attend_topk (benchmarks/sparse_attention.py:367-387) over the same selection, sentinel
    slots included. The reference rounds a bf16 call's softmax weights to bf16 before the
    weighted sum, hence the wider bf16 tolerance."""
    from bytes_b200 import sparse_attention as sa
    g = gen(122)
    B, Hq, S, D, ks = 2, 4, 600, 128, 48
    q = torch.randn(B, Hq, 1, D, generator=g).to(dt)
    k = torch.randn(B, Hq, S, D, generator=g).to(dt)
    v = torch.randn(B, Hq, S, D, generator=g).to(dt)
    idx = torch.randint(0, S, (B, Hq, 1, ks), generator=g)
    idx[0, 1, 0, :5] = S
    pos = torch.tensor([S - 1])
    args = [t.to(cuda) for t in (q, k, v, idx)]
    theirs = ref_sa.attend_topk(*args, pos.to(cuda), 0.088)
    ours = sa.attend_topk(*args, pos, 0.088)
    if dt == torch.float32:
        same(ours, theirs, max_abs=1e-4, mean_abs=1e-5)
    else:
        same(ours, theirs, max_abs=2e-2, mean_abs=2e-3)


@pytest.mark.parametrize("dt", [torch.float32, torch.float16])
def test_full_precision_scores_and_gather_vs_reference(ref, cuda, dt):
    """The reference's Triton score and gather kernels on fp32 / f16 inputs (they widen
    every load to fp32) against this engine's unrounded paths."""
    g = gen(123)
    B, Hq, Hk, S, D, kb = 2, 8, 2, 2000, 128, 100
    q = torch.randn(B, Hq, 1, D, generator=g).to(dt).to(cuda)
    k = torch.randn(B, Hk, S, D, generator=g).to(dt).to(cuda)
    v = torch.randn(B, Hk, S, D, generator=g).to(dt).to(cuda)
    same_scores(ak.sparse_score_scalar(q, k, 0.088), ref.sparse_score_scalar(q, k, 0.088))
    idx = torch.randint(0, S, (B, Hq, kb), generator=g).to(cuda)
    tol = 1e-4 if dt == torch.float32 else 2e-3
    same(ak.sparse_gather_attn(q, k, v, idx, 0.088), ref.sparse_gather_attn(q, k, v, idx, 0.088),
         max_abs=tol, mean_abs=tol / 10)


@pytest.mark.parametrize("selector", ["exact", "quest"])
def test_sparse_attention_chunked_vs_reference(ref_sa, cuda, selector):
    """The reference's own chunked prefill loop (benchmarks/sparse_attention.py:463-497) on the
    GPU against this engine's, fp32 inputs (bf16 values)."""
    from bytes_b200 import sparse_attention as sa
    g = gen(124)
    B, Hq, Hk, S, D = 1, 8, 2, 768, 64
    q = torch.randn(B, Hq, S, D, generator=g).bfloat16().float().to(cuda)
    k = torch.randn(B, Hk, S, D, generator=g).bfloat16().float().to(cuda)
    v = torch.randn(B, Hk, S, D, generator=g).bfloat16().float().to(cuda)
    theirs = ref_sa.sparse_attention_chunked(q, k, v, None, selector, 0.1, Hq // Hk, 0.125, page=16, q_chunk=256)
    ours = sa.sparse_attention_chunked(q, k, v, None, selector, 0.1, Hq // Hk, 0.125, page=16, q_chunk=256)
    d = (ours - theirs).abs()
    assert d.mean().item() <= 1e-4, d.mean().item()
    assert (d.amax(-1) > 1e-3).float().mean().item() <= 2e-3


@pytest.mark.parametrize("selector", ["random", "recent", "sparq", "approx"])
def test_other_selectors_vs_reference(ref_sa, cuda, selector):
    """The reference's select_topk for its other selectors on the GPU: 'random' from the same
    CUDA generator state and 'recent' give the same indices; 'sparq' and a soft selector
    ('approx', ranking approximate keys) the same key sets outside near-ties."""
    from bytes_b200 import sparse_attention as sa
    g = gen(125)
    B, Hq, S, D, q0, Qc, kb = 2, 4, 500, 64, 300, 60, 40
    q = torch.randn(B, Hq, Qc, D, generator=g).bfloat16().float().to(cuda)
    keys = torch.randn(B, Hq, S, D, generator=g).bfloat16().float().to(cuda)
    pos = torch.arange(q0, q0 + Qc)
    gens = [torch.Generator(device=cuda).manual_seed(5) for _ in range(2)]
    theirs = ref_sa.select_topk(selector, q, keys, pos.to(cuda), S, kb, 128, 0.125, generator=gens[0]).cpu()
    ours = sa.select_topk(selector, q, keys, pos, S, kb, 128, 0.125, generator=gens[1]).cpu()
    assert ours.shape == theirs.shape
    if selector in ("random", "recent"):
        assert torch.equal(ours, theirs)
        return
    qs = q.float().cpu()
    if selector == "sparq":
        _, topr = oracle.topk_lower_index(qs.abs(), ref_sa.SPARQ_R)
        qs = qs * torch.zeros_like(qs).scatter_(-1, topr, 1.0)
    sc = torch.einsum("bhqd,bhsd->bhqs", qs, keys.float().cpu()) * 0.125
    sc = sc.masked_fill(torch.arange(S)[None, None, None, :] > pos[None, None, :, None], float("-inf"))
    ok = _clear_rows(sc, kb)
    from conftest import sparq_tie_rows, valid_sets
    if selector == "sparq":
        ok &= ~sparq_tie_rows(q.cpu(), ref_sa.SPARQ_R)
    ok = ok.reshape(-1).tolist()
    a, b = valid_sets(ours, pos, S), valid_sets(theirs, pos, S)
    assert sum(ok) > 0.5 * len(ok)
    assert all(x == y or not o for x, y, o in zip(a, b, ok))


@pytest.mark.parametrize("kv", ["bf16", "fp8"])
def test_dense_decode_fp32_query_vs_reference(ref, cuda, kv):
    """The reference's dense Triton kernels widen an fp32 query; so does this engine."""
    g = gen(126)
    B, Hq, Hk, S, D = 2, 8, 2, 2000, 128
    q = (torch.randn(B, Hq, 1, D, generator=g) / math.sqrt(D)).to(cuda)
    k = torch.randn(B, Hk, S, D, generator=g).bfloat16().to(cuda)
    v = torch.randn(B, Hk, S, D, generator=g).bfloat16().to(cuda)
    if kv == "fp8":
        k, v = k.to(torch.float8_e4m3fn), v.to(torch.float8_e4m3fn)
        ours, theirs = ak.decode_attn_fp8(q, k, v), ref.decode_attn_fp8(q, k, v)
    else:
        ours, theirs = ak.decode_attn_bf16(q, k, v), ref.decode_attn_bf16(q, k, v)
    same(ours, theirs, max_abs=1e-4, mean_abs=1e-5)


def test_pq_lut_f16_values_vs_reference(ref, cuda):
    """decode_attn_pq_lut over an f16 value cache (the reference widens it to fp32)."""
    g = gen(127)
    B, Hq, Hk, S, D, K = 2, 8, 2, 1500, 128, 256
    _, codes, lut = _pq(g, B, Hq, Hk, S, D, K)
    v = torch.randn(B, Hk, S, D, generator=g).half()
    lut, codes, v = to(cuda, lut, codes, v)
    same(ak.decode_attn_pq_lut(lut, codes, v), ref.decode_attn_pq_lut(lut, codes, v), max_abs=2e-3, mean_abs=1e-4)


def _nan_same(ours, theirs):
    """Equal NaN pattern, and the finite entries within the attention tolerance."""
    assert ours.shape == theirs.shape and ours.dtype == theirs.dtype
    a, b = ours.float().cpu(), theirs.float().cpu()
    assert torch.equal(torch.isnan(a), torch.isnan(b))
    fin = ~torch.isnan(a)
    if fin.any():
        assert (a[fin] - b[fin]).abs().max().item() <= 4e-3


def test_empty_contexts_vs_reference(ref, cuda):
    """Empty inputs the reference's kernels accept: a paged sequence of length 0 and a gather
    with no positions give 0/0 = NaN rows there; the same rows here."""
    g = gen(128)
    B, Hq, Hk, D, bs = 2, 8, 2, 64, 16
    lens = torch.tensor([0, 45], dtype=torch.int32)
    _, codes, lut = _pq(g, B, Hq, Hk, 45, D, 16)
    vcent = torch.randn(D // 8, 16, 8, generator=g)
    vidx = torch.randint(0, 16, (B, Hk, 45, D // 8), generator=g).to(torch.uint8)
    kp, table = _paged(codes, torch.tensor([16, 45]), bs, 3)  # sequence 0 keeps one page it never reads
    vp, _ = _paged(vidx, torch.tensor([16, 45]), bs, 3)
    lut, kp, vp, vcent, table, lens = to(cuda, lut, kp, vp, vcent, table, lens)
    _nan_same(ak.paged_attn_pq_lut_kv(lut, kp, vp, vcent, table, lens, block_size=bs),
              ref.paged_attn_pq_lut_kv(lut, kp, vp, vcent, table, lens, block_size=bs))
    q = torch.randn(B, Hq, 1, D, generator=g).bfloat16().to(cuda)
    k = torch.randn(B, Hk, 100, D, generator=g).bfloat16().to(cuda)
    v = torch.randn(B, Hk, 100, D, generator=g).bfloat16().to(cuda)
    idx = torch.zeros(B, Hq, 0, dtype=torch.int64, device=cuda)
    _nan_same(ak.sparse_gather_attn(q, k, v, idx, 0.1), ref.sparse_gather_attn(q, k, v, idx, 0.1))


@pytest.mark.parametrize("gs", [16, 64, 128])
@pytest.mark.parametrize("bits", [4, 2])
def test_other_group_sizes_vs_reference(ref, cuda, gs, bits):
    """Score-key groups of 16, 64 and 128 channels: the packer bit-exact, the packed scores
    within 1e-4."""
    g = gen(129 + gs + bits)
    B, Hq, Hk, S, D = 2, 8, 2, 1200, 128
    q = torch.randn(B, Hq, 1, D, generator=g).bfloat16().to(cuda)
    k = (torch.randn(B, Hk, S, D, generator=g) * 2).bfloat16().to(cuda)
    ours = ak.quantize_and_pack_score_keys(k, bits, gs)
    theirs = ref.quantize_and_pack_score_keys(k, bits, gs)
    for a, b in zip(ours, theirs):
        assert a.dtype == b.dtype and a.shape == b.shape and torch.equal(a, b)
    kp, s_, z_ = theirs
    same_scores(ak.sparse_score_packed(q, kp, s_, z_, 0.1, score_bits=bits, group_size=gs),
                ref.sparse_score_packed(q, kp, s_, z_, 0.1, score_bits=bits, group_size=gs))


@pytest.mark.parametrize("d_sub", [4, 16])
def test_other_subvector_lengths_vs_reference(ref, cuda, d_sub):
    """PQ with sub-vectors of 4 and 16 channels: decode_attn_dequant and the PQ value path."""
    g = gen(130 + d_sub)
    B, Hq, Hk, S, D = 2, 8, 2, 600, 128
    M = D // d_sub
    cent = torch.randn(M, 16, d_sub, generator=g)
    codes = torch.randint(0, 16, (B, Hk, S, M), generator=g).to(torch.uint8)
    q = (torch.randn(B, Hq, 1, D, generator=g) / math.sqrt(D)).bfloat16()
    v = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    qd, cd, ced, vd = to(cuda, q, codes, cent, v)
    same(ak.decode_attn_dequant(qd, cd, ced, vd, d_sub=d_sub), ref.decode_attn_dequant(qd, cd, ced, vd, d_sub=d_sub))
    q_rot = torch.randn(B, Hq, D, generator=g) / math.sqrt(D)
    lut = torch.einsum("bhmd,mkd->bhmk", q_rot.view(B, Hq, M, d_sub), cent).contiguous().to(cuda)
    vcent = torch.randn(M, 16, d_sub, generator=g).to(cuda)
    vidx = torch.randint(0, 16, (B, Hk, S, M), generator=g).to(torch.uint8).to(cuda)
    same(ak.decode_attn_pq_lut_kv(lut, cd, vidx, vcent, d_sub_v=d_sub),
         ref.decode_attn_pq_lut_kv(lut, cd, vidx, vcent, d_sub_v=d_sub))
