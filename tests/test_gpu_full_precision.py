"""Full-precision inputs (fp32 / f16 queries, keys and values) through the sparse path.

The reference computes its sparse selection and attention in fp32 on whatever dtype the
caller passes: its score tiles cast to fp32 (benchmarks/sparse_attention.py:195-212, 342-345)
and its Triton kernels widen every load to fp32 (src/attention_kernels.py:1098-1110,
1169-1196, 1017-1027). This engine takes such inputs unrounded: a bf16 query against bf16
keys uses the tensor-core tiles (every product exact in fp32), anything else the fp32
CUDA-core score kernel, the gather kernel's f16 / fp32 forms and the Quest bound over f16 /
fp32 page metadata. Gates against the fp32 oracle: scores within 2e-5 relative, selections
equal to the oracle's own selection on every row whose cut-off is not a near-tie, attention
within 1e-4 (fp32 output) or 2e-3 (f16 output).
"""
import math

import pytest
import torch

import oracle
from bytes_b200 import _ops
from bytes_b200 import attention_kernels as ak
from bytes_b200 import sparse_attention as sa

pytestmark = pytest.mark.gpu

DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def gen(seed):
    return torch.Generator().manual_seed(seed)


def randn(g, *shape, dtype=torch.float32, scale=1.0):
    return (torch.randn(*shape, generator=g) * scale).to(dtype)


def clear_rows(scores, k, margin):
    """Rows whose k-th and (k+1)-th largest scores differ by more than `margin`."""
    v = scores.sort(-1, descending=True).values
    return (v[..., k - 1] - v[..., k]) > margin


@pytest.mark.parametrize("qd,kd", [("f32", "f32"), ("f32", "bf16"), ("f16", "f16"), ("f16", "bf16"),
                                   ("bf16", "f32"), ("bf16", "f16")])
@pytest.mark.parametrize("D,S", [(128, 1000), (64, 77)])
def test_scalar_scores(cuda, qd, kd, D, S):
    g = gen(D + S + len(qd + kd))
    q = randn(g, 2, 8, 1, D, dtype=DT[qd])
    k = randn(g, 2, 2, S, D, dtype=DT[kd], scale=2.0)
    out = ak.sparse_score_scalar(q.to(cuda), k.to(cuda), 1 / math.sqrt(D))
    ref = oracle.sparse_score_scalar(q, k, 1 / math.sqrt(D))
    assert out.dtype == torch.float32
    assert torch.allclose(out.cpu(), ref, rtol=2e-5, atol=2e-5), (out.cpu() - ref).abs().max()


@pytest.mark.parametrize("bits", [8, 4, 2])
def test_fp32_query_over_compressed_keys(cuda, bits):
    """An fp32 query keeps its precision over fp8 and packed keys (the tensor-core forms
    round the query to f16)."""
    g = gen(40 + bits)
    D, S = 128, 700
    q = randn(g, 1, 16, 1, D) * 3.0 + 1e-3 * randn(g, 1, 16, 1, D)
    k = randn(g, 1, 4, S, D, dtype=torch.bfloat16)
    if bits == 8:
        k8 = k.to(torch.float8_e4m3fn)
        out = ak.sparse_score_scalar(q.to(cuda), k8.to(cuda), 0.1, score_bits=8)
        ref = oracle.sparse_score_scalar(q, k8, 0.1)
    else:
        kp, s_, z_ = oracle.quantize_and_pack_score_keys(k, bits, 32)
        out = ak.sparse_score_packed(q.to(cuda), kp.to(cuda), s_.to(cuda), z_.to(cuda), 0.1, score_bits=bits,
                                     group_size=32)
        ref = oracle.sparse_score_packed(q, kp, s_, z_, 0.1, bits, 32)
    assert torch.allclose(out.cpu(), ref, rtol=2e-5, atol=2e-5), (out.cpu() - ref).abs().max()


@pytest.mark.parametrize("kvd", ["f32", "f16"])
@pytest.mark.parametrize("qd", ["f32", "bf16"])
@pytest.mark.parametrize("D", [128, 64, 32])
def test_gather_attn(cuda, kvd, qd, D):
    g = gen(60 + D + len(kvd + qd))
    B, Hq, Hk, S, kb = 2, 8, 2, 900, 150
    q = randn(g, B, Hq, 1, D, dtype=DT[qd])
    k = randn(g, B, Hk, S, D, dtype=DT[kvd])
    v = randn(g, B, Hk, S, D, dtype=DT[kvd])
    idx = torch.randint(0, S, (B, Hq, kb), generator=g)
    idx[0, 0, :4] = torch.tensor([3, 3, -1, S])  # a repeat, and two positions outside [0, S)
    out = ak.sparse_gather_attn(q.to(cuda), k.to(cuda), v.to(cuda), idx.to(cuda), 1 / math.sqrt(D))
    ref = oracle.sparse_gather_attn(q, k, v, idx, 1 / math.sqrt(D))
    assert out.dtype == DT[kvd]
    tol = 1e-4 if kvd == "f32" else 2e-3
    assert torch.allclose(out.float().cpu(), ref.float(), rtol=tol, atol=tol), (out.float().cpu() - ref.float()).abs().max()


@pytest.mark.parametrize("dt", ["f32", "f16"])
def test_select_topk_exact(cuda, dt):
    g = gen(80)
    B, Hq, S, D, kb = 2, 8, 3000, 128, 150
    q = randn(g, B, Hq, 1, D, dtype=DT[dt])
    keys = randn(g, B, Hq, S, D, dtype=DT[dt])
    idx = sa.select_topk("exact", q.to(cuda), keys.to(cuda), torch.tensor([S - 1]), S, kb, 512, 0.088)
    ref = oracle.select_topk_exact(q, keys, S, kb, 0.088)
    sc = torch.einsum("bhqd,bhsd->bhqs", q.float(), keys.float()) * 0.088
    ok = clear_rows(sc, kb, 1e-4)
    assert ok.float().mean() > 0.5
    a, b = idx.cpu().sort(-1).values, ref.sort(-1).values
    assert torch.equal(a[ok], b[ok])


@pytest.mark.parametrize("dt", ["f32", "f16"])
def test_quest_bounds_and_select(cuda, dt):
    g = gen(90)
    B, Hq, Hk, S, D, page, kb = 2, 8, 2, 1000, 128, 16, 160
    q = randn(g, B, Hq, 1, D, dtype=DT[dt])
    k = randn(g, B, Hk, S, D, dtype=DT[dt], scale=2.0)
    kmin, kmax = sa.quest_page_metadata(k.to(cuda), page)
    assert kmin.dtype == DT[dt]
    rmin, rmax = oracle.quest_page_minmax(k, page)
    assert torch.equal(kmin.cpu(), rmin) and torch.equal(kmax.cpu(), rmax)
    bounds = _ops.quest_page_bounds(q[:, :, 0].to(cuda), kmin, kmax, 0.088)
    rb = oracle.quest_page_bounds(q, rmin, rmax, 0.088)
    assert torch.allclose(bounds.cpu(), rb, rtol=2e-5, atol=2e-5), (bounds.cpu() - rb).abs().max()
    # the drop-in over GQA-expanded keys
    kr = k.repeat_interleave(Hq // Hk, dim=1)
    idx = sa._quest_select(q.to(cuda), kr.to(cuda), torch.tensor([S - 1]), S, kb, page, 0.088)
    ref = oracle.quest_select(q, kr, S, kb, page, 0.088)
    npick = kb // page
    ok = clear_rows(rb, npick, 1e-4)
    assert ok.float().mean() > 0.5
    assert torch.equal(idx.cpu()[:, :, 0][ok].sort(-1).values, ref[:, :, 0][ok].sort(-1).values)


def test_attend_topk_fp32(cuda):
    g = gen(100)
    B, Hq, S, D, ks = 2, 4, 500, 64, 40
    q = randn(g, B, Hq, 1, D)
    k = randn(g, B, Hq, S, D)
    v = randn(g, B, Hq, S, D)
    idx = torch.randint(0, S, (B, Hq, 1, ks), generator=g)
    idx[1, 2, 0, :3] = S  # sentinel slots
    pos = torch.tensor([S - 1])
    out = sa.attend_topk(q.to(cuda), k.to(cuda), v.to(cuda), idx.to(cuda), pos, 0.125)
    ref = oracle.attend_topk(q, k, v, idx, pos, 0.125)
    assert out.dtype == torch.float32
    assert torch.allclose(out.cpu(), ref, rtol=1e-4, atol=1e-4), (out.cpu() - ref).abs().max()


@pytest.mark.parametrize("qd", ["f32", "f16"])
@pytest.mark.parametrize("kv", ["bf16", "fp8"])
def test_dense_decode_unrounded_query(cuda, qd, kv):
    """decode_attn_bf16 / decode_attn_fp8 with an f16 or fp32 query: the reference widens it
    to fp32 (src/attention_kernels.py:8-63, 98-150); this engine computes those calls in
    fp32 over every position (an f16 query over fp8 keys stays on the exact f16 tiles)."""
    g = gen(140 + len(qd + kv))
    B, Hq, Hk, S, D = 2, 8, 2, 3000, 128
    q = (randn(g, B, Hq, 1, D) / math.sqrt(D) * 3.0).to(DT[qd])
    k = randn(g, B, Hk, S, D, dtype=torch.bfloat16)
    v = randn(g, B, Hk, S, D, dtype=torch.bfloat16)
    if kv == "fp8":
        k, v = k.to(torch.float8_e4m3fn), v.to(torch.float8_e4m3fn)
    fn = ak.decode_attn_bf16 if kv == "bf16" else ak.decode_attn_fp8
    out = fn(q.to(cuda), k.to(cuda), v.to(cuda))
    ref = oracle.decode_attn_dense(q.float(), k, v, 1.0)
    assert out.dtype == q.dtype and out.shape == (B, Hq, 1, D)
    tol = 1e-4 if qd == "f32" else 2e-3
    assert torch.allclose(out.float().cpu(), ref.float(), rtol=tol, atol=tol), (out.float().cpu() - ref.float()).abs().max()


def test_pq_family_f16_values(cuda):
    """f16 value caches go to the PQ kernels as they are (PV in f16 on the tensor cores),
    not through a bf16 copy: decode_attn_pq_lut, decode_attn_dequant and the outlier-aware
    form, against the fp32 oracle within the f16 output's rounding."""
    g = gen(150)
    B, Hq, Hk, S, D, K = 2, 8, 2, 900, 128, 256
    M = D // 8
    cent = torch.randn(M, K, 8, generator=g)
    codes = torch.randint(0, K, (B, Hk, S, M), generator=g).to(torch.uint8)
    lut = oracle.pq_lut(torch.randn(B, Hq, D, generator=g) / math.sqrt(D), cent)
    v = torch.randn(B, Hk, S, D, generator=g).half()
    out = ak.decode_attn_pq_lut(lut.to(cuda), codes.to(cuda), v.to(cuda))
    assert out.dtype == torch.float16
    ref = oracle.decode_attn_pq_lut(lut, codes, v)
    assert torch.allclose(out.float().cpu(), ref.float(), rtol=2e-3, atol=2e-3), (out.float().cpu() - ref.float()).abs().max()
    q = (torch.randn(B, Hq, 1, D, generator=g) / math.sqrt(D)).half()
    out = ak.decode_attn_dequant(q.to(cuda), codes.to(cuda), cent.to(cuda), v.to(cuda), d_sub=8)
    ref = oracle.decode_attn_dequant(q, codes, cent, v, 8)
    assert torch.allclose(out.float().cpu(), ref.float(), rtol=2e-3, atol=2e-3), (out.float().cpu() - ref.float()).abs().max()
    k_out = torch.randn(B, Hk, S, 2, generator=g).bfloat16() * 20
    q_out = torch.randn(B, Hq, 2, generator=g).bfloat16()
    out = ak.decode_attn_pq_lut_asym(lut.to(cuda), codes.to(cuda), k_out.to(cuda), q_out.to(cuda), v.to(cuda))
    assert out.dtype == torch.float16
    ref = oracle.decode_attn_pq_lut_asym(lut, codes, k_out, q_out, v)
    assert torch.allclose(out.float().cpu(), ref.float(), rtol=2e-3, atol=2e-3), (out.float().cpu() - ref.float()).abs().max()


@pytest.mark.parametrize("kvd", ["f16", "f32"])
def test_dense_decode_f16_f32_cache(cuda, kvd):
    """decode_attn_bf16 over an f16 / fp32 cache (the reference's kernel widens any dtype)."""
    g = gen(160)
    B, Hq, Hk, S, D = 2, 8, 2, 1500, 64
    q = (randn(g, B, Hq, 1, D) / math.sqrt(D)).bfloat16()
    k = randn(g, B, Hk, S, D, dtype=DT[kvd])
    v = randn(g, B, Hk, S, D, dtype=DT[kvd])
    out = ak.decode_attn_bf16(q.to(cuda), k.to(cuda), v.to(cuda))
    ref = oracle.decode_attn_dense(q, k, v, 1.0)
    assert out.dtype == torch.bfloat16
    assert torch.allclose(out.float().cpu(), ref.float(), rtol=8e-3, atol=8e-3), (out.float().cpu() - ref.float()).abs().max()
