"""GPU parity for the PQ-LUT decode family, PQ encode and the KIVI / asymmetric fake-quant.

Cases follow the reference's tests (benchmarks/test_correctness.py:117-594): paged block
tables with ragged lengths 45/78/55, outlier channels 12 and 45 scaled (randn+3)*50,
fp8 and bf16 values, G up to 16. Inputs are seeded; the oracle supplies the expected
outputs (attention within 2e-2 max-abs / 1e-3 mean-abs, quantizers bit-exact).
"""
import math

import pytest
import torch

import oracle
from bytes_b200 import attention_kernels as ak
from bytes_b200 import quantization as qz

pytestmark = pytest.mark.gpu


def gen(seed):
    return torch.Generator().manual_seed(seed)


def close(out, ref, max_abs=2e-2, mean_abs=1e-3):
    d = (out.float().cpu() - ref.float().cpu()).abs()
    assert torch.isfinite(out.float()).all()
    assert d.max().item() <= max_abs, f"max abs diff {d.max().item()}"
    assert d.mean().item() <= mean_abs, f"mean abs diff {d.mean().item()}"


def _pq_setup(g, B, Hq, Hk, S, D, d_sub=8, K=8):
    M = D // d_sub
    cent = torch.randn(M, K, d_sub, generator=g)
    codes = torch.randint(0, K, (B, Hk, S, M), generator=g).to(torch.uint8)
    q_rot = torch.randn(B, Hq, D, generator=g)
    lut = oracle.pq_lut(q_rot, cent)
    return cent, codes, q_rot, lut


@pytest.mark.parametrize("D", [64, 128])
def test_decode_attn_dequant(cuda, D):
    g = gen(1)
    B, Hq, Hk, S = 2, 8, 2, 128
    cent, codes, _, _ = _pq_setup(g, B, Hq, Hk, S, D)
    q = torch.randn(B, Hq, 1, D, generator=g).bfloat16()
    v = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    out = ak.decode_attn_dequant(q.to(cuda), codes.to(cuda), cent.to(cuda), v.to(cuda), d_sub=8)
    close(out, oracle.decode_attn_dequant(q, codes, cent, v, 8))


@pytest.mark.parametrize("B,Hq,Hk,S,D,K", [(2, 8, 2, 128, 64, 8), (1, 28, 4, 1000, 128, 256), (2, 16, 1, 300, 128, 256)])
def test_decode_attn_pq_lut(cuda, B, Hq, Hk, S, D, K):
    g = gen(S + K)
    cent, codes, _, lut = _pq_setup(g, B, Hq, Hk, S, D, K=K)
    v = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    out = ak.decode_attn_pq_lut(lut.to(cuda), codes.to(cuda), v.to(cuda))
    assert out.dtype == torch.bfloat16
    close(out, oracle.decode_attn_pq_lut(lut, codes, v))


def test_pq_lut_golden(cuda, golden):
    for c in golden["pq_lut_decode"]:
        if c["k_out"].shape[-1] == 0:
            out = ak.decode_attn_pq_lut(c["lut"].to(cuda), c["codes"].to(cuda), c["v"].to(cuda))
        else:
            out = ak.decode_attn_pq_lut_asym(c["lut"].to(cuda), c["codes"].to(cuda), c["k_out"].to(cuda),
                                             c["q_out"].to(cuda), c["v"].to(cuda))
        close(out, c["out"])


def test_decode_attn_pq_lut_kv(cuda):
    g = gen(3)
    B, Hq, Hk, S, D = 2, 8, 2, 128, 64
    cent, codes, _, lut = _pq_setup(g, B, Hq, Hk, S, D)
    vcent = torch.randn(D // 8, 8, 8, generator=g)
    vidx = torch.randint(0, 8, (B, Hk, S, D // 8), generator=g).to(torch.uint8)
    out = ak.decode_attn_pq_lut_kv(lut.to(cuda), codes.to(cuda), vidx.to(cuda), vcent.to(cuda), d_sub_v=8)
    assert out.dtype == torch.float32
    close(out, oracle.decode_attn_pq_lut_kv(lut, codes, vidx, vcent, 8))


def _page(x, lens, block_size):
    """Scatter [B,H,S,X] into a paged [NB,H,bs,X] layout with consecutive blocks per sequence."""
    B, H, S, X = x.shape
    nb = [math.ceil(int(l) / block_size) for l in lens]
    table = torch.full((B, max(nb)), -1, dtype=torch.int32)
    paged = torch.zeros(sum(nb), H, block_size, X, dtype=x.dtype)
    c = 0
    for b in range(B):
        for i in range(nb[b]):
            table[b, i] = c
            c += 1
        for t in range(int(lens[b])):
            paged[table[b, t // block_size], :, t % block_size] = x[b, :, t]
    return paged, table


def test_paged_attn_pq_lut_kv(cuda):
    """Reference fixture: lens 45/78, block size 16 (test_correctness.py:299-391)."""
    g = gen(4)
    B, Hq, Hk, D, bs = 2, 8, 2, 64, 16
    lens = torch.tensor([45, 78], dtype=torch.int32)
    S = int(lens.max())
    cent, codes, _, lut = _pq_setup(g, B, Hq, Hk, S, D)
    vcent = torch.randn(D // 8, 8, 8, generator=g)
    vidx = torch.randint(0, 8, (B, Hk, S, D // 8), generator=g).to(torch.uint8)
    kp, table = _page(codes, lens, bs)
    vp, _ = _page(vidx, lens, bs)
    out = ak.paged_attn_pq_lut_kv(lut.to(cuda), kp.to(cuda), vp.to(cuda), vcent.to(cuda), table.to(cuda),
                                  lens.to(cuda), block_size=bs)
    close(out, oracle.paged_attn_pq_lut_kv(lut, kp, vp, vcent, table, lens, bs))


def _asym_case(g, B, Hq, Hk, S, D, C_out, v_dtype, K=8):
    M = D // 8
    k_raw = torch.randn(B, Hk, S, D, generator=g)
    for ch in [12, 45][:C_out]:
        k_raw[:, :, :, ch] = (torch.randn(B, Hk, S, generator=g) + 3.0) * 50.0
    var = k_raw.reshape(-1, D).var(0)
    oi = torch.topk(var, k=C_out).indices
    q = torch.randn(B, Hq, 1, D, generator=g).bfloat16()
    k_out = k_raw[..., oi].bfloat16()
    q_out = q[:, :, 0][..., oi].bfloat16()
    cent = torch.randn(M, K, 8, generator=g)
    codes = torch.randint(0, K, (B, Hk, S, M), generator=g).to(torch.uint8)
    lut = oracle.pq_lut(torch.randn(B, Hq, D, generator=g), cent)
    v = torch.randn(B, Hk, S, D, generator=g).to(v_dtype)
    return lut, codes, k_out, q_out, v


@pytest.mark.parametrize("B,Hq,Hk,S,D,C_out,v_dtype", [
    (2, 8, 2, 128, 64, 2, torch.bfloat16),
    (2, 8, 2, 128, 64, 2, torch.float8_e4m3fn),
    (1, 4, 1, 64, 128, 1, torch.float8_e4m3fn),
    (2, 16, 1, 256, 128, 2, torch.bfloat16),
])
def test_decode_attn_pq_lut_asym(cuda, B, Hq, Hk, S, D, C_out, v_dtype):
    g = gen(S + C_out + D)
    lut, codes, k_out, q_out, v = _asym_case(g, B, Hq, Hk, S, D, C_out, v_dtype)
    out = ak.decode_attn_pq_lut_asym(lut.to(cuda), codes.to(cuda), k_out.to(cuda), q_out.to(cuda), v.to(cuda))
    assert out.dtype == torch.bfloat16
    close(out, oracle.decode_attn_pq_lut_asym(lut, codes, k_out, q_out, v))


@pytest.mark.parametrize("B,Hq,Hk,D,C_out,bs,v_dtype", [
    (2, 8, 2, 64, 2, 16, torch.bfloat16),
    (2, 8, 2, 64, 2, 16, torch.float8_e4m3fn),
    (1, 4, 1, 128, 1, 32, torch.float8_e4m3fn),
])
def test_paged_attn_pq_lut_asym(cuda, B, Hq, Hk, D, C_out, bs, v_dtype):
    g = gen(D + bs)
    lens = torch.tensor([45, 78] if B == 2 else [55], dtype=torch.int32)
    S = int(lens.max())
    lut, codes, k_out, q_out, v = _asym_case(g, B, Hq, Hk, S, D, C_out, v_dtype)
    kp, table = _page(codes, lens, bs)
    kop, _ = _page(k_out, lens, bs)
    vp, _ = _page(v.view(torch.uint8) if v.dtype == torch.float8_e4m3fn else v, lens, bs)
    if v.dtype == torch.float8_e4m3fn:
        vp = vp.view(torch.float8_e4m3fn)
    out = ak.paged_attn_pq_lut_asym(lut.to(cuda), kp.to(cuda), kop.to(cuda), q_out.to(cuda), vp.to(cuda),
                                    table.to(cuda), lens.to(cuda), block_size=bs)
    close(out, oracle.paged_attn_pq_lut_asym(lut, kp, kop, q_out, vp, table, lens, bs))


@pytest.mark.parametrize("B,Hq,Hk,S", [(2, 8, 2, 300), (4, 32, 8, 32768)])
def test_pq_lut_int8v_config2(cuda, B, Hq, Hk, S):
    """Config 2: 16 subspaces x 256 fp16 centroids ~N(0,1), uint8 codes U[0,256),
    int8 V per token with an f16 scale."""
    g = gen(S)
    D, M, K = 128, 16, 256
    cent = torch.randn(M, K, 8, generator=g).half().float()
    codes = torch.randint(0, K, (B, Hk, S, M), generator=g).to(torch.uint8)
    lut = oracle.pq_lut(torch.randn(B, Hq, D, generator=g) / math.sqrt(D), cent)
    v8 = torch.randint(-127, 128, (B, Hk, S, D), generator=g).to(torch.int8)
    vs = (torch.rand(B, Hk, S, generator=g) * 0.02 + 0.001).half()
    out = ak.decode_attn_pq_lut_int8v(lut.to(cuda), codes.to(cuda), v8.to(cuda), vs.to(cuda))
    close(out, oracle.decode_attn_pq_lut_int8v(lut, codes, v8, vs))


@pytest.mark.parametrize("M,code_pitch", [(8, 8), (16, 32), (32, 32)])
def test_pq_lut_int8v_code_layouts(cuda, M, code_pitch):
    """Subspace counts and code-row pitches on both tile paths: codes of 16 or 32 bytes in
    16-byte-multiple rows take tensor-map (TMA) loads, 8-byte codes the per-thread copies."""
    g = gen(100 + M + code_pitch)
    B, Hq, Hk, S, D, K = 2, 8, 2, 700, 128, 256
    cent = torch.randn(M, K, D // M, generator=g).half().float()
    codes = torch.randint(0, K, (B, Hk, S, M), generator=g).to(torch.uint8)
    lut = oracle.pq_lut(torch.randn(B, Hq, D, generator=g) / math.sqrt(D), cent)
    v8 = torch.randint(-127, 128, (B, Hk, S, D), generator=g).to(torch.int8)
    vs = (torch.rand(B, Hk, S, generator=g) * 0.02 + 0.001).half()
    buf = torch.zeros(B, Hk, S, code_pitch, dtype=torch.uint8, device=cuda)
    buf[..., :M] = codes.to(cuda)
    out = ak.decode_attn_pq_lut_int8v(lut.to(cuda), buf[..., :M], v8.to(cuda), vs.to(cuda))
    close(out, oracle.decode_attn_pq_lut_int8v(lut, codes, v8, vs))


def test_sparse_pq_lut_scores_and_pipeline(cuda):
    g = gen(9)
    B, Hq, Hk, S, D = 2, 8, 2, 512, 128
    lut, codes, k_out, q_out, _ = _asym_case(g, B, Hq, Hk, S, D, 2, torch.bfloat16, K=256)
    sc = ak.sparse_score_pq_lut_asym(lut.to(cuda), codes.to(cuda), k_out.to(cuda), q_out.to(cuda))
    ref = oracle.sparse_score_pq_lut_asym(lut, codes, k_out, q_out)
    assert torch.allclose(sc.cpu(), ref, rtol=1e-5, atol=1e-3)
    q = torch.randn(B, Hq, 1, D, generator=g).bfloat16()
    k = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    v = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    out = ak.sparse_decode_pq_lut(lut.to(cuda), codes.to(cuda), k_out.to(cuda), q_out.to(cuda), q.to(cuda),
                                  k.to(cuda), v.to(cuda), 0.05, 0.088)
    kb = max(1, int(round(0.05 * S)))
    _, idx = oracle.topk_lower_index(sc.cpu(), kb)
    close(out, oracle.sparse_gather_attn(q, k, v, idx, 0.088))


def test_pq_encode_matches_oracle_and_golden(cuda, golden_cuda):
    """Bit-exact against the oracle's CUDA rule; against the reference's Triton encoder
    (golden_cuda.pt) equal except between centroids whose scores tie to fp32 summation order."""
    for c in golden_cuda["pq_encode"]:
        M, K, d_sub = c["centroids"].shape
        pq = qz.ProductQuantizer(M * d_sub, d_sub, int(math.log2(K)), device=cuda)
        pq.centroids = c["centroids"].to(cuda)
        codes = pq.quantize(c["X"].to(cuda)).cpu()
        assert codes.dtype == torch.int64
        assert torch.equal(codes, oracle.pq_encode(c["X"], c["centroids"]))
        diff = codes != c["codes"]
        if diff.any():
            sc = oracle.quant.pq_encode_scores(c["X"], c["centroids"])
            a = sc.gather(-1, codes.unsqueeze(-1)).squeeze(-1)[diff]
            b = sc.gather(-1, c["codes"].unsqueeze(-1)).squeeze(-1)[diff]
            assert torch.allclose(a, b, rtol=1e-5, atol=1e-5)
        assert diff.float().mean() < 1e-3


def test_fakequant_and_kivi_quantizer_bit_exact(cuda, golden_cuda):
    """Against the reference's quantizers run on a CUDA device, and the oracle's CUDA rule."""
    for c in golden_cuda["fakequant"]:
        y = qz._asym_uniform_fakequant(c["x"].to(cuda), c["levels"], c["dim"])
        assert torch.equal(y.cpu(), c["y"])
    for c in golden_cuda["kivi_quantizer"]:
        q = qz.KIVIQuantizer(c["bits"], c["group_size"], c["residual_length"])
        assert torch.equal(q.quantize_key(c["k"].to(cuda)).cpu(), c["k_fq"])
        assert torch.equal(q.quantize_value(c["v"].to(cuda)).cpu(), c["v_fq"])
    g = gen(5)
    k = torch.randn(2, 4, 1000, 128, generator=g).bfloat16()
    for bits in (2, 4):
        q = qz.KIVIQuantizer(bits, 32, 128)
        assert torch.equal(q.quantize_key(k.to(cuda)).cpu(), oracle.kivi_quantize_key(k, bits, 32, 128))
        assert torch.equal(q.quantize_value(k.to(cuda)).cpu(), oracle.kivi_quantize_value(k, bits, 32, 128))
