"""GPU parity: dense bf16/fp8 decode and the KIVI path against the CPU oracle.

Tolerance: attention outputs agree within 2e-2 max-abs
and 1e-3 mean-abs; packing is bit-exact.
"""
import math

import pytest
import torch

import oracle
from bytes_b200 import attention_kernels as ak
from bytes_b200 import kivi as kv

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_ABS = 1e-3


def close(out, ref, max_abs=MAX_ABS, mean_abs=MEAN_ABS):
    d = (out.float().cpu() - ref.float().cpu()).abs()
    assert torch.isfinite(out.float()).all()
    assert d.max().item() <= max_abs, f"max abs diff {d.max().item()}"
    assert d.mean().item() <= mean_abs, f"mean abs diff {d.mean().item()}"


def gen(seed):
    return torch.Generator().manual_seed(seed)


@pytest.mark.parametrize("B,Hq,Hk,S,D", [
    (2, 8, 2, 128, 64),       # reference test shape (test_correctness.py:52-58)
    (1, 28, 4, 8192, 128),    # config 0
    (2, 8, 2, 1, 128),        # single key
    (1, 7, 1, 65, 128),       # ragged tail, G=7
    (2, 16, 1, 300, 128),     # G=16 (two head tiles)
    (1, 32, 1, 200, 64),      # G=32 (two head chunks)
    (3, 4, 4, 1000, 128),     # G=1
])
@pytest.mark.parametrize("kv_dtype", [torch.bfloat16, torch.float8_e4m3fn])
def test_dense_decode_matches_oracle(cuda, B, Hq, Hk, S, D, kv_dtype):
    g = gen(B * 1000 + S)
    q = torch.randn(B, Hq, 1, D, generator=g).bfloat16()
    k = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    v = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    if kv_dtype == torch.float8_e4m3fn:
        k, v = k.to(kv_dtype), v.to(kv_dtype)
    ref = oracle.decode_attn_dense(q, k, v, 1.0)
    fn = ak.decode_attn_bf16 if kv_dtype == torch.bfloat16 else ak.decode_attn_fp8
    out = fn(q.to(cuda), k.to(cuda), v.to(cuda))
    assert out.shape == (B, Hq, 1, D) and out.dtype == q.dtype
    close(out, ref)


def test_dense_decode_golden(cuda, golden):
    for c in golden["dense_decode"]:
        fn = ak.decode_attn_fp8 if c["k"].dtype == torch.float8_e4m3fn else ak.decode_attn_bf16
        out = fn(c["q"].to(cuda), c["k"].to(cuda), c["v"].to(cuda))
        close(out, c["out"])


def test_dense_decode_config0_outlier_channels(cuda):
    """Config 0: N(0,1) bf16 with 4 of 128 key channels x8, q pre-scaled by 1/sqrt(128)."""
    g = gen(0)
    B, Hq, Hk, S, D = 1, 28, 4, 8192, 128
    q = (torch.randn(B, Hq, 1, D, generator=g) / math.sqrt(D)).bfloat16()
    k = torch.randn(B, Hk, S, D, generator=g)
    ch = torch.randperm(D, generator=g)[:4]
    k[..., ch] *= 8
    k = k.bfloat16()
    v = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    out = ak.decode_attn_bf16(q.to(cuda), k.to(cuda), v.to(cuda))
    close(out, oracle.decode_attn_dense(q, k, v, 1.0))


def test_dense_decode_strided_inputs(cuda):
    g = gen(5)
    base_k = torch.randn(2, 2, 400, 128, generator=g).bfloat16().to(cuda)
    base_v = torch.randn(2, 2, 400, 128, generator=g).bfloat16().to(cuda)
    k, v = base_k[:, :, 50:350], base_v[:, :, 100:400]  # slices along S (row-aligned views)
    qb = torch.randn(2, 1, 8, 128, generator=g).bfloat16().to(cuda)
    q = qb.transpose(1, 2)  # [2,8,1,128] non-contiguous
    out = ak.decode_attn_bf16(q, k, v)
    close(out, oracle.decode_attn_dense(q.cpu(), k.cpu(), v.cpu(), 1.0))


def test_dense_decode_empty_context_is_nan(cuda):
    q = torch.randn(1, 4, 1, 128).bfloat16().to(cuda)
    k = torch.zeros(1, 1, 0, 128, dtype=torch.bfloat16, device=cuda)
    out = ak.decode_attn_bf16(q, k, k)
    assert torch.isnan(out.float()).all()


def test_dense_decode_graph_capture(cuda):
    g = gen(9)
    q = torch.randn(2, 28, 1, 128, generator=g).bfloat16().to(cuda)
    k = torch.randn(2, 4, 4096, 128, generator=g).bfloat16().to(cuda)
    v = torch.randn(2, 4, 4096, 128, generator=g).bfloat16().to(cuda)
    out = ak.decode_attn_bf16(q, k, v)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        o2 = ak.decode_attn_bf16(q, k, v)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, o2)


# ----------------------------------------------------------------------------- KIVI

def _kivi_inputs(B, Hq, Hk, S, R, D, seed, bits, outliers=True):
    g = gen(seed)
    k = torch.randn(B, Hk, S, D, generator=g)
    if outliers:
        ch = torch.randperm(D, generator=g)[:4]
        k[..., ch] *= 8
    k = k.bfloat16()
    v = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    q = torch.randn(B, Hq, 1, D, generator=g).bfloat16()
    Sq = S - R
    Kt = k[:, :, :Sq].transpose(2, 3).contiguous().to(torch.float16)
    Vt = v[:, :, :Sq].contiguous().to(torch.float16)
    return q, k, v, Kt, Vt, Sq


@pytest.mark.parametrize("bits", [2, 4])
def test_kivi_pack_bit_exact(cuda, bits):
    g = gen(11)
    x = torch.randn(2, 3, 128, 512, generator=g).to(torch.float16)
    x[0, 0, 5, 64:96] = 0.5  # constant group
    code, scale, mn = kv.triton_quantize_and_pack_along_last_dim(x.to(cuda), 32, bits)
    rc, rs, rm = oracle.kivi_pack_last_dim(x, 32, bits)
    assert torch.equal(code.cpu(), rc)
    assert torch.equal(scale.cpu(), rs)
    assert torch.equal(mn.cpu(), rm)


@pytest.mark.parametrize("bits", [2, 4])
@pytest.mark.parametrize("B,Hq,Hk,S,R", [
    (2, 8, 2, 256 + 128, 128),    # reference integrity-gate shape (kivi_latency.py:104-110)
    (8, 28, 4, 16384, 128),       # config 1
    (1, 7, 1, 32 + 16, 16),       # one group + small residual
    (1, 16, 1, 1024 + 5, 5),      # G=16 (two head chunks)
    (2, 4, 4, 96, 0),             # no residual window
    (1, 7, 1, 512 + 300, 300),    # window longer than a tile: spread over three splits
    (1, 7, 1, 40000 + 64, 64),    # long packed pass (> 256 tiles): the four-CTAs-per-SM build
])
def test_kivi_decode_matches_oracle(cuda, bits, B, Hq, Hk, S, R):
    D = 128
    q, k, v, Kt, Vt, Sq = _kivi_inputs(B, Hq, Hk, S, R, D, seed=S + bits, bits=bits)
    Kq, Ks, Km = oracle.kivi_pack_last_dim(Kt, 32, bits)
    Vq, Vs, Vm = oracle.kivi_pack_last_dim(Vt, 32, bits)
    Kr, Vr = k[:, :, Sq:].contiguous(), v[:, :, Sq:].contiguous()
    ref = oracle.kivi_decode_attn(q, Kq, Ks, Km, Kr, Vq, Vs, Vm, Vr, bits)
    dev = [t.to(cuda) for t in (q, Kq, Ks, Km, Kr, Vq, Vs, Vm, Vr)]
    out = kv.kivi_decode_attn(*dev, bits, 32)
    assert out.shape == (B, Hq, 1, D) and out.dtype == torch.bfloat16
    close(out, ref)


@pytest.mark.parametrize("bits", [2, 4])
def test_kivi_decode_padded_cache_rows(cuda, bits):
    """Caches living inside wider buffers (row pitch > row length): the packed pass then
    stages tiles with per-thread async copies instead of tensor-map (TMA) loads."""
    B, Hq, Hk, S, R, D = 2, 14, 2, 1024 + 64 + 32, 32, 128
    q, k, v, Kt, Vt, Sq = _kivi_inputs(B, Hq, Hk, S, R, D, seed=77 + bits, bits=bits)
    Kq, Ks, Km = oracle.kivi_pack_last_dim(Kt, 32, bits)
    Vq, Vs, Vm = oracle.kivi_pack_last_dim(Vt, 32, bits)
    Kr, Vr = k[:, :, Sq:].contiguous(), v[:, :, Sq:].contiguous()
    ref = oracle.kivi_decode_attn(q, Kq, Ks, Km, Kr, Vq, Vs, Vm, Vr, bits)

    def padded(t, extra):  # same values, last-dim rows padded by `extra` elements
        buf = torch.full(t.shape[:-1] + (t.shape[-1] + extra,), 7, dtype=t.dtype, device=cuda)
        buf[..., :t.shape[-1]] = t.to(cuda)
        return buf[..., :t.shape[-1]]

    Kq_d, Vq_d = padded(Kq, 4), padded(Vq, 4)  # 16 extra bytes per row
    assert Kq_d.stride(2) != Kq_d.shape[3] and Vq_d.stride(2) != Vq_d.shape[3]
    dev = [t.to(cuda) for t in (q, Ks, Km, Kr, Vs, Vm, Vr)]
    out = kv.kivi_decode_attn(dev[0], Kq_d, dev[1], dev[2], dev[3], Vq_d, dev[4], dev[5], dev[6], bits, 32)
    close(out, ref)


def test_kivi_decode_unaligned_output_rows(cuda):
    """Output rows whose pitch takes no 8-byte stores: the split slots are merged by the
    separate combine kernel instead of the last CTA of each group."""
    from bytes_b200 import _ops
    bits, D = 2, 128
    B, Hq, Hk, S, R = 2, 14, 2, 1024 + 128, 128
    q, k, v, Kt, Vt, Sq = _kivi_inputs(B, Hq, Hk, S, R, D, seed=91, bits=bits)
    Kq, Ks, Km = oracle.kivi_pack_last_dim(Kt, 32, bits)
    Vq, Vs, Vm = oracle.kivi_pack_last_dim(Vt, 32, bits)
    Kr, Vr = k[:, :, Sq:].contiguous(), v[:, :, Sq:].contiguous()
    ref = oracle.kivi_decode_attn(q, Kq, Ks, Km, Kr, Vq, Vs, Vm, Vr, bits)
    dev = [t.to(cuda) for t in (q, Kq, Ks, Km, Kr, Vq, Vs, Vm, Vr)]
    buf = torch.zeros(B, Hq, D + 2, dtype=torch.bfloat16, device=cuda)
    out = buf[..., :D]
    _ops.kivi_decode(dev[0][:, :, 0, :], *dev[1:], bits, 32, 1.0 / D ** 0.5, out)
    close(out.unsqueeze(2), ref)
    assert (buf[..., D:] == 0).all()


def test_kivi_gemv_matches_oracle(cuda):
    g = gen(13)
    bits = 2
    fA = torch.randn(2, 8, 1, 128, generator=g).half()
    x = torch.randn(2, 2, 128, 256, generator=g).half()
    qB, sc, zr = oracle.kivi_pack_last_dim(x, 32, bits)
    out = kv.cuda_bmm_fA_qB_outer(32, fA.to(cuda), qB.to(cuda), sc.to(cuda), zr.to(cuda), bits)
    ref = oracle.kivi_gemv_outer(32, fA, qB, sc, zr, bits)
    assert out.dtype == torch.float16 and out.shape == (2, 8, 1, 256)
    d = (out.float().cpu() - ref.float()).abs().max().item()
    assert d < 5e-2 * max(1.0, ref.float().abs().max().item() / 10)


def test_kivi_decode_graph_capture(cuda):
    bits, D = 2, 128
    q, k, v, Kt, Vt, Sq = _kivi_inputs(2, 28, 4, 2048 + 128, 128, D, seed=3, bits=bits)
    Kq, Ks, Km = kv.triton_quantize_and_pack_along_last_dim(Kt.to(cuda), 32, bits)
    Vq, Vs, Vm = kv.triton_quantize_and_pack_along_last_dim(Vt.to(cuda), 32, bits)
    Kr, Vr = k[:, :, Sq:].contiguous().to(cuda), v[:, :, Sq:].contiguous().to(cuda)
    qd = q.to(cuda)
    out = kv.kivi_decode_attn(qd, Kq, Ks, Km, Kr, Vq, Vs, Vm, Vr, bits)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        o2 = kv.kivi_decode_attn(qd, Kq, Ks, Km, Kr, Vq, Vs, Vm, Vr, bits)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, o2)
