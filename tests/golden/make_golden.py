"""Generate golden vectors by running the reference project's own CPU-runnable code.

Usage (in a container where the reference checkout is present):

    python tests/golden/make_golden.py --reference <path-to-saifmb0-bytes-checkout>

Every output tensor in ``tests/golden/*.pt`` is produced by a function of the
reference itself (``src.attention_kernels``, ``src.quantization``,
``benchmarks.sparse_attention``, ``benchmarks.kivi_latency``), imported from the
checkout and run on the CPU with fixed seeds. Where the reference's entry point is a
Triton kernel (the decode-attention kernels), the golden output comes from the
reference's own exact attention routine ``attend_topk`` over all keys, which is the
math those kernels implement. ``benchmarks.kivi_latency`` insists on a KIVI checkout
at import time; a stub ``quant`` package in a temporary directory satisfies that
import (only its pure-torch helpers are called).
"""
import argparse
import math
import os
import sys
import tempfile

import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _kivi_stub_dir():
    d = tempfile.mkdtemp(prefix="kivi_stub_")
    os.makedirs(os.path.join(d, "quant"))
    open(os.path.join(d, "quant", "__init__.py"), "w").close()
    for name, fn in (("matmul", "cuda_bmm_fA_qB_outer"),
                     ("new_pack", "triton_quantize_and_pack_along_last_dim")):
        with open(os.path.join(d, "quant", name + ".py"), "w") as f:
            f.write(f"def {fn}(*a, **k):\n    raise RuntimeError('stub')\n")
    return d


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    os.environ["KIVI_REPO"] = _kivi_stub_dir()

    from src.attention_kernels import quantize_and_pack_score_keys
    from src.quantization import _asym_uniform_fakequant, KIVIQuantizer, ProductQuantizer
    from benchmarks.sparse_attention import select_topk, _quest_select, attend_topk, repeat_kv
    from benchmarks import kivi_latency as kl

    g = torch.Generator().manual_seed(20260101)

    def randn(*s, dtype=torch.float32):
        return torch.randn(*s, generator=g).to(dtype)

    out = {}

    # a6: score-key pack (per-token groups of 32 channels), bf16 / fp16 / fp32 inputs
    pack = []
    for dt in (torch.bfloat16, torch.float16, torch.float32):
        for bits in (2, 4):
            k = randn(1, 2, 24, 128, dtype=dt)
            k[0, 0, 3, 32:64] = 0.75  # a constant group: range 0 -> scale clamp(1e-8)
            k[0, 1, 5, :] = k[0, 1, 5, :] * 40.0  # wide-range token
            p, s, z = quantize_and_pack_score_keys(k, bits, 32)
            pack.append(dict(k=k, bits=bits, group_size=32, packed=p, scale=s, zero=z))
    out["pack_score_keys"] = pack

    # a5: asymmetric uniform fake-quant and the KIVI quantizer
    fq = []
    for levels, dim in ((4, 3), (16, 3), (4, 2), (16, 2)):
        x = randn(2, 2, 40, 32)
        fq.append(dict(x=x, levels=levels, dim=dim, y=_asym_uniform_fakequant(x, levels, dim)))
    out["fakequant"] = fq
    kq = []
    for bits in (2, 4):
        for S in (200, 20):
            k = randn(1, 2, S, 32, dtype=torch.bfloat16)
            v = randn(1, 2, S, 32, dtype=torch.bfloat16)
            qz = KIVIQuantizer(bits=bits, group_size=32, residual_length=32)
            kq.append(dict(k=k, v=v, bits=bits, group_size=32, residual_length=32,
                           k_fq=qz.quantize_key(k), v_fq=qz.quantize_value(v)))
    out["kivi_quantizer"] = kq

    # a16: PQ encode, CPU cdist path of ProductQuantizer.quantize
    pqe = []
    for bits, d_sub in ((8, 8), (3, 8), (8, 4)):
        D = 64
        pq = ProductQuantizer(D, d_sub, bits, device="cpu")
        pq.centroids = randn(D // d_sub, 2 ** bits, d_sub)
        X = randn(200, D)
        pqe.append(dict(X=X, centroids=pq.centroids.clone(), codes=pq.quantize(X)))
    out["pq_encode"] = pqe

    # a9/a10/a11: streaming exact top-k, Quest page selection, exact attend (decode row)
    sel = []
    for (B, Hq, S, D, kb, kc) in ((2, 4, 300, 32, 20, 64), (1, 2, 96, 16, 200, 32)):
        q = randn(B, Hq, 1, D)
        keys = randn(B, Hq, S, D)
        qpos = torch.tensor([S - 1])
        idx = select_topk("exact", q, keys, qpos, S, kb, kc, 0.17)
        sel.append(dict(q=q, keys=keys, S=S, kb=kb, k_chunk=kc, scaling=0.17, idx=idx))
    out["select_topk"] = sel
    quest = []
    for (B, Hk, G, S, D, kb, page) in ((2, 2, 2, 300, 32, 40, 16), (1, 1, 4, 256, 64, 64, 16)):
        k = randn(B, Hk, S, D, dtype=torch.bfloat16)
        v = randn(B, Hk, S, D, dtype=torch.bfloat16)
        q = randn(B, Hk * G, 1, D, dtype=torch.bfloat16)
        kr = repeat_kv(k, G)
        vr = repeat_kv(v, G)
        qpos = torch.tensor([S - 1])
        idx = _quest_select(q.float(), kr.float(), qpos, S, kb, page, 0.125)
        o = attend_topk(q.float(), kr.float(), vr.float(), idx, qpos, 0.125)
        quest.append(dict(q=q, k=k, v=v, S=S, kb=kb, page=page, scaling=0.125, idx=idx, out=o))
    out["quest"] = quest

    # a1/a2 dense decode and a13/a14 PQ-LUT decode: the reference's exact attention
    # (attend_topk over every key) is the math of its Triton decode kernels.
    dense = []
    for (B, Hk, G, S, D, fp8) in ((2, 2, 4, 128, 64, False), (2, 2, 4, 128, 64, True),
                                  (1, 4, 7, 96, 128, False)):
        q = randn(B, Hk * G, 1, D, dtype=torch.bfloat16)
        k = randn(B, Hk, S, D, dtype=torch.bfloat16)
        v = randn(B, Hk, S, D, dtype=torch.bfloat16)
        if fp8:
            k, v = k.to(torch.float8_e4m3fn), v.to(torch.float8_e4m3fn)
        idx = torch.arange(S).expand(B, Hk * G, 1, S)
        o = attend_topk(q.float(), repeat_kv(k.float(), G), repeat_kv(v.float(), G), idx,
                        torch.tensor([S - 1]), 1.0)
        dense.append(dict(q=q, k=k, v=v, out=o))
    out["dense_decode"] = dense

    pql = []
    for (B, Hk, G, S, D, C_out) in ((1, 2, 4, 128, 64, 0), (1, 2, 4, 128, 64, 2)):
        d_sub, M = 8, D // 8
        pq = ProductQuantizer(D, d_sub, 8, device="cpu")
        pq.centroids = randn(M, 256, d_sub)
        codes = torch.randint(0, 256, (B, Hk, S, M), generator=g).to(torch.uint8)
        k_hat = pq.dequantize(codes)  # [B,Hk,S,D]
        q_rot = randn(B, Hk * G, D)
        lut = torch.einsum("bhmd,mkd->bhmk", q_rot.view(B, Hk * G, M, d_sub), pq.centroids)
        v = randn(B, Hk, S, D, dtype=torch.bfloat16)
        k_out = randn(B, Hk, S, C_out, dtype=torch.bfloat16) * 20
        q_out = randn(B, Hk * G, C_out, dtype=torch.bfloat16)
        qc = torch.cat([q_rot, q_out.float()], -1).unsqueeze(2)
        kc = torch.cat([k_hat, k_out.float()], -1)
        idx = torch.arange(S).expand(B, Hk * G, 1, S)
        # attend_topk takes one width for q, k and v: pad v with C_out zero columns
        vpad = torch.cat([v.float(), torch.zeros(B, Hk, S, C_out)], -1)
        o = attend_topk(qc, repeat_kv(kc, G), repeat_kv(vpad, G), idx,
                        torch.tensor([S - 1]), 1.0)[..., :D]
        pql.append(dict(lut=lut, codes=codes, centroids=pq.centroids.clone(), v=v,
                        k_out=k_out, q_out=q_out, out=o))
    out["pq_lut_decode"] = pql

    # a3/a4: KIVI in-tree unpack, dequant and dense reference decode
    kv = []
    for bits in (2, 4):
        B, Hk, G, D, Sq, R = 1, 2, 4, 128, 128, 64
        fpi = 32 // bits
        Kq = torch.randint(-2 ** 31, 2 ** 31 - 1, (B, Hk, D, Sq // fpi), generator=g, dtype=torch.int64).to(torch.int32)
        Vq = torch.randint(-2 ** 31, 2 ** 31 - 1, (B, Hk, Sq, D // fpi), generator=g, dtype=torch.int64).to(torch.int32)
        K_scale = (torch.rand(B, Hk, D, Sq // 32, generator=g) * 0.5 + 0.05).to(torch.float16)
        K_mn = (randn(B, Hk, D, Sq // 32) - 1.0).to(torch.float16)
        V_scale = (torch.rand(B, Hk, Sq, D // 32, generator=g) * 0.5 + 0.05).to(torch.float16)
        V_mn = (randn(B, Hk, Sq, D // 32) - 1.0).to(torch.float16)
        K_res = randn(B, Hk, R, D, dtype=torch.bfloat16)
        V_res = randn(B, Hk, R, D, dtype=torch.bfloat16)
        Q = randn(B, Hk * G, 1, D, dtype=torch.bfloat16)
        K_dq = kl.dequant_k(Kq, K_scale, K_mn, 32, bits)
        V_dq = kl.dequant_v(Vq, V_scale, V_mn, 32, bits)
        o = kl.kivi_decode_attn_ref(Q.float(), K_dq.float(), K_res.float(), V_dq.float(),
                                    V_res.float(), G)
        kv.append(dict(bits=bits, Q=Q, Kq=Kq, K_scale=K_scale, K_mn=K_mn, Vq=Vq,
                       V_scale=V_scale, V_mn=V_mn, K_res=K_res, V_res=V_res,
                       K_unpacked=kl.unpack_tensor_last_dim(Kq, bits),
                       K_dq=K_dq, V_dq=V_dq, out=o))
    out["kivi"] = kv

    path = os.path.join(HERE, "golden.pt")
    torch.save(out, path)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
