"""Generate golden vectors by running the reference's quantizers on a CUDA device.

Usage (on a machine with a GPU and the reference installed, e.g. into ``baseline/_ref``):

    python tests/golden/make_golden_cuda.py [--reference baseline/_ref]

The reference's quantize / pack / encode steps are PyTorch expressions (and, for
``ProductQuantizer.quantize``, a Triton kernel) whose results depend on the device:
PyTorch divides a tensor by a Python number on a CUDA device as a multiplication by the
number's fp32 reciprocal and on the CPU as a true division, and ``ProductQuantizer``
encodes with an f16 dot-product kernel on CUDA and with cdist + argmin on the CPU. The
decode path runs on a GPU, so the engine follows the CUDA results. This script runs the
reference's own functions (``src.attention_kernels.quantize_and_pack_score_keys``,
``src.quantization._asym_uniform_fakequant``, ``KIVIQuantizer``, ``ProductQuantizer``) on
CUDA tensors with fixed seeds, and writes inputs and outputs to
``tests/golden/golden_cuda.pt``. For each case it also records how many output elements
the same call on the CPU gives differently (``cpu_differs``), which shows the fixture
separates the two device rules.
"""
import argparse
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def _ndiff(a, b):
    if isinstance(a, (tuple, list)):
        return sum(_ndiff(x, y) for x, y in zip(a, b))
    return int((a.cpu() != b.cpu()).sum())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.path.join(ROOT, "baseline", "_ref"))
    ap.add_argument("--out", default=os.path.join(HERE, "golden_cuda.pt"))
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from src.attention_kernels import quantize_and_pack_score_keys
    from src.quantization import _asym_uniform_fakequant, KIVIQuantizer, ProductQuantizer

    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(20261202)

    def randn(*s, dtype=torch.float32, scale=1.0):
        return (torch.randn(*s, generator=g) * scale).to(dtype)

    out = {"device": torch.cuda.get_device_name(0), "torch": str(torch.__version__)}

    pack = []
    for dt in (torch.bfloat16, torch.float16, torch.float32):
        for bits in (2, 4):
            k = randn(1, 2, 48, 128, dtype=dt, scale=3.0)
            k[0, 0, 3, 32:64] = 0.75  # a constant group: range 0 -> scale clamp(1e-8)
            k[0, 1, 5, :] = k[0, 1, 5, :] * 40.0  # wide-range token
            p, s, z = quantize_and_pack_score_keys(k.to(dev), bits, 32)
            cpu = quantize_and_pack_score_keys(k, bits, 32)
            pack.append(dict(k=k, bits=bits, group_size=32, packed=p.cpu(), scale=s.cpu(), zero=z.cpu(),
                             cpu_differs=_ndiff((p, s, z), cpu)))
    out["pack_score_keys"] = pack

    fq = []
    for dt in (torch.float32, torch.bfloat16):
        for levels, dim in ((4, 3), (16, 3), (4, 2), (16, 2)):
            x = randn(2, 2, 40, 32, dtype=dt, scale=2.0)
            y = _asym_uniform_fakequant(x.to(dev), levels, dim).cpu()
            fq.append(dict(x=x, levels=levels, dim=dim, y=y,
                           cpu_differs=_ndiff(y, _asym_uniform_fakequant(x, levels, dim))))
    out["fakequant"] = fq

    kq = []
    for dt in (torch.bfloat16, torch.float16, torch.float32):
        for bits in (2, 4):
            for S in (100, 20):
                k = randn(1, 2, S, 32, dtype=dt, scale=2.0)
                v = randn(1, 2, S, 32, dtype=dt, scale=2.0)
                qz = KIVIQuantizer(bits=bits, group_size=32, residual_length=32)
                kf, vf = qz.quantize_key(k.to(dev)).cpu(), qz.quantize_value(v.to(dev)).cpu()
                kq.append(dict(k=k, v=v, bits=bits, group_size=32, residual_length=32, k_fq=kf, v_fq=vf,
                               cpu_differs=_ndiff((kf, vf), (qz.quantize_key(k), qz.quantize_value(v)))))
    out["kivi_quantizer"] = kq

    pqe = []
    for bits, d_sub in ((8, 8), (3, 8), (4, 16)):
        D = 64
        C = randn(D // d_sub, 2 ** bits, d_sub)
        for dt in (torch.float32, torch.bfloat16, torch.float16):
            X = randn(160, D, dtype=dt)
            pq = ProductQuantizer(D, d_sub, bits, device="cuda")
            pq.centroids = C.to(dev)
            codes = pq.quantize(X.to(dev)).cpu()
            pc = ProductQuantizer(D, d_sub, bits, device="cpu")
            pc.centroids = C.clone()
            pqe.append(dict(X=X, centroids=C.clone(), codes=codes,
                            cpu_differs=_ndiff(codes, pc.quantize(X.float()))))
    out["pq_encode"] = pqe

    torch.save(out, args.out)
    for name in ("pack_score_keys", "fakequant", "kivi_quantizer", "pq_encode"):
        print(name, [c["cpu_differs"] for c in out[name]])
    print("wrote", args.out, os.path.getsize(args.out), "bytes")


if __name__ == "__main__":
    main()
