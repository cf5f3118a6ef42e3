"""Thin torch-facing wrappers over the C ABI: descriptor building, layout
normalisation, workspace allocation and error mapping. Every function launches
CUDA kernels through ``libbdecode.so`` on the current stream; none has a CPU path.
"""
import ctypes
import math

import torch

from . import _native as N

_f = {}


def _fn(name, argtypes, restype=ctypes.c_int):
    f = _f.get(name)
    if f is None:
        f = getattr(N.lib(), name)
        f.argtypes = argtypes
        f.restype = restype
        _f[name] = f
    return f


P = ctypes.POINTER(N.BdTensor)
VP = ctypes.c_void_p
SZ = ctypes.c_size_t
I = ctypes.c_int
F = ctypes.c_float


def rows_aligned(t, align=16):
    """Return t, or a contiguous copy when its rows are not `align`-byte addressable."""
    es = t.element_size()
    ok = t.data_ptr() % align == 0 and (t.dim() == 0 or t.stride(-1) == 1 or t.shape[-1] <= 1)
    if ok:
        for i in range(t.dim() - 1):
            if t.shape[i] > 1 and (t.stride(i) * es) % align:
                ok = False
                break
    return t if ok else t.contiguous()


def inner_contig(t):
    return t if (t.dim() == 0 or t.stride(-1) == 1 or t.shape[-1] <= 1) else t.contiguous()


def _ws(nbytes, device):
    if nbytes == 0:
        return None, 0
    buf = torch.empty(int(nbytes), dtype=torch.uint8, device=device)
    return buf, int(nbytes)


def _ptr(buf):
    return VP(buf.data_ptr()) if buf is not None else VP(0)


def decode_attn(q3, k, v, scaling, out):
    """q3 [B,Hq,D], k/v [B,Hk,S,D] bf16|fp8 -> writes out [B,Hq,D]."""
    N.require_cuda(q3, k, v, out)
    k = rows_aligned(k)
    v = rows_aligned(v)
    q3 = inner_contig(q3)
    dq, dk, dv, do = N.desc(q3), N.desc(k), N.desc(v), N.desc(out)
    nws = _fn("bd_decode_attn_workspace", [P, P], SZ)(ctypes.byref(dq), ctypes.byref(dk))
    buf, nb = _ws(nws, q3.device)
    st = N.stream_of(q3)
    rc = _fn("bd_decode_attn", [P, P, P, P, F, VP, SZ, VP])(
        ctypes.byref(dq), ctypes.byref(dk), ctypes.byref(dv), ctypes.byref(do), float(scaling), _ptr(buf), nb, st)
    N.check(rc, "bd_decode_attn")
    return out


def decode_attn_partial(q3, k, v, scaling):
    """Shard partials (m, l, o) of dense decode over this device's keys."""
    N.require_cuda(q3, k, v)
    k = rows_aligned(k)
    v = rows_aligned(v)
    q3 = inner_contig(q3)
    B, Hq, D = q3.shape
    m = torch.empty(B, Hq, dtype=torch.float32, device=q3.device)
    l = torch.empty_like(m)
    o = torch.empty(B, Hq, D, dtype=torch.float32, device=q3.device)
    dq, dk, dv = N.desc(q3), N.desc(k), N.desc(v)
    nws = _fn("bd_decode_attn_workspace", [P, P], SZ)(ctypes.byref(dq), ctypes.byref(dk))
    buf, nb = _ws(nws, q3.device)
    dm, dl, dO = N.desc(m), N.desc(l), N.desc(o)
    rc = _fn("bd_decode_attn_partial", [P, P, P, F, P, P, P, VP, SZ, VP])(
        ctypes.byref(dq), ctypes.byref(dk), ctypes.byref(dv), float(scaling), ctypes.byref(dm), ctypes.byref(dl),
        ctypes.byref(dO), _ptr(buf), nb, N.stream_of(q3))
    N.check(rc, "bd_decode_attn_partial")
    return m, l, o


def lse_combine(m, l, o, out_dtype=torch.bfloat16):
    """m,l [n,B,Hq], o [n,B,Hq,D] fp32 -> [B,Hq,D]."""
    N.require_cuda(m, l, o)
    m, l, o = m.contiguous(), l.contiguous(), o.contiguous()
    n, B, Hq, D = o.shape
    out = torch.empty(B, Hq, D, dtype=out_dtype, device=o.device)
    dm, dl, dO, dout = N.desc(m), N.desc(l), N.desc(o), N.desc(out)
    rc = _fn("bd_lse_combine", [P, P, P, P, VP])(
        ctypes.byref(dm), ctypes.byref(dl), ctypes.byref(dO), ctypes.byref(dout), N.stream_of(o))
    N.check(rc, "bd_lse_combine")
    return out


def kivi_decode(Q3, Kq, Ks, Km, Kr, Vq, Vs, Vm, Vr, bits, group_size, scaling, out):
    N.require_cuda(Q3, Kq, Ks, Km, Kr, Vq, Vs, Vm, Vr, out)
    Kq, Vq = rows_aligned(Kq, 16), rows_aligned(Vq, 16)
    Ks, Km, Vs, Vm = (rows_aligned(t, 8) for t in (Ks, Km, Vs, Vm))
    Kr, Vr = rows_aligned(Kr), rows_aligned(Vr)
    Q3 = inner_contig(Q3)
    ds = [N.desc(t) for t in (Q3, Kq, Ks, Km, Kr, Vq, Vs, Vm, Vr)]
    nws = _fn("bd_kivi_decode_attn_workspace", [P, P, P, I], SZ)(
        ctypes.byref(ds[0]), ctypes.byref(ds[1]), ctypes.byref(ds[4]), int(bits))
    buf, nb = _ws(nws, Q3.device)
    do = N.desc(out)
    rc = _fn("bd_kivi_decode_attn", [P] * 9 + [I, I, F, P, VP, SZ, VP])(
        *[ctypes.byref(d) for d in ds], int(bits), int(group_size), float(scaling), ctypes.byref(do), _ptr(buf), nb,
        N.stream_of(Q3))
    N.check(rc, "bd_kivi_decode_attn")
    return out


def kivi_pack(x, group_size, bits):
    N.require_cuda(x)
    x = inner_contig(x)
    lead = tuple(x.shape[:-1])
    n = x.shape[-1]
    fpi = 32 // bits
    if n % group_size:
        raise ValueError("last dim must be a multiple of group_size")
    code = torch.empty(lead + (n // fpi,), dtype=torch.int32, device=x.device)
    scale = torch.empty(lead + (n // group_size,), dtype=x.dtype, device=x.device)
    mn = torch.empty_like(scale)
    if x.dim() > 4:
        x = x.reshape((-1,) + tuple(x.shape[-3:])) if x.is_contiguous() else x.contiguous().reshape(
            (-1,) + tuple(x.shape[-3:]))
    dx = N.desc(x)
    dc, ds_, dm = (N.desc(t.reshape(tuple(x.shape[:-1]) + (t.shape[-1],))) for t in (code, scale, mn))
    rc = _fn("bd_kivi_pack_last_dim", [P, I, I, P, P, P, VP])(
        ctypes.byref(dx), int(group_size), int(bits), ctypes.byref(dc), ctypes.byref(ds_), ctypes.byref(dm),
        N.stream_of(x))
    N.check(rc, "bd_kivi_pack_last_dim")
    return code, scale, mn


def kivi_gemv(group_size, fA, qB, scales, zeros, bits):
    N.require_cuda(fA, qB, scales, zeros)
    fA = inner_contig(fA.to(torch.float16))
    qB, scales, zeros = inner_contig(qB), inner_contig(scales.to(torch.float16)), inner_contig(zeros.to(torch.float16))
    B, Hq, M, K = fA.shape
    Ncols = qB.shape[-1] * (32 // bits)
    out = torch.empty(B, Hq, M, Ncols, dtype=torch.float16, device=fA.device)
    ds = [N.desc(t) for t in (fA, qB, scales, zeros, out)]
    rc = _fn("bd_kivi_gemv_outer", [I, P, P, P, P, I, P, VP])(
        int(group_size), ctypes.byref(ds[0]), ctypes.byref(ds[1]), ctypes.byref(ds[2]), ctypes.byref(ds[3]),
        int(bits), ctypes.byref(ds[4]), N.stream_of(fA))
    N.check(rc, "bd_kivi_gemv_outer")
    return out
