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


def _is_rows_aligned(t, align):
    es = t.element_size()
    if t.data_ptr() % align or not (t.dim() == 0 or t.stride(-1) == 1 or t.shape[-1] <= 1):
        return False
    return all(t.shape[i] <= 1 or (t.stride(i) * es) % align == 0 for i in range(t.dim() - 1))


def rows_aligned(t, align=16):
    """Return t, or a copy whose rows start on `align`-byte boundaries.

    The copy pads the innermost dim of its storage (the returned view has t's shape),
    so every leading stride is a multiple of `align` bytes.
    """
    if _is_rows_aligned(t, align):
        return t
    es = t.element_size()
    n = t.shape[-1]
    per = max(1, align // es)
    n_pad = (n + per - 1) // per * per
    buf = torch.zeros(tuple(t.shape[:-1]) + (n_pad,), dtype=t.dtype, device=t.device)
    buf[..., :n] = t
    return buf[..., :n]


def inner_contig(t):
    return t if (t.dim() == 0 or t.stride(-1) == 1 or t.shape[-1] <= 1) else t.contiguous()


def _ws(nbytes, device):
    if nbytes == 0:
        return None, 0
    buf = torch.empty(int(nbytes), dtype=torch.uint8, device=device)
    return buf, int(nbytes)


def _ptr(buf):
    return VP(buf.data_ptr()) if buf is not None else VP(0)


# status codes after which a call is retried with re-laid-out copies of its inputs
_RELAYOUT = (4, 5)  # BD_ERR_STRIDE, BD_ERR_ALIGN


def decode_attn(q3, k, v, scaling, out):
    """q3 [B,Hq,D], k/v [B,Hk,S,D] bf16|fp8 -> writes out [B,Hq,D]."""
    rc = N.glue().decode_attn(q3, k, v, out, float(scaling))
    if rc == 0:
        return out
    if rc not in _RELAYOUT:
        N.check(rc, "bd_decode_attn")
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


def peer_exchange_combine(m, l, o, peers_dev, rank, world, out_dtype=torch.bfloat16):
    """bd_peer_exchange_combine: this rank's m,l [B,Hq], o [B,Hq,D] fp32 -> [B,Hq,D] over all ranks.
    peers_dev: device address of the [world] table of exchange-buffer bases."""
    N.require_cuda(m, l, o)
    m, l, o = m.contiguous(), l.contiguous(), o.contiguous()
    B, Hq, D = o.shape
    out = torch.empty(B, Hq, D, dtype=out_dtype, device=o.device)
    dm, dl, do_, dout = N.desc(m), N.desc(l), N.desc(o), N.desc(out)
    rc = _fn("bd_peer_exchange_combine", [P, P, P, VP, I, I, P, VP])(
        ctypes.byref(dm), ctypes.byref(dl), ctypes.byref(do_), VP(peers_dev), int(rank), int(world),
        ctypes.byref(dout), N.stream_of(o))
    N.check(rc, "bd_peer_exchange_combine")
    return out


def split_kv_decode_peer(q3, k, v, scaling, peers_dev, rank, world, out_dtype=torch.bfloat16):
    """bd_split_kv_decode_peer: dense split pass over this rank's token shard k,v and the
    fused NVLink exchange + combine -> [B,Hq,D] over all ranks' shards."""
    N.require_cuda(q3, k, v)
    k = rows_aligned(k)
    v = rows_aligned(v)
    q3 = inner_contig(q3)
    B, Hq, D = q3.shape
    out = torch.empty(B, Hq, D, dtype=out_dtype, device=q3.device)
    dq, dk, dv, dout = N.desc(q3), N.desc(k), N.desc(v), N.desc(out)
    nws = _fn("bd_decode_attn_workspace", [P, P], SZ)(ctypes.byref(dq), ctypes.byref(dk))
    buf, nb = _ws(nws, q3.device)
    rc = _fn("bd_split_kv_decode_peer", [P, P, P, F, VP, I, I, P, VP, SZ, VP])(
        ctypes.byref(dq), ctypes.byref(dk), ctypes.byref(dv), float(scaling), VP(peers_dev), int(rank), int(world),
        ctypes.byref(dout), _ptr(buf), nb, N.stream_of(q3))
    N.check(rc, "bd_split_kv_decode_peer")
    return out


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


def kivi_decode(Q3, Kq, Ks, Km, Kr, Vq, Vs, Vm, Vr, bits, group_size, scaling, out, stages=7):
    rc = N.glue().kivi_decode(Q3, Kq, Ks, Km, Kr, Vq, Vs, Vm, Vr, int(bits), int(group_size), float(scaling), out,
                              int(stages))
    if rc == 0:
        return out
    if rc not in _RELAYOUT:
        N.check(rc, "bd_kivi_decode_attn")
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
    rc = _fn("bd_kivi_decode_attn_stages", [P] * 9 + [I, I, F, P, VP, SZ, I, VP])(
        *[ctypes.byref(d) for d in ds], int(bits), int(group_size), float(scaling), ctypes.byref(do), _ptr(buf), nb,
        int(stages), N.stream_of(Q3))
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


def kivi_append(k_new, v_new, bits, group_size, token_offset, Kq, K_scale, K_mn, Vq, V_scale, V_mn):
    """Quantize whole 32-token groups of k_new/v_new [B,Hk,Tn,D] into the caches in place."""
    N.require_cuda(k_new, v_new, Kq, K_scale, K_mn, Vq, V_scale, V_mn)
    k_new, v_new = inner_contig(k_new), inner_contig(v_new)
    if v_new.dtype != k_new.dtype:
        v_new = v_new.to(k_new.dtype)
    ds = [N.desc(t) for t in (k_new, v_new, Kq, K_scale, K_mn, Vq, V_scale, V_mn)]
    rc = _fn("bd_kivi_append", [P, P, I, I, ctypes.c_int64, P, P, P, P, P, P, VP])(
        ctypes.byref(ds[0]), ctypes.byref(ds[1]), int(bits), int(group_size), int(token_offset),
        *[ctypes.byref(d) for d in ds[2:]], N.stream_of(k_new))
    N.check(rc, "bd_kivi_append")


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


def _token_major_aligned(t):
    """[B,H,S,G] with contiguous (S,G) rows per (b,h) and every (b,h) block starting on a
    16-byte boundary (the score kernel stages whole tiles of it with 16-byte copies)."""
    B, H, S, G = t.shape
    es = t.element_size()
    ok = (t.stride(3) == 1 or G == 1) and (t.stride(2) == G or S == 1) and t.data_ptr() % 16 == 0
    ok = ok and (H == 1 or (t.stride(1) * es) % 16 == 0) and (B == 1 or (t.stride(0) * es) % 16 == 0)
    if ok:
        return t
    per = max(1, 16 // (G * es)) if (G * es) < 16 else 1
    S_pad = (S + per - 1) // per * per
    while (S_pad * G * es) % 16:
        S_pad += 1
    buf = torch.zeros(B, H, S_pad, G, dtype=t.dtype, device=t.device)
    buf[:, :, :S] = t
    return buf[:, :, :S]


def sparse_score(q3, k, scale, zero, scaling, bits, group_size):
    """q3 [B,Hq,D]; k bf16/fp8 [B,Hk,S,D] or packed u8 -> scores [B,Hq,S] f32."""
    N.require_cuda(q3, k, scale, zero)
    k = rows_aligned(k)
    q3 = inner_contig(q3)
    B, Hq, D = q3.shape
    S = k.shape[2]
    if bits in (2, 4):
        if scale is None or zero is None:
            raise ValueError("packed scores need scale and zero")
        if scale.dtype not in (torch.bfloat16, torch.float16):
            scale = scale.to(torch.bfloat16)
            zero = zero.to(torch.bfloat16)
        scale = _token_major_aligned(scale)
        zero = _token_major_aligned(zero)
    scores = torch.empty(B, Hq, S, dtype=torch.float32, device=q3.device)
    ds = [N.desc(q3), N.desc(k), N.desc(scale), N.desc(zero), N.desc(scores)]
    rc = _fn("bd_sparse_score", [P, P, P, P, F, I, I, P, VP])(
        ctypes.byref(ds[0]), ctypes.byref(ds[1]), N.ref(ds[2]), N.ref(ds[3]), float(scaling), int(bits),
        int(group_size), ctypes.byref(ds[4]), N.stream_of(q3))
    N.check(rc, "bd_sparse_score")
    return scores


def pack_score_keys(k, bits, group_size):
    N.require_cuda(k)
    k = inner_contig(k)
    B, H, S, D = k.shape
    packed = torch.empty(B, H, S, D * bits // 8, dtype=torch.uint8, device=k.device)
    scale = torch.empty(B, H, S, D // group_size, dtype=k.dtype, device=k.device)
    zero = torch.empty_like(scale)
    ds = [N.desc(t) for t in (k, packed, scale, zero)]
    rc = _fn("bd_pack_score_keys", [P, I, I, P, P, P, VP])(
        ctypes.byref(ds[0]), int(bits), int(group_size), ctypes.byref(ds[1]), ctypes.byref(ds[2]),
        ctypes.byref(ds[3]), N.stream_of(k))
    N.check(rc, "bd_pack_score_keys")
    return packed, scale, zero


def topk(scores, k, sorted=True, want_values=True, idx_dtype=torch.int64):
    """Top-k over the last dim (lower index wins ties); scores f32 with <= 3 dims."""
    N.require_cuda(scores)
    if scores.dtype != torch.float32:
        scores = scores.float()
    lead = scores.shape[:-1]
    n = scores.shape[-1]
    s = scores if scores.dim() <= 3 else scores.reshape(-1, n)
    s = inner_contig(s)
    idx = torch.empty(tuple(s.shape[:-1]) + (k,), dtype=idx_dtype, device=s.device)
    vals = torch.empty(tuple(s.shape[:-1]) + (k,), dtype=torch.float32, device=s.device) if want_values else None
    ds, di, dv = N.desc(s), N.desc(idx), N.desc(vals)
    rc = _fn("bd_topk", [P, I, I, P, P, VP])(ctypes.byref(ds), int(k), int(bool(sorted)), N.ref(dv), ctypes.byref(di),
                                             N.stream_of(s))
    N.check(rc, "bd_topk")
    idx = idx.reshape(tuple(lead) + (k,))
    return (vals.reshape(tuple(lead) + (k,)) if vals is not None else None), idx


def gather_attn(q3, k, v, idx, scaling, out):
    N.require_cuda(q3, k, v, idx, out)
    k, v = rows_aligned(k), rows_aligned(v)
    q3 = inner_contig(q3)
    idx = inner_contig(idx)
    if idx.dtype not in (torch.int32, torch.int64):
        idx = idx.long()
    dq, di = N.desc(q3), N.desc(idx)
    nws = _fn("bd_sparse_gather_attn_workspace", [P, P], SZ)(ctypes.byref(dq), ctypes.byref(di))
    buf, nb = _ws(nws, q3.device)
    dk, dv, do = N.desc(k), N.desc(v), N.desc(out)
    rc = _fn("bd_sparse_gather_attn", [P, P, P, P, F, P, VP, SZ, VP])(
        ctypes.byref(dq), ctypes.byref(dk), ctypes.byref(dv), ctypes.byref(di), float(scaling), ctypes.byref(do),
        _ptr(buf), nb, N.stream_of(q3))
    N.check(rc, "bd_sparse_gather_attn")
    return out


def gather_attn_partial(q3, k, v, idx, scaling):
    """Shard partials (m, l, o) of gather-attend over this device's positions in idx."""
    N.require_cuda(q3, k, v, idx)
    k, v = rows_aligned(k), rows_aligned(v)
    q3 = inner_contig(q3)
    idx = inner_contig(idx)
    if idx.dtype not in (torch.int32, torch.int64):
        idx = idx.long()
    B, Hq, D = q3.shape
    m = torch.empty(B, Hq, dtype=torch.float32, device=q3.device)
    l = torch.empty_like(m)
    o = torch.empty(B, Hq, D, dtype=torch.float32, device=q3.device)
    dq, di = N.desc(q3), N.desc(idx)
    nws = _fn("bd_sparse_gather_attn_workspace", [P, P], SZ)(ctypes.byref(dq), ctypes.byref(di))
    buf, nb = _ws(nws, q3.device)
    dk, dv, dm, dl, dO = N.desc(k), N.desc(v), N.desc(m), N.desc(l), N.desc(o)
    rc = _fn("bd_sparse_gather_attn_partial", [P, P, P, P, F, P, P, P, VP, SZ, VP])(
        ctypes.byref(dq), ctypes.byref(dk), ctypes.byref(dv), ctypes.byref(di), float(scaling), ctypes.byref(dm),
        ctypes.byref(dl), ctypes.byref(dO), _ptr(buf), nb, N.stream_of(q3))
    N.check(rc, "bd_sparse_gather_attn_partial")
    return m, l, o


def quest_page_minmax(k, page):
    N.require_cuda(k)
    k = inner_contig(k)
    B, H, S, D = k.shape
    np_ = (S + page - 1) // page
    kmin = torch.empty(B, H, np_, D, dtype=k.dtype, device=k.device)
    kmax = torch.empty_like(kmin)
    dk, dmn, dmx = N.desc(k), N.desc(kmin), N.desc(kmax)
    rc = _fn("bd_quest_page_minmax", [P, I, P, P, VP])(ctypes.byref(dk), int(page), ctypes.byref(dmn),
                                                       ctypes.byref(dmx), N.stream_of(k))
    N.check(rc, "bd_quest_page_minmax")
    return kmin, kmax


def quest_page_minmax_into(k, page, kmin, kmax):
    """Page min/max of k [B,H,S,D] written into the (possibly strided) views kmin/kmax."""
    N.require_cuda(k, kmin, kmax)
    k = inner_contig(k)
    dk, dmn, dmx = N.desc(k), N.desc(kmin), N.desc(kmax)
    rc = _fn("bd_quest_page_minmax", [P, I, P, P, VP])(ctypes.byref(dk), int(page), ctypes.byref(dmn),
                                                       ctypes.byref(dmx), N.stream_of(k))
    N.check(rc, "bd_quest_page_minmax")


def _page_meta(t):
    """Quest page metadata as the kernels read it: bf16 / f16 / fp32 as given (other float
    dtypes widened to fp32), rows on 16-byte boundaries."""
    if t.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        t = t.float()
    return rows_aligned(t)


def quest_page_bounds(q3, kmin, kmax, scaling, force_from_page=None):
    N.require_cuda(q3, kmin, kmax)
    q3 = inner_contig(q3)
    kmin, kmax = _page_meta(kmin), _page_meta(kmax)
    B, Hq, _ = q3.shape
    np_ = kmin.shape[2]
    bounds = torch.empty(B, Hq, np_, dtype=torch.float32, device=q3.device)
    ff = np_ if force_from_page is None else int(force_from_page)
    ds = [N.desc(t) for t in (q3, kmin, kmax, bounds)]
    rc = _fn("bd_quest_page_bounds", [P, P, P, F, I, P, VP])(
        ctypes.byref(ds[0]), ctypes.byref(ds[1]), ctypes.byref(ds[2]), float(scaling), ff, ctypes.byref(ds[3]),
        N.stream_of(q3))
    N.check(rc, "bd_quest_page_bounds")
    return bounds


def quest_select(q3, kmin, kmax, S, kb, page, scaling, force_from_page=None, idx_dtype=torch.int64):
    N.require_cuda(q3, kmin, kmax)
    q3 = inner_contig(q3)
    kmin, kmax = _page_meta(kmin), _page_meta(kmax)
    B, Hq, _ = q3.shape
    np_ = kmin.shape[2]
    npick = min(max(1, (kb + page - 1) // page), np_)
    idx = torch.empty(B, Hq, npick * page, dtype=idx_dtype, device=q3.device)
    ff = np_ if force_from_page is None else int(force_from_page)
    dq, dmn, dmx, di = N.desc(q3), N.desc(kmin), N.desc(kmax), N.desc(idx)
    nws = _fn("bd_quest_select_workspace", [P, P, I, I], SZ)(ctypes.byref(dq), ctypes.byref(dmn), int(kb), int(page))
    buf, nb = _ws(nws, q3.device)
    rc = _fn("bd_quest_select", [P, P, P, I, I, I, F, I, P, VP, SZ, VP])(
        ctypes.byref(dq), ctypes.byref(dmn), ctypes.byref(dmx), int(S), int(kb), int(page), float(scaling), ff,
        ctypes.byref(di), _ptr(buf), nb, N.stream_of(q3))
    N.check(rc, "bd_quest_select")
    return idx


def pq_decode(lut, k_idx, v=None, v_scale=None, v_idx=None, v_cent=None, k_out=None, q_out=None,
              block_table=None, context_lens=None, block_size=0, out_dtype=torch.bfloat16):
    """PQ-LUT decode; returns [B,Hq,D]."""
    N.require_cuda(lut, k_idx, v, v_scale, v_idx, v_cent, k_out, q_out, block_table, context_lens)
    lut = lut if lut.dtype == torch.float32 else lut.float()
    k_idx = inner_contig(k_idx)
    if v is not None:
        v = rows_aligned(v)
    if v_cent is not None and v_cent.dtype != torch.float32:
        v_cent = v_cent.float()
    if k_out is not None and k_out.shape[-1] == 0:
        k_out, q_out = None, None
    if k_out is not None and k_out.dtype not in (torch.bfloat16, torch.float16):
        k_out = k_out.to(torch.bfloat16)
    if block_table is not None:
        block_table = block_table.to(torch.int32)
        context_lens = context_lens.to(torch.int32)
    B, Hq = lut.shape[:2]
    D = v.shape[-1] if v is not None else v_cent.shape[0] * v_cent.shape[2]
    out = torch.empty(B, Hq, D, dtype=out_dtype, device=lut.device)
    ds = {n: N.desc(t) for n, t in dict(lut=lut, k_idx=k_idx, k_out=k_out, q_out=q_out, v=v, v_scale=v_scale,
                                        v_idx=v_idx, v_cent=v_cent, bt=block_table, cl=context_lens,
                                        out=out).items()}
    nws = _fn("bd_pq_decode_workspace", [P, P, P, P, P, P, P, I], SZ)(
        N.ref(ds["lut"]), N.ref(ds["k_idx"]), N.ref(ds["v"]), N.ref(ds["v_idx"]), N.ref(ds["v_cent"]),
        N.ref(ds["bt"]), N.ref(ds["cl"]), int(block_size))
    buf, nb = _ws(nws, lut.device)
    rc = _fn("bd_pq_decode", [P] * 10 + [I, P, VP, SZ, VP])(
        N.ref(ds["lut"]), N.ref(ds["k_idx"]), N.ref(ds["k_out"]), N.ref(ds["q_out"]), N.ref(ds["v"]),
        N.ref(ds["v_scale"]), N.ref(ds["v_idx"]), N.ref(ds["v_cent"]), N.ref(ds["bt"]), N.ref(ds["cl"]),
        int(block_size), N.ref(ds["out"]), _ptr(buf), nb, N.stream_of(lut))
    N.check(rc, "bd_pq_decode")
    return out


def pq_scores(lut, k_idx, k_out=None, q_out=None):
    N.require_cuda(lut, k_idx, k_out, q_out)
    lut = lut if lut.dtype == torch.float32 else lut.float()
    k_idx = inner_contig(k_idx)
    if k_out is not None and k_out.shape[-1] == 0:
        k_out, q_out = None, None
    if k_out is not None and k_out.dtype not in (torch.bfloat16, torch.float16):
        k_out = k_out.to(torch.bfloat16)
    B, Hq = lut.shape[:2]
    S = k_idx.shape[2]
    scores = torch.empty(B, Hq, S, dtype=torch.float32, device=lut.device)
    ds = [N.desc(t) for t in (lut, k_idx, k_out, q_out, scores)]
    rc = _fn("bd_pq_scores", [P, P, P, P, P, VP])(N.ref(ds[0]), N.ref(ds[1]), N.ref(ds[2]), N.ref(ds[3]),
                                                  N.ref(ds[4]), N.stream_of(lut))
    N.check(rc, "bd_pq_scores")
    return scores


def pq_build_lut(q3, centroids):
    N.require_cuda(q3, centroids)
    centroids = centroids if centroids.dtype == torch.float32 else centroids.float()
    B, H, D = q3.shape
    M, K, _ = centroids.shape
    lut = torch.empty(B, H, M, K, dtype=torch.float32, device=q3.device)
    ds = [N.desc(t) for t in (q3, centroids, lut)]
    rc = _fn("bd_pq_build_lut", [P, P, P, VP])(*[ctypes.byref(d) for d in ds], N.stream_of(q3))
    N.check(rc, "bd_pq_build_lut")
    return lut


def pq_encode(x2, centroids, codes_dtype=torch.int64):
    N.require_cuda(x2, centroids)
    x2 = inner_contig(x2)
    centroids = centroids if centroids.dtype == torch.float32 else centroids.float()
    codes = torch.empty(x2.shape[0], centroids.shape[0], dtype=codes_dtype, device=x2.device)
    ds = [N.desc(t) for t in (x2, centroids, codes)]
    rc = _fn("bd_pq_encode", [P, P, P, VP])(*[ctypes.byref(d) for d in ds], N.stream_of(x2))
    N.check(rc, "bd_pq_encode")
    return codes


def asym_fakequant_5d(x5, levels):
    """x5: a 5-d strided view (o0, o1, o2, group axis, inner) -> contiguous fake-quant output."""
    N.require_cuda(x5)
    y = torch.empty(x5.shape, dtype=x5.dtype, device=x5.device)
    dx, dy = N.desc(x5), N.desc(y)
    rc = _fn("bd_asym_fakequant", [P, I, P, VP])(ctypes.byref(dx), int(levels), ctypes.byref(dy), N.stream_of(x5))
    N.check(rc, "bd_asym_fakequant")
    return y
