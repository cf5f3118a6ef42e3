"""bd_decode_attn_noalloc: decode attention for callers that cannot allocate device memory.

A serving runtime that has reserved all of HBM for its KV pages, or a plain C / FFI host
holding only the q/k/v/out buffers, cannot hand the engine a workspace. This entry point
keeps its split partials in a fixed device array inside the library instead. The test
calls it through the C ABI twice in a row (the array keeps the previous call's contents)
and compares each result with bd_decode_attn given a normal workspace.

This file is collected last (after test_zzz_wait_timeouts.py), so a run that stops at the
first failure has run every other test before it.
"""
import ctypes

import pytest
import torch

from bytes_b200 import _native as N

pytestmark = pytest.mark.gpu


def _call_with_workspace(lib, q3, k, v, out):
    dq, dk, dv, do = N.desc(q3), N.desc(k), N.desc(v), N.desc(out)
    f = lib.bd_decode_attn_workspace
    f.restype = ctypes.c_size_t
    nws = f(ctypes.byref(dq), ctypes.byref(dk))
    ws = torch.empty(max(nws, 1), dtype=torch.uint8, device=q3.device)
    rc = lib.bd_decode_attn(ctypes.byref(dq), ctypes.byref(dk), ctypes.byref(dv), ctypes.byref(do),
                            ctypes.c_float(1.0), ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(nws),
                            N.stream_of(q3))
    assert rc == 0, lib.bd_last_error()


def _call_noalloc(lib, q3, k, v, out):
    dq, dk, dv, do = N.desc(q3), N.desc(k), N.desc(v), N.desc(out)
    rc = lib.bd_decode_attn_noalloc(ctypes.byref(dq), ctypes.byref(dk), ctypes.byref(dv), ctypes.byref(do),
                                    ctypes.c_float(1.0), N.stream_of(q3))
    assert rc == 0, lib.bd_last_error()


def test_noalloc_matches_workspace_entry_point_twice(cuda):
    lib = N.lib()
    lib.bd_decode_attn.restype = ctypes.c_int
    lib.bd_decode_attn_noalloc.restype = ctypes.c_int
    g = torch.Generator().manual_seed(77)
    # two different problems in a row: the second must not see the first one's partials
    for (B, Hq, Hk, S) in ((1, 28, 4, 8192), (2, 8, 2, 3000)):
        q3 = torch.randn(B, Hq, 128, generator=g).bfloat16().to(cuda)
        k = torch.randn(B, Hk, S, 128, generator=g).bfloat16().to(cuda)
        v = torch.randn(B, Hk, S, 128, generator=g).bfloat16().to(cuda)
        ref = torch.empty(B, Hq, 128, dtype=torch.bfloat16, device=cuda)
        out = torch.empty_like(ref)
        _call_with_workspace(lib, q3, k, v, ref)
        _call_noalloc(lib, q3, k, v, out)
        torch.cuda.synchronize()
        d = (out.float() - ref.float()).abs()
        assert torch.isfinite(out.float()).all()
        assert d.max().item() <= 2e-2 and d.mean().item() <= 1e-3


def test_noalloc_scratch_covers_every_plan_on_this_device(cuda):
    """The split plan targets two CTAs per SM (three for fp8 caches), so a plan that splits
    at all needs at most 16 heads x 3 x SMs x (D+2) floats of scratch plus 256 bytes of
    alignment slack, i.e. 24,960 bytes per SM (about 3.7 MB on a 148-SM part): the 4 MiB
    static array holds every such plan on parts with up to 168 SMs, this device included.
    (Larger plans are rejected with BD_ERR_UNSUPPORTED before any launch; no device this
    test runs on reaches that.)"""
    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    assert 24960 * sms + 256 <= 4 << 20
    lib = N.lib()
    f = lib.bd_decode_attn_workspace
    f.restype = ctypes.c_size_t

    def fake(shape, dt=N.BD_BF16, ptr=0x100000):
        d = N.BdTensor()
        d.data, d.dtype, d.ndim = ptr, dt, len(shape)
        st = 1
        for i in range(len(shape) - 1, -1, -1):
            d.shape[i], d.stride[i] = shape[i], st
            st *= shape[i]
        return d

    worst = 0
    for B in (1, 2, 3, 8):
        for Hk in (1, 2, 4, 8):
            for G in (1, 4, 7, 8, 9, 16, 17, 32, 64, 128):
                for D, kdt in ((64, N.BD_BF16), (128, N.BD_BF16), (64, N.BD_F8E4M3), (128, N.BD_F8E4M3)):
                    q = fake((B, Hk * G, D))
                    k = fake((B, Hk, 1 << 20, D), kdt)
                    ws = f(ctypes.byref(q), ctypes.byref(k))
                    splits = (ws - 256) // (B * Hk * G * (D + 2) * 4)
                    if splits > 1:  # a one-split plan writes the output directly, no scratch
                        worst = max(worst, ws)
    assert 0 < worst <= 4 << 20, worst
