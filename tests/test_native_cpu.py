"""CPU-side checks of the C-ABI library: it loads, exports every entry point the header
declares, and rejects malformed requests on the host before any launch."""
import ctypes

import pytest
import torch

from bytes_b200 import _native as N


def test_library_loads_and_exports_header_symbols():
    lib = N.lib()
    names = N.exported_symbols()
    assert len(names) >= 5
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert lib.bd_abi_version() == 1


def test_status_names():
    lib = N.lib()
    assert lib.bd_status_name(0) == b"BD_OK"
    assert lib.bd_status_name(3) == b"BD_ERR_SHAPE"


def _fake(shape, dtype, ptr=0x10000):
    """Descriptor with a fake (never dereferenced) device pointer and contiguous strides."""
    d = N.BdTensor()
    d.data = ptr
    d.dtype = dtype
    d.ndim = len(shape)
    s = 1
    for i in range(len(shape) - 1, -1, -1):
        d.shape[i] = shape[i]
        d.stride[i] = s
        s *= shape[i]
    return d


def _call_decode(q, k, v, out):
    lib = N.lib()
    f = lib.bd_decode_attn
    f.restype = ctypes.c_int
    return f(ctypes.byref(q), ctypes.byref(k), ctypes.byref(v), ctypes.byref(out), ctypes.c_float(1.0),
             ctypes.c_void_p(0), ctypes.c_size_t(0), ctypes.c_void_p(0))


def test_decode_rejects_bad_shapes_and_dtypes_on_host():
    q = _fake((2, 8, 128), N.BD_BF16)
    k = _fake((2, 3, 64, 128), N.BD_BF16)  # 8 % 3 != 0
    v = _fake((2, 3, 64, 128), N.BD_BF16)
    out = _fake((2, 8, 128), N.BD_BF16)
    assert _call_decode(q, k, v, out) == 3  # BD_ERR_SHAPE
    assert b"multiple" in N.lib().bd_last_error()
    k = _fake((2, 2, 64, 128), N.BD_F32)
    v = _fake((2, 2, 64, 128), N.BD_F32)
    assert _call_decode(q, k, v, out) == 2  # BD_ERR_DTYPE
    k = _fake((2, 2, 64, 96), N.BD_BF16)
    v = _fake((2, 2, 64, 96), N.BD_BF16)
    q = _fake((2, 8, 96), N.BD_BF16)
    out = _fake((2, 8, 96), N.BD_BF16)
    assert _call_decode(q, k, v, out) == 7  # BD_ERR_UNSUPPORTED (head_dim 96)


def test_decode_rejects_misaligned_rows_on_host():
    q = _fake((1, 4, 128), N.BD_BF16)
    k = _fake((1, 1, 64, 128), N.BD_BF16, ptr=0x10002)
    v = _fake((1, 1, 64, 128), N.BD_BF16)
    out = _fake((1, 4, 128), N.BD_BF16)
    assert _call_decode(q, k, v, out) == 5  # BD_ERR_ALIGN


def test_kivi_rejects_bad_bits_on_host():
    lib = N.lib()
    f = lib.bd_kivi_decode_attn
    f.restype = ctypes.c_int
    Q = _fake((1, 4, 128), N.BD_BF16)
    Kq = _fake((1, 1, 128, 8), N.BD_I32)
    Ks = _fake((1, 1, 128, 4), N.BD_F16)
    Kr = _fake((1, 1, 16, 128), N.BD_BF16)
    Vq = _fake((1, 1, 128, 8), N.BD_I32)
    Vs = _fake((1, 1, 128, 4), N.BD_F16)
    out = _fake((1, 4, 128), N.BD_BF16)
    args = [ctypes.byref(t) for t in (Q, Kq, Ks, Ks, Kr, Vq, Vs, Vs, Kr)]
    rc = f(*args, 3, 32, ctypes.c_float(0.1), ctypes.byref(out), ctypes.c_void_p(0), ctypes.c_size_t(0),
           ctypes.c_void_p(0))
    assert rc == 9  # BD_ERR_VALUE
    rc = f(*args, 2, 64, ctypes.c_float(0.1), ctypes.byref(out), ctypes.c_void_p(0), ctypes.c_size_t(0),
           ctypes.c_void_p(0))
    assert rc == 7


def test_kivi_append_rejects_bad_requests_on_host():
    lib = N.lib()
    f = lib.bd_kivi_append
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int64] + [ctypes.c_void_p] * 7
    kn = _fake((1, 1, 32, 128), N.BD_F16)
    Kq = _fake((1, 1, 128, 8), N.BD_I32)    # capacity 128 tokens at 2 bits
    Ks = _fake((1, 1, 128, 4), N.BD_F16)
    Vq = _fake((1, 1, 128, 8), N.BD_I32)
    Vs = _fake((1, 1, 128, 4), N.BD_F16)

    def call(k, bits, off, kq=Kq):
        return f(ctypes.addressof(k), ctypes.addressof(k), bits, 32, off, ctypes.addressof(kq), ctypes.addressof(Ks),
                 ctypes.addressof(Ks), ctypes.addressof(Vq), ctypes.addressof(Vs), ctypes.addressof(Vs), None)

    assert call(kn, 3, 0) == 9                                   # bits
    assert call(kn, 2, 16) == 9                                  # offset inside a group
    assert call(_fake((1, 1, 48, 128), N.BD_F16), 2, 0) == 3     # partial group
    assert call(kn, 2, 128) == 3                                 # past the key capacity
    assert call(_fake((1, 1, 32, 128), N.BD_I8), 2, 0) == 2      # dtype


def test_python_layer_refuses_cpu_tensors():
    from bytes_b200 import attention_kernels as ak
    q = torch.randn(1, 4, 1, 128).bfloat16()
    k = torch.randn(1, 1, 16, 128).bfloat16()
    with pytest.raises(ValueError):
        ak.decode_attn_bf16(q, k, k)
