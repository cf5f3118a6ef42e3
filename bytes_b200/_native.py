"""ctypes bridge to the C-ABI library ``libbdecode.so`` (declared in include/bdecode.h).

The library is loaded once, from ``bytes_b200/lib/libbdecode.so`` (build it with
``python -m bytes_b200.build``). There is no fallback: if the library is missing
or a call fails, the error propagates to the caller.
"""
import ctypes
import os

import torch

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "lib", "libbdecode.so")

MAX_DIMS = 6
BD_F32, BD_F16, BD_BF16, BD_F8E4M3, BD_U8, BD_I8, BD_I32, BD_I64 = range(8)

_DTYPES = {
    torch.float32: BD_F32,
    torch.float16: BD_F16,
    torch.bfloat16: BD_BF16,
    torch.float8_e4m3fn: BD_F8E4M3,
    torch.uint8: BD_U8,
    torch.int8: BD_I8,
    torch.int32: BD_I32,
    torch.int64: BD_I64,
}

# status codes whose meaning is "the caller passed something invalid"
_VALUE_ERRORS = {1, 2, 3, 4, 5, 7, 9}


class BdTensor(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("ndim", ctypes.c_int32),
        ("shape", ctypes.c_int64 * MAX_DIMS),
        ("stride", ctypes.c_int64 * MAX_DIMS),
    ]


_lib = None


def lib():
    """Load (once) and return the native library; raises if it is absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"bytes_b200 native library not found at {LIB_PATH}; build it with "
                "`python -m bytes_b200.build` (nvcc, sm_100a). There is no CPU fallback.")
        # RTLD_GLOBAL: the torch glue module resolves its bd_* symbols against this copy
        L = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)
        L.bd_last_error.restype = ctypes.c_char_p
        L.bd_status_name.restype = ctypes.c_char_p
        L.bd_abi_version.restype = ctypes.c_int
        _lib = L
    return _lib


GLUE_PATH = os.path.join(_PKG, "lib", "glue", "bd_glue.so")
_glue = None


def glue():
    """The compiled torch glue module (csrc/torch_glue.cpp); raises if it is absent."""
    global _glue
    if _glue is None:
        lib()
        if not os.path.exists(GLUE_PATH):
            raise RuntimeError(f"bytes_b200 glue module not found at {GLUE_PATH}; build it with "
                               "`python -m bytes_b200.build`.")
        import importlib.util
        spec = importlib.util.spec_from_file_location("bd_glue", GLUE_PATH)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        _glue = mod
    return _glue


def fn(name, restype=ctypes.c_int):
    f = getattr(lib(), name)
    f.restype = restype
    return f


def desc(t, ndim=None):
    """bd_tensor descriptor for a torch tensor (None -> NULL pointer)."""
    if t is None:
        return None
    if t.dtype not in _DTYPES:
        raise ValueError(f"unsupported dtype {t.dtype}")
    if t.dim() > MAX_DIMS:
        raise ValueError("too many dimensions")
    d = BdTensor()
    d.data = t.data_ptr() if t.numel() > 0 else 0
    d.dtype = _DTYPES[t.dtype]
    d.ndim = t.dim()
    for i in range(t.dim()):
        d.shape[i] = t.shape[i]
        d.stride[i] = t.stride(i)
    return d


def ref(d):
    return ctypes.byref(d) if d is not None else None


def stream_of(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def check(status, what):
    if status == 0:
        return
    msg = lib().bd_last_error().decode(errors="replace")
    if status in _VALUE_ERRORS:
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what}: {msg}")


def workspace(nbytes, device):
    if nbytes == 0:
        return None, 0
    return torch.empty(int(nbytes), dtype=torch.uint8, device=device), int(nbytes)


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("bytes_b200 kernels take CUDA tensors (there is no CPU path)")


def exported_symbols():
    """Names of the C-ABI entry points declared in include/bdecode.h."""
    import re
    hdr = os.path.join(os.path.dirname(_PKG), "include", "bdecode.h")
    src = open(hdr).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(bd_[a-z0-9_]+)\s*\(", src)))
