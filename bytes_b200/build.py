"""Build the sm_100a C-ABI library ``bytes_b200/lib/libbdecode.so`` with nvcc.

Every ``bytes_b200/csrc/*.cu`` compiles to an object (in parallel, skipped when
its sources are unchanged) and links into one shared library exporting the
``extern "C"`` entry points declared in ``include/bdecode.h``. Then the torch glue
module ``bytes_b200/lib/glue/bd_glue.so`` (``csrc/torch_glue.cpp``: descriptors
filled in C++ for the per-token decode calls) is compiled against the installed torch.

    python -m bytes_b200.build [--verbose-ptxas]
"""
import argparse
import concurrent.futures as cf
import ctypes
import hashlib
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(PKG, "lib", "obj")
LIB = os.path.join(PKG, "lib", "libbdecode.so")
GLUE_DIR = os.path.join(PKG, "lib", "glue")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I" + os.path.join(ROOT, "include")]


def _digest(path, extra):
    h = hashlib.sha256()
    for p in sorted([path] + extra):
        with open(p, "rb") as f:
            h.update(f.read())
    h.update(" ".join(ARCH + FLAGS).encode())
    return h.hexdigest()[:16]


def _compile(src, headers, ptxas_verbose):
    name = os.path.splitext(os.path.basename(src))[0]
    obj = os.path.join(OBJ, name + ".o")
    stamp = obj + ".stamp"
    dig = _digest(src, headers)
    if os.path.exists(obj) and os.path.exists(stamp) and open(stamp).read() == dig and not ptxas_verbose:
        return obj, ""
    cmd = [NVCC] + ARCH + FLAGS + (["-Xptxas", "-v"] if ptxas_verbose else []) + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed for %s:\n%s\n%s" % (src, r.stdout, r.stderr))
    with open(stamp, "w") as f:
        f.write(dig)
    return obj, r.stderr


def build(ptxas_verbose=False, quiet=False):
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))
    headers = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cuh"))
    headers.append(os.path.join(ROOT, "include", "bdecode.h"))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        results = list(ex.map(lambda s: _compile(s, headers, ptxas_verbose), srcs))
    objs = [o for o, _ in results]
    if ptxas_verbose:
        for _, log in results:
            sys.stderr.write(log)
    newest = max(os.path.getmtime(o) for o in objs)
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n%s\n%s" % (r.stdout, r.stderr))
    build_glue()
    if not quiet:
        print("built", LIB)
    return LIB


def build_glue():
    """Compile (when changed) and import the torch glue module against libbdecode.so."""
    from torch.utils import cpp_extension
    ctypes.CDLL(LIB, mode=ctypes.RTLD_GLOBAL)  # the glue resolves bd_* against it
    os.makedirs(GLUE_DIR, exist_ok=True)
    return cpp_extension.load(name="bd_glue", sources=[os.path.join(CSRC, "torch_glue.cpp")],
                              extra_include_paths=[os.path.join(ROOT, "include")], extra_cflags=["-O2"],
                              build_directory=GLUE_DIR, with_cuda=True, verbose=False)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    a = ap.parse_args()
    build(a.verbose_ptxas)
