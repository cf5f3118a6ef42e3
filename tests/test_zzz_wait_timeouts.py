"""Collected after every kernel test (only the no-alloc entry point's own test follows; its
dense kernels have no bounded waits): no bounded device wait (TMA tile barriers of the KIVI and PQ kernels,
the bulk copy of the window-merge pass) ran past its iteration limit during this GPU
session — every tile those tests checked arrived before its consumers read it."""
import ctypes

import pytest
import torch

from bytes_b200 import _native as N

pytestmark = pytest.mark.gpu


def test_no_bounded_wait_ran_out(cuda):
    lib = N.lib()
    f = lib.bd_wait_timeouts
    f.restype = ctypes.c_longlong
    torch.cuda.synchronize()
    assert f() == 0
