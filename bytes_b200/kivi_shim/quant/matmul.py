"""KIVI GEMV entry point (``quant.matmul``) backed by bytes_b200."""
from . import _ROOT  # noqa: F401  (puts the repository root on sys.path)
from bytes_b200.kivi import cuda_bmm_fA_qB_outer  # noqa: F401
