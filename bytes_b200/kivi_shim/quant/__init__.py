"""Stand-in for the KIVI ``quant`` package: point ``KIVI_REPO`` at ``bytes_b200/kivi_shim``
and ``from quant.matmul import cuda_bmm_fA_qB_outer`` / ``from quant.new_pack import
triton_quantize_and_pack_along_last_dim`` resolve to this engine's sm_100a kernels."""
import os
import sys

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)
