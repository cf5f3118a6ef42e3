"""KIVI packer entry point (``quant.new_pack``) backed by bytes_b200."""
from . import _ROOT  # noqa: F401  (puts the repository root on sys.path)
from bytes_b200.kivi import triton_quantize_and_pack_along_last_dim  # noqa: F401
