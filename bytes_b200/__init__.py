"""bytes_b200 — a B200-native (sm_100a) decode-attention engine.

Drop-in modules mirroring the reference project saifmb0/bytes:
  bytes_b200.attention_kernels  <- src/attention_kernels.py
  bytes_b200.quantization       <- src/quantization.py (hot-path parts)
  bytes_b200.sparse_attention   <- benchmarks/sparse_attention.py (decode selection)
  bytes_b200.kivi               <- benchmarks/kivi_latency.py + the KIVI quant package
  bytes_b200/kivi_shim/quant    <- set KIVI_REPO to this directory
The kernels live in the C-ABI library lib/libbdecode.so (include/bdecode.h).
"""
__version__ = "0.1.0"
