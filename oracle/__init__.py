"""CPU oracle for the decode-attention hot path — TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU and in fp32 PyTorch/numpy, the algorithms of the
reference project saifmb0/bytes for the decode-attention path (dense BF16/FP8 decode,
KIVI 2/4-bit decode and packing, PQ-LUT decode and encode, score passes, top-k,
Quest page selection, sparse gather-attention). Every function cites the reference
file:line it follows (paths are relative to the reference project's root).

Only the test-suite, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it, and only as the checker or
as the timed CPU baseline. The product package ``bytes_b200`` never imports it; its
entry points run the CUDA kernels or raise.

Parity pinning: the restatement is checked against golden vectors produced by
running the reference's own CPU-runnable functions (``tests/golden/make_golden.py``) and
its quantizers on a CUDA device (``tests/golden/make_golden_cuda.py``): those PyTorch
expressions round differently on the two devices, and the quantizers here take
``rule="cuda"`` (default, what the GPU engine must match) or ``rule="cpu"``.
The external KIVI packer (jy-yuan/KIVI @ 876b4d2d, not vendored by the reference)
is the one piece whose bit-exact output is not pinned: its layout is pinned by the
reference's in-tree ``unpack_tensor_last_dim`` and its quantisation formula follows
the reference's in-tree ``_asym_uniform_fakequant``.
"""

from .attention import (  # noqa: F401
    repeat_kv,
    decode_attn_dense,
    decode_attn_dequant,
    decode_attn_pq_lut,
    decode_attn_pq_lut_kv,
    paged_attn_pq_lut_kv,
    decode_attn_pq_lut_asym,
    paged_attn_pq_lut_asym,
    decode_attn_pq_lut_int8v,
    sparse_score_pq_lut_asym,
    sparse_score_scalar,
    sparse_score_packed,
    sparse_gather_attn,
    sparse_decode_scalar,
    sparse_decode_pq_lut,
    split_partials,
    lse_combine,
)
from .quant import (  # noqa: F401
    asym_uniform_fakequant,
    kivi_quantize_key,
    kivi_quantize_value,
    quantize_and_pack_score_keys,
    unpack_score_keys,
    kivi_pack_last_dim,
    kivi_unpack_last_dim,
    kivi_dequant_k,
    kivi_dequant_v,
    kivi_decode_attn,
    kivi_gemv_outer,
    pq_encode,
    pq_dequantize,
    pq_lut,
)
from .select import (  # noqa: F401
    topk_lower_index,
    select_topk_exact,
    quest_page_minmax,
    quest_page_bounds,
    quest_select,
    quest_select_from_meta,
    attend_topk,
    select_topk_exact_window,
    quest_bounds_window,
    quest_select_window,
    select_topk_window,
    sparse_attention_chunked,
)
