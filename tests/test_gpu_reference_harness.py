"""The reference's own test and harness code, run unchanged against this engine.

``baseline/_ref`` holds an installed copy of the reference project (its ``src`` and
``benchmarks`` packages, unmodified). These tests make the drop-in swap a maintainer would
make -- ``src.attention_kernels`` resolves to ``bytes_b200.attention_kernels`` and
``KIVI_REPO`` points at ``bytes_b200/kivi_shim`` -- and then call the reference's own test
functions (benchmarks/test_correctness.py) and its KIVI integrity gate
(benchmarks/kivi_latency.py:102-146). Each reference test builds its own inputs and its own
PyTorch reference and asserts with its own tolerances. Skipped when the install is absent.
"""
import importlib
import os
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")

# kernels the reference's test file checks (the rest test calibration utilities and the
# Hadamard/JL helpers of src/quantization.py, which are not on the decode path)
KERNEL_TESTS = [
    "test_bf16_attention_correctness",
    "test_fp8_attention_correctness",
    "test_dequant_attention_correctness",
    "test_pq_lut_attention_correctness",
    "test_pq_lut_kv_attention_correctness",
    "test_paged_pq_lut_kv_attention_correctness",
    "test_pq_lut_asym_attention_correctness",
    "test_paged_pq_lut_asym_attention_correctness",
    "test_sparse_scalar_score_correctness",
    "test_sparse_pipeline_correctness",
]


@pytest.fixture(scope="module")
def swapped(cuda):
    if not os.path.isdir(os.path.join(REF, "src")) or not os.path.isdir(os.path.join(REF, "benchmarks")):
        pytest.skip("reference install (baseline/_ref) not present")
    saved_path = list(sys.path)
    saved_mods = {k: v for k, v in sys.modules.items() if k == "src" or k.startswith(("src.", "benchmarks", "quant"))}
    saved_env = os.environ.get("KIVI_REPO")
    for k in saved_mods:
        del sys.modules[k]
    sys.path.insert(0, REF)
    import bytes_b200.attention_kernels as ours
    import bytes_b200.quantization as ours_q
    import src  # the reference's package
    sys.modules["src.attention_kernels"] = ours
    src.attention_kernels = ours
    # the hot-path quantizers are re-exported over the reference's module; its calibration,
    # Hadamard and JL utilities stay as they are
    import src.quantization as ref_q
    for name in ("ProductQuantizer", "KIVIQuantizer", "_asym_uniform_fakequant"):
        setattr(ref_q, name, getattr(ours_q, name))
    os.environ["KIVI_REPO"] = os.path.join(ROOT, "bytes_b200", "kivi_shim")
    yield
    for k in [k for k in sys.modules if k == "src" or k.startswith(("src.", "benchmarks", "quant"))]:
        del sys.modules[k]
    sys.modules.update(saved_mods)
    sys.path[:] = saved_path
    if saved_env is None:
        os.environ.pop("KIVI_REPO", None)
    else:
        os.environ["KIVI_REPO"] = saved_env


@pytest.mark.parametrize("name", KERNEL_TESTS)
def test_reference_correctness_suite(swapped, name):
    import torch
    tc = importlib.import_module("benchmarks.test_correctness")
    assert tc.decode_attn_bf16.__module__ == "bytes_b200.attention_kernels"
    torch.manual_seed(1234)
    getattr(tc, name)()


def test_reference_kivi_integrity_gate(swapped):
    kl = importlib.import_module("benchmarks.kivi_latency")
    assert kl.cuda_bmm_fA_qB_outer.__module__ == "bytes_b200.kivi"
    assert kl.triton_quantize_and_pack_along_last_dim.__module__ == "bytes_b200.kivi"
    errors = kl.run_integrity_gate()  # exits the process if an error reaches 1 %
    assert set(errors) == {2, 4} and max(errors.values()) < 0.01
    # the reference's fused step itself (GEMV + residual + softmax + GEMV through the shim)
    # against the engine's single fused call on the gate's inputs
    import torch
    from bytes_b200 import kivi as ours
    torch.manual_seed(42)
    B, Hq, Hk, D, Sq, R = 2, 8, 2, 128, 256, 128
    Q = torch.randn(B, Hq, 1, D, device="cuda", dtype=torch.bfloat16)
    K = torch.randn(B, Hk, Sq, D, device="cuda", dtype=torch.bfloat16)
    Kr = torch.randn(B, Hk, R, D, device="cuda", dtype=torch.bfloat16)
    V = torch.randn(B, Hk, Sq, D, device="cuda", dtype=torch.bfloat16)
    Vr = torch.randn(B, Hk, R, D, device="cuda", dtype=torch.bfloat16)
    for bits in (2, 4):
        Kq, Ks, Km = kl.triton_quantize_and_pack_along_last_dim(K.transpose(2, 3).contiguous().half(), 32, bits)
        Vq, Vs, Vm = kl.triton_quantize_and_pack_along_last_dim(V.contiguous().half(), 32, bits)
        ref_path = kl.kivi_decode_attn(Q, Kq, Ks, Km, Kr, Vq, Vs, Vm, Vr, bits, 32)
        fused = ours.kivi_decode_attn(Q, Kq, Ks, Km, Kr, Vq, Vs, Vm, Vr, bits, 32)
        d = (ref_path.float() - fused.float()).abs()
        assert d.max().item() < 2e-2 and d.mean().item() < 1e-3
