"""Pin the CPU oracle against golden vectors produced by the reference's own code.

``golden.pt`` comes from tests/golden/make_golden.py, which imports the reference project
and runs its CPU-runnable functions; ``golden_cuda.pt`` from tests/golden/make_golden_cuda.py,
which runs the reference's quantizers on a CUDA device, where PyTorch evaluates their
division by levels-1 as a reciprocal multiply and ``ProductQuantizer`` encodes with its
f16 Triton kernel. The oracle's quantizers take ``rule="cpu"`` / ``rule="cuda"`` for the
two. Integer / byte / index outputs must be bit-exact; floating outputs agree to fp32
summation-order noise.
"""
import math

import torch

import oracle
from conftest import chunked_mismatch, valid_sets


def test_pack_score_keys_bit_exact(golden):
    for c in golden["pack_score_keys"]:
        p, s, z = oracle.quantize_and_pack_score_keys(c["k"], c["bits"], c["group_size"], rule="cpu")
        assert torch.equal(p, c["packed"])
        assert torch.equal(s, c["scale"]) and s.dtype == c["scale"].dtype
        assert torch.equal(z, c["zero"])
        codes = oracle.unpack_score_keys(p, c["bits"])
        assert codes.shape == c["k"].shape


def test_fakequant_bit_exact(golden):
    for c in golden["fakequant"]:
        y = oracle.asym_uniform_fakequant(c["x"], c["levels"], c["dim"], rule="cpu")
        assert torch.equal(y, c["y"])


def test_kivi_quantizer_bit_exact(golden):
    for c in golden["kivi_quantizer"]:
        kf = oracle.kivi_quantize_key(c["k"], c["bits"], c["group_size"], c["residual_length"], rule="cpu")
        vf = oracle.kivi_quantize_value(c["v"], c["bits"], c["group_size"], c["residual_length"], rule="cpu")
        assert torch.equal(kf, c["k_fq"])
        assert torch.equal(vf, c["v_fq"])


def test_pq_encode_matches_reference_cpu_path(golden):
    """cdist+argmin (reference) vs direct fp32 distances (oracle): equal codes, except
    where the two candidates' distances tie within float noise."""
    for c in golden["pq_encode"]:
        codes = oracle.pq_encode(c["X"], c["centroids"], rule="cpu")
        ref = c["codes"]
        diff = codes != ref
        if diff.any():
            d2 = oracle.quant.pq_distances(c["X"], c["centroids"])
            a = d2.gather(-1, codes.unsqueeze(-1)).squeeze(-1)[diff]
            b = d2.gather(-1, ref.unsqueeze(-1)).squeeze(-1)[diff]
            assert torch.allclose(a, b, rtol=1e-5, atol=1e-5)
        assert diff.float().mean() < 1e-3


def test_quantizers_match_reference_on_cuda(golden_cuda):
    """rule="cuda" reproduces the reference's quantizers run on a GPU bit for bit, and the
    fixture separates the device rules (the CPU rule misses some of its bytes)."""
    cpu_miss = 0
    for c in golden_cuda["pack_score_keys"]:
        out = oracle.quantize_and_pack_score_keys(c["k"], c["bits"], c["group_size"])
        for a, b in zip(out, (c["packed"], c["scale"], c["zero"])):
            assert a.dtype == b.dtype and torch.equal(a, b)
        cpu = oracle.quantize_and_pack_score_keys(c["k"], c["bits"], c["group_size"], rule="cpu")
        n = sum(int((a != b).sum()) for a, b in zip(cpu, (c["packed"], c["scale"], c["zero"])))
        assert n == c["cpu_differs"]
        cpu_miss += n
    for c in golden_cuda["fakequant"]:
        assert torch.equal(oracle.asym_uniform_fakequant(c["x"], c["levels"], c["dim"]), c["y"])
        cpu = oracle.asym_uniform_fakequant(c["x"], c["levels"], c["dim"], rule="cpu")
        assert int((cpu != c["y"]).sum()) == c["cpu_differs"]
        cpu_miss += c["cpu_differs"]
    for c in golden_cuda["kivi_quantizer"]:
        args = (c["bits"], c["group_size"], c["residual_length"])
        assert torch.equal(oracle.kivi_quantize_key(c["k"], *args), c["k_fq"])
        assert torch.equal(oracle.kivi_quantize_value(c["v"], *args), c["v_fq"])
    assert cpu_miss > 0


def test_pq_encode_matches_reference_cuda_kernel(golden_cuda):
    """rule="cuda" (f16 dot products minus norms, argmax) against the reference's Triton
    encoder: equal codes except between centroids whose scores agree to fp32 summation
    order; its CPU path (rule="cpu") differs on more codes."""
    for c in golden_cuda["pq_encode"]:
        codes = oracle.pq_encode(c["X"], c["centroids"])
        ref = c["codes"]
        diff = codes != ref
        if diff.any():
            sc = oracle.quant.pq_encode_scores(c["X"], c["centroids"])
            a = sc.gather(-1, codes.unsqueeze(-1)).squeeze(-1)[diff]
            b = sc.gather(-1, ref.unsqueeze(-1)).squeeze(-1)[diff]
            assert torch.allclose(a, b, rtol=1e-5, atol=1e-5)
        assert diff.float().mean() < 1e-3
    assert sum(c["cpu_differs"] for c in golden_cuda["pq_encode"]) > 0


def test_select_topk_exact_matches_reference(golden):
    for c in golden["select_topk"]:
        idx = oracle.select_topk_exact(c["q"], c["keys"], c["S"], c["kb"], c["scaling"])
        assert torch.equal(idx, c["idx"])


def test_quest_select_and_attend_match_reference(golden):
    for c in golden["quest"]:
        q, k, v = c["q"], c["k"], c["v"]
        G = q.shape[1] // k.shape[1]
        kr = oracle.repeat_kv(k, G)
        idx = oracle.quest_select(q.float(), kr.float(), c["S"], c["kb"], c["page"], c["scaling"])
        # page sets are what matter; the reference's torch.topk orders them by bound too
        assert torch.equal(idx, c["idx"])
        kmin, kmax = oracle.quest_page_minmax(k, c["page"])
        idx2 = oracle.quest_select_from_meta(q, kmin, kmax, c["S"], c["kb"], c["page"], c["scaling"])
        assert torch.equal(idx2, c["idx"])
        o = oracle.attend_topk(q.float(), kr.float(), oracle.repeat_kv(v, G).float(), idx,
                               torch.tensor([c["S"] - 1]), c["scaling"])
        assert torch.allclose(o, c["out"], atol=1e-5, rtol=1e-5)


def test_dense_decode_matches_reference_attention(golden):
    for c in golden["dense_decode"]:
        o = oracle.decode_attn_dense(c["q"], c["k"], c["v"], 1.0, out_dtype=torch.float32)
        assert torch.allclose(o, c["out"], atol=1e-5, rtol=1e-5)


def test_pq_lut_decode_matches_reference_attention(golden):
    for c in golden["pq_lut_decode"]:
        if c["k_out"].shape[-1] == 0:
            o = oracle.decode_attn_pq_lut(c["lut"], c["codes"], c["v"].float())
        else:
            o = oracle.decode_attn_pq_lut_asym(c["lut"], c["codes"], c["k_out"], c["q_out"],
                                               c["v"].float())
        assert torch.allclose(o, c["out"], atol=1e-4, rtol=1e-4)
        # the dequant kernel computes the same thing from codes + centroids
        q_rot = None  # the LUT already folds q; reconstruct via dequantize for K3's check
        k_hat = oracle.pq_dequantize(c["codes"], c["centroids"])
        assert k_hat.shape[-1] == c["v"].shape[-1]


def test_kivi_unpack_dequant_and_decode_match_reference(golden):
    for c in golden["kivi"]:
        bits = c["bits"]
        un = oracle.kivi_unpack_last_dim(c["Kq"], bits)
        assert torch.equal(un.to(torch.float16), c["K_unpacked"])
        kdq = oracle.kivi_dequant_k(c["Kq"], c["K_scale"], c["K_mn"], 32, bits)
        vdq = oracle.kivi_dequant_v(c["Vq"], c["V_scale"], c["V_mn"], 32, bits)
        # reference dequant runs in fp16 (one rounding per mul and add)
        assert torch.allclose(kdq, c["K_dq"].float(), atol=4e-3, rtol=2e-3)
        assert torch.allclose(vdq, c["V_dq"].float(), atol=4e-3, rtol=2e-3)
        o = oracle.kivi_decode_attn(c["Q"].float(), c["Kq"], c["K_scale"], c["K_mn"], c["K_res"],
                                    c["Vq"], c["V_scale"], c["V_mn"], c["V_res"], bits)
        assert (o - c["out"]).abs().max() < 2e-3


def test_kivi_pack_round_trip_through_reference_layout():
    """Pack -> in-tree unpack layout -> dequant is within half a quantisation step."""
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 2, 64, 256, generator=g).to(torch.float16)
    for bits in (2, 4):
        code, scale, mn = oracle.kivi_pack_last_dim(x, 32, bits)
        assert code.dtype == torch.int32 and code.shape[-1] == 256 * bits // 32
        codes = oracle.kivi_unpack_last_dim(code, bits)
        assert int(codes.max()) <= 2 ** bits - 1
        deq = oracle.kivi_dequant_v(code, scale, mn, 32, bits)
        step = scale.float().repeat_interleave(32, -1)
        assert ((deq - x.float()).abs() <= 0.5 * step + 2e-3 * x.float().abs() + 1e-3).all()


def test_topk_lower_index_tie_rule():
    s = torch.tensor([[1.0, 3.0, 3.0, 2.0, 3.0, 0.0]])
    v, i = oracle.topk_lower_index(s, 2)
    assert i.tolist() == [[1, 2]]
    v, i = oracle.topk_lower_index(s, 4)
    assert i.tolist() == [[1, 2, 4, 3]]


def test_lse_combine_equals_dense():
    g = torch.Generator().manual_seed(1)
    q = torch.randn(2, 8, 1, 64, generator=g)
    k = torch.randn(2, 2, 300, 64, generator=g)
    v = torch.randn(2, 2, 300, 64, generator=g)
    m, l, o = oracle.split_partials(q, k, v, 0.125, 5)
    comb = oracle.lse_combine(m, l, o)
    ref = oracle.decode_attn_dense(q, k, v, 0.125, out_dtype=torch.float32)[:, :, 0]
    assert torch.allclose(comb, ref, atol=1e-5, rtol=1e-5)


def _near_tie_rows(scores, kb, tol=1e-5):
    """Rows whose kb-th and (kb+1)-th largest finite scores agree within tol."""
    v = scores.sort(-1, descending=True).values
    if v.shape[-1] <= kb:
        return torch.zeros(v.shape[:-1], dtype=torch.bool)
    a, b = v[..., kb - 1], v[..., kb]
    return torch.isfinite(a) & torch.isfinite(b) & ((a - b).abs() <= tol)


def test_select_exact_window_matches_reference(golden_window):
    for c in golden_window["select_exact_window"]:
        q, keys = c["q"].float(), c["keys"].float()
        idx = oracle.select_topk_exact_window(q, keys, c["q_pos"], c["S"], c["kb"], c["scaling"], c["local_w"])
        assert idx.shape == c["idx"].shape
        sc = torch.einsum("bhqd,bhsd->bhqs", q, keys) * c["scaling"]
        tie = _near_tie_rows(sc, c["kb"]).reshape(-1)
        a, b = valid_sets(idx, c["q_pos"], c["S"]), valid_sets(c["idx"], c["q_pos"], c["S"])
        assert all(x == y or t for x, y, t in zip(a, b, tie.tolist()))
        assert tie.float().mean() < 0.05


def test_quest_window_matches_reference(golden_window):
    for c in golden_window["quest_window"]:
        q, k_r = c["q"].float(), c["k_r"].float()
        idx = oracle.quest_select_window(q, k_r, c["q_pos"], c["S"], c["kb"], c["page"], c["scaling"], c["local_w"])
        assert idx.shape == c["idx"].shape
        assert valid_sets(idx, c["q_pos"], c["S"]) == valid_sets(c["idx"], c["q_pos"], c["S"])


def test_attend_and_chunked_window_match_reference(golden_window):
    for c in golden_window["attend_window"]:
        o = oracle.attend_topk(c["q"].float(), c["k_r"].float(), c["v"].float(), c["idx"], c["q_pos"], c["scaling"])
        assert torch.allclose(o, c["out"], rtol=1e-5, atol=1e-5, equal_nan=True)
    for c in golden_window["chunked"]:
        so = c.get("sel_override")
        o = oracle.sparse_attention_chunked(c["q_r"].float(), c["k_r"].float(), c["v"].float(), c["selector"],
                                            c["frac"], c["n_kv_groups"], c["scaling"], c["page"], c["q_chunk"],
                                            sel_override=None if so is None else so.float())
        assert chunked_mismatch(o, c["out"], c, 1e-4) <= 1e-4, c["selector"]
