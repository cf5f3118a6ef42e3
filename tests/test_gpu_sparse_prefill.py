"""The selection primitives of ``benchmarks/sparse_attention.py`` over prefill windows.

The reference runs select_topk / _quest_select / attend_topk over blocks of query rows at
positions q_pos (keys causal per row, an optional forced recent window), and
sparse_attention_chunked loops them over a whole prefill window
(benchmarks/sparse_attention.py:226-387, 463-497), for the 'exact', 'quest', soft
(approximate-key), 'sparq', 'recent' and 'random' selectors. This engine folds a block's rows into the
head axis and runs the decode kernels with per-row causal limits. Gates: the golden vectors
made by running the reference's code (tests/golden/make_golden_window.py) and the fp32
oracle; selections compared as sets of usable (causal, in-range) positions per row, exact
except on rows whose cut-off is a near-tie; attention within 1e-4 for fp32 inputs and
within 1e-3 mean-abs for bf16 outputs, with at most 0.2 % of rows past 2e-2 max-abs.
"""
import pytest
import torch

import oracle
from bytes_b200 import sparse_attention as sa
from conftest import chunked_mismatch, valid_sets

pytestmark = pytest.mark.gpu


def _near_tie_rows(scores, kb, tol=1e-5):
    v = scores.sort(-1, descending=True).values
    if v.shape[-1] <= kb:
        return torch.zeros(v.shape[:-1], dtype=torch.bool)
    a, b = v[..., kb - 1], v[..., kb]
    return torch.isfinite(a) & torch.isfinite(b) & ((a - b).abs() <= tol)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_select_exact_window_golden(cuda, golden_window, dt):
    for c in golden_window["select_exact_window"]:
        q, keys = c["q"].to(dt), c["keys"].to(dt)
        idx = sa.select_topk("exact", q.to(cuda), keys.to(cuda), c["q_pos"], c["S"], c["kb"], 64, c["scaling"],
                             local_w=c["local_w"]).cpu()
        assert idx.shape == c["idx"].shape and idx.dtype == torch.int64
        sc = torch.einsum("bhqd,bhsd->bhqs", q.float(), keys.float()) * c["scaling"]
        tie = _near_tie_rows(sc, c["kb"]).reshape(-1).tolist()
        a, b = valid_sets(idx, c["q_pos"], c["S"]), valid_sets(c["idx"], c["q_pos"], c["S"])
        assert all(x == y or t for x, y, t in zip(a, b, tie))


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_quest_window_golden(cuda, golden_window, dt):
    for c in golden_window["quest_window"]:
        idx = sa._quest_select(c["q"].to(dt).to(cuda), c["k_r"].to(dt).to(cuda), c["q_pos"], c["S"], c["kb"],
                               c["page"], c["scaling"], c["local_w"]).cpu()
        assert idx.shape == c["idx"].shape
        assert valid_sets(idx, c["q_pos"], c["S"]) == valid_sets(c["idx"], c["q_pos"], c["S"])


def test_attend_window_golden(cuda, golden_window):
    for c in golden_window["attend_window"]:
        args = [c[n].float().to(cuda) for n in ("q", "k_r", "v")]
        o = sa.attend_topk(*args, c["idx"].to(cuda), c["q_pos"], c["scaling"]).cpu()
        assert torch.allclose(o, c["out"], rtol=1e-4, atol=1e-4, equal_nan=True), (o - c["out"]).abs().max()


def test_chunked_golden(cuda, golden_window):
    for c in golden_window["chunked"]:
        args = [c[n].float().to(cuda) for n in ("q_r", "k_r", "v")]
        so = c.get("sel_override")
        o = sa.sparse_attention_chunked(*args, None if so is None else so.float().to(cuda), c["selector"], c["frac"],
                                        c["n_kv_groups"], c["scaling"], page=c["page"], q_chunk=c["q_chunk"]).cpu()
        assert chunked_mismatch(o, c["out"], c, 1e-4) <= 1e-4, c["selector"]


@pytest.mark.parametrize("selector,local_w", [("exact", 0), ("exact", 32), ("quest", 0), ("quest", 48)])
def test_chunked_vs_oracle(cuda, selector, local_w):
    """bf16 window of 1000 tokens (28/4 heads, D=128), chunks of 256 rows, 10 % budget."""
    g = torch.Generator().manual_seed(7 + local_w)
    B, Hq, Hk, S, D = 1, 28, 4, 1000, 128
    q = torch.randn(B, Hq, S, D, generator=g).bfloat16()
    k = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    v = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    o = sa.sparse_attention_chunked(q.to(cuda), k.to(cuda), v.to(cuda), None, selector, 0.1, Hq // Hk, 0.088,
                                    page=16, q_chunk=256, local_w=local_w).cpu()
    ref = oracle.sparse_attention_chunked(q, k, v, selector, 0.1, Hq // Hk, 0.088, 16, 256, local_w)
    assert o.dtype == torch.bfloat16 and o.shape == q.shape
    d = (o.float() - ref.float()).abs()
    assert torch.isfinite(o.float()).all()
    assert d.mean().item() <= 1e-3, d.mean().item()
    # a row whose cut-off is a near-tie may take the other key: allow a handful of rows
    bad = (d.amax(-1) > 2e-2).float().mean().item()
    assert bad <= 2e-3, bad


def test_decode_row_with_local_window(cuda):
    """A decode row (q_pos = S-1) with a forced recent window takes the window form."""
    g = torch.Generator().manual_seed(11)
    B, Hq, S, D, kb = 2, 8, 700, 64, 50
    q = torch.randn(B, Hq, 1, D, generator=g)
    keys = torch.randn(B, Hq, S, D, generator=g)
    pos = torch.tensor([S - 1])
    idx = sa.select_topk("exact", q.to(cuda), keys.to(cuda), pos, S, kb, 512, 0.125, local_w=16).cpu()
    ref = oracle.select_topk_exact_window(q, keys, pos, S, kb, 0.125, 16)
    assert valid_sets(idx, pos, S) == valid_sets(ref, pos, S)
    assert all(set(range(S - 16, S)) <= set(r) for r in valid_sets(idx, pos, S))
