"""Shared pytest configuration: the ``gpu`` marker and common fixtures."""
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    return torch.load(os.path.join(ROOT, "tests", "golden", "golden.pt"))


@pytest.fixture(scope="session")
def golden_cuda():
    """The reference's quantizers run on a CUDA device (tests/golden/make_golden_cuda.py)."""
    return torch.load(os.path.join(ROOT, "tests", "golden", "golden_cuda.pt"))


@pytest.fixture(scope="session")
def golden_window():
    """The reference's selection code over prefill windows (tests/golden/make_golden_window.py)."""
    return torch.load(os.path.join(ROOT, "tests", "golden", "golden_window.pt"))


def valid_sets(idx, q_pos, S):
    """Per query row, the sorted set of causal in-range positions of an index tensor
    [..., Qc, k] (slots the reference fills with a sentinel or with -inf-tied future keys
    carry no weight and are dropped)."""
    out = []
    flat = idx.reshape(-1, idx.shape[-2], idx.shape[-1])
    for m in range(flat.shape[0]):
        for r in range(flat.shape[1]):
            row = flat[m, r]
            out.append(sorted(set(int(x) for x in row[(row <= int(q_pos[r])) & (row < S) & (row >= 0)])))
    return out


def sparq_tie_rows(q, r=16):
    """Query rows [..., S, D] whose r-th and (r+1)-th largest |q| are equal: which channel
    SparQ keeps there is the tie order of torch.topk, which is unspecified."""
    v = q.float().abs().sort(-1, descending=True).values
    return v[..., r - 1] == v[..., r]


def chunked_mismatch(o, ref, c, tol):
    """Largest difference between two chunked-attention outputs over the rows where both
    are defined (SparQ rows with a tie at the channel cut excluded)."""
    d = (o.float() - ref.float()).abs().amax(-1)
    if c["selector"] == "sparq":
        d = d.masked_fill(sparq_tie_rows(c["q_r"]), 0.0)
    return d.max().item()


@pytest.fixture(scope="session")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
