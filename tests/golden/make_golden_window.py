"""Generate golden vectors for the prefill-window forms of the reference's selection code.

Usage (in a container where the reference checkout is present):

    python tests/golden/make_golden_window.py --reference <path-to-saifmb0-bytes-checkout>

Runs ``benchmarks.sparse_attention`` of the reference on the CPU with fixed seeds over
blocks of query rows at positions inside the context (per-row causal limits), with and
without the forced recent window: ``select_topk('exact')``, ``_quest_select``,
``attend_topk`` (including sentinel and future positions) and ``sparse_attention_chunked``
for the 'exact', 'quest', 'approx' (approximate keys as ``sel_override``), 'sparq' and
'recent' selectors. Inputs are bf16 values (stored as bf16, passed to
the reference as fp32), so every product is exact in fp32. Output:
``tests/golden/golden_window.pt``.
"""
import argparse
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from benchmarks.sparse_attention import select_topk, _quest_select, attend_topk, sparse_attention_chunked

    g = torch.Generator().manual_seed(20261203)

    def randn(*s):
        return torch.randn(*s, generator=g).bfloat16()

    out = {}
    sel = []
    for (B, Hq, S, D, q0, Qc, kb, local_w) in ((2, 2, 256, 32, 100, 40, 24, 0), (1, 2, 256, 32, 200, 50, 24, 8),
                                               (1, 2, 160, 32, 0, 20, 30, 0)):
        q = randn(B, Hq, Qc, D)
        keys = randn(B, Hq, S, D)
        pos = torch.arange(q0, q0 + Qc)
        idx = select_topk("exact", q.float(), keys.float(), pos, S, kb, 64, 0.15, local_w=local_w)
        sel.append(dict(q=q, keys=keys, q_pos=pos, S=S, kb=kb, scaling=0.15, local_w=local_w, idx=idx))
    out["select_exact_window"] = sel

    quest = []
    for (B, Hq, S, D, q0, Qc, kb, page, local_w) in ((2, 2, 256, 32, 100, 40, 48, 16, 0),
                                                     (1, 2, 256, 32, 180, 60, 48, 16, 20)):
        q = randn(B, Hq, Qc, D)
        k_r = randn(B, Hq, S, D)
        pos = torch.arange(q0, q0 + Qc)
        idx = _quest_select(q.float(), k_r.float(), pos, S, kb, page, 0.15, local_w)
        quest.append(dict(q=q, k_r=k_r, q_pos=pos, S=S, kb=kb, page=page, scaling=0.15, local_w=local_w, idx=idx))
    out["quest_window"] = quest

    att = []
    B, Hq, S, D, q0, Qc, ks = 1, 2, 200, 32, 120, 30, 40
    q = randn(B, Hq, Qc, D)
    k_r = randn(B, Hq, S, D)
    v = randn(B, Hq, S, D)
    idx = torch.randint(0, S + 1, (B, Hq, Qc, ks), generator=g)  # S = sentinel; > q_pos = future
    pos = torch.arange(q0, q0 + Qc)
    att.append(dict(q=q, k_r=k_r, v=v, idx=idx, q_pos=pos, scaling=0.15,
                    out=attend_topk(q.float(), k_r.float(), v.float(), idx, pos, 0.15)))
    out["attend_window"] = att

    chunked = []
    for selector in ("exact", "quest"):
        B, Hq, Hk, S, D = 1, 4, 2, 192, 32
        q_r = randn(B, Hq, S, D)
        k_r = randn(B, Hk, S, D)
        v = randn(B, Hk, S, D)
        o = sparse_attention_chunked(q_r.float(), k_r.float(), v.float(), None, selector, 0.1, Hq // Hk, 0.15,
                                     page=16, q_chunk=64, k_chunk=64)
        chunked.append(dict(selector=selector, q_r=q_r, k_r=k_r, v=v, frac=0.1, n_kv_groups=Hq // Hk,
                            scaling=0.15, page=16, q_chunk=64, out=o))
    # the soft selectors (ranking by approximate keys passed as sel_override), SparQ and the
    # recent window (the random selector's draws depend on the device's generator)
    for selector in ("approx", "sparq", "recent"):
        B, Hq, Hk, S, D = 1, 4, 2, 192, 32
        q_r = randn(B, Hq, S, D)
        k_r = randn(B, Hk, S, D)
        v = randn(B, Hk, S, D)
        approx = (k_r.float() + 0.3 * randn(B, Hk, S, D).float()).bfloat16()
        o = sparse_attention_chunked(q_r.float(), k_r.float(), v.float(), approx.float(), selector, 0.1, Hq // Hk,
                                     0.15, page=16, q_chunk=64, k_chunk=64)
        chunked.append(dict(selector=selector, q_r=q_r, k_r=k_r, v=v, sel_override=approx, frac=0.1,
                            n_kv_groups=Hq // Hk, scaling=0.15, page=16, q_chunk=64, out=o))
    out["chunked"] = chunked

    path = os.path.join(HERE, "golden_window.pt")
    torch.save(out, path)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
