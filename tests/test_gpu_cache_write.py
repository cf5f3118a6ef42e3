"""Cache-write side of the decode path: streaming KIVI appends and Quest metadata refresh.

The reference packs whole tensors (external KIVI packer, benchmarks/kivi_latency.py:123,127)
and recomputes Quest page min/max on every call (benchmarks/sparse_attention.py:334-341).
The incremental forms must leave the caches exactly as the whole-tensor forms would.
"""
import pytest
import torch

import oracle
from bytes_b200 import kivi as kv
from bytes_b200 import sparse_attention as sa

pytestmark = pytest.mark.gpu


def gen(seed):
    return torch.Generator().manual_seed(seed)


@pytest.mark.parametrize("bits", [2, 4])
def test_kivi_append_equals_whole_pack(cuda, bits):
    g = gen(40 + bits)
    B, Hk, S, D, cap = 2, 2, 320, 128, 384
    fpi = 32 // bits
    k = torch.randn(B, Hk, S, D, generator=g).half()
    v = torch.randn(B, Hk, S, D, generator=g).half()
    k[:, :, 100:132] = 0.25  # one constant key group (range clamp)
    Kq_ref, Ks_ref, Km_ref = oracle.kivi_pack_last_dim(k.transpose(2, 3).contiguous(), 32, bits)
    Vq_ref, Vs_ref, Vm_ref = oracle.kivi_pack_last_dim(v, 32, bits)
    Kq = torch.full((B, Hk, D, cap // fpi), -1, dtype=torch.int32, device=cuda)
    Ks = torch.full((B, Hk, D, cap // 32), float("nan"), dtype=torch.float16, device=cuda)
    Km = Ks.clone()
    Vq = torch.full((B, Hk, cap, D // fpi), -1, dtype=torch.int32, device=cuda)
    Vs = torch.full((B, Hk, cap, D // 32), float("nan"), dtype=torch.float16, device=cuda)
    Vm = Vs.clone()
    kd, vd = k.to(cuda), v.to(cuda)
    for t0, t1 in ((0, 64), (64, 96), (96, S)):
        kv.kivi_append(kd[:, :, t0:t1], vd[:, :, t0:t1], bits, t0, Kq, Ks, Km, Vq, Vs, Vm)
    torch.cuda.synchronize()
    assert torch.equal(Kq[..., :S // fpi].cpu(), Kq_ref)
    assert torch.equal(Ks[..., :S // 32].cpu(), Ks_ref) and torch.equal(Km[..., :S // 32].cpu(), Km_ref)
    assert torch.equal(Vq[:, :, :S].cpu(), Vq_ref)
    assert torch.equal(Vs[:, :, :S].cpu(), Vs_ref) and torch.equal(Vm[:, :, :S].cpu(), Vm_ref)
    # nothing past the appended tokens is touched
    assert (Kq[..., S // fpi:] == -1).all() and (Vq[:, :, S:] == -1).all()
    assert torch.isnan(Ks[..., S // 32:]).all() and torch.isnan(Vs[:, :, S:]).all()


def test_kivi_append_rejects_partial_groups(cuda):
    B, Hk, D = 1, 1, 128
    k = torch.zeros(B, Hk, 48, D, dtype=torch.float16, device=cuda)
    Kq = torch.zeros(B, Hk, D, 8, dtype=torch.int32, device=cuda)
    Ks = torch.zeros(B, Hk, D, 4, dtype=torch.float16, device=cuda)
    Vq = torch.zeros(B, Hk, 128, 8, dtype=torch.int32, device=cuda)
    Vs = torch.zeros(B, Hk, 128, 4, dtype=torch.float16, device=cuda)
    with pytest.raises(ValueError):
        kv.kivi_append(k, k, 2, 0, Kq, Ks, Ks, Vq, Vs, Vs)  # 48 tokens: not whole groups
    with pytest.raises(ValueError):
        kv.kivi_append(k[:, :, :32], k[:, :, :32], 2, 16, Kq, Ks, Ks, Vq, Vs, Vs)  # offset not a group start
    with pytest.raises(ValueError):
        kv.kivi_append(k[:, :, :32], k[:, :, :32], 2, 128, Kq, Ks, Ks, Vq, Vs, Vs)  # past the capacity


def test_quest_metadata_update_equals_recompute(cuda):
    g = gen(44)
    B, H, S, D, page, cap_pages = 2, 3, 100, 64, 16, 10
    k = torch.randn(B, H, S, D, generator=g).bfloat16().to(cuda)
    kmin_ref, kmax_ref = sa.quest_page_metadata(k, page)
    kmin = torch.zeros(B, H, cap_pages, D, dtype=k.dtype, device=cuda)
    kmax = torch.zeros_like(kmin)
    sa.quest_page_metadata_update(k, kmin, kmax, page, 0, 3)
    sa.quest_page_metadata_update(k, kmin, kmax, page, 3, 7)  # last page holds 4 tokens
    np_ = (S + page - 1) // page
    assert torch.equal(kmin[:, :, :np_], kmin_ref) and torch.equal(kmax[:, :, :np_], kmax_ref)
    assert (kmin[:, :, np_:] == 0).all()
    rmin, rmax = oracle.quest_page_minmax(k.cpu(), page)
    assert torch.equal(kmin[:, :, :np_].cpu(), rmin) and torch.equal(kmax[:, :, :np_].cpu(), rmax)
