"""Sparse decode over a paged KV cache (vLLM's flash layout) against the contiguous decode.

A contiguous cache is scattered into a shuffled page pool; the paged decode must give
exactly the contiguous decode's output (same keys in the same order, same arithmetic),
and an out-of-range table entry must be reported in the error word without a fault.
"""
from __future__ import annotations

import math

import pytest
import torch

import tasft_b200 as T
from tasft_b200 import masks as M

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(B, Hq, Hk, Lc, D, page, dtype=torch.bfloat16, density=0.25, seed=0, spare=3):
    g = torch.Generator(device=DEV).manual_seed(seed)
    q = torch.randn(B, Hq, D, device=DEV, generator=g).to(dtype)
    kc = torch.randn(B, Hk, Lc, D, device=DEV, generator=g).to(dtype)
    vc = torch.randn(B, Hk, Lc, D, device=DEV, generator=g).to(dtype)
    kv_len = torch.randint(Lc // 3, Lc + 1, (B,), device=DEV, generator=g).to(torch.int32)
    nb = math.ceil(Lc / 64)
    mask = M.decode_mask(torch.rand(B, Hk, nb, device=DEV, generator=g), (kv_len + 63) // 64, density, nb)
    kept = T.KeptBlocks(*M.lists_from_mask(mask))
    max_pages = Lc // page
    num_pages = B * max_pages + spare
    perm = torch.randperm(num_pages, device=DEV, generator=g)[: B * max_pages].to(torch.int32)
    table = perm.view(B, max_pages)
    kp = torch.zeros(num_pages, page, Hk, D, device=DEV, dtype=dtype)
    vp = torch.zeros_like(kp)
    # logical page p of sequence b -> physical page table[b, p]; pool rows are [token, head, d]
    kp[table.flatten().long()] = kc.view(B, Hk, max_pages, page, D).permute(0, 2, 3, 1, 4).reshape(-1, page, Hk, D)
    vp[table.flatten().long()] = vc.view(B, Hk, max_pages, page, D).permute(0, 2, 3, 1, 4).reshape(-1, page, Hk, D)
    return q, kc, vc, kp, vp, table, kv_len, kept


@pytest.mark.parametrize("page", [16, 32, 64, 128])
@pytest.mark.parametrize("splits", [1, 4])
def test_paged_equals_contiguous(page, splits):
    q, kc, vc, kp, vp, table, kv_len, kept = _case(4, 32, 8, 2048, 128, page)
    ref = T.bsa_decode(q, kc, vc, kv_len, kept, 64, num_splits=splits)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = T.bsa_decode_paged(q, kp, vp, table, kv_len, kept, 64, num_splits=splits, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(out, ref)


@pytest.mark.parametrize("dtype,Hq,Hk,D", [(torch.float16, 28, 4, 128), (torch.bfloat16, 8, 8, 64)])
def test_paged_other_shapes(dtype, Hq, Hk, D):
    q, kc, vc, kp, vp, table, kv_len, kept = _case(2, Hq, Hk, 4096, D, 16, dtype=dtype, density=0.1, seed=3)
    ref = T.bsa_decode(q, kc, vc, kv_len, kept, 64)
    out = T.bsa_decode_paged(q, kp, vp, table, kv_len, kept, 64)
    assert torch.equal(out, ref)


def test_paged_bad_table_entry_is_reported_not_loaded():
    q, kc, vc, kp, vp, table, kv_len, kept = _case(2, 8, 2, 1024, 128, 64, density=1.0, seed=5)
    bad = table.clone()
    bad[0, 0] = kp.shape[0] + 7  # outside the pool
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = T.bsa_decode_paged(q, kp, vp, bad, kv_len, kept, 64, num_splits=1, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) & 1  # TASFT_DEVERR_INDEX
    assert torch.isfinite(out.float()).all()
    # the other sequence does not touch the bad entry and is unaffected
    ref = T.bsa_decode(q, kc, vc, kv_len, kept, 64, num_splits=1)
    assert torch.equal(out[1], ref[1])
