"""The quad-tile tcgen05 prefill kernel (per-kv-head lists, GQA groups >= 3) against the
oracle, against the two-slot tcgen05 kernel it replaces for those shapes, and at its
edges: odd list lengths (a lone 64-key block in the last stage), ragged S, groups of 3, 7
and 8 (an idle slot; two quads per kv-head), D 64, fp16, non-causal, empty rows, many
quads per CTA, bad indices."""
from __future__ import annotations

import math

import pytest
import torch

import oracle as O
import tasft_b200 as T
from tasft_b200 import _lib as L
from tasft_b200 import masks as M

pytestmark = pytest.mark.gpu
DEV = "cuda"
BF16_ABS = 2e-2
BF16_REL = 1e-2


def _close(out, ref):
    o, r = out.float().cpu(), ref.float()
    assert (o - r).abs().max().item() <= BF16_ABS
    assert ((o - r).abs().sum() / r.abs().sum().clamp_min(1e-6)).item() <= BF16_REL


def _case(B, Hq, Hk, S, D, dtype, density, seed, causal=True, odd=False):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, S, D, generator=g).to(dtype)
    k = torch.randn(B, Hk, S, D, generator=g).to(dtype)
    v = torch.randn(B, Hk, S, D, generator=g).to(dtype)
    nb = math.ceil(S / 64)
    if causal:
        mask = M.prefill_mask(torch.rand(B, Hk, nb, nb, generator=g), density)
    else:
        mask = torch.rand(B, Hk, nb, nb, generator=g) < density
    if odd:  # drop block 0 from rows with an even count (rows > 0): every list has odd length
        even = (mask.sum(-1) % 2 == 0) & (torch.arange(nb) > 0)
        mask[..., 0] &= ~even
    return q, k, v, mask


def _run(kern_mode, q, k, v, mask, causal=True):
    kern = T.BlockSparseFlashAttention(block_size=64)
    kern.force_simt = kern_mode
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = kern.forward(q.to(DEV), k.to(DEV), v.to(DEV), mask.to(DEV), causal=causal, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out


@pytest.mark.parametrize("B,Hq,Hk,S,D,density,odd", [
    (1, 4, 1, 512, 128, 0.3, False),
    (1, 4, 1, 512, 128, 0.3, True),    # odd lists: N64 S chain + K64 P.V for the last block
    (2, 8, 2, 700, 128, 0.25, False),  # ragged S
    (1, 7, 1, 384, 128, 0.4, False),   # group 7: second quad has an idle slot
    (1, 8, 1, 640, 128, 0.5, True),    # group 8: two quads per kv-head
    (1, 3, 1, 448, 64, 0.5, False),    # group 3, D 64
    (1, 4, 1, 2048, 128, 0.6, False),  # long lists: deep ring reuse
    (2, 4, 2, 1024, 64, 1.0, False),   # dense
])
def test_quad_vs_oracle(B, Hq, Hk, S, D, density, odd):
    q, k, v, mask = _case(B, Hq, Hk, S, D, torch.bfloat16, density, seed=S + Hq + D, odd=odd)
    out = _run(0, q, k, v, mask)
    _close(out, O.bsa_prefill_masked_dense(q, k, v, mask, 64))
    # the two-slot kernel on the same inputs agrees within the same tolerance
    out2 = _run(2, q, k, v, mask)
    assert (out.float() - out2.float()).abs().max().item() <= BF16_ABS


def test_quad_fp16_noncausal():
    q, k, v, mask = _case(1, 4, 1, 320, 128, torch.float16, 0.5, seed=3, causal=False)
    out = _run(0, q, k, v, mask, causal=False)
    _close(out, O.bsa_prefill_masked_dense(q, k, v, mask, 64, causal=False))


@pytest.mark.parametrize("gain", [6.0, 20.0])
def test_quad_lazy_rescale(gain):
    q, k, v, mask = _case(1, 4, 1, 1024, 128, torch.bfloat16, 0.5, seed=31)
    q = (q.float() * gain).to(torch.bfloat16)
    ramp = torch.linspace(0.2, 3.0, 1024).view(1, 1, 1024, 1)
    k = (k.float() * ramp).to(torch.bfloat16)
    _close(_run(0, q, k, v, mask), O.bsa_prefill_masked_dense(q, k, v, mask, 64))


def test_quad_empty_rows_and_many_quads_per_cta(monkeypatch):
    monkeypatch.setenv("TASFT_PREFILL_GRID", "3")
    q, k, v, mask = _case(2, 8, 2, 1024, 128, torch.bfloat16, 0.4, seed=41)
    mask[:, :, 5, :] = False
    mask[1, 1, 9, :] = False
    out = _run(0, q, k, v, mask)
    assert out[:, :, 320:384].abs().max().item() == 0.0
    _close(out, O.bsa_prefill_masked_dense(q, k, v, mask, 64))


def test_quad_deterministic_and_lists_input():
    q, k, v, mask = _case(2, 8, 2, 2048, 128, torch.bfloat16, 0.3, seed=33)
    a = _run(0, q, k, v, mask)
    b = _run(0, q, k, v, mask)
    assert torch.equal(a, b)
    idx, cnt = M.lists_from_mask(mask)
    kern = T.BlockSparseFlashAttention()
    c = kern.forward(q.to(DEV), k.to(DEV), v.to(DEV), T.KeptBlocks(idx.to(DEV), cnt.to(DEV)))
    assert torch.equal(a, c)


def test_quad_bad_index_reported():
    q, k, v, mask = _case(1, 4, 1, 256, 128, torch.bfloat16, 1.0, seed=15)
    idx, cnt = M.lists_from_mask(mask)
    idx[0, 0, 3, 0] = 99
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    T.BlockSparseFlashAttention().forward(q.to(DEV), k.to(DEV), v.to(DEV), T.KeptBlocks(idx.to(DEV), cnt.to(DEV)),
                                          err=err)
    assert int(err.item()) & L.DEVERR_INDEX
