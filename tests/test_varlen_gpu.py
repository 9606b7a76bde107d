"""Prefill of packed sequences of different lengths (cu_seqlens) against the padded
prefill run on each sequence alone: the same kept blocks in the same order, so the
outputs must agree exactly, and no sequence may see another's keys."""
from __future__ import annotations

import math

import pytest
import torch

import tasft_b200 as T
from tasft_b200 import masks as M

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(lens, Hq, Hk, D, dtype=torch.bfloat16, density=0.3, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    tot = sum(lens)
    q = torch.randn(tot, Hq, D, device=DEV, generator=g).to(dtype)
    k = torch.randn(tot, Hk, D, device=DEV, generator=g).to(dtype)
    v = torch.randn(tot, Hk, D, device=DEV, generator=g).to(dtype)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32, device=DEV)
    nb = math.ceil(max(lens) / 64)
    mask = M.prefill_mask(torch.rand(len(lens), Hk, nb, nb, device=DEV, generator=g), density)
    return q, k, v, cu, mask, nb


@pytest.mark.parametrize("lens,Hq,Hk,D", [
    ([100, 500, 64, 1000], 8, 2, 128),
    ([4096, 33, 2048], 32, 8, 128),
    ([70, 130, 129], 4, 4, 64),        # MHA: two q-blocks per tile
    ([1, 64, 65, 127, 128], 6, 2, 64),  # GQA 3: a head pair and a single head
])
def test_varlen_equals_per_sequence(lens, Hq, Hk, D):
    q, k, v, cu, mask, nb = _case(lens, Hq, Hk, D)
    kern = T.BlockSparseFlashAttention()
    out = kern.forward_varlen(q, k, v, cu, max(lens), mask)
    for b, n in enumerate(lens):
        s0 = int(cu[b])
        nbs = math.ceil(n / 64)
        qs = q[s0:s0 + n].transpose(0, 1).unsqueeze(0)
        ks = k[s0:s0 + n].transpose(0, 1).unsqueeze(0)
        vs = v[s0:s0 + n].transpose(0, 1).unsqueeze(0)
        ref = kern.forward(qs, ks, vs, mask[b:b + 1, :, :nbs, :nbs].contiguous())
        assert torch.equal(out[s0:s0 + n], ref[0].transpose(0, 1)), f"sequence {b}"


def test_varlen_fp16_noncausal_rows_isolated():
    lens = [300, 77]
    q, k, v, cu, mask, nb = _case(lens, 4, 2, 128, dtype=torch.float16, density=1.0, seed=3)
    full = torch.ones(len(lens), 2, nb, nb, dtype=torch.bool, device=DEV)
    kern = T.BlockSparseFlashAttention()
    out = kern.forward_varlen(q, k, v, cu, max(lens), full, causal=False)
    # sequence 1 attends to its own 77 keys only, even though its blocks overlap nothing else
    s0, n = int(cu[1]), lens[1]
    ref = torch.nn.functional.scaled_dot_product_attention(
        q[s0:s0 + n].transpose(0, 1).float(), k[s0:s0 + n].transpose(0, 1).float().repeat_interleave(2, 0),
        v[s0:s0 + n].transpose(0, 1).float().repeat_interleave(2, 0))
    assert (out[s0:s0 + n].transpose(0, 1).float() - ref).abs().max().item() <= 2e-2


@pytest.mark.parametrize("dtype,block,force_simt", [(torch.float32, 64, False), (torch.float32, 32, False),
                                                      (torch.float32, 128, False), (torch.bfloat16, 64, True)])
def test_varlen_cuda_core_kernel_equals_per_sequence(dtype, block, force_simt):
    lens = [90, 300, 33]
    g = torch.Generator(device=DEV).manual_seed(7)
    Hq, Hk, D = 4, 2, 64
    tot = sum(lens)
    q = torch.randn(tot, Hq, D, device=DEV, generator=g).to(dtype)
    k = torch.randn(tot, Hk, D, device=DEV, generator=g).to(dtype)
    v = torch.randn(tot, Hk, D, device=DEV, generator=g).to(dtype)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32, device=DEV)
    nb = math.ceil(max(lens) / block)
    mask = torch.rand(len(lens), Hk, nb, nb, device=DEV, generator=g) < 0.6
    mask |= torch.eye(nb, dtype=torch.bool, device=DEV)
    kern = T.BlockSparseFlashAttention(block_size=block)
    kern.force_simt = force_simt
    out = kern.forward_varlen(q, k, v, cu, max(lens), mask)
    for b, n in enumerate(lens):
        s0, nbs = int(cu[b]), math.ceil(n / block)
        ref = kern.forward(q[s0:s0 + n].transpose(0, 1).unsqueeze(0), k[s0:s0 + n].transpose(0, 1).unsqueeze(0),
                           v[s0:s0 + n].transpose(0, 1).unsqueeze(0), mask[b:b + 1, :, :nbs, :nbs].contiguous())
        assert torch.equal(out[s0:s0 + n], ref[0].transpose(0, 1)), f"sequence {b}"
