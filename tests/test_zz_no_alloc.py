"""The decode entry point that allocates nothing (tasft_bsa_decode_fwd_noalloc).

It exists for callers that cannot allocate device memory themselves -- a plugin whose
host process owns every allocation, or a serving loop that must not call cudaMalloc --
so its split-KV scratch is a fixed 4 MiB array inside the library. These tests call it
through the C ABI and compare it with the regular entry point (which takes a
caller-allocated workspace), twice in a row, since every call reuses the same scratch.
The file name makes pytest collect it last.
"""
from __future__ import annotations

import ctypes as C
import math

import pytest
import torch

import tasft_b200 as T
from tasft_b200 import _lib as L
from tasft_b200 import masks as M

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(B=8, Hq=32, Hk=8, Lc=2048, D=128, seed=77):
    g = torch.Generator(device=DEV).manual_seed(seed)
    q = torch.randn(B, Hq, D, device=DEV, dtype=torch.bfloat16, generator=g)
    kc = torch.randn(B, Hk, Lc, D, device=DEV, dtype=torch.bfloat16, generator=g)
    vc = torch.randn(B, Hk, Lc, D, device=DEV, dtype=torch.bfloat16, generator=g)
    kv_len = torch.randint(Lc // 2, Lc + 1, (B,), device=DEV, generator=g).to(torch.int32)
    nb = math.ceil(Lc / 64)
    mask = M.decode_mask(torch.rand(B, Hk, nb, device=DEV, generator=g), (kv_len + 63) // 64, 0.3, nb)
    idx, cnt = M.lists_from_mask(mask)
    return q, kc, vc, kv_len, idx, cnt


def _args(q, kc, vc, kv_len, idx, cnt, out, splits):
    B, Hq, D = q.shape
    return L.DecodeArgs(
        q=q.data_ptr(), k_cache=kc.data_ptr(), v_cache=vc.data_ptr(), out=out.data_ptr(),
        q_stride=L.strides3(q), k_stride=L.strides4(kc), v_stride=L.strides4(vc), o_stride=L.strides3(out),
        B=B, Hq=Hq, Hk=kc.shape[1], L=kc.shape[2], D=D, block=64, dtype=L.BF16, scale=1.0 / math.sqrt(D),
        kv_len=kv_len.data_ptr(), kept_idx=idx.data_ptr(), kept_cnt=cnt.data_ptr(), nb_max=idx.shape[-1],
        num_splits=splits, part_o=None, part_ml=None, workspace=None, workspace_bytes=0, err=None,
    )


# (B, Lc, splits): one split (no scratch), 3 splits within the resident CTA slots, and 64
# sequences x 8 kv-heads x 3 splits = 1536 work items, more than the 6 x 148 resident
# CTAs, so the persistent kernel claims items from the work counters in the scratch.
@pytest.mark.parametrize("B,Lc,splits", [(8, 2048, 1), (8, 2048, 3), (64, 1024, 3)])
def test_noalloc_matches_workspace_entry_point_twice(B, Lc, splits):
    q, kc, vc, kv_len, idx, cnt = _inputs(B=B, Lc=Lc)
    ref = T.bsa_decode(q, kc, vc, kv_len, T.KeptBlocks(idx, cnt), 64, num_splits=splits)
    lib = L.lib()
    stream = L.stream_ptr(q.device)
    for _ in range(2):  # the scratch keeps the previous call's contents
        out = torch.full_like(q, float("nan"))
        rc = lib.tasft_bsa_decode_fwd_noalloc(C.byref(_args(q, kc, vc, kv_len, idx, cnt, out, splits)), stream)
        assert rc == 0, lib.tasft_status_string(rc)
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        # same kernels, same split boundaries and merge order: bit-identical
        assert torch.equal(out, ref)


def test_noalloc_rejects_scratch_beyond_capacity():
    lib = L.lib()
    cap = lib.tasft_decode_noalloc_capacity()
    assert cap == 4 << 20
    q, kc, vc, kv_len, idx, cnt = _inputs(B=2, Lc=256)
    out = torch.empty_like(q)
    a = _args(q, kc, vc, kv_len, idx, cnt, out, splits=1)
    # enough splits that the partials exceed the fixed scratch: rejected before launching
    a.num_splits = int(cap // (a.B * a.Hq * (a.D + 2) * 4)) + 1
    assert lib.tasft_bsa_decode_fwd_noalloc(C.byref(a), L.stream_ptr(q.device)) == -5
