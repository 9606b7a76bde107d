"""Split-KV long-context decode on the GPU: per-rank slabs through the CUDA decode with
partials, merged by the combine kernel, against the unsplit decode (one GPU emulates the
ranks), and the real exchange over NCCL when two GPUs are present."""
from __future__ import annotations

import math
import os
import socket

import pytest
import torch

import tasft_b200 as T
from tasft_b200 import masks as M
from tasft_b200 import shards as SH

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(dev, B=1, Hq=28, Hk=4, Lc=8192, D=128, density=0.1, seed=11):
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(B, Hq, D, device=dev, dtype=torch.bfloat16, generator=g)
    kc = torch.randn(B, Hk, Lc, D, device=dev, dtype=torch.bfloat16, generator=g)
    vc = torch.randn(B, Hk, Lc, D, device=dev, dtype=torch.bfloat16, generator=g)
    kv_len = torch.full((B,), Lc - 37, dtype=torch.int32, device=dev)
    nb = math.ceil(Lc / 64)
    mask = M.decode_mask(torch.rand(B, Hk, nb, device=dev, generator=g), (kv_len + 63) // 64, density, nb)
    idx, cnt = M.lists_from_mask(mask)
    return q, kc, vc, kv_len, T.KeptBlocks(idx, cnt)


@pytest.mark.parametrize("world", [2, 3, 8])
def test_emulated_ranks_match_unsplit(world):
    q, kc, vc, kv_len, kept = _inputs(DEV)
    ref = T.bsa_decode(q, kc, vc, kv_len, kept, 64).float()
    nb = kc.shape[2] // 64
    pos, pms = [], []
    for r in range(world):
        lo, hi = SH.block_range(nb, r, world)
        kl = SH.local_kept(kept, lo, hi)
        po = torch.empty(q.shape, dtype=torch.float32, device=DEV)
        pm = torch.empty(*q.shape[:2], 2, dtype=torch.float32, device=DEV)
        T.bsa_decode(q, kc[:, :, lo * 64 : hi * 64].contiguous(), vc[:, :, lo * 64 : hi * 64].contiguous(),
                     SH.local_kv_len(kv_len, lo, hi, 64), kl, 64, partials=(po, pm))
        pos.append(po)
        pms.append(pm)
    out = T.decode_combine(torch.stack(pos), torch.stack(pms), torch.bfloat16).float()
    # bf16 output tolerance of the suite
    assert (out - ref).abs().max().item() <= 2e-2


def _rank(rank, world, port, res):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist  # noqa: PLC0415

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        q, kc, vc, kv_len, kept = _inputs(dev)
        lo, hi = SH.block_range(kc.shape[2] // 64, rank, world)
        out = SH.long_context_decode(q, kc[:, :, lo * 64 : hi * 64].contiguous(),
                                     vc[:, :, lo * 64 : hi * 64].contiguous(), kv_len, kept, lo)
        ref = T.bsa_decode(q, kc, vc, kv_len, kept, 64)
        res.put((rank, (out.float() - ref.float()).abs().max().item()))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nccl_two_ranks_match_unsplit():
    import torch.multiprocessing as mp  # noqa: PLC0415

    ctx = mp.get_context("spawn")
    res = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_rank, args=(r, 2, port, res)) for r in range(2)]
    for p in procs:
        p.start()
    errs = dict(res.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert max(errs.values()) <= 2e-2


@pytest.mark.parametrize("world", [1, 3, 8])
def test_sharded_prefill_units_equal_full_batch(world):
    """LPT-sharded prefill: every rank runs its (sequence, kv-head) units; scattered back,
    the result is exactly the one-call prefill's."""
    g = torch.Generator(device=DEV).manual_seed(31)
    B, Hq, Hk, S, D = 2, 32, 8, 1024, 128
    q = torch.randn(B, Hq, S, D, device=DEV, generator=g).bfloat16()
    k = torch.randn(B, Hk, S, D, device=DEV, generator=g).bfloat16()
    v = torch.randn(B, Hk, S, D, device=DEV, generator=g).bfloat16()
    mask = M.prefill_mask(torch.rand(B, Hk, S // 64, S // 64, device=DEV, generator=g), 0.2)
    kern = T.BlockSparseFlashAttention()
    kept = T.mask_to_kept(mask, True)
    full = kern.forward(q, k, v, kept)
    parts = SH.assign_units(SH.unit_weights(kept, Hk), world)
    out = torch.zeros_like(full)
    for units in parts:
        if units:
            SH.scatter_units(out, SH.prefill_units(kern, q, k, v, kept, units), units, Hk)
    assert torch.equal(out, full)


def _rank_decoder(rank, world, port, res):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist  # noqa: PLC0415

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        q, kc, vc, kv_len, kept = _inputs(dev)
        lo, hi = SH.block_range(kc.shape[2] // 64, rank, world)
        dec = SH.SplitKVDecoder(q.shape[0], q.shape[1], kc.shape[1], q.shape[2], dev)
        kl, vl = kc[:, :, lo * 64 : hi * 64].contiguous(), vc[:, :, lo * 64 : hi * 64].contiguous()
        loc = dec.local(kept, lo, hi - lo)
        ref = T.bsa_decode(q, kc, vc, kv_len, kept, 64)
        errs = [(dec(q, kl, vl, kv_len, kept, lo, local=loc).float() - ref.float()).abs().max().item()
                for _ in range(3)]  # buffers reused across calls
        res.put((rank, max(errs)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_split_kv_decoder_reuses_buffers_two_ranks():
    import torch.multiprocessing as mp  # noqa: PLC0415

    ctx = mp.get_context("spawn")
    res = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_rank_decoder, args=(r, 2, port, res)) for r in range(2)]
    for p in procs:
        p.start()
    errs = dict(res.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert max(errs.values()) <= 2e-2


@pytest.mark.parametrize("world", [3, 8])
def test_long_prefill_qblock_ranges_sum_to_full(world):
    """One long sequence, 4 kv-heads: ranks split the q-blocks by kept work; each rank's
    rows outside its range are zero, so the ranks' outputs sum to the one-call prefill."""
    g = torch.Generator(device=DEV).manual_seed(32)
    B, Hq, Hk, S, D = 1, 28, 4, 8192, 128
    q = torch.randn(B, Hq, S, D, device=DEV, generator=g).bfloat16()
    k = torch.randn(B, Hk, S, D, device=DEV, generator=g).bfloat16()
    v = torch.randn(B, Hk, S, D, device=DEV, generator=g).bfloat16()
    mask = M.prefill_mask(torch.rand(B, Hk, S // 64, S // 64, device=DEV, generator=g), 0.1)
    kern = T.BlockSparseFlashAttention()
    kept = T.mask_to_kept(mask, True)
    full = kern.forward(q, k, v, kept)
    acc = torch.zeros_like(full, dtype=torch.float32)
    for lo, hi in SH.qblock_ranges(kept, world):
        part = kern.forward(q, k, v, SH.restrict_qblocks(kept, lo, hi))
        assert part[:, :, : lo * 64].eq(0).all() and part[:, :, hi * 64:].eq(0).all()
        acc += part.float()
    assert torch.equal(acc.to(full.dtype), full)


@pytest.mark.parametrize("grp", [7, 1])
def test_long_prefill_qblock_window_writes_only_its_rows(grp):
    """q_block_range: the tensor-core kernel visits only the window's tiles. Rows inside the
    window equal the full call bit for bit; rows outside keep what the output held (NaN
    here). GQA (7 q-heads per kv-head) and MHA (pairs of q-blocks per tile, odd window
    ends)."""
    g = torch.Generator(device=DEV).manual_seed(33)
    B, Hk, S, D = 1, 2, 4096, 128
    Hq = Hk * grp
    q = torch.randn(B, Hq, S, D, device=DEV, generator=g).bfloat16()
    k = torch.randn(B, Hk, S, D, device=DEV, generator=g).bfloat16()
    v = torch.randn(B, Hk, S, D, device=DEV, generator=g).bfloat16()
    mask = M.prefill_mask(torch.rand(B, Hk, S // 64, S // 64, device=DEV, generator=g), 0.2)
    kern = T.BlockSparseFlashAttention()
    kept = T.mask_to_kept(mask, True)
    full = kern.forward(q, k, v, kept)
    for lo, hi in [(0, 21), (21, 47), (47, 64)]:
        out = torch.full_like(full, float("nan"))
        kern.forward(q, k, v, SH.restrict_qblocks(kept, lo, hi), out=out, q_block_range=(lo, hi))
        assert torch.equal(out[:, :, lo * 64: hi * 64], full[:, :, lo * 64: hi * 64])
        assert out[:, :, : lo * 64].isnan().all() and out[:, :, hi * 64:].isnan().all()
