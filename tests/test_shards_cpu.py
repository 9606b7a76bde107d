"""Host-side multi-GPU logic on CPU: unit assignment, per-rank lists, and the split-KV
long-context decode exchange run as two ``gloo`` ranks (the per-rank partials come from
the oracle, since there is no GPU here; the exchange and the rebasing are the product's)."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from tasft_b200 import shards as SH
from tasft_b200.types import KeptBlocks


def test_assign_units_balances_and_covers():
    w = [13, 1, 7, 7, 2, 9, 4, 4, 11, 3]
    for world in (1, 2, 3, 4, 8):
        parts = SH.assign_units(w, world)
        assert sorted(i for p in parts for i in p) == list(range(len(w)))
        loads = [sum(w[i] for i in p) for p in parts]
        # LPT bound: max load <= mean + largest item
        assert max(loads) <= sum(w) / world + max(w)
    assert SH.assign_units([5, 5], 2) == [[0], [1]]
    with pytest.raises(ValueError):
        SH.assign_units([1], 0)


def test_block_range_partitions():
    for nb in (1, 7, 64, 513):
        for world in (1, 2, 3, 8):
            rs = [SH.block_range(nb, r, world) for r in range(world)]
            assert rs[0][0] == 0 and rs[-1][1] == nb
            assert all(rs[i][1] == rs[i + 1][0] for i in range(world - 1))
            assert max(h - lo for lo, h in rs) - min(h - lo for lo, h in rs) <= 1


def test_local_kept_rebases_in_order():
    idx = torch.tensor([[[0, 3, 5, 9, -1, -1], [2, 4, 6, 8, 10, 11]]], dtype=torch.int32)
    cnt = torch.tensor([[4, 6]], dtype=torch.int32)
    kl = SH.local_kept(KeptBlocks(idx, cnt), 4, 9)
    assert kl.cnt.tolist() == [[1, 3]]
    assert kl.idx[0, 0].tolist() == [1, -1, -1, -1, -1, -1]
    assert kl.idx[0, 1].tolist() == [0, 2, 4, -1, -1, -1]
    # entries past cnt are ignored even if they hold in-range values
    kl2 = SH.local_kept(KeptBlocks(idx, torch.tensor([[1, 0]], dtype=torch.int32)), 0, 12)
    assert kl2.cnt.tolist() == [[1, 0]]


def test_local_kv_len():
    kv = torch.tensor([0, 100, 640, 1000], dtype=torch.int32)
    assert SH.local_kv_len(kv, 2, 5, 64).tolist() == [0, 0, 192, 192]
    assert SH.local_kv_len(kv, 0, 2, 64).tolist() == [0, 100, 128, 128]


def _inputs(seed=3):
    g = torch.Generator().manual_seed(seed)
    B, Hq, Hk, Lc, D, nb = 2, 4, 2, 640, 32, 10
    q = torch.randn(B, Hq, D, generator=g)
    kc = torch.randn(B, Hk, Lc, D, generator=g)
    vc = torch.randn(B, Hk, Lc, D, generator=g)
    kv_len = torch.tensor([640, 411], dtype=torch.int32)
    keep = torch.rand(B, Hk, nb, generator=g) < 0.5
    keep[:, :, 0] = True
    idx = torch.full((B, Hk, nb), -1, dtype=torch.int32)
    cnt = keep.sum(-1).to(torch.int32)
    for b in range(B):
        for h in range(Hk):
            ks = keep[b, h].nonzero().flatten().to(torch.int32)
            idx[b, h, : ks.numel()] = ks
    return q, kc, vc, kv_len, idx, cnt


def _rank_main(rank, world, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, kc, vc, kv_len, idx, cnt = _inputs()
        lo, hi = SH.block_range(kc.shape[2] // 64, rank, world)
        kl = SH.local_kept(KeptBlocks(idx, cnt), lo, hi)
        o, m, l = O.bsa_decode(q, kc[:, :, lo * 64 : hi * 64], vc[:, :, lo * 64 : hi * 64],
                               SH.local_kv_len(kv_len, lo, hi, 64), kl.idx, kl.cnt, 64, return_lse=True)
        ml = torch.stack([m, l], dim=-1)
        ao, am = SH.gather_partials(o.float(), ml.float())
        out = O.decode_combine(ao, am[..., 0], am[..., 1])
        if rank == 0:
            out_q.put(out)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 3])
def test_split_kv_decode_over_gloo_matches_unsplit(world):
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, out_q)) for r in range(world)]
    for p in procs:
        p.start()
    got = out_q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    q, kc, vc, kv_len, idx, cnt = _inputs()
    ref = O.bsa_decode(q, kc, vc, kv_len, idx, cnt, 64)
    torch.testing.assert_close(got, ref.float(), atol=1e-5, rtol=1e-5)


def test_unit_weights_sum_kept_blocks_per_kv_head():
    cnt = torch.tensor([[[1, 2], [3, 4], [5, 6], [7, 8]]], dtype=torch.int32)  # B=1, Hm=4 (q-heads), NB=2
    kept = KeptBlocks(torch.zeros(1, 4, 2, 2, dtype=torch.int32), cnt)
    assert SH.unit_weights(kept, 2).tolist() == [1 + 2 + 3 + 4, 5 + 6 + 7 + 8]
    kv = KeptBlocks(torch.zeros(1, 2, 2, 2, dtype=torch.int32), cnt[:, :2])
    assert SH.unit_weights(kv, 2).tolist() == [3, 7]


def test_qblock_ranges_partition_and_balance():
    nb = 64
    cnt = torch.arange(1, nb + 1, dtype=torch.int32).view(1, 1, nb).expand(1, 4, nb)  # causal-like growth
    kept = KeptBlocks(torch.zeros(1, 4, nb, nb, dtype=torch.int32), cnt.contiguous())
    for world in (1, 2, 3, 8):
        rs = SH.qblock_ranges(kept, world)
        assert rs[0][0] == 0 and rs[-1][1] == nb and all(rs[i][1] == rs[i + 1][0] for i in range(world - 1))
        work = [int(cnt[0, 0, lo:hi].sum()) * 4 for lo, hi in rs]
        assert max(work) <= sum(work) / world + 4 * nb  # within one q-block of the mean
    r = SH.restrict_qblocks(kept, 10, 20)
    assert r.cnt[0, 0, :10].eq(0).all() and r.cnt[0, 0, 20:].eq(0).all()
    assert torch.equal(r.cnt[0, 0, 10:20], cnt[0, 0, 10:20])
