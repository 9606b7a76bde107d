"""Split-KV decode partials merged over peer memory (tasft_peer_combine, and the decode
whose merge kernel exchanges itself, tasft_bsa_decode_peer_fwd).

On one GPU the other rank is emulated by the host: its partial and its flag are written
into this rank's mailbox before the call (no kernel ever waits for another kernel on the
same GPU). The merged output must equal the NCCL path's combine kernel on the same
partials; this rank's own partial must land in the other rank's mailbox with its flag;
a flag that nobody raises must end the wait with TASFT_DEVERR_TIMEOUT. The two-rank test
maps real peer memory over CUDA IPC (two GPUs) and replays the decode step from a CUDA
graph.
"""
from __future__ import annotations

import ctypes as C
import os
import socket

import pytest
import torch

import tasft_b200 as T
from tasft_b200 import _lib as L
from tasft_b200 import masks as M
from tasft_b200 import shards as SH

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _mailbox(world, rows, D):
    nbytes = int(L.lib().tasft_peer_mailbox_bytes(world, rows, D))
    return torch.zeros(nbytes // 4, dtype=torch.int32, device=DEV)


def _flags_bytes(world):
    return ((world + 1) * 4 + 255) // 256 * 256


def _part_off(world, rows, D):
    """Float offset of the partials in a mailbox: call flags (world + 1 words, padded to 256
    bytes), then the row words (2 x world x rows x (D + 2) 8-byte words)."""
    return (_flags_bytes(world) + 2 * world * rows * (D + 2) * 8) // 4


def _words(box, world, rows, D, par, r):
    """Slot [par][r] of the row words, [rows, D + 2] int64 (fp32 bits | epoch << 32)."""
    base = _flags_bytes(world) // 8 + (par * world + r) * rows * (D + 2)
    return box.view(torch.int64)[base: base + rows * (D + 2)].view(rows, D + 2)


def _pack(values, epoch):
    bits = values.contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    return bits | (epoch << 32)


def _slot(box, world, rows, D, par, r):
    foff = _part_off(world, rows, D)
    slab = rows * (D + 2)
    return box.view(torch.float32)[foff + (par * world + r) * slab: foff + (par * world + r + 1) * slab].view(rows, D + 2)


def _call(boxes, rank, po, pm, out, epoch, err, timeout_ns=int(2e8)):
    table = torch.tensor([b.data_ptr() for b in boxes], dtype=torch.int64, device=DEV)
    rows, D = po.shape
    args = L.PeerCombineArgs(part_o=po.data_ptr(), part_ml=pm.data_ptr(), rows=rows, D=D, world=len(boxes), rank=rank,
                             mailboxes=table.data_ptr(), epoch=epoch.data_ptr(), out=out.data_ptr(),
                             dtype=L.dtype_code(out), timeout_ns=timeout_ns, err=err.data_ptr())
    rc = L.lib().tasft_peer_combine(C.byref(args), L.stream_ptr(out.device))
    torch.cuda.synchronize()
    assert rc == 0
    return table


def _partials(rows, D, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    po = torch.randn(rows, D, device=DEV, generator=g)
    pm = torch.stack([torch.randn(rows, device=DEV, generator=g) * 3, torch.rand(rows, device=DEV, generator=g) * 5],
                     -1)
    pm[3, 1] = 0.0  # a rank with nothing kept for this row
    return po, pm


def test_two_ranks_emulated_twice_matches_combine_kernel():
    rows, D, world = 28, 128, 2
    boxes = [_mailbox(world, rows, D), _mailbox(world, rows, D)]
    epoch = torch.zeros(1, dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    for call in (1, 2):
        par = call & 1
        po0, pm0 = _partials(rows, D, 10 * call)
        po1, pm1 = _partials(rows, D, 10 * call + 1)
        # rank 1 (emulated): its partial in our mailbox, then its flag
        _slot(boxes[0], world, rows, D, par, 1).copy_(torch.cat([po1, pm1], -1))
        boxes[0][1] = call
        out = torch.empty(rows, D, dtype=torch.bfloat16, device=DEV)
        _call(boxes, 0, po0, pm0, out, epoch, err)
        assert int(err.item()) == 0 and int(epoch.item()) == call
        ref = T.decode_combine(torch.stack([po0, po1]), torch.stack([pm0, pm1]), torch.bfloat16)
        assert torch.equal(out, ref)
        # our partial and flag reached the other rank's mailbox
        assert torch.equal(_slot(boxes[1], world, rows, D, par, 0), torch.cat([po0, pm0], -1))
        assert int(boxes[1][0].item()) == call


def test_missing_peer_times_out_with_error_bit():
    rows, D, world = 8, 64, 2
    boxes = [_mailbox(world, rows, D), _mailbox(world, rows, D)]
    epoch = torch.zeros(1, dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    po, pm = _partials(rows, D, 3)
    out = torch.empty(rows, D, dtype=torch.bfloat16, device=DEV)
    _call(boxes, 0, po, pm, out, epoch, err, timeout_ns=int(5e7))  # flag of rank 1 never raised
    assert int(err.item()) & L.DEVERR_TIMEOUT


class _Peer:
    """The fields of shards.PeerExchange that bsa_decode_peer reads, over local mailboxes."""

    def __init__(self, boxes, rank, timeout_ns):
        self.table = torch.tensor([b.data_ptr() for b in boxes], dtype=torch.int64, device=DEV)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=DEV)
        self.err = torch.zeros(1, dtype=torch.int32, device=DEV)
        self.world, self.rank, self.timeout_ns = len(boxes), rank, timeout_ns


def _slab_case():
    g = torch.Generator(device=DEV).manual_seed(8)
    B, Hq, Hk, Lc, D = 1, 28, 4, 8192, 128
    q = torch.randn(B, Hq, D, device=DEV, generator=g).bfloat16()
    kc = torch.randn(B, Hk, Lc, D, device=DEV, generator=g).bfloat16()
    vc = torch.randn(B, Hk, Lc, D, device=DEV, generator=g).bfloat16()
    kv_len = torch.full((B,), Lc - 37, dtype=torch.int32, device=DEV)
    nb = Lc // 64
    mask = M.decode_mask(torch.rand(B, Hk, nb, device=DEV, generator=g), (kv_len + 63) // 64, 0.15, nb)
    return q, kc, vc, kv_len, T.KeptBlocks(*M.lists_from_mask(mask)), nb


def test_fused_decode_exchange_emulated_twice():
    """Rank 0 of 2 on one GPU: rank 1's rows (its own slab decoded with partials) and row
    flags are written into rank 0's mailbox by the host; the fused call must agree with the
    NCCL path's combine of the two slabs' partials and with a one-rank decode of the whole
    cache, leave its own rows (tagged with the epoch) in rank 1's mailbox, and advance the
    epoch."""
    q, kc, vc, kv_len, kept, nb = _slab_case()
    B, Hq, D = q.shape
    rows, world, half = B * Hq, 2, nb // 2
    boxes = [_mailbox(world, rows, D), _mailbox(world, rows, D)]
    peer = _Peer(boxes, 0, int(2e8))
    ws = T.DecodeWorkspace(B, Hq, 4, D, 64, DEV)
    slabs = [(kc[:, :, :half * 64].contiguous(), vc[:, :, :half * 64].contiguous(), 0),
             (kc[:, :, half * 64:].contiguous(), vc[:, :, half * 64:].contiguous(), half)]
    parts = []
    for k_s, v_s, lo in slabs:
        kl = SH.local_kept(kept, lo, lo + half)
        po = torch.empty(B, Hq, D, device=DEV)
        pm = torch.empty(B, Hq, 2, device=DEV)
        T.bsa_decode(q, k_s, v_s, kv_len, kl, 64, workspace=ws, partials=(po, pm), kv_offset=lo * 64)
        parts.append((po.view(rows, D), pm.view(rows, 2), kl))
    full = T.bsa_decode(q, kc, vc, kv_len, kept, 64)
    for call in (1, 2):
        par = call & 1
        _words(boxes[0], world, rows, D, par, 1).copy_(_pack(torch.cat([parts[1][0], parts[1][1]], -1), call))
        out = torch.empty(B, Hq, D, dtype=torch.bfloat16, device=DEV)
        T.decode.bsa_decode_peer(q, slabs[0][0], slabs[0][1], kv_len, parts[0][2], peer, 64, workspace=ws, out=out)
        torch.cuda.synchronize()
        assert int(peer.err.item()) == 0 and int(peer.epoch.item()) == call
        ref = T.decode_combine(torch.stack([parts[0][0], parts[1][0]]).view(2, B, Hq, D),
                               torch.stack([parts[0][1], parts[1][1]]).view(2, B, Hq, 2), torch.bfloat16)
        # this rank's rows come from the separate merge kernel, the reference partials from the
        # in-kernel merge (16 splits): same maths, fp32 summation orders differ
        assert (out.float() - ref.float()).abs().max().item() <= 1e-2
        assert (out.float() - full.float()).abs().max().item() <= 2e-2
        pushed = _words(boxes[1], world, rows, D, par, 0)
        assert bool(((pushed >> 32) == call).all())  # every word carries this call's epoch
        vals = (pushed & 0xFFFFFFFF).to(torch.int32).view(torch.float32)
        own = torch.cat([parts[0][0], parts[0][1]], -1)
        assert torch.allclose(vals, own, rtol=1e-4, atol=1e-5)


def test_fused_decode_exchange_missing_peer_times_out():
    q, kc, vc, kv_len, kept, nb = _slab_case()
    B, Hq, D = q.shape
    boxes = [_mailbox(2, B * Hq, D), _mailbox(2, B * Hq, D)]
    peer = _Peer(boxes, 0, int(5e7))  # rank 1's words never arrive
    ws = T.DecodeWorkspace(B, Hq, 4, D, 64, DEV)
    half = nb // 2
    out = torch.empty(B, Hq, D, dtype=torch.bfloat16, device=DEV)
    T.decode.bsa_decode_peer(q, kc[:, :, :half * 64].contiguous(), vc[:, :, :half * 64].contiguous(), kv_len,
                             SH.local_kept(kept, 0, half), peer, 64, workspace=ws, out=out)
    torch.cuda.synchronize()
    assert int(peer.err.item()) & L.DEVERR_TIMEOUT


def _inputs(dev):
    g = torch.Generator(device=dev).manual_seed(5)
    B, Hq, Hk, Lc, D = 1, 28, 4, 32768, 128
    q = torch.randn(B, Hq, D, device=dev, generator=g).bfloat16()
    kc = torch.randn(B, Hk, Lc, D, device=dev, generator=g).bfloat16()
    vc = torch.randn(B, Hk, Lc, D, device=dev, generator=g).bfloat16()
    kv_len = torch.full((B,), Lc - 100, dtype=torch.int32, device=dev)
    nb = Lc // 64
    idx, cnt = M.lists_from_mask(M.decode_mask(torch.rand(B, Hk, nb, device=dev, generator=g),
                                               (kv_len + 63) // 64, 0.1, nb))
    return q, kc, vc, kv_len, T.KeptBlocks(idx, cnt)


def _rank_peer(rank, world, port, res):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist  # noqa: PLC0415

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    dec = None
    try:
        q, kc, vc, kv_len, kept = _inputs(dev)
        lo, hi = SH.block_range(kc.shape[2] // 64, rank, world)
        dec = SH.SplitKVDecoder(q.shape[0], q.shape[1], kc.shape[1], q.shape[2], dev, exchange="peer")
        kl, vl = kc[:, :, lo * 64: hi * 64].contiguous(), vc[:, :, lo * 64: hi * 64].contiguous()
        loc = dec.local(kept, lo, hi - lo)
        ref = T.bsa_decode(q, kc, vc, kv_len, kept, 64)
        errs = [(dec(q, kl, vl, kv_len, kept, lo, local=loc).float() - ref.float()).abs().max().item()
                for _ in range(3)]
        # the same step replayed from a CUDA graph (no host work, no NCCL)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            dec(q, kl, vl, kv_len, kept, lo, local=loc)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = dec(q, kl, vl, kv_len, kept, lo, local=loc)
        for _ in range(5):
            graph.replay()
            torch.cuda.synchronize(dev)
            errs.append((out.float() - ref.float()).abs().max().item())
        res.put((rank, (max(errs), int(dec.peer.err.item()))))
    finally:
        if dec is not None and dec.peer is not None:
            dist.barrier()
            dec.peer.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_exchange_two_ranks_and_graph_replay():
    import torch.multiprocessing as mp  # noqa: PLC0415

    ctx = mp.get_context("spawn")
    res = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_rank_peer, args=(r, 2, port, res)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(res.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, (err, dev_err) in out.items():
        assert dev_err == 0, rank
        assert err <= 2e-2, rank
