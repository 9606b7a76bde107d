"""Multi-GPU sharding of the sparse-attention path: one process per GPU, ``torch.distributed``.

Prefill, the gate and batched decode split into independent units (sequence, kv-head):
every unit reads only its own Q/K/V slice, so ranks share nothing and exchange nothing.
``assign_units`` balances units over ranks by their kept-block counts (longest first).

Long-context decode (one sequence, few kv-heads, a KV cache too large or too slow for one
GPU) is the one path with an exchange. Rank r holds a contiguous range of KV blocks
(``block_range``) of every kv-head. It decodes over the kept blocks that fall in its range
and writes, per q-head, its normalised output with (max, sum). Then the partials of all
ranks are all-gathered (NCCL over NVLink; 4*(D+2) bytes per q-head per rank) and merged
locally by the log-sum-exp combine kernel. The reference has no sparse decode at all; the
per-rank kernel follows the single-GPU decode's contract.
"""
from __future__ import annotations

import heapq

import torch

from tasft_b200.types import KeptBlocks


def assign_units(weights, world: int) -> list[list[int]]:
    """Longest-processing-time assignment of unit ids to ``world`` ranks.

    ``weights[i]`` is unit i's work (its kept-block count). Returns one ascending id list
    per rank; ties go to the lower rank, so every rank computes the same answer.
    """
    if world <= 0:
        raise ValueError("world must be positive")
    w = [float(x) for x in (weights.tolist() if isinstance(weights, torch.Tensor) else weights)]
    order = sorted(range(len(w)), key=lambda i: (-w[i], i))
    heap = [(0.0, r) for r in range(world)]
    out: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + w[i], r))
    return [sorted(x) for x in out]


def unit_weights(kept: KeptBlocks, hk: int) -> torch.Tensor:
    """Kept blocks per prefill unit (sequence, kv-head), ``[B * Hk]`` in unit order
    ``b * Hk + hk``: the work measure ``assign_units`` balances."""
    cnt = kept.cnt  # [B, Hm, NB]
    B, hm = cnt.shape[0], cnt.shape[1]
    return cnt.reshape(B, hk, hm // hk, -1).sum(dim=(2, 3)).reshape(-1)


def unit_slices(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kept: KeptBlocks, units):
    """The Q/K/V slices and kept lists of the (sequence, kv-head) units ``units`` (ids
    ``b * Hk + hk``) as one batch: ``q [U, grp, S, D]``, ``k, v [U, 1, S, D]`` and lists
    ``[U, mg, NB, NB]`` (mg = 1 for kv-head lists, grp for per-q-head lists)."""
    Hk = k.shape[1]
    grp = q.shape[1] // Hk
    hm = kept.idx.shape[1]
    mg = hm // Hk
    ids = torch.as_tensor(list(units), dtype=torch.long, device=q.device)
    b, h = ids // Hk, ids % Hk
    hq = (h[:, None] * grp + torch.arange(grp, device=q.device)[None, :])
    hl = (h[:, None] * mg + torch.arange(mg, device=q.device)[None, :])
    return (q[b[:, None], hq], k[b, h].unsqueeze(1), v[b, h].unsqueeze(1),
            KeptBlocks(kept.idx[b[:, None], hl].contiguous(), kept.cnt[b[:, None], hl].contiguous()))


def prefill_units(kern, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kept: KeptBlocks, units,
                  causal: bool = True) -> torch.Tensor:
    """Prefill of the (sequence, kv-head) units ``units`` only (ids ``b * Hk + hk``), as
    one call over a batch of units: returns ``[len(units), Hq/Hk, S, D]``, the q-heads of
    each unit's group. A rank of a sharded prefill passes the units ``assign_units`` gave
    it; the tensors may be the full batch or just those units' slices gathered by the
    caller (then ``units`` are indices into that smaller batch)."""
    qu, ku, vu, ku_kept = unit_slices(q, k, v, kept, units)
    return kern.forward(qu, ku, vu, ku_kept, causal=causal)


def scatter_units(out: torch.Tensor, parts: torch.Tensor, units, Hk: int) -> None:
    """Write unit outputs ``[U, grp, S, D]`` back into the full ``[B, Hq, S, D]`` tensor."""
    grp = out.shape[1] // Hk
    for i, u in enumerate(units):
        b, h = divmod(int(u), Hk)
        out[b, h * grp:(h + 1) * grp] = parts[i]


def qblock_ranges(kept: KeptBlocks, world: int) -> list[tuple[int, int]]:
    """Contiguous q-block ranges ``[lo, hi)`` with about equal kept work each, for a
    prefill with too few (sequence, kv-head) units to go around (one long sequence): the
    boundaries cut the cumulative kept-block count summed over batch and heads."""
    per_q = kept.cnt.sum(dim=tuple(range(kept.cnt.ndim - 1))).double().cpu()  # [NB], host-side planning
    cum = torch.cumsum(per_q, 0)
    total = float(cum[-1]) if cum.numel() else 0.0
    nb = per_q.numel()
    cuts = [0]
    for r in range(1, world):
        c = int(torch.searchsorted(cum, torch.tensor(total * r / world, dtype=cum.dtype)).item()) + 1
        cuts.append(min(max(c, cuts[-1]), nb))
    cuts.append(nb)
    return [(cuts[r], cuts[r + 1]) for r in range(world)]


def restrict_qblocks(kept: KeptBlocks, lo: int, hi: int) -> KeptBlocks:
    """The prefill lists with every q-block outside ``[lo, hi)`` emptied: a prefill on them
    computes only those q-blocks (the other rows come out as zeros)."""
    nb = kept.cnt.shape[-1]
    inside = (torch.arange(nb, device=kept.cnt.device) >= lo) & (torch.arange(nb, device=kept.cnt.device) < hi)
    return KeptBlocks(kept.idx, torch.where(inside, kept.cnt, torch.zeros_like(kept.cnt)).contiguous())


def block_range(nb: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous KV-block range ``[lo, hi)`` of ``rank`` when ``nb`` blocks split over ``world``."""
    base, extra = divmod(nb, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def local_kept(kept: KeptBlocks, lo: int, hi: int) -> KeptBlocks:
    """Decode lists ``[B, Hk, NBmax]`` restricted to blocks in ``[lo, hi)`` and rebased to
    the local cache slab (block ``lo`` becomes 0), ascending order kept, padded with -1."""
    idx, cnt = kept.idx, kept.cnt
    pos = torch.arange(idx.shape[-1], device=idx.device)
    inside = (pos < cnt.unsqueeze(-1)) & (idx >= lo) & (idx < hi)
    big = torch.iinfo(torch.int32).max
    key = torch.where(inside, idx - lo, torch.full_like(idx, big))
    key = torch.sort(key, dim=-1).values  # lists are ascending, so this only compacts
    key = torch.where(key == big, torch.full_like(key, -1), key)
    return KeptBlocks(key.to(torch.int32).contiguous(), inside.sum(-1).to(torch.int32).contiguous())


def local_kv_len(kv_len: torch.Tensor, lo: int, hi: int, block: int) -> torch.Tensor:
    """Valid tokens of the local slab ``[lo*block, hi*block)`` for each sequence."""
    return (kv_len.to(torch.int64) - lo * block).clamp(0, (hi - lo) * block).to(torch.int32)


def gather_partials(part_o: torch.Tensor, part_ml: torch.Tensor, group=None):
    """All-gather ``o [B,Hq,D]`` and ``ml [B,Hq,2]`` (fp32) from every rank of ``group``:
    returns ``[G,B,Hq,D]`` and ``[G,B,Hq,2]`` in rank order. Both travel in ONE collective
    (a flat ``[o | ml]`` buffer per rank): the exchange is a few KB, so its cost is the
    collective's latency, paid once."""
    import torch.distributed as dist  # noqa: PLC0415

    g = dist.get_world_size(group)
    no, nm = part_o.numel(), part_ml.numel()
    flat = torch.cat([part_o.reshape(-1), part_ml.reshape(-1)])
    out = torch.empty(g * (no + nm), dtype=flat.dtype, device=flat.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, flat, group=group)
    else:  # gloo takes the list form
        dist.all_gather(list(out.view(g, no + nm).unbind(0)), flat, group=group)
    rows = out.view(g, no + nm)
    return rows[:, :no].reshape(g, *part_o.shape), rows[:, no:].reshape(g, *part_ml.shape)


def long_context_decode(
    q: torch.Tensor,
    k_local: torch.Tensor,
    v_local: torch.Tensor,
    kv_len: torch.Tensor,
    kept: KeptBlocks,
    block_lo: int,
    group=None,
    block: int = 64,
    num_splits: int = 0,
) -> torch.Tensor:
    """Sparse decode of a KV cache split by position over the ranks of ``group``.

    ``k_local``/``v_local`` ``[B,Hk,Lloc,D]`` hold global blocks ``[block_lo, block_lo +
    Lloc/block)``; ``kept`` and ``kv_len`` are the global lists and lengths (the same on
    every rank). Every rank returns the full ``[B,Hq,D]`` result.
    """
    from tasft_b200.decode import bsa_decode, decode_combine  # noqa: PLC0415

    B, Hq, D = q.shape
    nloc = k_local.shape[2] // block
    lo, hi = block_lo, block_lo + nloc
    kl = local_kept(kept, lo, hi)
    po = torch.empty(B, Hq, D, dtype=torch.float32, device=q.device)
    pm = torch.empty(B, Hq, 2, dtype=torch.float32, device=q.device)
    bsa_decode(q, k_local, v_local, kv_len, kl, block, num_splits=num_splits, partials=(po, pm),
               kv_offset=lo * block)
    ao, am = gather_partials(po, pm, group)
    return decode_combine(ao, am, q.dtype)


class PeerExchange:
    """Mailboxes for exchanging split-KV decode partials across the ranks of ``group`` over
    peer memory: every rank's mailbox is mapped into every other rank through CUDA IPC.
    ``bsa_decode_peer`` uses them from inside the decode's merge kernel (each rank stores its
    rows into every mailbox and merges what its own holds); calling the object runs the
    stand-alone merge kernel (``tasft_peer_combine``) on given partials. No NCCL call per
    step, so the step can be captured in a CUDA graph. Set up once (collective: every rank
    constructs it in the same order); ``close()`` unmaps and frees."""

    def __init__(self, rows: int, D: int, device, group=None, timeout_s: float = 1.0) -> None:
        import ctypes as C  # noqa: PLC0415

        import torch.distributed as dist  # noqa: PLC0415

        from tasft_b200 import _lib as L  # noqa: PLC0415

        self._L, self._C = L, C
        lib = L.lib()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.rows, self.D, self.device = rows, D, torch.device(device)
        self.timeout_ns = int(timeout_s * 1e9)
        nbytes = int(lib.tasft_peer_mailbox_bytes(self.world, rows, D))
        box = C.c_void_p()
        L.check(lib.tasft_peer_alloc(nbytes, C.byref(box)), "tasft_peer_alloc")
        self._own = box.value
        h = C.create_string_buffer(64)
        L.check(lib.tasft_ipc_handle(self._own, h), "tasft_ipc_handle")
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(h.raw), group=group)
        self._opened = []
        ptrs = []
        for r, hr in enumerate(handles):
            if r == self.rank:
                ptrs.append(self._own)
                continue
            p = C.c_void_p()
            L.check(lib.tasft_ipc_open(C.c_char_p(hr), C.byref(p)), "tasft_ipc_open", peer=r)
            self._opened.append(p.value)
            ptrs.append(p.value)
        self.table = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)

    def __call__(self, part_o: torch.Tensor, part_ml: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        L = self._L
        args = L.PeerCombineArgs(
            part_o=part_o.data_ptr(), part_ml=part_ml.data_ptr(), rows=self.rows, D=self.D, world=self.world,
            rank=self.rank, mailboxes=self.table.data_ptr(), epoch=self.epoch.data_ptr(), out=out.data_ptr(),
            dtype=L.dtype_code(out), timeout_ns=self.timeout_ns, err=self.err.data_ptr(),
        )
        L.check(L.lib().tasft_peer_combine(args, L.stream_ptr(out.device)), "tasft_peer_combine")
        return out

    def close(self) -> None:
        lib = self._L.lib()
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            lib.tasft_ipc_close(p)
        self._opened = []
        if self._own:
            lib.tasft_peer_free(self._own)
            self._own = None


class SplitKVDecoder:
    """``long_context_decode`` with its buffers kept across calls (workspace, partials, the
    gather buffer), for a serving loop that decodes one token per step. ``local`` lets the
    caller pass the rank's rebased kept lists when they did not change since the last step."""

    def __init__(self, B: int, Hq: int, Hk: int, D: int, device, group=None, block: int = 64,
                 num_splits: int = 0, exchange: str = "nccl", out_dtype=torch.bfloat16, fused: bool = True) -> None:
        import torch.distributed as dist  # noqa: PLC0415

        from tasft_b200.decode import DecodeWorkspace  # noqa: PLC0415

        if exchange not in ("nccl", "peer"):
            raise ValueError(f"exchange must be 'nccl' or 'peer', got {exchange!r}")
        self.group, self.block, self.num_splits = group, block, num_splits
        # "peer" + fused: the exchange runs inside the decode's merge kernel
        # (tasft_bsa_decode_peer_fwd) where that kernel applies (bf16/f16, block 64, D 64/128,
        # up to 8 q-heads per kv-head); otherwise decode, then the separate merge kernel
        from tasft_b200.decode import max_splits_for  # noqa: PLC0415

        self.fused = fused and exchange == "peer" and max_splits_for(out_dtype, block, D, Hq // Hk) == 64
        self.world = dist.get_world_size(group)
        self.nccl = dist.get_backend(group) == "nccl"
        # "peer": partials merged over peer memory by one kernel (graph-capturable step)
        self.peer = PeerExchange(B * Hq, D, device, group) if exchange == "peer" else None
        self.out = torch.empty(B, Hq, D, dtype=out_dtype, device=device) if self.peer is not None else None
        self.ws = DecodeWorkspace(B, Hq, Hk, D, max(num_splits, 64), device)
        self.no, self.nm = B * Hq * D, B * Hq * 2
        self.flat = torch.empty(self.no + self.nm, dtype=torch.float32, device=device)
        self.po = self.flat[: self.no].view(B, Hq, D)
        self.pm = self.flat[self.no:].view(B, Hq, 2)
        self.gathered = torch.empty(self.world * (self.no + self.nm), dtype=torch.float32, device=device)
        self.shape = (B, Hq, D)

    def local(self, kept: KeptBlocks, block_lo: int, nloc: int) -> KeptBlocks:
        return local_kept(kept, block_lo, block_lo + nloc)

    def __call__(self, q, k_local, v_local, kv_len, kept: KeptBlocks, block_lo: int,
                 local: KeptBlocks | None = None) -> torch.Tensor:
        import torch.distributed as dist  # noqa: PLC0415

        from tasft_b200.decode import bsa_decode, bsa_decode_peer, decode_combine  # noqa: PLC0415

        nloc = k_local.shape[2] // self.block
        kl = local if local is not None else local_kept(kept, block_lo, block_lo + nloc)
        if self.peer is not None and self.fused:
            # the decode's own merge kernel pushes this rank's rows to every rank and merges
            return bsa_decode_peer(q, k_local, v_local, kv_len, kl, self.peer, self.block, workspace=self.ws,
                                   out=self.out, num_splits=self.num_splits, kv_offset=block_lo * self.block)
        # the slab's valid length comes from kv_len and the slab offset inside the kernel (no
        # per-step tensor ops)
        bsa_decode(q, k_local, v_local, kv_len, kl, self.block, num_splits=self.num_splits, workspace=self.ws,
                   partials=(self.po, self.pm), kv_offset=block_lo * self.block)
        if self.peer is not None:
            return self.peer(self.po, self.pm, self.out)
        if self.nccl:
            dist.all_gather_into_tensor(self.gathered, self.flat, group=self.group)
        else:
            dist.all_gather(list(self.gathered.view(self.world, -1).unbind(0)), self.flat, group=self.group)
        rows = self.gathered.view(self.world, self.no + self.nm)
        return decode_combine(rows[:, : self.no].view(self.world, *self.shape),
                              rows[:, self.no:].view(self.world, self.shape[0], self.shape[1], 2), q.dtype)


__all__ = ["assign_units", "block_range", "gather_partials", "local_kept", "local_kv_len", "long_context_decode",
           "prefill_units", "qblock_ranges", "restrict_qblocks", "scatter_units", "unit_slices", "unit_weights",
           "PeerExchange", "SplitKVDecoder"]
