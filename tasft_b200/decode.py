"""Block-sparse decode (one query token per sequence) and the split-KV combine.

New capability: the reference has no sparse decode (``tasft/inference/vllm_patch.py:189-196``
hands decode to vLLM's dense forward). Queries of the q-heads of one GQA group attend
over the kept KV blocks of their kv-head, bounded by ``kv_len``.
"""
from __future__ import annotations

import math

import torch

from tasft_b200 import _lib as L
from tasft_b200.exceptions import KernelError
from tasft_b200.types import KeptBlocks


class DecodeWorkspace:
    """Caller-owned split-KV scratch (partials + zeroed tickets), reused across calls."""

    def __init__(self, B: int, Hq: int, Hk: int, D: int, max_splits: int, device) -> None:
        self.max_splits = max_splits
        self.bytes = int(L.lib().tasft_decode_workspace_size(B, Hq, Hk, D, max_splits))
        self.buf = torch.zeros(self.bytes, dtype=torch.uint8, device=device)
        self.key = (B, Hq, Hk, D)


def max_splits_for(dtype: torch.dtype, block: int, D: int, group: int) -> int:
    """Most splits the decode takes: 64 on the tensor-core path (bf16/f16, block 64, D 64 or
    128, group <= 8), whose wide splits merge in a separate kernel; 16 elsewhere (the last
    split of a unit merges all partials with one warp)."""
    mma = dtype in (torch.bfloat16, torch.float16) and block == 64 and D in (64, 128) and group <= 8
    return 64 if mma else 16


def default_splits(B: int, Hk: int, mean_kept: float, sms: int = 148, most: int = 16) -> int:
    """Splits per (sequence, kv-head) for the persistent decode kernel.

    As many splits as keep the work items within the resident CTA slots (6 per SM), so
    each CTA owns one item and no dynamic claiming is needed; at least two kept blocks
    per split, at most ``most`` (``max_splits_for``).
    """
    units = max(1, B * Hk)
    fit = max(1, (6 * sms) // units)
    by_size = max(1, int(mean_kept // 2))
    return max(1, min(fit, by_size, most))


def _decode_args(q, k, v, kv_len, kept: KeptBlocks, block, L_logical, Hk, num_splits, workspace, out, partials,
                 err, kv_offset: int = 0):
    """The ``tasft_decode_args`` both decode entry points share (``k``/``v`` are the caches,
    or the page pools for the paged call), with the split count and workspace resolved."""
    B, Hq, D = q.shape
    idx = kept.idx.contiguous()
    cnt = kept.cnt.contiguous()
    ws_ptr, ws_bytes = None, 0
    if num_splits != 1:
        most = max_splits_for(q.dtype, block, D, Hq // Hk)
        if workspace is None:
            ms = num_splits if num_splits > 0 else most
            workspace = DecodeWorkspace(B, Hq, Hk, D, ms, q.device)
        ws_ptr, ws_bytes = workspace.buf.data_ptr(), workspace.bytes
        if num_splits <= 0:
            num_splits = min(workspace.max_splits, default_splits(B, Hk, idx.shape[-1] / 4, most=most))
    args = L.DecodeArgs(
        q=q.data_ptr(), k_cache=k.data_ptr(), v_cache=v.data_ptr(), out=L.ptr(out),
        q_stride=L.strides3(q), k_stride=L.strides4(k), v_stride=L.strides4(v),
        o_stride=L.strides3(out) if out is not None else L.I64x3(0, 0, 0),
        B=B, Hq=Hq, Hk=Hk, L=L_logical, D=D, block=block, dtype=L.dtype_code(q), scale=1.0 / math.sqrt(D),
        kv_len=kv_len.data_ptr(), kept_idx=idx.data_ptr(), kept_cnt=cnt.data_ptr(), nb_max=idx.shape[-1],
        num_splits=num_splits, part_o=L.ptr(partials[0]) if partials else None,
        part_ml=L.ptr(partials[1]) if partials else None, workspace=ws_ptr, workspace_bytes=ws_bytes,
        err=L.ptr(err), kv_offset=int(kv_offset),
    )
    # keep the tensors the struct points into alive until the call returns
    return args, num_splits, (idx, cnt, workspace)


def bsa_decode(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    kv_len: torch.Tensor,
    kept: KeptBlocks,
    block: int = 64,
    *,
    num_splits: int = 0,
    workspace: DecodeWorkspace | None = None,
    out: torch.Tensor | None = None,
    partials: tuple[torch.Tensor, torch.Tensor] | None = None,
    err: torch.Tensor | None = None,
    kv_offset: int = 0,
) -> torch.Tensor | None:
    """Decode attention: q ``[B,Hq,D]``, caches ``[B,Hk,L,D]``, ``kv_len`` int32 ``[B]``,
    ``kept`` lists ``[B,Hk,NBmax]`` / ``[B,Hk]``. Returns ``[B,Hq,D]`` (``out``) and, when
    ``partials=(o [B,Hq,D] f32, ml [B,Hq,2] f32)`` is given, also writes the normalised
    output with its (max, sum) for a cross-GPU combine. ``kv_offset``: the cache is the slab
    of a longer sequence starting at that token (one rank's share of a split cache); the
    valid rows are ``clamp(kv_len - kv_offset, 0, L)``, computed in the kernel."""
    L.require_cuda(q, k_cache, v_cache, kv_len)
    if q.ndim != 3 or k_cache.ndim != 4 or k_cache.shape != v_cache.shape:
        raise KernelError("decode expects q [B,Hq,D] and caches [B,Hk,L,D]",
                          context={"q": list(q.shape), "k": list(k_cache.shape), "v": list(v_cache.shape)})
    B, Hq, D = q.shape
    Hk, Lc = k_cache.shape[1], k_cache.shape[2]
    if Hq % Hk or k_cache.shape[0] != B or k_cache.shape[3] != D:
        raise KernelError("decode shape mismatch", context={"q": list(q.shape), "k": list(k_cache.shape)})
    q = q.contiguous()
    k_cache = k_cache.contiguous()
    v_cache = v_cache.contiguous()
    if out is None and partials is None:
        out = torch.empty_like(q)
    args, num_splits, _keep = _decode_args(q, k_cache, v_cache, kv_len, kept, block, Lc, Hk, num_splits, workspace,
                                           out, partials, err, kv_offset)
    L.check(L.lib().tasft_bsa_decode_fwd(args, L.stream_ptr(q.device)), "tasft_bsa_decode_fwd",
            shape=[B, Hq, Hk, Lc, D], splits=num_splits)
    return out


def bsa_decode_peer(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    kv_len: torch.Tensor,
    kept: KeptBlocks,
    peer,
    block: int = 64,
    *,
    workspace: DecodeWorkspace,
    out: torch.Tensor,
    num_splits: int = 0,
    kv_offset: int = 0,
) -> torch.Tensor:
    """One rank's share of a split-KV decode with the cross-GPU merge fused into its merge
    kernel (``tasft_bsa_decode_peer_fwd``): decodes this rank's slab (``kv_offset`` as in
    :func:`bsa_decode`), pushes the rank's ``(o, m, l)`` rows into every rank's mailbox of
    ``peer`` (a :class:`tasft_b200.shards.PeerExchange`) and writes the merge of all ranks
    into ``out``. Every rank makes the same calls; a wait that runs out sets ``peer.err``."""
    L.require_cuda(q, k_cache, v_cache, kv_len)
    B, Hq, D = q.shape
    Hk, Lc = k_cache.shape[1], k_cache.shape[2]
    q = q.contiguous()
    args, num_splits, _keep = _decode_args(q, k_cache.contiguous(), v_cache.contiguous(), kv_len, kept, block, Lc, Hk,
                                           num_splits, workspace, out, None, peer.err, kv_offset)
    pa = L.DecodePeerArgs(mailboxes=peer.table.data_ptr(), epoch=peer.epoch.data_ptr(), world=peer.world,
                          rank=peer.rank, timeout_ns=peer.timeout_ns)
    L.check(L.lib().tasft_bsa_decode_peer_fwd(args, pa, L.stream_ptr(q.device)), "tasft_bsa_decode_peer_fwd",
            shape=[B, Hq, Hk, Lc, D], splits=num_splits)
    return out


def bsa_decode_paged(
    q: torch.Tensor,
    k_pages: torch.Tensor,
    v_pages: torch.Tensor,
    block_table: torch.Tensor,
    kv_len: torch.Tensor,
    kept: KeptBlocks,
    block: int = 64,
    *,
    num_splits: int = 0,
    workspace: DecodeWorkspace | None = None,
    out: torch.Tensor | None = None,
    partials: tuple[torch.Tensor, torch.Tensor] | None = None,
    err: torch.Tensor | None = None,
) -> torch.Tensor | None:
    """Sparse decode over a paged KV cache (vLLM's flash layout).

    ``k_pages`` / ``v_pages`` ``[num_pages, page_size, Hk, D]``; ``block_table``
    ``[B, max_pages]`` int32 maps logical page ``t // page_size`` of sequence b to a
    physical page; ``kept`` lists are in logical 64-token blocks, as for ``bsa_decode``.
    The reference's vLLM backend decodes paged caches densely
    (``tasft/inference/vllm_patch.py:189-196``); this is the sparse call for that site.
    """
    L.require_cuda(q, k_pages, v_pages, block_table, kv_len)
    if q.ndim != 3 or k_pages.ndim != 4 or k_pages.shape != v_pages.shape or block_table.ndim != 2:
        raise KernelError("paged decode expects q [B,Hq,D], pages [P,page,Hk,D], block_table [B,max_pages]",
                          context={"q": list(q.shape), "k": list(k_pages.shape), "table": list(block_table.shape)})
    B, Hq, D = q.shape
    num_pages, page_size, Hk, _ = k_pages.shape
    max_pages = block_table.shape[1]
    if Hq % Hk or k_pages.shape[3] != D or block_table.shape[0] != B:
        raise KernelError("paged decode shape mismatch", context={"q": list(q.shape), "k": list(k_pages.shape)})
    q = q.contiguous()
    table = block_table.to(torch.int32).contiguous()
    if out is None and partials is None:
        out = torch.empty_like(q)
    base, num_splits, _keep = _decode_args(q, k_pages, v_pages, kv_len, kept, block, max_pages * page_size, Hk,
                                           num_splits, workspace, out, partials, err)
    args = L.PagedDecodeArgs(base=base, block_table=table.data_ptr(), max_pages=max_pages, page_size=page_size,
                             num_pages=num_pages)
    L.check(L.lib().tasft_bsa_decode_paged_fwd(args, L.stream_ptr(q.device)), "tasft_bsa_decode_paged_fwd",
            shape=[B, Hq, Hk, num_pages, page_size, D], splits=num_splits)
    return out


def decode_combine(part_o: torch.Tensor, part_ml: torch.Tensor, out_dtype=torch.bfloat16) -> torch.Tensor:
    """Merge G partials ``o [G,B,Hq,D]`` / ``ml [G,B,Hq,2]`` (e.g. all-gathered from G GPUs)."""
    L.require_cuda(part_o, part_ml)
    G = part_o.shape[0]
    D = part_o.shape[-1]
    rows = part_o[0].numel() // D
    out = torch.empty(part_o.shape[1:], dtype=out_dtype, device=part_o.device)
    po = part_o.float().contiguous()
    pm = part_ml.float().contiguous()
    args = L.CombineArgs(part_o=po.data_ptr(), part_ml=pm.data_ptr(), G=G, rows=rows, D=D, out=out.data_ptr(),
                         dtype=L.dtype_code(out))
    L.check(L.lib().tasft_bsa_decode_combine(args, L.stream_ptr(po.device)), "tasft_bsa_decode_combine")
    return out


__all__ = ["DecodeWorkspace", "bsa_decode", "bsa_decode_paged", "bsa_decode_peer", "decode_combine", "default_splits"]
