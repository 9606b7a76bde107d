"""Benchmark mask rules (workload generation, not reference behaviour).

The reference derives masks as ``soft >= tau`` (``tasft/modules/attn_gate.py:475``). With
random-init gates the scores cluster at 0.5, so a fixed tau gives an uncontrolled
sparsity. The benchmark therefore keeps a fixed fraction of blocks per row, chosen by
the gate's fp32 scores. Every such mask is expressible as ``soft >= tau_row`` for a
per-row threshold, so the reference API accepts it unchanged. All functions are plain
torch ops and run on any device; ties go to the lower block index (stable sort).
"""
from __future__ import annotations

import torch


def _rank_desc(scores: torch.Tensor) -> torch.Tensor:
    """0-based rank of each entry along the last dim, highest score first, stable."""
    order = torch.sort(scores, dim=-1, descending=True, stable=True).indices
    rank = torch.empty_like(order)
    rank.scatter_(-1, order, torch.arange(scores.shape[-1], device=scores.device).expand_as(order))
    return rank


def prefill_mask(scores: torch.Tensor, density: float) -> torch.Tensor:
    """Causal rule for the Llama/Qwen prefill configs.

    Row i keeps blocks 0 and i plus the top-scored of 1..i-1, ``max(2, round(d (i+1)))``
    in total (row 0 keeps block 0). ``scores`` ``[..., NB, NB]`` fp32.
    """
    nb = scores.shape[-1]
    dev = scores.device
    i = torch.arange(nb, device=dev).view(nb, 1)
    j = torch.arange(nb, device=dev).view(1, nb)
    cand = (j >= 1) & (j < i)
    s = torch.where(cand, scores.float(), torch.full_like(scores.float(), float("-inf")))
    rank = _rank_desc(s)
    total = torch.clamp(torch.round(density * (i + 1).float()), min=2).long()
    total = torch.minimum(total, i + 1)
    extra = (total - 2).clamp(min=0)
    keep = (j == 0) | (j == i) | (cand & (rank < extra))
    return keep & (j <= i)


def diag_topk_mask(scores: torch.Tensor, density: float) -> torch.Tensor:
    """CPU-config rule: row i keeps block i plus the top ``round(d (i+1)) - 1`` of 0..i-1."""
    nb = scores.shape[-1]
    dev = scores.device
    i = torch.arange(nb, device=dev).view(nb, 1)
    j = torch.arange(nb, device=dev).view(1, nb)
    cand = j < i
    s = torch.where(cand, scores.float(), torch.full_like(scores.float(), float("-inf")))
    rank = _rank_desc(s)
    extra = (torch.round(density * (i + 1).float()).long() - 1).clamp(min=0)
    return (j == i) | (cand & (rank < extra))


def decode_mask(scores: torch.Tensor, nb_valid: torch.Tensor, density: float, nb_total: int) -> torch.Tensor:
    """Decode rule: per (sequence, kv-head) keep the first block, the last (partial) block
    and the top-scored others, ``round(d NB)`` in total. ``scores`` ``[B, Hk, NB]``,
    ``nb_valid`` ``[B]`` blocks holding valid tokens."""
    B, H, nb = scores.shape
    dev = scores.device
    j = torch.arange(nb, device=dev).view(1, 1, nb)
    last = (nb_valid.view(B, 1, 1) - 1)
    valid = j <= last
    cand = valid & (j > 0) & (j < last)
    s = torch.where(cand, scores.float(), torch.full_like(scores.float(), float("-inf")))
    rank = _rank_desc(s)
    total = max(2, int(round(density * nb_total)))
    keep = (j == 0) | (j == last) | (cand & (rank < total - 2))
    return keep & valid


def group_max(scores: torch.Tensor, hk: int) -> torch.Tensor:
    """Aggregate q-head scores ``[B, Hq, ...]`` to kv-heads by max over each GQA group."""
    B, Hq = scores.shape[:2]
    return scores.view(B, hk, Hq // hk, *scores.shape[2:]).amax(dim=2)


def lists_from_mask(mask: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Ascending kept indices (-1 padded) and counts along the last dim (torch ops)."""
    nb = mask.shape[-1]
    ar = torch.arange(nb, device=mask.device, dtype=torch.int64).expand_as(mask)
    key = torch.where(mask, ar, ar + nb)
    srt = key.sort(dim=-1).values
    idx = torch.where(srt < nb, srt, torch.full_like(srt, -1)).to(torch.int32)
    return idx, mask.sum(-1).to(torch.int32)


__all__ = ["decode_mask", "diag_topk_mask", "group_max", "lists_from_mask", "prefill_mask"]
