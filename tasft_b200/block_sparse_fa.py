"""Drop-in ``BlockSparseFlashAttention`` backed by hand-written sm_100a CUDA.

Mirrors the reference API of ``tasft/kernels/block_sparse_fa.py`` (class at :299-618,
``forward`` :361-411, ``_validate_inputs`` :413-452, ``compute_sparsity_stats``
:574-595, ``estimate_speedup`` :597-618, ``detect_kernels`` :63-90). Differences, all
additive or stricter:

* K/V may have fewer heads than Q (GQA, ``Hq % Hk == 0``); no ``repeat_interleave``.
* ``block_mask`` may be a bool ``[B, Hm, NB, NB]`` mask with ``Hm`` = q-heads or
  kv-heads, or a precomputed :class:`~tasft_b200.types.KeptBlocks`.
* There is one compute backend (the CUDA library). Under ``AUTO`` a call below
  ``min_sparsity_for_speedup`` still runs the sparse kernel on the given mask (the
  reference would run dense SDPA and ignore the mask, :393-399), with no host sync. An
  explicit ``DENSE_FALLBACK`` backend is accepted as the reference accepts it
  (:340-359) and, like the reference's dense path, ignores the mask: it runs full
  (causal) attention through the same kernel with every block kept.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from enum import Enum, auto

import torch

from tasft_b200 import _lib as L
from tasft_b200.exceptions import KernelError
from tasft_b200.types import VALID_BLOCK_SIZES, KeptBlocks

_EXPECTED_TENSOR_NDIM = 4
_VALID_HEAD_DIMS = frozenset({32, 64, 128})


class KernelBackend(Enum):
    """Backend selector kept for signature compatibility with the reference enum."""

    AUTO = auto()
    FLASH_ATTN_SPARSE = auto()
    TRITON = auto()
    DENSE_FALLBACK = auto()
    SM100_CUDA = auto()


def detect_kernels() -> list[KernelBackend]:
    """Available backends in priority order; ``DENSE_FALLBACK`` is always the last element
    (the reference's guarantee, block_sparse_fa.py:63-90). ``SM100_CUDA`` is listed when
    the sm_100a library loads. Both run on that library: without it the constructor
    raises, there is no CPU path."""
    try:
        L.lib()
    except KernelError:
        return [KernelBackend.DENSE_FALLBACK]
    return [KernelBackend.SM100_CUDA, KernelBackend.DENSE_FALLBACK]


_FULL_LISTS: dict = {}


def full_kept(B: int, H: int, nb: int, causal: bool, device) -> KeptBlocks:
    """Kept lists with every block (of the lower triangle when causal): dense attention
    through the block-sparse kernel. Cached per shape and device."""
    key = (B, H, nb, causal, str(device))
    kb = _FULL_LISTS.get(key)
    if kb is None:
        ar = torch.arange(nb, dtype=torch.int32, device=device)
        idx = ar.view(1, nb).expand(nb, nb).clone()
        if causal:
            idx = torch.where(ar.view(nb, 1) >= ar.view(1, nb), idx, torch.full_like(idx, -1))
            cnt = ar + 1
        else:
            cnt = torch.full((nb,), nb, dtype=torch.int32, device=device)
        kb = KeptBlocks(idx.expand(B, H, nb, nb).contiguous(), cnt.expand(B, H, nb).contiguous())
        _FULL_LISTS[key] = kb
    return kb


@dataclass(frozen=True, slots=True)
class SparsityStats:
    """Same record as ``tasft/kernels/block_sparse_fa.py:277-291``."""

    total_blocks: int
    active_blocks: int
    sparsity_ratio: float
    estimated_speedup: float


def mask_to_kept(block_mask: torch.Tensor, causal: bool) -> KeptBlocks:
    """Bool block mask -> ascending kept lists on the device (one kernel, no host sync).

    Follows the reference host step ``block_mask & tril`` (block_sparse_fa.py:497-508)
    and the kernel's ascending visiting order (:192-203).
    """
    L.require_cuda(block_mask)
    m = block_mask
    if m.dtype != torch.bool:
        m = m != 0
    m = m.contiguous()
    nbq, nbk = m.shape[-2], m.shape[-1]
    rows = m.numel() // max(nbk, 1)
    idx = torch.empty(m.shape, dtype=torch.int32, device=m.device)
    cnt = torch.empty(m.shape[:-1], dtype=torch.int32, device=m.device)
    args = L.MaskArgs(
        mask=m.data_ptr(), rows=rows, NBq=nbq, NBk=nbk, causal=int(causal),
        kept_idx=idx.data_ptr(), kept_cnt=cnt.data_ptr(), num_kept=None,
    )
    L.check(L.lib().tasft_mask_to_kept(args, L.stream_ptr(m.device)), "tasft_mask_to_kept")
    return KeptBlocks(idx, cnt)


class BlockSparseFlashAttention:
    """Block-sparse causal (GQA-aware) flash attention on B200.

    Args:
        block_size: 32, 64 or 128 (64 runs on the tcgen05 tensor-core kernel for bf16/fp16).
        min_sparsity_for_speedup: validated and kept for API compatibility.
        backend: ``AUTO`` / ``SM100_CUDA`` (block-sparse), or ``DENSE_FALLBACK`` (full
            attention, mask ignored, as the reference's dense backend); the reference's
            ``TRITON`` and ``FLASH_ATTN_SPARSE`` raise ``KernelError``.
    """

    def __init__(
        self,
        block_size: int = 64,
        min_sparsity_for_speedup: float = 0.5,
        backend: KernelBackend = KernelBackend.AUTO,
    ) -> None:
        if block_size not in VALID_BLOCK_SIZES:
            raise ValueError(f"block_size must be one of {sorted(VALID_BLOCK_SIZES)}, got {block_size}")
        if not 0.0 <= min_sparsity_for_speedup <= 1.0:
            raise ValueError(f"min_sparsity_for_speedup must be in [0, 1], got {min_sparsity_for_speedup}")
        self.block_size = block_size
        self.min_sparsity_for_speedup = min_sparsity_for_speedup
        self._available_backends = detect_kernels()
        if backend not in self._available_backends + [KernelBackend.AUTO] or \
                KernelBackend.SM100_CUDA not in self._available_backends:
            names = [b.name for b in self._available_backends]
            raise KernelError(
                f"Requested backend {backend.name} is not available. Available: {names}",
                context={"requested": backend.name, "available": names},
            )
        self.backend = KernelBackend.DENSE_FALLBACK if backend == KernelBackend.DENSE_FALLBACK \
            else KernelBackend.SM100_CUDA
        self.force_simt = False  # testing hook: run the CUDA-core kernel instead of tcgen05

    # ------------------------------------------------------------------
    def forward(
        self,
        q: torch.Tensor,
        k: torch.Tensor,
        v: torch.Tensor,
        block_mask: torch.Tensor | KeptBlocks,
        *,
        causal: bool = True,
        out: torch.Tensor | None = None,
        err: torch.Tensor | None = None,
        q_block_range: tuple[int, int] | None = None,
    ) -> torch.Tensor:
        """Block-sparse attention; returns a new ``[B, Hq, S, D]`` tensor in q's dtype.

        ``q_block_range=(lo, hi)``: compute only the rows of q-blocks ``[lo, hi)`` (one rank's
        share of a long sequence, ``shards.qblock_ranges``); the tensor-core kernel then visits
        only those tiles and leaves the other rows of ``out`` as they were (the CUDA-core
        kernel computes every row)."""
        self._validate_inputs(q, k, v, block_mask)
        B, Hq, S, D = q.shape
        Hk = k.shape[1]
        q = q.contiguous()
        k = k.contiguous()
        v = v.contiguous()
        if self.backend == KernelBackend.DENSE_FALLBACK:
            kept = full_kept(B, Hk, math.ceil(S / self.block_size), causal, q.device)
        else:
            kept = block_mask if isinstance(block_mask, KeptBlocks) else mask_to_kept(block_mask, causal)
        if out is None:
            out = torch.empty_like(q)
        idx = kept.idx.contiguous()
        cnt = kept.cnt.contiguous()
        args = L.PrefillArgs(
            q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), out=out.data_ptr(),
            q_stride=L.strides4(q), k_stride=L.strides4(k), v_stride=L.strides4(v), o_stride=L.strides4(out),
            B=B, Hq=Hq, Hk=Hk, S=S, D=D, block=self.block_size, dtype=L.dtype_code(q), causal=int(causal),
            scale=1.0 / math.sqrt(D), kept_idx=idx.data_ptr(), kept_cnt=cnt.data_ptr(), Hm=idx.shape[1],
            err=L.ptr(err), force_simt=int(self.force_simt),
            qb_lo=int(q_block_range[0]) if q_block_range else 0, qb_hi=int(q_block_range[1]) if q_block_range else 0,
        )
        L.check(L.lib().tasft_bsa_prefill_fwd(args, L.stream_ptr(q.device)), "tasft_bsa_prefill_fwd",
                shape=[B, Hq, Hk, S, D], block=self.block_size)
        return out

    __call__ = forward

    def forward_varlen(
        self,
        q: torch.Tensor,
        k: torch.Tensor,
        v: torch.Tensor,
        cu_seqlens: torch.Tensor,
        max_seqlen: int,
        block_mask: torch.Tensor | KeptBlocks,
        *,
        causal: bool = True,
        out: torch.Tensor | None = None,
        err: torch.Tensor | None = None,
    ) -> torch.Tensor:
        """Block-sparse attention over sequences of different lengths packed along the
        token axis: q ``[T, Hq, D]``, k/v ``[T, Hk, D]``, ``cu_seqlens`` int32 ``[B + 1]``
        (sequence b is rows ``cu_seqlens[b]:cu_seqlens[b+1]``), masks per sequence
        ``[B, H, NB, NB]`` with ``NB = ceil(max_seqlen / block)``. Each sequence attends only
        within itself -- unlike the reference's vLLM prefill, which flattens the batch into one
        causal sequence (``tasft/inference/vllm_patch.py:172-196``). Every dtype and block
        size of ``forward``."""
        if q.ndim != 3 or k.ndim != 3 or k.shape != v.shape or k.shape[0] != q.shape[0] or \
                k.shape[2] != q.shape[2] or q.shape[1] % max(k.shape[1], 1) != 0:
            raise KernelError("varlen expects q [T, Hq, D] and k, v [T, Hk, D]",
                              context={"q": list(q.shape), "k": list(k.shape), "v": list(v.shape)})
        L.require_cuda(q, k, v, cu_seqlens)
        T_, Hq, D = q.shape
        Hk = k.shape[1]
        B = cu_seqlens.numel() - 1
        nb = math.ceil(max_seqlen / self.block_size)
        kept = block_mask if isinstance(block_mask, KeptBlocks) else mask_to_kept(block_mask, causal)
        if kept.idx.shape[0] != B or tuple(kept.idx.shape[2:]) != (nb, nb):
            raise KernelError("block_mask shape mismatch for varlen",
                              context={"expected": [B, "H", nb, nb], "got": list(kept.idx.shape)})
        q = q.contiguous()
        k = k.contiguous()
        v = v.contiguous()
        cu = cu_seqlens.to(torch.int32).contiguous()
        if out is None:
            out = torch.empty_like(q)
        idx = kept.idx.contiguous()
        cnt = kept.cnt.contiguous()

        def packed(x):  # [T, H, D] seen as [1, H, T, D] (the batch stride is never stepped)
            return L.I64x4(x.numel(), x.stride(1), x.stride(0), x.stride(2))

        base = L.PrefillArgs(
            q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), out=out.data_ptr(),
            q_stride=packed(q), k_stride=packed(k), v_stride=packed(v), o_stride=packed(out),
            B=B, Hq=Hq, Hk=Hk, S=int(max_seqlen), D=D, block=self.block_size, dtype=L.dtype_code(q),
            causal=int(causal), scale=1.0 / math.sqrt(D), kept_idx=idx.data_ptr(), kept_cnt=cnt.data_ptr(),
            Hm=idx.shape[1], err=L.ptr(err), force_simt=int(self.force_simt),
        )
        args = L.PrefillVarlenArgs(base=base, cu_seqlens=cu.data_ptr(), total=T_)
        L.check(L.lib().tasft_bsa_prefill_varlen_fwd(args, L.stream_ptr(q.device)), "tasft_bsa_prefill_varlen_fwd",
                shape=[B, Hq, Hk, T_, D], block=self.block_size)
        return out

    def _validate_inputs(self, q, k, v, block_mask) -> None:
        if q.ndim != _EXPECTED_TENSOR_NDIM:
            raise KernelError(f"Expected 4D tensors [B, H, S, D], got q.ndim={q.ndim}",
                              context={"q_shape": list(q.shape)})
        if k.ndim != 4 or v.ndim != 4 or k.shape != v.shape or k.shape[0] != q.shape[0] \
                or k.shape[2:] != q.shape[2:] or q.shape[1] % max(k.shape[1], 1) != 0:
            raise KernelError(
                "Q, K, V shapes must match (K/V may have Hq/n heads for GQA)",
                context={"q": list(q.shape), "k": list(k.shape), "v": list(v.shape)},
            )
        if not q.is_cuda:
            raise KernelError("Tensors must be on CUDA device", context={"device": str(q.device)})
        if q.dtype != k.dtype or q.dtype != v.dtype:
            raise KernelError("Q, K, V dtypes must match",
                              context={"q": str(q.dtype), "k": str(k.dtype), "v": str(v.dtype)})
        B, Hq, S, D = q.shape
        if D not in _VALID_HEAD_DIMS:
            raise KernelError(f"head_dim must be in {sorted(_VALID_HEAD_DIMS)}, got {D}",
                              context={"head_dim": D, "supported": sorted(_VALID_HEAD_DIMS)})
        nb = math.ceil(S / self.block_size)
        shape = block_mask.idx.shape if isinstance(block_mask, KeptBlocks) else block_mask.shape
        hm = shape[1] if len(shape) == 4 else -1
        if len(shape) != 4 or shape[0] != B or shape[2:] != (nb, nb) or hm not in (Hq, k.shape[1]):
            raise KernelError(
                f"block_mask shape mismatch: expected {(B, Hq, nb, nb)}, got {tuple(shape)}",
                context={"expected": [B, Hq, nb, nb], "got": list(shape), "block_size": self.block_size},
            )

    # ------------------------------------------------------------------
    def compute_sparsity_stats(self, block_mask: torch.Tensor) -> SparsityStats:
        """Same statistics as the reference (one host sync, like the reference)."""
        total = block_mask.numel()
        active = int(block_mask.sum().item())
        ratio = 1.0 - active / max(total, 1)
        return SparsityStats(total, active, ratio, self.estimate_speedup(ratio))

    @staticmethod
    def sparsity_stats_device(block_mask: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """``(active_blocks, sparsity_ratio)`` as device scalars: the statistics of
        :meth:`compute_sparsity_stats` without its host synchronisation."""
        active = block_mask.sum()
        return active, 1.0 - active.float() / max(block_mask.numel(), 1)

    @staticmethod
    def estimate_speedup(sparsity_ratio: float) -> float:
        """The reference's model ``1 / (1 - s (1 - 0.02))`` (block_sparse_fa.py:597-618)."""
        return 1.0 / max(1e-6, 1.0 - sparsity_ratio * (1.0 - 0.02))


__all__ = ["BlockSparseFlashAttention", "KernelBackend", "SparsityStats", "detect_kernels", "full_kept", "mask_to_kept"]
