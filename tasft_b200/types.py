"""Shared constants and result types (mirrors ``tasft/types.py:12-22``)."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Final

import torch

VALID_BLOCK_SIZES: Final[frozenset[int]] = frozenset({32, 64, 128})


@dataclass(frozen=True)
class KeptBlocks:
    """Compact block mask: ascending kept k-block indices per (batch, head, q-block).

    ``idx`` is ``[B, Hm, NBq, NBk]`` int32 padded with ``-1``; ``cnt`` is ``[B, Hm, NBq]``.
    ``Hm`` is the q-head count (per-head masks, the reference's granularity) or the
    kv-head count (one list shared by the q-heads of each GQA group).
    For decode, ``idx`` is ``[B, Hk, NBmax]`` and ``cnt`` ``[B, Hk]``.
    """

    idx: torch.Tensor
    cnt: torch.Tensor

    @property
    def heads(self) -> int:
        return int(self.idx.shape[1])
