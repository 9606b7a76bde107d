"""Exception hierarchy with the reference's names and ``(message, context)`` convention.

Mirrors ``tasft/exceptions.py:7-43``. When the reference package ``tasft`` is importable
(the drop-in case), each class also derives from the reference class of the same name,
so ``except tasft.exceptions.KernelError`` in reference callers catches errors raised here.
"""
from __future__ import annotations

from typing import Any

try:  # pragma: no cover - depends on the environment
    from tasft import exceptions as _ref  # type: ignore
except Exception:  # noqa: BLE001
    _ref = None


def _bases(name: str, *local):
    ref_cls = getattr(_ref, name, None) if _ref is not None else None
    return (ref_cls, *local) if ref_cls is not None else local


class TASFTError(*_bases("TASFTError", Exception)):
    """Base error; carries a structured ``context`` dict (tasft/exceptions.py:7-13)."""

    def __init__(self, message: str, context: dict[str, Any] | None = None) -> None:
        Exception.__init__(self, message)
        self.context: dict[str, Any] = context or {}


class KernelError(*_bases("KernelError", TASFTError)):
    """The sparse attention kernels rejected a call or failed (tasft/exceptions.py:36)."""


class ValidationError(*_bases("ValidationError", TASFTError)):
    """Input validation failed (tasft/exceptions.py:32)."""


class TrainingError(*_bases("TrainingError", TASFTError)):
    """Unrecoverable training-path error (tasft/exceptions.py:16)."""


class NaNDetectedError(*_bases("NaNDetectedError", TrainingError)):
    """NaN/Inf found in a tensor (tasft/exceptions.py:20)."""


__all__ = ["KernelError", "NaNDetectedError", "TASFTError", "TrainingError", "ValidationError"]
