"""Swap this package's classes into an imported reference ``tasft`` package.

The reference's callers resolve the hot-path classes by module attribute:
``BlockSparseFlashAttention`` lazily at ``tasft/modules/tasft_attention.py:189``,
``tasft/inference/tasft_model.py:198``, ``tasft/inference/vllm_patch.py:136`` and
``tasft/eval/long_context_bench.py:226``; ``AttnGate`` at import time in
``tasft/modules/tasft_attention.py:31``, ``tasft/inference/tasft_model.py:48``,
``tasft/inference/vllm_patch.py:48``, ``tasft/bundle/export.py:37`` and
``tasft/eval/gate_quality.py:39``. ``patch()`` rebinds those names (in every module
that is already imported) so newly built layers and the vLLM prefill patch use the
B200 kernels; ``unpatch()`` restores the originals.
"""
from __future__ import annotations

import importlib
import sys

_SAVED: dict[tuple[str, str], object] = {}

_TARGETS = {
    "BlockSparseFlashAttention": ["tasft.kernels.block_sparse_fa", "tasft.kernels"],
    "AttnGate": ["tasft.modules.attn_gate", "tasft.modules", "tasft.modules.tasft_attention",
                 "tasft.inference.tasft_model", "tasft.inference.vllm_patch", "tasft.bundle.export",
                 "tasft.eval.gate_quality"],
    "GateOutput": ["tasft.modules.attn_gate", "tasft.modules", "tasft.modules.tasft_attention",
                   "tasft.inference.tasft_model"],
}


def patch(import_missing: bool = True) -> list[str]:
    """Rebind the hot-path classes in the reference modules; returns the patched names."""
    from tasft_b200.attn_gate import AttnGate, GateOutput  # noqa: PLC0415
    from tasft_b200.block_sparse_fa import BlockSparseFlashAttention  # noqa: PLC0415

    repl = {"BlockSparseFlashAttention": BlockSparseFlashAttention, "AttnGate": AttnGate, "GateOutput": GateOutput}
    done = []
    for name, mods in _TARGETS.items():
        for mod_name in mods:
            mod = sys.modules.get(mod_name)
            if mod is None and import_missing and mod_name in ("tasft.kernels.block_sparse_fa",
                                                                "tasft.modules.attn_gate"):
                try:
                    mod = importlib.import_module(mod_name)
                except Exception:  # noqa: BLE001 - the reference may be absent
                    mod = None
            if mod is None or not hasattr(mod, name):
                continue
            _SAVED.setdefault((mod_name, name), getattr(mod, name))
            setattr(mod, name, repl[name])
            done.append(f"{mod_name}.{name}")
    return done


def unpatch() -> None:
    """Restore every name :func:`patch` replaced."""
    for (mod_name, name), obj in list(_SAVED.items()):
        mod = sys.modules.get(mod_name)
        if mod is not None:
            setattr(mod, name, obj)
    _SAVED.clear()


__all__ = ["patch", "unpatch"]
