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

``patch(training=True)`` also swaps the training step's two score-tensor consumers: the
reference ``TASFTAttention._training_forward`` (``tasft/modules/tasft_attention.py:363-468``)
for :func:`training_forward`, which runs :func:`tasft_b200.training_attention` (attention
output and gate target in one pass, no ``[B, H, S, S]`` scores) and stores the gate TARGET
``[B, H, NBq, NBk]`` in ``_last_attn_weights``; and ``TASFTObjective`` in
``tasft.training.objectives`` / ``tasft.training.trainer`` for this package's, whose
``compute`` takes such a target in place of a score tensor.
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


_TRAINING_TARGETS = {
    "TASFTObjective": ["tasft.training.objectives", "tasft.training.trainer", "tasft.training"],
}


def training_forward(self, hidden_states, attention_mask=None, position_ids=None, past_key_value=None,
                     use_cache=False, cache_position=None, position_embeddings=None, **kwargs):
    """Replacement for ``TASFTAttention._training_forward`` (tasft_attention.py:363-468).

    Same projections (the layer's own ``_prepare_qkv``), same gate call, same output
    projection and return value; the score matrix, its softmax and P V are one
    :func:`tasft_b200.training_attention` pass that also yields the gate target, stored in
    ``_last_attn_weights`` (the patched ``TASFTObjective.compute`` takes it as is). Falls
    back to the reference method for what that pass does not cover: a padding
    ``attention_mask`` or a base module without q/k/v/o projections.
    """
    from tasft_b200.training import training_attention  # noqa: PLC0415

    attn = self.base_attn
    if attention_mask is not None or not all(hasattr(attn, p) for p in ("q_proj", "k_proj", "v_proj", "o_proj")):
        return _SAVED_METHODS["_training_forward"](self, hidden_states, attention_mask=attention_mask,
                                                  position_ids=position_ids, past_key_value=past_key_value,
                                                  use_cache=use_cache, cache_position=cache_position,
                                                  position_embeddings=position_embeddings, **kwargs)
    bsz, q_len, hidden_dim = hidden_states.shape
    q, k, v, head_dim = self._prepare_qkv(attn, hidden_states, bsz, q_len, position_ids, position_embeddings,
                                          past_key_value)
    new_past = (k, v) if use_cache else None
    self._last_gate_output = self.gate(q, k)
    out, target = training_attention(q, k, v, self.gate.block_size)
    self._last_attn_weights = target
    out = attn.o_proj(out.transpose(1, 2).contiguous().reshape(bsz, q_len, hidden_dim))
    return self._pack_output(out, None, new_past)


_SAVED_METHODS: dict[str, object] = {}


def patch(import_missing: bool = True, training: bool = False) -> list[str]:
    """Rebind the hot-path classes in the reference modules; returns the patched names.
    ``training=True`` also installs :func:`training_forward` and this package's
    ``TASFTObjective`` (see the module docstring)."""
    from tasft_b200.attn_gate import AttnGate, GateOutput  # noqa: PLC0415
    from tasft_b200.block_sparse_fa import BlockSparseFlashAttention  # noqa: PLC0415
    from tasft_b200.training import TASFTObjective  # noqa: PLC0415

    repl = {"BlockSparseFlashAttention": BlockSparseFlashAttention, "AttnGate": AttnGate, "GateOutput": GateOutput,
            "TASFTObjective": TASFTObjective}
    done = []
    targets = dict(_TARGETS)
    if training:
        targets.update(_TRAINING_TARGETS)
        mod = sys.modules.get("tasft.modules.tasft_attention")
        if mod is None and import_missing:
            try:
                mod = importlib.import_module("tasft.modules.tasft_attention")
            except Exception:  # noqa: BLE001 - the reference may be absent
                mod = None
        if mod is not None and hasattr(mod, "TASFTAttention"):
            cls = mod.TASFTAttention
            _SAVED_METHODS.setdefault("_training_forward", cls._training_forward)
            cls._training_forward = training_forward
            done.append("tasft.modules.tasft_attention.TASFTAttention._training_forward")
    for name, mods in targets.items():
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
    if "_training_forward" in _SAVED_METHODS:
        mod = sys.modules.get("tasft.modules.tasft_attention")
        if mod is not None:
            mod.TASFTAttention._training_forward = _SAVED_METHODS["_training_forward"]
        _SAVED_METHODS.clear()


__all__ = ["patch", "training_forward", "unpatch"]
