"""tasft_b200: B200-native (sm_100a) gated block-sparse attention for TASFT.

Drop-in replacements for the reference's hot-path API:
``BlockSparseFlashAttention`` (tasft/kernels/block_sparse_fa.py), ``AttnGate``
(tasft/modules/attn_gate.py) and the gate-target objective (tasft/training/objectives.py),
plus a block-sparse decode and its split-KV combine. Compute runs in
``libtasft_b200.so`` (hand-written CUDA, C ABI in ``include/tasft_b200.h``).
"""
from tasft_b200.attn_gate import (
    AttnGate,
    GateOutput,
    calibrate_tau,
    measured_sparsity_profile,
    qkv_rope_pool,
    threshold_scores,
)
from tasft_b200.block_sparse_fa import (
    BlockSparseFlashAttention,
    KernelBackend,
    SparsityStats,
    detect_kernels,
    mask_to_kept,
)
from tasft_b200.decode import DecodeWorkspace, bsa_decode, bsa_decode_paged, decode_combine
from tasft_b200.exceptions import KernelError, NaNDetectedError, TASFTError, ValidationError
from tasft_b200.patch import patch, unpatch
from tasft_b200 import shards
from tasft_b200.training import (
    ObjectiveLossOutput,
    TASFTObjective,
    gate_losses,
    gate_objective,
    gate_target_from_qk,
    gate_target_from_scores,
    training_attention,
)
from tasft_b200.types import VALID_BLOCK_SIZES, KeptBlocks

__all__ = [
    "VALID_BLOCK_SIZES",
    "AttnGate",
    "BlockSparseFlashAttention",
    "DecodeWorkspace",
    "GateOutput",
    "KeptBlocks",
    "KernelBackend",
    "KernelError",
    "NaNDetectedError",
    "ObjectiveLossOutput",
    "SparsityStats",
    "TASFTError",
    "TASFTObjective",
    "ValidationError",
    "bsa_decode",
    "calibrate_tau",
    "bsa_decode_paged",
    "decode_combine",
    "detect_kernels",
    "gate_losses",
    "gate_objective",
    "gate_target_from_qk",
    "gate_target_from_scores",
    "mask_to_kept",
    "measured_sparsity_profile",
    "patch",
    "qkv_rope_pool",
    "shards",
    "threshold_scores",
    "training_attention",
    "unpatch",
]
