"""ctypes binding of ``libtasft_b200.so`` (declarations in ``include/tasft_b200.h``).

The library is loaded from ``tasft_b200/_lib/`` inside the source tree. There is no
fallback: if the shared object is missing or fails to load, every op raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import torch

from tasft_b200.exceptions import KernelError, ValidationError

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libtasft_b200.so"

TASFT_OK = 0
STATUS = {
    -1: "invalid argument",
    -2: "unsupported dtype, head_dim or block size",
    -3: "CUDA runtime error",
    -4: "workspace missing or too small",
    -5: "size exceeds a fixed capacity",
}
DEVERR_INDEX, DEVERR_TIMEOUT, DEVERR_ORDER = 1, 2, 4

F32, BF16, F16 = 0, 1, 2
_DTYPES = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}

I64x4 = C.c_int64 * 4
I64x3 = C.c_int64 * 3
vp = C.c_void_p


class GateArgs(C.Structure):
    _fields_ = [
        ("q", vp), ("k", vp), ("q_stride", I64x4), ("k_stride", I64x4),
        ("B", C.c_int32), ("Hq", C.c_int32), ("Hk", C.c_int32), ("Sq", C.c_int32), ("Sk", C.c_int32),
        ("D", C.c_int32), ("block", C.c_int32), ("dtype", C.c_int32), ("hidden", C.c_int32),
        ("w_in", vp), ("b_in", vp), ("w_out", vp), ("causal", C.c_int32), ("tau", C.c_float),
        ("soft", vp), ("hard", vp), ("kept_idx", vp), ("kept_cnt", vp), ("num_kept", vp),
        ("pooled_q", vp), ("pooled_k", vp), ("workspace", vp), ("workspace_bytes", C.c_int64),
    ]


class QkvArgs(C.Structure):
    _fields_ = [
        ("q_in", vp), ("k_in", vp), ("v_in", vp), ("q_in_stride", C.c_int64 * 2), ("k_in_stride", C.c_int64 * 2),
        ("v_in_stride", C.c_int64 * 2), ("cos", vp), ("sin", vp), ("cs_stride", C.c_int64 * 2),
        ("q_out", vp), ("k_out", vp), ("v_out", vp), ("pooled_q", vp), ("pooled_k", vp),
        ("B", C.c_int32), ("Hq", C.c_int32), ("Hk", C.c_int32), ("S", C.c_int32), ("D", C.c_int32),
        ("block", C.c_int32), ("dtype", C.c_int32), ("rope", C.c_int32),
    ]


class ThresholdArgs(C.Structure):
    _fields_ = [
        ("soft", vp), ("rows", C.c_int64), ("NBq", C.c_int32), ("NBk", C.c_int32), ("causal", C.c_int32),
        ("tau", C.c_float), ("hard", vp), ("kept_idx", vp), ("kept_cnt", vp), ("num_kept", vp),
    ]


class CalibArgs(C.Structure):
    _fields_ = [("scores", vp), ("n", C.c_int64), ("keep", C.c_int64), ("tau", vp), ("kept", vp)]


class MaskArgs(C.Structure):
    _fields_ = [
        ("mask", vp), ("rows", C.c_int64), ("NBq", C.c_int32), ("NBk", C.c_int32), ("causal", C.c_int32),
        ("kept_idx", vp), ("kept_cnt", vp), ("num_kept", vp),
    ]


class PrefillArgs(C.Structure):
    _fields_ = [
        ("q", vp), ("k", vp), ("v", vp), ("out", vp),
        ("q_stride", I64x4), ("k_stride", I64x4), ("v_stride", I64x4), ("o_stride", I64x4),
        ("B", C.c_int32), ("Hq", C.c_int32), ("Hk", C.c_int32), ("S", C.c_int32), ("D", C.c_int32),
        ("block", C.c_int32), ("dtype", C.c_int32), ("causal", C.c_int32), ("scale", C.c_float),
        ("kept_idx", vp), ("kept_cnt", vp), ("Hm", C.c_int32), ("err", vp), ("force_simt", C.c_int32), ("qb_lo", C.c_int32),
        ("qb_hi", C.c_int32),
    ]


class TrainFwdArgs(C.Structure):
    _fields_ = [
        ("base", PrefillArgs), ("block_max", vp), ("target", vp), ("temperature", C.c_float), ("clamp", C.c_float),
        ("emulate_bf16_scores", C.c_int32),
    ]


class PrefillVarlenArgs(C.Structure):
    _fields_ = [("base", PrefillArgs), ("cu_seqlens", vp), ("total", C.c_int32)]


class DecodeArgs(C.Structure):
    _fields_ = [
        ("q", vp), ("k_cache", vp), ("v_cache", vp), ("out", vp),
        ("q_stride", I64x3), ("k_stride", I64x4), ("v_stride", I64x4), ("o_stride", I64x3),
        ("B", C.c_int32), ("Hq", C.c_int32), ("Hk", C.c_int32), ("L", C.c_int32), ("D", C.c_int32),
        ("block", C.c_int32), ("dtype", C.c_int32), ("scale", C.c_float),
        ("kv_len", vp), ("kept_idx", vp), ("kept_cnt", vp), ("nb_max", C.c_int32), ("num_splits", C.c_int32),
        ("part_o", vp), ("part_ml", vp), ("workspace", vp), ("workspace_bytes", C.c_int64), ("err", vp),
        ("kv_offset", C.c_int32),
    ]


class PagedDecodeArgs(C.Structure):
    _fields_ = [
        ("base", DecodeArgs), ("block_table", vp), ("max_pages", C.c_int32), ("page_size", C.c_int32),
        ("num_pages", C.c_int32),
    ]


class CombineArgs(C.Structure):
    _fields_ = [
        ("part_o", vp), ("part_ml", vp), ("G", C.c_int32), ("rows", C.c_int64), ("D", C.c_int32),
        ("out", vp), ("dtype", C.c_int32),
    ]


class DecodePeerArgs(C.Structure):
    _fields_ = [("mailboxes", vp), ("epoch", vp), ("world", C.c_int32), ("rank", C.c_int32), ("timeout_ns", C.c_uint64)]


class PeerCombineArgs(C.Structure):
    _fields_ = [
        ("part_o", vp), ("part_ml", vp), ("rows", C.c_int64), ("D", C.c_int32), ("world", C.c_int32),
        ("rank", C.c_int32), ("mailboxes", vp), ("epoch", vp), ("out", vp), ("dtype", C.c_int32),
        ("timeout_ns", C.c_uint64), ("err", vp),
    ]


class TargetArgs(C.Structure):
    _fields_ = [
        ("q", vp), ("k", vp), ("q_stride", I64x4), ("k_stride", I64x4),
        ("B", C.c_int32), ("Hq", C.c_int32), ("Hk", C.c_int32), ("S", C.c_int32), ("D", C.c_int32),
        ("block", C.c_int32), ("dtype", C.c_int32), ("scale", C.c_float), ("emulate_bf16_scores", C.c_int32),
        ("temperature", C.c_float), ("clamp", C.c_float), ("block_max", vp), ("target", vp),
        ("workspace", vp), ("workspace_bytes", C.c_int64), ("force_simt", C.c_int32), ("err", vp),
    ]


class ScoresTargetArgs(C.Structure):
    _fields_ = [
        ("scores", vp), ("stride", I64x4), ("B", C.c_int32), ("H", C.c_int32), ("Sq", C.c_int32),
        ("Sk", C.c_int32), ("block", C.c_int32), ("dtype", C.c_int32), ("temperature", C.c_float),
        ("clamp", C.c_float), ("block_max", vp), ("target", vp), ("flags", vp), ("workspace", vp),
        ("workspace_bytes", C.c_int64),
    ]


class LossArgs(C.Structure):
    _fields_ = [
        ("soft", vp), ("target", vp), ("B", C.c_int32), ("H", C.c_int32), ("NBq", C.c_int32), ("NBk", C.c_int32),
        ("tau_target", C.c_float), ("w_kl", C.c_float), ("w_sparse", C.c_float),
        ("kl", vp), ("sparse", vp), ("d_soft", vp), ("workspace", vp), ("workspace_bytes", C.c_int64),
    ]


class GateBwdArgs(C.Structure):
    _fields_ = [
        ("pooled_q", vp), ("pooled_k", vp), ("d_soft", vp), ("soft", vp),
        ("B", C.c_int32), ("Hq", C.c_int32), ("Hk", C.c_int32), ("NBq", C.c_int32), ("NBk", C.c_int32),
        ("D", C.c_int32), ("hidden", C.c_int32), ("causal", C.c_int32),
        ("w_in", vp), ("b_in", vp), ("w_out", vp),
        ("d_w_in", vp), ("d_b_in", vp), ("d_w_out", vp), ("d_pooled_q", vp), ("d_pooled_k", vp),
        ("workspace", vp), ("workspace_bytes", C.c_int64),
    ]


# name -> (argtypes, restype); every symbol declared in include/tasft_b200.h
SIGNATURES = {
    "tasft_gate_workspace_size": ([C.c_int32] * 8, C.c_int64),
    "tasft_gate_mask_build": ([C.POINTER(GateArgs), vp], C.c_int),
    "tasft_mask_from_scores": ([C.POINTER(ThresholdArgs), vp], C.c_int),
    "tasft_qkv_rope_pool": ([C.POINTER(QkvArgs), vp], C.c_int),
    "tasft_mask_to_kept": ([C.POINTER(MaskArgs), vp], C.c_int),
    "tasft_calibrate_tau": ([C.POINTER(CalibArgs), vp], C.c_int),
    "tasft_bsa_prefill_fwd": ([C.POINTER(PrefillArgs), vp], C.c_int),
    "tasft_bsa_prefill_varlen_fwd": ([C.POINTER(PrefillVarlenArgs), vp], C.c_int),
    "tasft_attention_train_fwd": ([C.POINTER(TrainFwdArgs), vp], C.c_int),
    "tasft_decode_workspace_size": ([C.c_int32] * 5, C.c_int64),
    "tasft_bsa_decode_fwd": ([C.POINTER(DecodeArgs), vp], C.c_int),
    "tasft_bsa_decode_combine": ([C.POINTER(CombineArgs), vp], C.c_int),
    "tasft_bsa_decode_fwd_noalloc": ([C.POINTER(DecodeArgs), vp], C.c_int),
    "tasft_bsa_decode_paged_fwd": ([C.POINTER(PagedDecodeArgs), vp], C.c_int),
    "tasft_decode_noalloc_capacity": ([], C.c_int64),
    "tasft_peer_mailbox_bytes": ([C.c_int32, C.c_int64, C.c_int32], C.c_int64),
    "tasft_peer_alloc": ([C.c_int64, C.POINTER(vp)], C.c_int),
    "tasft_peer_free": ([vp], C.c_int),
    "tasft_ipc_handle": ([vp, C.c_char_p], C.c_int),
    "tasft_ipc_open": ([C.c_char_p, C.POINTER(vp)], C.c_int),
    "tasft_ipc_close": ([vp], C.c_int),
    "tasft_peer_combine": ([C.POINTER(PeerCombineArgs), vp], C.c_int),
    "tasft_bsa_decode_peer_fwd": ([C.POINTER(DecodeArgs), C.POINTER(DecodePeerArgs), vp], C.c_int),
    "tasft_gate_target_workspace_size": ([C.c_int32] * 4, C.c_int64),
    "tasft_gate_target_fwd": ([C.POINTER(TargetArgs), vp], C.c_int),
    "tasft_scores_target_workspace_size": ([C.c_int32] * 5, C.c_int64),
    "tasft_gate_target_from_scores": ([C.POINTER(ScoresTargetArgs), vp], C.c_int),
    "tasft_gate_loss_workspace_size": ([C.c_int32] * 2, C.c_int64),
    "tasft_gate_loss_fwd_bwd": ([C.POINTER(LossArgs), vp], C.c_int),
    "tasft_gate_bwd_workspace_size": ([C.c_int32] * 6, C.c_int64),
    "tasft_gate_bwd": ([C.POINTER(GateBwdArgs), vp], C.c_int),
    "tasft_status_string": ([C.c_int], C.c_char_p),
    "tasft_abi_version": ([], C.c_int),
    "tasft_launch_count": ([], C.c_int64),
}

_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    """Load the shared library once; raise KernelError if it cannot be loaded."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise KernelError(
                "libtasft_b200.so is not built; run `python -m tasft_b200.build` (needs nvcc)",
                context={"path": str(LIB_PATH)},
            )
        try:
            handle = C.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | os.RTLD_GLOBAL)
        except OSError as e:
            raise KernelError(f"cannot load {LIB_PATH}: {e}", context={"path": str(LIB_PATH)}) from e
        for name, (argt, rest) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = argt
            fn.restype = rest
        _lib = handle
    return _lib


def check(rc: int, what: str, **context) -> None:
    if rc != TASFT_OK:
        msg = STATUS.get(rc, f"status {rc}")
        cls = ValidationError if rc in (-1,) else KernelError
        raise cls(f"{what}: {msg}", context={"status": rc, **context})


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError as e:
        raise KernelError(f"unsupported dtype {t.dtype}", context={"dtype": str(t.dtype)}) from e


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def strides4(t: torch.Tensor):
    return I64x4(*t.stride())


def strides3(t: torch.Tensor):
    return I64x3(*t.stride())


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise KernelError("Tensors must be on CUDA device", context={"device": str(t.device)})


def launch_count() -> int:
    return int(lib().tasft_launch_count())
