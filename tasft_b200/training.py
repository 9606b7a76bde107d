"""Training-time gate-target path on the GPU.

Reference: ``TASFTAttention._training_forward`` builds the full ``[B, H, S, S]`` score
matrix (``tasft/modules/tasft_attention.py:427-458``) and ``TASFTObjective`` max-pools it,
softmaxes the block grid and takes the KL against the gate
(``tasft/training/objectives.py:128-241``). Here :func:`gate_target_from_qk` goes from Q
and K to the target without storing the score matrix, and :func:`gate_losses` returns the
KL and sparsity losses with the gradient w.r.t. the soft scores in one pass.
:class:`TASFTObjective` keeps the reference's static-method API for scores given as a
tensor.
"""
from __future__ import annotations

import math

import torch

from tasft_b200 import _lib as L
from tasft_b200.exceptions import NaNDetectedError


def gate_target_from_qk(
    q: torch.Tensor,
    k: torch.Tensor,
    block: int = 64,
    *,
    emulate_bf16_scores: bool | None = None,
    temperature: float = 1.0,
    clamp: float | None = None,
    return_block_max: bool = False,
    force_simt: bool = False,
):
    """Block-importance target from Q ``[B,Hq,S,D]`` and K ``[B,Hk,S,D]`` (causal).

    ``emulate_bf16_scores`` (default: on for bf16 inputs) rounds each block max as the
    reference's bf16 ``(Q K^T) * scale`` would be rounded, so the result matches a bf16
    training forward; rounding is monotone, so the max of rounded scores equals the
    rounded max.
    """
    L.require_cuda(q, k)
    q = q.contiguous()
    k = k.contiguous()
    B, Hq, S, D = q.shape
    Hk = k.shape[1]
    nb = math.ceil(S / block)
    if emulate_bf16_scores is None:
        emulate_bf16_scores = q.dtype == torch.bfloat16
    bm = torch.empty(B, Hq, nb, nb, dtype=torch.float32, device=q.device)
    tgt = torch.empty_like(bm)
    args = L.TargetArgs(
        q=q.data_ptr(), k=k.data_ptr(), q_stride=L.strides4(q), k_stride=L.strides4(k),
        B=B, Hq=Hq, Hk=Hk, S=S, D=D, block=block, dtype=L.dtype_code(q), scale=1.0 / math.sqrt(D),
        emulate_bf16_scores=int(emulate_bf16_scores), temperature=float(temperature),
        clamp=float(clamp) if clamp is not None else 0.0, block_max=bm.data_ptr(), target=tgt.data_ptr(),
        workspace=None, workspace_bytes=0, force_simt=int(force_simt), err=None,
    )
    L.check(L.lib().tasft_gate_target_fwd(args, L.stream_ptr(q.device)), "tasft_gate_target_fwd",
            shape=[B, Hq, Hk, S, D])
    return (tgt, bm) if return_block_max else tgt


def gate_losses(soft: torch.Tensor, target: torch.Tensor, tau_target: float = 0.8,
                w_kl: float = 1.0, w_sparse: float = 0.0, want_grad: bool = True):
    """KL(target || soft/sum) batchmean, (mean(soft) - tau)^2 and d(w_kl KL + w_sparse sparse)/d soft."""
    L.require_cuda(soft, target)
    s = soft.float().contiguous()
    t = target.float().contiguous()
    B, H, nq, nk = s.shape
    kl = torch.empty((), dtype=torch.float32, device=s.device)
    sp = torch.empty((), dtype=torch.float32, device=s.device)
    d = torch.empty_like(s) if want_grad else None
    ws_bytes = L.lib().tasft_gate_loss_workspace_size(B, H)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=s.device)
    args = L.LossArgs(soft=s.data_ptr(), target=t.data_ptr(), B=B, H=H, NBq=nq, NBk=nk, tau_target=tau_target,
                      w_kl=w_kl, w_sparse=w_sparse, kl=kl.data_ptr(), sparse=sp.data_ptr(), d_soft=L.ptr(d),
                      workspace=ws.data_ptr(), workspace_bytes=ws_bytes)
    L.check(L.lib().tasft_gate_loss_fwd_bwd(args, L.stream_ptr(s.device)), "tasft_gate_loss_fwd_bwd")
    return kl, sp, d


def gate_backward(pooled_q, pooled_k, soft, d_soft, w_in, b_in, w_out, causal: bool, need_inputs: bool = True):
    """Gradients of the gate MLP given d(loss)/d(soft) (used by ``AttnGate``'s autograd)."""
    B, Hq, nq, D = pooled_q.shape
    Hk, nk = pooled_k.shape[1], pooled_k.shape[2]
    hid = w_in.shape[0]
    dev = soft.device
    w_in_f = w_in.detach().float().contiguous()
    b_in_f = b_in.detach().float().contiguous()
    w_out_f = w_out.detach().float().contiguous().view(-1)
    out = {
        "d_w_in": torch.empty(hid, 2 * D, dtype=torch.float32, device=dev),
        "d_b_in": torch.empty(hid, dtype=torch.float32, device=dev),
        "d_w_out": torch.empty(hid, dtype=torch.float32, device=dev),
        "d_pooled_q": torch.empty_like(pooled_q) if need_inputs else None,
        "d_pooled_k": torch.empty_like(pooled_k) if need_inputs else None,
    }
    ws_bytes = L.lib().tasft_gate_bwd_workspace_size(B, Hq, Hk, nq, nk, hid)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    args = L.GateBwdArgs(
        pooled_q=pooled_q.data_ptr(), pooled_k=pooled_k.data_ptr(), d_soft=d_soft.data_ptr(),
        soft=soft.data_ptr(), B=B, Hq=Hq, Hk=Hk, NBq=nq, NBk=nk, D=D, hidden=hid, causal=int(causal),
        w_in=w_in_f.data_ptr(), b_in=b_in_f.data_ptr(), w_out=w_out_f.data_ptr(),
        d_w_in=out["d_w_in"].data_ptr(), d_b_in=out["d_b_in"].data_ptr(), d_w_out=out["d_w_out"].data_ptr(),
        d_pooled_q=L.ptr(out["d_pooled_q"]), d_pooled_k=L.ptr(out["d_pooled_k"]),
        workspace=ws.data_ptr(), workspace_bytes=ws_bytes,
    )
    L.check(L.lib().tasft_gate_bwd(args, L.stream_ptr(dev)), "tasft_gate_bwd")
    out["d_w_in"] = out["d_w_in"].to(w_in.dtype)
    out["d_b_in"] = out["d_b_in"].to(b_in.dtype)
    out["d_w_out"] = out["d_w_out"].to(w_out.dtype)
    return out


class _GateLossFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, soft, target, tau, w_kl, w_sparse):
        kl, sp, d = gate_losses(soft, target, tau, w_kl, w_sparse, want_grad=True)
        ctx.save_for_backward(d)
        ctx.dtype = soft.dtype
        return w_kl * kl + w_sparse * sp, kl, sp

    @staticmethod
    def backward(ctx, g_total, _gk, _gs):
        (d,) = ctx.saved_tensors
        return (d * g_total).to(ctx.dtype), None, None, None, None


def gate_objective(soft: torch.Tensor, target: torch.Tensor, tau_target: float = 0.8,
                   w_kl: float = 1.0, w_sparse: float = 0.01):
    """Differentiable ``w_kl * KL + w_sparse * sparse`` (trainer.py:442-447 weighting); returns (total, kl, sparse)."""
    return _GateLossFn.apply(soft, target, tau_target, w_kl, w_sparse)


def _check_finite_scores(attn_scores: torch.Tensor) -> None:
    has_nan = bool(torch.isnan(attn_scores).any())
    has_pos_inf = bool((attn_scores == float("inf")).any())
    if has_nan or has_pos_inf:
        raise NaNDetectedError(
            f"Non-finite values detected in attn_scores: NaN={has_nan}, Inf={has_pos_inf}",
            context={"tensor_name": "attn_scores", "has_nan": has_nan, "has_inf": has_pos_inf,
                     "shape": list(attn_scores.shape), "dtype": str(attn_scores.dtype)},
        )


def _check_finite(t: torch.Tensor, name: str) -> None:
    if not torch.isfinite(t).all():
        has_nan = bool(torch.isnan(t).any())
        has_inf = bool(torch.isinf(t).any())
        raise NaNDetectedError(f"Non-finite values detected in {name}: NaN={has_nan}, Inf={has_inf}",
                               context={"tensor_name": name, "has_nan": has_nan, "has_inf": has_inf,
                                        "shape": list(t.shape), "dtype": str(t.dtype)})


class TASFTObjective:
    """GPU versions of the reference's gate-target static methods (objectives.py:128-241)."""

    @staticmethod
    def compute_gate_target_from_qk(q, k, block_size: int = 64, **kw):
        return gate_target_from_qk(q, k, block_size, **kw)

    @staticmethod
    def compute_gate_loss(gate_soft_scores: torch.Tensor, gate_target: torch.Tensor) -> torch.Tensor:
        _check_finite(gate_soft_scores, "gate_soft_scores")
        _check_finite(gate_target, "gate_target")
        kl, _, _ = gate_losses(gate_soft_scores, gate_target, want_grad=False)
        return kl

    @staticmethod
    def compute_sparsity_loss(gate_soft_scores: torch.Tensor, tau_target: float) -> torch.Tensor:
        _check_finite(gate_soft_scores, "gate_soft_scores")
        _, sp, _ = gate_losses(gate_soft_scores, torch.zeros_like(gate_soft_scores, dtype=torch.float32),
                               tau_target, want_grad=False)
        return sp


__all__ = ["TASFTObjective", "gate_backward", "gate_losses", "gate_objective", "gate_target_from_qk"]
