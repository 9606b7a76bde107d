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
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from tasft_b200 import _lib as L
from tasft_b200.exceptions import KernelError, NaNDetectedError


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
    """(w_kl KL + w_sparse sparse, KL, sparse). The kernel writes the gradient of the
    weighted total; the KL and sparse outputs carry the gradient of their own term
    (KL: the total's gradient at w_sparse = 0; sparse: at w_kl = 0), so a caller
    differentiates whichever output it uses. ``target`` None = sparsity only."""

    @staticmethod
    def forward(ctx, soft, target, tau, w_kl, w_sparse):
        if target is None:
            target = torch.zeros_like(soft, dtype=torch.float32)
        want = soft.requires_grad
        kl, sp, d = gate_losses(soft, target, tau, w_kl, w_sparse, want_grad=want)
        ctx.save_for_backward(d if want else None)
        ctx.dtype = soft.dtype
        ctx.w = (w_kl, w_sparse)
        ctx.n = soft.numel()
        ctx.mean_dev = None
        if want:
            # d sparse / d soft is the constant 2 (mean - tau) / N; keep it for the sparse output
            ctx.mean_dev = (soft.detach().float().mean() - tau)
        return w_kl * kl + w_sparse * sp, kl, sp

    @staticmethod
    def backward(ctx, g_total, g_kl, g_sp):
        (d,) = ctx.saved_tensors
        if d is None:
            return None, None, None, None, None
        w_kl, w_sparse = ctx.w
        g_sparse_const = 2.0 * ctx.mean_dev / ctx.n  # d sparse / d soft
        grad = d * g_total if g_total is not None else torch.zeros_like(d)
        if g_kl is not None and w_kl != 0.0:
            # d holds w_kl dKL + w_sparse dSparse; recover dKL
            grad = grad + (d - w_sparse * g_sparse_const) / w_kl * g_kl
        if g_sp is not None:
            grad = grad + g_sparse_const * g_sp
        return grad.to(ctx.dtype), None, None, None, None


def gate_objective(soft: torch.Tensor, target: torch.Tensor, tau_target: float = 0.8,
                   w_kl: float = 1.0, w_sparse: float = 0.01):
    """Differentiable ``w_kl * KL + w_sparse * sparse`` (trainer.py:442-447 weighting); returns (total, kl, sparse)."""
    return _GateLossFn.apply(soft, target, tau_target, w_kl, w_sparse)


def gate_target_from_scores(
    attn_scores: torch.Tensor,
    block: int = 64,
    *,
    temperature: float = 1.0,
    clamp: float | None = None,
    check_finite: bool = True,
    return_block_max: bool = False,
    out_dtype: torch.dtype | None = None,
):
    """Block-importance target from a score tensor ``[B, H, Sq, Sk]`` the caller holds.

    The reference's ``compute_gate_target`` (``tasft/training/objectives.py:128-185``):
    -inf padding to whole blocks, ``block x block`` max-pool, softmax over the flattened
    grid; with ``temperature=2, clamp=50`` it is ``TASFTAttention._compute_gate_target``
    (``tasft/modules/tasft_attention.py:220-290``). One streaming read of the scores
    (``tasft_gate_target_from_scores``). With ``check_finite`` NaN or +inf in the scores
    raise ``NaNDetectedError`` as the reference does (one host read of a flag word). The
    target is returned in ``out_dtype`` (default: the scores' dtype, as the reference's
    softmax returns it).
    """
    if block <= 0:
        raise ValueError(f"block_size must be > 0, got {block}")
    L.require_cuda(attn_scores)
    if attn_scores.ndim != 4:
        raise ValueError(f"attn_scores must be [B, H, Sq, Sk], got shape {tuple(attn_scores.shape)}")
    sc = attn_scores if attn_scores.stride(-1) == 1 else attn_scores.contiguous()
    B, H, Sq, Sk = sc.shape
    nq, nk = math.ceil(Sq / block), math.ceil(Sk / block)
    bm = torch.empty(B, H, nq, nk, dtype=torch.float32, device=sc.device)
    tgt = torch.empty_like(bm)
    flags = torch.zeros(1, dtype=torch.int32, device=sc.device) if check_finite else None
    args = L.ScoresTargetArgs(
        scores=sc.data_ptr(), stride=L.strides4(sc), B=B, H=H, Sq=Sq, Sk=Sk, block=block, dtype=L.dtype_code(sc),
        temperature=float(temperature), clamp=float(clamp) if clamp is not None else 0.0, block_max=bm.data_ptr(),
        target=tgt.data_ptr(), flags=L.ptr(flags), workspace=None, workspace_bytes=0,
    )
    L.check(L.lib().tasft_gate_target_from_scores(args, L.stream_ptr(sc.device)), "tasft_gate_target_from_scores",
            shape=[B, H, Sq, Sk], block=block)
    if flags is not None:
        f = int(flags.item())
        if f:
            has_nan, has_pos_inf = bool(f & 1), bool(f & 2)
            raise NaNDetectedError(
                f"Non-finite values detected in attn_scores: NaN={has_nan}, Inf={has_pos_inf}",
                context={"tensor_name": "attn_scores", "has_nan": has_nan, "has_inf": has_pos_inf,
                         "shape": list(attn_scores.shape), "dtype": str(attn_scores.dtype)},
            )
    od = out_dtype or attn_scores.dtype
    if od != torch.float32:
        tgt = tgt.to(od)
    return (tgt, bm) if return_block_max else tgt


def _train_fwd(q, k, v, block, temperature, clamp, emulate):
    """Attention output + block maxima + target in one tcgen05 pass (dense causal lists);
    for shapes that kernel does not take, the CUDA-core prefill and the target kernels."""
    from tasft_b200.block_sparse_fa import BlockSparseFlashAttention, full_kept  # noqa: PLC0415

    B, Hq, S, D = q.shape
    Hk = k.shape[1]
    nb = math.ceil(S / block)
    kept = full_kept(B, Hk, nb, True, q.device)
    out = torch.empty_like(q)
    bm = torch.empty(B, Hq, nb, nb, dtype=torch.float32, device=q.device)
    tgt = torch.empty_like(bm)
    if block == 64 and q.dtype in (torch.bfloat16, torch.float16) and D in (64, 128):
        base = L.PrefillArgs(
            q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), out=out.data_ptr(), q_stride=L.strides4(q),
            k_stride=L.strides4(k), v_stride=L.strides4(v), o_stride=L.strides4(out), B=B, Hq=Hq, Hk=Hk, S=S, D=D,
            block=block, dtype=L.dtype_code(q), causal=1, scale=1.0 / math.sqrt(D), kept_idx=kept.idx.data_ptr(),
            kept_cnt=kept.cnt.data_ptr(), Hm=Hk, err=None, force_simt=0,
        )
        args = L.TrainFwdArgs(base=base, block_max=bm.data_ptr(), target=tgt.data_ptr(), temperature=float(temperature),
                              clamp=float(clamp) if clamp is not None else 0.0, emulate_bf16_scores=int(emulate))
        rc = L.lib().tasft_attention_train_fwd(args, L.stream_ptr(q.device))
        if rc == 0:
            return out, tgt, bm
        if rc != -2:
            L.check(rc, "tasft_attention_train_fwd", shape=[B, Hq, Hk, S, D])
    # other dtypes / blocks / head dims: the two kernels separately
    out = BlockSparseFlashAttention(block_size=block).forward(q, k, v, kept) if block in (32, 64, 128) else None
    if out is None:
        raise KernelError(f"training attention: unsupported block size {block}", context={"block": block})
    tgt, bm = gate_target_from_qk(q, k, block, emulate_bf16_scores=emulate, temperature=temperature, clamp=clamp,
                                  return_block_max=True)
    return out, tgt, bm


class _TrainAttnFn(torch.autograd.Function):
    """Forward: this library's fused attention + gate-target pass. Backward: the gradient of
    dense causal attention w.r.t. q, k, v, recomputed by PyTorch's scaled_dot_product_attention
    (the reference's training path differentiates its dense matmul/softmax the same way;
    the target is a detached distillation signal, tasft_attention.py:446-453)."""

    @staticmethod
    def forward(ctx, q, k, v, block, temperature, clamp, emulate):
        out, tgt, bm = _train_fwd(q, k, v, block, temperature, clamp, emulate)
        ctx.save_for_backward(q, k, v)
        ctx.mark_non_differentiable(tgt, bm)
        return out, tgt, bm

    @staticmethod
    def backward(ctx, g_out, _g_tgt, _g_bm):
        q, k, v = ctx.saved_tensors
        with torch.enable_grad():
            qq, kk, vv = (t.detach().requires_grad_(True) for t in (q, k, v))
            o = F.scaled_dot_product_attention(qq, kk, vv, is_causal=True, enable_gqa=q.shape[1] != k.shape[1])
            dq, dk, dv = torch.autograd.grad(o, (qq, kk, vv), g_out)
        return dq, dk, dv, None, None, None, None


def training_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, block: int = 64, *,
                       temperature: float = 1.0, clamp: float | None = None,
                       emulate_bf16_scores: bool | None = None, return_block_max: bool = False):
    """Dense causal attention for the training forward together with the gate target.

    The reference forms the ``[B, H, S, S]`` scores, softmaxes them for the output and keeps
    them for ``compute_gate_target`` (``tasft/modules/tasft_attention.py:427-466``,
    ``tasft/training/objectives.py:128-185``). Here one kernel pass produces the output and the
    per-tile score maxima (``tasft_attention_train_fwd``); the score tensor never exists.
    K/V may have fewer heads (GQA). Returns ``(out, target)`` (and the block maxima when
    asked); ``out`` is differentiable in q, k, v.
    """
    L.require_cuda(q, k, v)
    if emulate_bf16_scores is None:
        emulate_bf16_scores = q.dtype == torch.bfloat16
    out, tgt, bm = _TrainAttnFn.apply(q.contiguous(), k.contiguous(), v.contiguous(), block, temperature, clamp,
                                      bool(emulate_bf16_scores))
    return (out, tgt, bm) if return_block_max else (out, tgt)


def _check_finite(t: torch.Tensor, name: str, context: dict | None = None) -> None:
    if not torch.isfinite(t).all():
        has_nan = bool(torch.isnan(t).any())
        has_inf = bool(torch.isinf(t).any())
        raise NaNDetectedError(f"Non-finite values detected in {name}: NaN={has_nan}, Inf={has_inf}",
                               context={"tensor_name": name, "has_nan": has_nan, "has_inf": has_inf,
                                        "shape": list(t.shape), "dtype": str(t.dtype), **(context or {})})


@dataclass(frozen=True, slots=True)
class ObjectiveLossOutput:
    """Same record as ``tasft/training/objectives.py:40-63``."""

    total: torch.Tensor
    task: torch.Tensor
    gate: torch.Tensor
    sparse: torch.Tensor
    per_layer_gate_loss: dict[int, float]
    per_layer_sparsity: dict[int, float]
    active_layers: list[int]


class TASFTObjective:
    """Drop-in for the reference's dual objective (``tasft/training/objectives.py:66-361``).

    Same constructor validation, static methods and ``compute``. The gate-side steps run
    on this library's kernels: the target from a score tensor
    (``tasft_gate_target_from_scores``), and the KL and sparsity losses with their
    gradient w.r.t. the gate scores from one kernel pass (``tasft_gate_loss_fwd_bwd``),
    wrapped in autograd so ``loss.backward()`` reaches the gate as ``F.kl_div`` would.
    The task loss is the plain cross-entropy the reference uses.
    ``compute_gate_target_from_qk`` is the path that needs no score tensor at all.
    """

    def __init__(self, lambda_gate: float = 0.1, beta_sparse: float = 0.01, tau_target: float = 0.8,
                 label_smoothing: float = 0.0) -> None:
        if not 0.0 < lambda_gate <= 10.0:
            raise ValueError(f"lambda_gate must be in (0, 10], got {lambda_gate}")
        if beta_sparse < 0.0:
            raise ValueError(f"beta_sparse must be >= 0, got {beta_sparse}")
        if not 0.0 < tau_target < 1.0:
            raise ValueError(f"tau_target must be in (0, 1), got {tau_target}")
        if not 0.0 <= label_smoothing < 1.0:
            raise ValueError(f"label_smoothing must be in [0, 1), got {label_smoothing}")
        self._lambda_gate = lambda_gate
        self._beta_sparse = beta_sparse
        self._tau_target = tau_target
        self._label_smoothing = label_smoothing

    @staticmethod
    def compute_gate_target(attn_scores: torch.Tensor, block_size: int) -> torch.Tensor:
        """objectives.py:128-185 on the GPU (see :func:`gate_target_from_scores`)."""
        return gate_target_from_scores(attn_scores, block_size)

    @staticmethod
    def compute_gate_target_from_qk(q, k, block_size: int = 64, **kw):
        """The same target from Q and K, never forming the score tensor."""
        return gate_target_from_qk(q, k, block_size, **kw)

    @staticmethod
    def compute_gate_loss(gate_soft_scores: torch.Tensor, gate_target: torch.Tensor) -> torch.Tensor:
        """KL(target || soft / sum soft), batchmean (objectives.py:187-221); differentiable in the scores."""
        _check_finite(gate_soft_scores, "gate_soft_scores")
        _check_finite(gate_target, "gate_target")
        _, kl, _ = _GateLossFn.apply(gate_soft_scores, gate_target.detach(), 0.5, 1.0, 0.0)
        return kl

    @staticmethod
    def compute_sparsity_loss(gate_soft_scores: torch.Tensor, tau_target: float) -> torch.Tensor:
        """(mean(soft) - tau)^2 (objectives.py:223-241); differentiable in the scores."""
        _check_finite(gate_soft_scores, "gate_soft_scores")
        _, _, sp = _GateLossFn.apply(gate_soft_scores, None, tau_target, 0.0, 1.0)
        return sp

    def compute_task_loss(self, logits: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        """Next-token cross-entropy (objectives.py:243-266)."""
        _check_finite(logits, "logits")
        shift_logits = logits[..., :-1, :].contiguous()
        shift_labels = labels[..., 1:].contiguous()
        return F.cross_entropy(shift_logits.view(-1, shift_logits.size(-1)), shift_labels.view(-1),
                               ignore_index=-100, label_smoothing=self._label_smoothing)

    def compute(self, logits: torch.Tensor, labels: torch.Tensor, gate_outputs_by_layer: dict,
                attn_scores_by_layer: dict, active_layer_indices: list[int], block_size: int = 64,
                ) -> ObjectiveLossOutput:
        """``L_task + lambda (L_gate + beta L_sparse)`` with the per-layer gate and sparsity
        losses accumulated by Kahan summation (objectives.py:268-361).

        ``attn_scores_by_layer[i]`` may be the score tensor (as the reference's trainer
        passes it) or a ready target: a tensor of the gate's ``[B, H, NBq, NBk]`` shape
        is taken as the target (e.g. from :func:`gate_target_from_qk` or
        :func:`tasft_b200.training_attention`), so the score tensor need not exist.
        """
        device = logits.device
        task_loss = self.compute_task_loss(logits, labels)
        _check_finite(task_loss, "task_loss")
        zero = lambda: torch.tensor(0.0, device=device, dtype=logits.dtype)  # noqa: E731
        gate_sum, gate_comp, sparse_sum, sparse_comp = zero(), zero(), zero(), zero()
        per_layer_gate: dict[int, float] = {}
        per_layer_sparsity: dict[int, float] = {}
        active: list[int] = []
        for layer_idx in active_layer_indices:
            active.append(layer_idx)
            gate_scores = gate_outputs_by_layer[layer_idx]
            given = attn_scores_by_layer[layer_idx]
            if given.shape == gate_scores.shape:
                gate_target = given
            else:
                gate_target = self.compute_gate_target(given, block_size)
            layer_gate_loss = self.compute_gate_loss(gate_scores, gate_target)
            _check_finite(layer_gate_loss, "layer_gate_loss", {"layer": layer_idx})
            per_layer_gate[layer_idx] = layer_gate_loss.item()
            y = layer_gate_loss - gate_comp
            t = gate_sum + y
            gate_comp = (t - gate_sum) - y
            gate_sum = t
            layer_sparse_loss = self.compute_sparsity_loss(gate_scores, self._tau_target)
            _check_finite(layer_sparse_loss, "layer_sparse_loss", {"layer": layer_idx})
            per_layer_sparsity[layer_idx] = gate_scores.mean().item()
            y = layer_sparse_loss - sparse_comp
            t = sparse_sum + y
            sparse_comp = (t - sparse_sum) - y
            sparse_sum = t
        gate_total = gate_sum + self._beta_sparse * sparse_sum
        total_loss = task_loss + self._lambda_gate * gate_total
        _check_finite(total_loss, "total_loss")
        return ObjectiveLossOutput(total=total_loss, task=task_loss, gate=gate_sum, sparse=sparse_sum,
                                   per_layer_gate_loss=per_layer_gate, per_layer_sparsity=per_layer_sparsity,
                                   active_layers=active)


__all__ = ["ObjectiveLossOutput", "TASFTObjective", "gate_backward", "gate_losses", "gate_objective",
           "gate_target_from_qk", "gate_target_from_scores", "training_attention"]
