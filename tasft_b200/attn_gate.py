"""Drop-in ``AttnGate`` whose forward is the fused sm_100a mask builder.

Mirrors ``tasft/modules/attn_gate.py``: same constructor and validation (:271-338), the
same parameters ``gate_proj_in.{weight,bias}`` / ``gate_proj_out.weight`` and init
(:340-349) so bundle state dicts load unchanged, and ``forward(q, k, threshold)``
returning :class:`GateOutput` (:230-246, :377-485). Additions: K may carry the kv-heads
of a GQA group (no ``repeat_interleave``), ``Sq`` may differ from ``Sk`` (decode
scoring), and the output also carries the kept-block lists. Scores are fp32. The
sparsity ratio is read from the device lazily, on first access.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass, field

import torch
from torch import nn

from tasft_b200 import _lib as L
from tasft_b200.exceptions import ValidationError
from tasft_b200.types import KeptBlocks


@dataclass(frozen=True)
class GateOutput:
    """Result of :meth:`AttnGate.forward` (fields of ``tasft/modules/attn_gate.py:230-246``)."""

    soft_scores: torch.Tensor
    hard_mask: torch.Tensor
    num_blocks_q: int
    num_blocks_k: int
    kept: KeptBlocks | None = None
    _num_kept: torch.Tensor | None = field(default=None, repr=False)
    _ratio: list = field(default_factory=list, repr=False)

    @property
    def sparsity_ratio_device(self) -> torch.Tensor:
        """``1 - mean(hard_mask)`` as a device scalar (fp32): no host synchronisation, for
        callers that branch on the device or log asynchronously."""
        total = self.hard_mask.numel()
        kept = self._num_kept if self._num_kept is not None else self.hard_mask.sum()
        return 1.0 - kept.reshape(()).float() / max(total, 1)

    @property
    def sparsity_ratio(self) -> float:
        """``1 - mean(hard_mask)`` over the full grid (host sync on first access)."""
        if not self._ratio:
            total = self.hard_mask.numel()
            kept = int(self._num_kept.item()) if self._num_kept is not None else int(self.hard_mask.sum().item())
            self._ratio.append(1.0 - kept / max(total, 1))
        return self._ratio[0]


class _GateFn(torch.autograd.Function):
    """Soft scores with a CUDA backward to the gate parameters and to q/k."""

    @staticmethod
    def forward(ctx, q, k, w_in, b_in, w_out, gate, tau):  # noqa: D401
        res = gate._launch(q, k, tau, want_pooled=True)
        ctx.save_for_backward(res["pooled_q"], res["pooled_k"], res["soft"], w_in, b_in, w_out)
        ctx.meta = (q.shape, k.shape, q.dtype, gate.block_size, gate.is_causal)
        ctx.mark_non_differentiable(res["hard"])
        return res["soft"], res["hard"], res["kept_idx"], res["kept_cnt"], res["num_kept"]

    @staticmethod
    def backward(ctx, d_soft, *_):
        from tasft_b200.training import gate_backward  # noqa: PLC0415

        pq, pk, soft, w_in, b_in, w_out = ctx.saved_tensors
        qshape, kshape, qdtype, block, causal = ctx.meta
        g = gate_backward(pq, pk, soft, d_soft.contiguous().float(), w_in, b_in, w_out, causal,
                          need_inputs=ctx.needs_input_grad[0] or ctx.needs_input_grad[1])
        dq = dk = None
        if ctx.needs_input_grad[0]:
            dq = _unpool(g["d_pooled_q"], qshape, block).to(qdtype)
        if ctx.needs_input_grad[1]:
            dk = _unpool(g["d_pooled_k"], kshape, block).to(qdtype)
        return dq, dk, g["d_w_in"], g["d_b_in"], g["d_w_out"].view(1, -1), None, None


def _unpool(d_pooled: torch.Tensor, shape, block: int) -> torch.Tensor:
    """Gradient of the zero-padded block mean: every token of block i gets d_i / block."""
    b, h, s, d = shape
    rep = (d_pooled / block).repeat_interleave(block, dim=2)
    return rep[:, :, :s, :]


class AttnGate(nn.Module):
    """Learnable block-importance predictor (see ``tasft/modules/attn_gate.py:249-338``)."""

    def __init__(
        self,
        num_heads: int,
        head_dim: int,
        block_size: int = 64,
        gate_hidden_dim: int | None = None,
        default_threshold: float = 0.5,
        is_causal: bool = True,
    ) -> None:
        super().__init__()
        if num_heads <= 0:
            raise ValidationError(f"num_heads must be positive, got {num_heads}", context={"num_heads": num_heads})
        if head_dim <= 0:
            raise ValidationError(f"head_dim must be positive, got {head_dim}", context={"head_dim": head_dim})
        if block_size <= 0:
            raise ValidationError(f"block_size must be positive, got {block_size}", context={"block_size": block_size})
        if not 0.0 <= default_threshold <= 1.0:
            raise ValidationError(f"default_threshold must be in [0, 1], got {default_threshold}",
                                  context={"default_threshold": default_threshold})
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.block_size = block_size
        self.default_threshold = default_threshold
        self.is_causal = is_causal
        hid = gate_hidden_dim if gate_hidden_dim is not None else max(32, head_dim // 4)
        self.gate_hidden_dim = hid
        self.gate_proj_in = nn.Linear(2 * head_dim, hid, bias=True)
        self.gate_proj_out = nn.Linear(hid, 1, bias=False)
        self._init_weights()

    def _init_weights(self) -> None:
        nn.init.xavier_uniform_(self.gate_proj_in.weight)
        nn.init.zeros_(self.gate_proj_in.bias)
        nn.init.normal_(self.gate_proj_out.weight, std=0.01)

    # ------------------------------------------------------------------
    def _validate(self, q: torch.Tensor, k: torch.Tensor) -> None:
        if q.ndim != 4:
            raise ValidationError(f"Expected 4D Q tensor [B, H, S, D], got ndim={q.ndim}",
                                  context={"q_shape": list(q.shape)})
        if k.ndim != 4:
            raise ValidationError(f"Expected 4D K tensor [B, H, S, D], got ndim={k.ndim}",
                                  context={"k_shape": list(k.shape)})
        B, H, S, D = q.shape
        if k.shape[0] != B or k.shape[3] != D or k.shape[1] <= 0 or H % k.shape[1] != 0:
            raise ValidationError(f"Q and K must have same shape, got {q.shape} vs {k.shape}",
                                  context={"q_shape": list(q.shape), "k_shape": list(k.shape)})
        if self.num_heads != H:
            raise ValidationError(f"Expected {self.num_heads} heads, got {H}",
                                  context={"expected_heads": self.num_heads, "actual_heads": H})
        if self.head_dim != D:
            raise ValidationError(f"Expected head_dim={self.head_dim}, got {D}",
                                  context={"expected_dim": self.head_dim, "actual_dim": D})
        if S == 0 or k.shape[2] == 0:
            raise ValidationError("Sequence length must be > 0", context={"seq_len": S})
        L.require_cuda(q, k)

    def _launch(self, q: torch.Tensor, k: torch.Tensor, tau: float, want_pooled: bool = False,
                want_lists: bool = True) -> dict:
        q = q.detach().contiguous()
        k = k.detach().contiguous()
        B, Hq, Sq, D = q.shape
        Hk, Sk = k.shape[1], k.shape[2]
        blk = self.block_size
        nbq, nbk = math.ceil(Sq / blk), math.ceil(Sk / blk)
        dev = q.device
        hid = self.gate_hidden_dim
        w_in = self.gate_proj_in.weight.detach().float().contiguous()
        b_in = self.gate_proj_in.bias.detach().float().contiguous()
        w_out = self.gate_proj_out.weight.detach().float().contiguous().view(-1)
        soft = torch.empty(B, Hq, nbq, nbk, dtype=torch.float32, device=dev)
        hard = torch.empty(B, Hq, nbq, nbk, dtype=torch.bool, device=dev)
        idx = torch.empty(B, Hq, nbq, nbk, dtype=torch.int32, device=dev) if want_lists else None
        cnt = torch.empty(B, Hq, nbq, dtype=torch.int32, device=dev) if want_lists else None
        num = torch.zeros(1, dtype=torch.int32, device=dev)
        pq = torch.empty(B, Hq, nbq, D, dtype=torch.float32, device=dev) if want_pooled else None
        pk = torch.empty(B, Hk, nbk, D, dtype=torch.float32, device=dev) if want_pooled else None
        lib = L.lib()
        ws_bytes = lib.tasft_gate_workspace_size(B, Hq, Hk, Sq, Sk, blk, hid, D)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        args = L.GateArgs(
            q=q.data_ptr(), k=k.data_ptr(), q_stride=L.strides4(q), k_stride=L.strides4(k),
            B=B, Hq=Hq, Hk=Hk, Sq=Sq, Sk=Sk, D=D, block=blk, dtype=L.dtype_code(q), hidden=hid,
            w_in=w_in.data_ptr(), b_in=b_in.data_ptr(), w_out=w_out.data_ptr(),
            causal=int(self.is_causal), tau=float(tau), soft=soft.data_ptr(), hard=hard.data_ptr(),
            kept_idx=L.ptr(idx), kept_cnt=L.ptr(cnt), num_kept=num.data_ptr(),
            pooled_q=L.ptr(pq), pooled_k=L.ptr(pk), workspace=ws.data_ptr(), workspace_bytes=ws_bytes,
        )
        L.check(lib.tasft_gate_mask_build(args, L.stream_ptr(dev)), "tasft_gate_mask_build",
                shape=[B, Hq, Hk, Sq, Sk, D])
        return {"soft": soft, "hard": hard, "kept_idx": idx, "kept_cnt": cnt, "num_kept": num,
                "pooled_q": pq, "pooled_k": pk, "nbq": nbq, "nbk": nbk}

    def forward(self, q: torch.Tensor, k: torch.Tensor, threshold: float | None = None) -> GateOutput:
        tau = threshold if threshold is not None else self.default_threshold
        self._validate(q, k)
        params = (self.gate_proj_in.weight, self.gate_proj_in.bias, self.gate_proj_out.weight)
        needs_grad = torch.is_grad_enabled() and (
            q.requires_grad or k.requires_grad or any(p.requires_grad for p in params))
        if needs_grad:
            soft, hard, idx, cnt, num = _GateFn.apply(q, k, *params, self, tau)
            nbq, nbk = soft.shape[2], soft.shape[3]
        else:
            r = self._launch(q, k, tau)
            soft, hard, idx, cnt, num, nbq, nbk = (r["soft"], r["hard"], r["kept_idx"], r["kept_cnt"],
                                                   r["num_kept"], r["nbq"], r["nbk"])
        return GateOutput(soft_scores=soft, hard_mask=hard, num_blocks_q=nbq, num_blocks_k=nbk,
                          kept=KeptBlocks(idx, cnt), _num_kept=num)

    def forward_pooled(self, pooled_q: torch.Tensor, pooled_k: torch.Tensor, seq_q: int, seq_k: int,
                       threshold: float | None = None) -> GateOutput:
        """The gate from block means already computed by :func:`qkv_rope_pool`
        (``pooled_q [B, Hq, NBq, D]``, ``pooled_k [B, Hk, NBk, D]`` fp32): the projection and
        pair kernels only, no pass over Q and K. Inference only (no autograd)."""
        tau = threshold if threshold is not None else self.default_threshold
        L.require_cuda(pooled_q, pooled_k)
        B, Hq, nbq, D = pooled_q.shape
        Hk, nbk = pooled_k.shape[1], pooled_k.shape[2]
        if Hq != self.num_heads or D != self.head_dim or Hq % Hk:
            raise ValidationError("pooled means do not match the gate",
                                  context={"pooled_q": list(pooled_q.shape), "pooled_k": list(pooled_k.shape)})
        blk = self.block_size
        if math.ceil(seq_q / blk) != nbq or math.ceil(seq_k / blk) != nbk:
            raise ValidationError("sequence lengths do not match the pooled block counts",
                                  context={"seq_q": seq_q, "seq_k": seq_k, "nbq": nbq, "nbk": nbk})
        dev = pooled_q.device
        pq = pooled_q.float().contiguous()
        pk = pooled_k.float().contiguous()
        hid = self.gate_hidden_dim
        w_in = self.gate_proj_in.weight.detach().float().contiguous()
        b_in = self.gate_proj_in.bias.detach().float().contiguous()
        w_out = self.gate_proj_out.weight.detach().float().contiguous().view(-1)
        soft = torch.empty(B, Hq, nbq, nbk, dtype=torch.float32, device=dev)
        hard = torch.empty(B, Hq, nbq, nbk, dtype=torch.bool, device=dev)
        idx = torch.empty(B, Hq, nbq, nbk, dtype=torch.int32, device=dev)
        cnt = torch.empty(B, Hq, nbq, dtype=torch.int32, device=dev)
        num = torch.zeros(1, dtype=torch.int32, device=dev)
        lib = L.lib()
        ws_bytes = lib.tasft_gate_workspace_size(B, Hq, Hk, seq_q, seq_k, blk, hid, D)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        args = L.GateArgs(
            q=None, k=None, B=B, Hq=Hq, Hk=Hk, Sq=seq_q, Sk=seq_k, D=D, block=blk, dtype=L.F32, hidden=hid,
            w_in=w_in.data_ptr(), b_in=b_in.data_ptr(), w_out=w_out.data_ptr(), causal=int(self.is_causal),
            tau=float(tau), soft=soft.data_ptr(), hard=hard.data_ptr(), kept_idx=idx.data_ptr(),
            kept_cnt=cnt.data_ptr(), num_kept=num.data_ptr(), pooled_q=pq.data_ptr(), pooled_k=pk.data_ptr(),
            workspace=ws.data_ptr(), workspace_bytes=ws_bytes,
        )
        L.check(lib.tasft_gate_mask_build(args, L.stream_ptr(dev)), "tasft_gate_mask_build (pooled)",
                shape=[B, Hq, Hk, nbq, nbk, D])
        return GateOutput(soft_scores=soft, hard_mask=hard, num_blocks_q=nbq, num_blocks_k=nbk,
                          kept=KeptBlocks(idx, cnt), _num_kept=num)

    def compute_sparsity(self, soft_scores: torch.Tensor, threshold: float) -> float:
        """``1 - mean(soft >= tau)`` (attn_gate.py:487-497)."""
        return 1.0 - (soft_scores >= threshold).float().mean().item()

    @property
    def num_parameters(self) -> int:
        return sum(p.numel() for p in self.parameters() if p.requires_grad)

    def extra_repr(self) -> str:
        return (f"num_heads={self.num_heads}, head_dim={self.head_dim}, block_size={self.block_size}, "
                f"gate_hidden_dim={self.gate_hidden_dim}, default_threshold={self.default_threshold}, "
                f"is_causal={self.is_causal}, params={self.num_parameters}")


def threshold_scores(soft: torch.Tensor, tau: float, causal: bool) -> tuple[torch.Tensor, KeptBlocks, torch.Tensor]:
    """Hard mask and kept lists from given fp32 scores (bit-exact ``soft >= tau``)."""
    L.require_cuda(soft)
    s = soft.float().contiguous()
    nbq, nbk = s.shape[-2], s.shape[-1]
    rows = s.numel() // nbk
    hard = torch.empty(s.shape, dtype=torch.bool, device=s.device)
    idx = torch.empty(s.shape, dtype=torch.int32, device=s.device)
    cnt = torch.empty(s.shape[:-1], dtype=torch.int32, device=s.device)
    num = torch.zeros(1, dtype=torch.int32, device=s.device)
    args = L.ThresholdArgs(soft=s.data_ptr(), rows=rows, NBq=nbq, NBk=nbk, causal=int(causal), tau=float(tau),
                           hard=hard.data_ptr(), kept_idx=idx.data_ptr(), kept_cnt=cnt.data_ptr(),
                           num_kept=num.data_ptr())
    L.check(L.lib().tasft_mask_from_scores(args, L.stream_ptr(s.device)), "tasft_mask_from_scores")
    return hard, KeptBlocks(idx, cnt), num


def qkv_rope_pool(q_lin: torch.Tensor, k_lin: torch.Tensor, v_lin: torch.Tensor, num_heads: int,
                  num_kv_heads: int, cos: torch.Tensor | None = None, sin: torch.Tensor | None = None,
                  block: int = 64):
    """Projection epilogue (``tasft_qkv_rope_pool``): ``[B, S, H*D]`` projection outputs ->
    rotated ``q [B, Hq, S, D]``, ``k, v [B, Hk, S, D]`` and the fp32 block means of q and k
    for :meth:`AttnGate.forward_pooled`, in one pass. ``cos`` / ``sin`` ``[B or 1, S, D]`` in
    the model dtype as a HF rotary embedding returns them (None: no rotation). Follows
    ``TASFTAttention._prepare_qkv`` (``tasft/modules/tasft_attention.py:615-742``) and
    ``_apply_rotary_pos_emb`` (``:872-908``) without the per-q-head repeat of K/V."""
    L.require_cuda(q_lin, k_lin, v_lin)
    B, S, qd = q_lin.shape
    D = qd // num_heads
    if qd != num_heads * D or k_lin.shape != (B, S, num_kv_heads * D) or v_lin.shape != k_lin.shape:
        raise ValidationError("projection shapes do not match the head counts",
                              context={"q": list(q_lin.shape), "k": list(k_lin.shape), "v": list(v_lin.shape)})
    dev, dt = q_lin.device, q_lin.dtype
    qi, ki, vi = (x if x.stride(-1) == 1 else x.contiguous() for x in (q_lin, k_lin, v_lin))
    nb = math.ceil(S / block)
    q = torch.empty(B, num_heads, S, D, dtype=dt, device=dev)
    k = torch.empty(B, num_kv_heads, S, D, dtype=dt, device=dev)
    v = torch.empty_like(k)
    pq = torch.empty(B, num_heads, nb, D, dtype=torch.float32, device=dev)
    pk = torch.empty(B, num_kv_heads, nb, D, dtype=torch.float32, device=dev)
    rope = cos is not None
    if rope:
        if cos.ndim == 2:
            cos, sin = cos.unsqueeze(0), sin.unsqueeze(0)
        cos = cos.to(dt).contiguous()
        sin = sin.to(dt).contiguous()
        cs_stride = (cos.stride(0) if cos.shape[0] == B and B > 1 else 0, cos.stride(1))
    else:
        cs_stride = (0, 0)
    args = L.QkvArgs(
        q_in=qi.data_ptr(), k_in=ki.data_ptr(), v_in=vi.data_ptr(), q_in_stride=(C.c_int64 * 2)(qi.stride(0), qi.stride(1)),
        k_in_stride=(C.c_int64 * 2)(ki.stride(0), ki.stride(1)), v_in_stride=(C.c_int64 * 2)(vi.stride(0), vi.stride(1)),
        cos=cos.data_ptr() if rope else None, sin=sin.data_ptr() if rope else None,
        cs_stride=(C.c_int64 * 2)(*cs_stride), q_out=q.data_ptr(), k_out=k.data_ptr(), v_out=v.data_ptr(),
        pooled_q=pq.data_ptr(), pooled_k=pk.data_ptr(), B=B, Hq=num_heads, Hk=num_kv_heads, S=S, D=D, block=block,
        dtype=L.dtype_code(q_lin), rope=int(rope),
    )
    L.check(L.lib().tasft_qkv_rope_pool(args, L.stream_ptr(dev)), "tasft_qkv_rope_pool", shape=[B, S, num_heads, D])
    return q, k, v, pq, pk


def calibrate_tau(soft_scores: torch.Tensor, target_sparsity: float, *, sync: bool = True):
    """Threshold that keeps ``round((1 - target_sparsity) * numel)`` of the given gate scores.

    Measured replacement for the reference bundle's weight-norm sparsity estimate
    (``tasft/bundle/export.py:327-360``): run the gate on calibration inputs, pass its
    ``soft_scores`` (the full grid: causal zeros count, as in the reference's
    ``sparsity_ratio``, ``attn_gate.py:477``), get the layer's tau. Exact (a radix select on
    the device, ``tasft_calibrate_tau``); ties at tau are kept, so the achieved sparsity can
    only be lower. Returns ``(tau, achieved_sparsity)`` as floats (one host sync), or as
    device scalars with ``sync=False``.
    """
    L.require_cuda(soft_scores)
    if not 0.0 <= target_sparsity <= 1.0:
        raise ValidationError(f"target_sparsity must be in [0, 1], got {target_sparsity}",
                              context={"target_sparsity": target_sparsity})
    s = soft_scores.detach().float().contiguous().view(-1)
    n = s.numel()
    keep = int(round((1.0 - target_sparsity) * n))
    tau = torch.empty((), dtype=torch.float32, device=s.device)
    kept = torch.empty((), dtype=torch.int64, device=s.device)
    args = L.CalibArgs(scores=s.data_ptr(), n=n, keep=keep, tau=tau.data_ptr(), kept=kept.data_ptr())
    L.check(L.lib().tasft_calibrate_tau(args, L.stream_ptr(s.device)), "tasft_calibrate_tau")
    achieved = 1.0 - kept.double() / n
    if not sync:
        return tau, achieved
    return float(tau.item()), float(achieved.item())


def measured_sparsity_profile(gates: dict, calib_qk: dict, target_sparsity: float) -> dict:
    """Per-layer ``(tau, achieved_sparsity)`` measured on calibration Q/K, in the shape of the
    reference exporter's ``_compute_sparsity_profile`` (``tasft/bundle/export.py:327-360``):
    ``gates[i]`` an ``AttnGate``, ``calib_qk[i] = (q, k)`` that layer's inputs."""
    out = {}
    with torch.no_grad():
        for i in sorted(gates):
            q, k = calib_qk[i]
            out[i] = calibrate_tau(gates[i](q, k).soft_scores, target_sparsity)
    return out


__all__ = ["AttnGate", "GateOutput", "calibrate_tau", "measured_sparsity_profile", "qkv_rope_pool",
           "threshold_scores"]
