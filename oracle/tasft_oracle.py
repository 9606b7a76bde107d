"""CPU restatement of TASFT's gated block-sparse attention path.

TEST INFRASTRUCTURE ONLY. This module is the checker that the CUDA path in
``tasft_b200`` is compared against; it is never the thing measured or shipped.
Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` import it.

Every function restates one step of the reference (``v-code01/tasft``) and cites
the file:line it follows. Parity pins (checked by ``tests/test_oracle_golden.py``):

* the reference's own known-answer tests, restated as golden vectors
  (``tests/unit/test_numerical_correctness.py:40-98``, ``:119-184``, ``:196-238``,
  ``:407-443``, ``:714-721``; ``tests/unit/test_objectives.py:166-227``);
* fixtures produced by importing the reference in the build container
  (``tests/golden/make_golden.py``): ``AttnGate.forward`` outputs,
  ``compute_gate_target``/``compute_gate_loss``/``compute_sparsity_loss`` outputs,
  and the reference Triton kernel run under ``TRITON_INTERPRET=1`` in fp32.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

__all__ = [
    "pool_to_blocks",
    "apply_rotary",
    "gate_forward",
    "gate_forward_gqa",
    "kept_from_mask",
    "mask_from_kept",
    "bsa_prefill_masked_dense",
    "bsa_prefill_blockwise",
    "bsa_decode",
    "decode_combine",
    "training_scores",
    "gate_target",
    "gate_target_from_qk",
    "gate_loss",
    "sparsity_loss",
]


# ---------------------------------------------------------------------------
# AttnGate (tasft/modules/attn_gate.py)
# ---------------------------------------------------------------------------


def pool_to_blocks(x: torch.Tensor, block: int) -> torch.Tensor:
    """Zero-pad S up to a multiple of ``block`` and average each block of tokens.

    Follows ``tasft/modules/attn_gate.py:351-375``: the padding zeros are part of the
    mean (a ragged last block of r tokens is divided by ``block``, not r).
    """
    b, h, s, d = x.shape
    pad = (block - s % block) % block
    if pad:
        x = F.pad(x, (0, 0, 0, pad))
    nb = x.shape[2] // block
    return x.view(b, h, nb, block, d).mean(dim=3)


def gate_forward(
    q: torch.Tensor,
    k: torch.Tensor,
    w_in: torch.Tensor,
    b_in: torch.Tensor,
    w_out: torch.Tensor,
    block: int,
    tau: float,
    is_causal: bool = True,
) -> tuple[torch.Tensor, torch.Tensor, float]:
    """AttnGate forward: pooled pair MLP -> sigmoid -> causal zeroing -> threshold.

    Follows ``tasft/modules/attn_gate.py:377-485`` step for step: pool Q and K
    (``:442-443``), build every (q-block, k-block) pair ``[q_i; k_j]`` (``:450-453``),
    ``Linear(2D->hid) -> ReLU -> Linear(hid->1)`` (``:456-457``), sigmoid (``:459``),
    zero the upper block triangle when causal and ``NB_q == NB_k`` (``:466-473``),
    hard mask ``soft >= tau`` (``:475``) and the sparsity over the full grid (``:477``).
    Computed in the dtype of ``q`` like the reference module. ``w_in`` is
    ``[hid, 2D]``, ``b_in`` ``[hid]``, ``w_out`` ``[1, hid]`` (nn.Linear layouts).
    """
    qb = pool_to_blocks(q, block)
    kb = pool_to_blocks(k, block)
    b, h, nbq, d = qb.shape
    nbk = kb.shape[2]
    q_exp = qb.unsqueeze(3).expand(b, h, nbq, nbk, d)
    k_exp = kb.unsqueeze(2).expand(b, h, nbq, nbk, d)
    cat = torch.cat([q_exp, k_exp], dim=-1)
    dt = q.dtype
    hidden = F.relu(F.linear(cat, w_in.to(dt), b_in.to(dt)))
    logits = F.linear(hidden, w_out.to(dt)).squeeze(-1)
    soft = torch.sigmoid(logits)
    if is_causal and nbq == nbk:
        tri = torch.ones(nbq, nbk, dtype=torch.bool).tril()
        soft = soft * tri
    hard = soft >= tau
    sparsity = 1.0 - hard.float().mean().item()
    return soft, hard, sparsity


def gate_forward_gqa(q, k_kv, w_in, b_in, w_out, block, tau, is_causal=True):
    """Gate over GQA K: expand K to the q-heads first, as every reference caller does.

    The callers repeat K per q-head before calling the gate
    (``tasft/modules/tasft_attention.py:725-729``, ``tasft/inference/tasft_model.py:267-271``,
    ``tasft/inference/vllm_patch.py:183-187``).
    """
    n_rep = q.shape[1] // k_kv.shape[1]
    k = k_kv.repeat_interleave(n_rep, dim=1) if n_rep > 1 else k_kv
    return gate_forward(q, k, w_in, b_in, w_out, block, tau, is_causal)


# ---------------------------------------------------------------------------
# Kept-block index lists (the compact form of a block mask)
# ---------------------------------------------------------------------------


def kept_from_mask(mask: torch.Tensor, causal: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """Ascending kept-KV-block indices per mask row, ``-1`` padded, plus counts.

    The reference kernel visits the kept blocks of a row in ascending order
    (``tasft/kernels/block_sparse_fa.py:192-203``) after the block mask is ANDed with
    the block lower triangle when causal (``:502-508``). The list is that visiting order.
    """
    m = mask.bool().clone()
    nbq, nbk = m.shape[-2], m.shape[-1]
    if causal:
        m &= torch.ones(nbq, nbk, dtype=torch.bool).tril()
    cnt = m.sum(-1).to(torch.int32)
    ar = torch.arange(nbk, dtype=torch.int64).expand_as(m)
    key = torch.where(m, ar, ar + nbk)  # kept first, ascending
    order = key.sort(dim=-1).values
    idx = torch.where(order < nbk, order, torch.full_like(order, -1)).to(torch.int32)
    return idx, cnt


def mask_from_kept(idx: torch.Tensor, cnt: torch.Tensor, nbk: int) -> torch.Tensor:
    """Inverse of :func:`kept_from_mask` (entries past ``cnt`` are ignored)."""
    out = torch.zeros(*idx.shape[:-1], nbk + 1, dtype=torch.bool)
    pos = torch.arange(idx.shape[-1])
    valid = pos < cnt.unsqueeze(-1).long()
    tgt = torch.where(valid, idx.long().clamp(min=0), torch.full_like(idx.long(), nbk))
    out.scatter_(-1, tgt, torch.ones_like(valid))
    out = out[..., :nbk]
    return out


# ---------------------------------------------------------------------------
# Block-sparse prefill (tasft/kernels/block_sparse_fa.py)
# ---------------------------------------------------------------------------


def _expand_kv(q, k, v):
    n_rep = q.shape[1] // k.shape[1]
    if n_rep > 1:
        k = k.repeat_interleave(n_rep, dim=1)
        v = v.repeat_interleave(n_rep, dim=1)
    return k, v


def bsa_prefill_masked_dense(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    block_mask: torch.Tensor,
    block: int,
    causal: bool = True,
) -> torch.Tensor:
    """Masked-dense restatement of the reference block-sparse kernel.

    Element mask = ``repeat(block_mask & tril_blocks) & tril_elements`` (plus the
    ``< S`` bounds), ``-inf`` fill, fp32 softmax, ``p`` cast to the value dtype
    before ``P @ V`` (``tasft/kernels/block_sparse_fa.py:252``) with fp32 accumulation,
    and rows with no kept key give 0 (``:257-258``). K/V may have fewer heads (GQA);
    they are expanded per q-head. ``block_mask`` is ``[B, Hm, NB, NB]`` with ``Hm``
    equal to the q-heads or the kv-heads (then shared by the heads of each group).
    Processed one (b, q-head) at a time to bound memory.
    """
    bsz, hq, s, d = q.shape
    k, v = _expand_kv(q, k, v)
    nb = math.ceil(s / block)
    hm = block_mask.shape[1]
    grp = hq // hm
    scale = 1.0 / math.sqrt(d)
    out = torch.empty_like(q)
    pos = torch.arange(s)
    tri_blocks = torch.ones(nb, nb, dtype=torch.bool).tril()
    for b in range(bsz):
        for h in range(hq):
            bm = block_mask[b, h // grp].bool()
            if causal:
                bm = bm & tri_blocks
            em = bm.repeat_interleave(block, 0).repeat_interleave(block, 1)[:s, :s]
            if causal:
                em = em & (pos[:, None] >= pos[None, :])
            qk = (q[b, h].float() @ k[b, h].float().T) * scale
            qk = qk.masked_fill(~em, float("-inf"))
            m = qk.max(dim=-1, keepdim=True).values
            m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
            p = torch.exp(qk - m)
            l = p.sum(dim=-1, keepdim=True)
            acc = p.to(v.dtype).float() @ v[b, h].float()
            l_safe = torch.where(l > 0, l, torch.ones_like(l))
            out[b, h] = (acc / l_safe).to(q.dtype)
    return out


def bsa_prefill_blockwise(q, k, v, block_mask, block, causal=True):
    """Literal restatement of the reference kernel loop (small shapes only).

    Per (b, h, q-block): ``m=-inf, l=0, acc=0``; for each kept k-block in ascending
    order: ``qk = q k^T * scale``, element causal/bounds ``-inf``, ``m' = max(m, rowmax)``,
    ``alpha = e^(m-m')``, ``p = e^(qk-m')``, ``l = alpha l + sum p``,
    ``acc = alpha acc + (p -> v.dtype) v``; finally ``acc / (l>0 ? l : 1)``.
    Follows ``tasft/kernels/block_sparse_fa.py:169-269`` and the host-side causal
    block triangle at ``:502-508``.
    """
    bsz, hq, s, d = q.shape
    k, v = _expand_kv(q, k, v)
    nb = math.ceil(s / block)
    grp = hq // block_mask.shape[1]
    scale = 1.0 / math.sqrt(d)
    out = torch.zeros_like(q)
    for b in range(bsz):
        for h in range(hq):
            for qb in range(nb):
                q0 = qb * block
                qi = torch.arange(q0, q0 + block)
                qt = torch.zeros(block, d)
                rows = min(block, s - q0)
                qt[:rows] = q[b, h, q0 : q0 + rows].float()
                m_i = torch.full((block,), float("-inf"))
                l_i = torch.zeros(block)
                acc = torch.zeros(block, d)
                for kb in range(nb):
                    if not bool(block_mask[b, h // grp, qb, kb]):
                        continue
                    if causal and kb > qb:
                        continue
                    k0 = kb * block
                    krows = min(block, s - k0)
                    kt = torch.zeros(block, d)
                    vt = torch.zeros(block, d, dtype=v.dtype)
                    kt[:krows] = k[b, h, k0 : k0 + krows].float()
                    vt[:krows] = v[b, h, k0 : k0 + krows]
                    ki = torch.arange(k0, k0 + block)
                    qk = (qt @ kt.T) * scale
                    valid = (qi[:, None] < s) & (ki[None, :] < s)
                    if causal:
                        valid &= qi[:, None] >= ki[None, :]
                    qk = torch.where(valid, qk, torch.full_like(qk, float("-inf")))
                    m_new = torch.maximum(m_i, qk.max(dim=1).values)
                    alpha = torch.exp(m_i - m_new)
                    p = torch.exp(qk - m_new[:, None])
                    # rows that are still fully masked: exp(-inf - -inf) = nan -> treat as 0
                    alpha = torch.nan_to_num(alpha, nan=1.0)
                    p = torch.nan_to_num(p, nan=0.0)
                    l_i = alpha * l_i + p.sum(dim=1)
                    acc = alpha[:, None] * acc + p.to(v.dtype).float() @ vt.float()
                    m_i = m_new
                l_safe = torch.where(l_i > 0, l_i, torch.ones_like(l_i))
                res = acc / l_safe[:, None]
                out[b, h, q0 : q0 + rows] = res[:rows].to(q.dtype)
    return out


# ---------------------------------------------------------------------------
# Block-sparse decode (new capability; no reference counterpart)
# ---------------------------------------------------------------------------


def bsa_decode(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    kv_len: torch.Tensor,
    kept_idx: torch.Tensor,
    kept_cnt: torch.Tensor,
    block: int,
    return_lse: bool = False,
):
    """Single-query attention over the kept KV blocks of each (sequence, kv-head).

    The reference has no sparse decode (vLLM decode is delegated to the dense
    PagedAttention forward, ``tasft/inference/vllm_patch.py:189-196``). Specification:
    the query of q-head h attends to the keys of kv-head ``h // (Hq/Hkv)`` at positions
    in the kept blocks and below ``kv_len[b]``, with the reference kernel's softmax
    (``tasft/kernels/block_sparse_fa.py:245-258``, fp32, empty -> 0), scale ``1/sqrt(D)``.
    ``q`` ``[B,Hq,D]``, caches ``[B,Hkv,L,D]``, lists ``[B,Hkv,NBmax]``/``[B,Hkv]``.
    With ``return_lse`` also returns ``(m, l)`` in base-e units for split combines.
    """
    bsz, hq, d = q.shape
    hkv = k_cache.shape[1]
    grp = hq // hkv
    scale = 1.0 / math.sqrt(d)
    out = torch.zeros(bsz, hq, d, dtype=torch.float32)
    m_out = torch.full((bsz, hq), float("-inf"))
    l_out = torch.zeros(bsz, hq)
    for b in range(bsz):
        n = int(kv_len[b])
        for g in range(hkv):
            c = int(kept_cnt[b, g])
            blocks = kept_idx[b, g, :c].long()
            if c == 0:
                continue
            pos = (blocks[:, None] * block + torch.arange(block)[None, :]).reshape(-1)
            pos = pos[pos < n]
            if pos.numel() == 0:
                continue
            kk = k_cache[b, g, pos].float()
            vv = v_cache[b, g, pos].float()
            for j in range(grp):
                h = g * grp + j
                s = (kk @ q[b, h].float()) * scale
                m = s.max()
                p = torch.exp(s - m)
                l = p.sum()
                out[b, h] = (p @ vv) / l
                m_out[b, h] = m
                l_out[b, h] = l
    out = out.to(q.dtype)
    if return_lse:
        return out, m_out, l_out
    return out


def decode_combine(o_parts, m_parts, l_parts):
    """Log-sum-exp combine of split-KV partial results (``o`` normalised per part).

    ``o_parts`` ``[G, ..., D]`` fp32, ``m_parts``/``l_parts`` ``[G, ...]`` base-e.
    Parts with ``l == 0`` contribute nothing; all-empty rows give 0.
    """
    m = m_parts.max(dim=0).values
    m_safe = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    w = torch.where(l_parts > 0, l_parts * torch.exp(m_parts - m_safe), torch.zeros_like(l_parts))
    denom = w.sum(dim=0)
    num = (w.unsqueeze(-1) * o_parts).sum(dim=0)
    return torch.where(denom.unsqueeze(-1) > 0, num / denom.clamp_min(1e-38).unsqueeze(-1), torch.zeros_like(num))


# ---------------------------------------------------------------------------
# Gate target and losses (tasft/training/objectives.py)
# ---------------------------------------------------------------------------


def apply_rotary(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotary embedding as ``_apply_rotary_pos_emb`` applies it
    (``tasft/modules/tasft_attention.py:872-908``): ``x * cos + rotate_half(x) * sin`` with
    ``rotate_half(x) = cat(-x[..., D/2:], x[..., :D/2])``, element-wise in ``x``'s dtype;
    ``cos`` / ``sin`` ``[B, S, D]`` gain a head axis."""
    if cos.ndim == 3:
        cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return (x * cos) + (rot * sin)


def training_scores(q: torch.Tensor, k: torch.Tensor) -> torch.Tensor:
    """Pre-softmax training scores as ``TASFTAttention._training_forward`` builds them.

    ``(Q K^T) * scale`` in the model dtype, then ``+ triu(-inf, 1)``
    (``tasft/modules/tasft_attention.py:427-443``). K is GQA-expanded by the caller.
    """
    d = q.shape[-1]
    scale = 1.0 / (d**0.5)
    w = torch.matmul(q, k.transpose(-2, -1)) * scale
    sq, sk = q.shape[2], k.shape[2]
    cm = torch.triu(torch.full((sq, sk), float("-inf"), dtype=w.dtype), diagonal=1)
    return w + cm


def gate_target(
    scores: torch.Tensor,
    block: int,
    temperature: float = 1.0,
    clamp: float | None = None,
) -> torch.Tensor:
    """Block importance target: ``-inf`` pad, 2-D max-pool, softmax over the NB^2 grid.

    ``temperature=1, clamp=None`` follows ``tasft/training/objectives.py:128-185`` (the
    one the trainer uses, ``tasft/training/trainer.py:421``); ``temperature=2, clamp=50``
    follows the alternate ``TASFTAttention._compute_gate_target``
    (``tasft/modules/tasft_attention.py:220-290``: clamp finite values, softmax(x/T)).
    """
    if torch.isnan(scores).any() or (scores == float("inf")).any():
        raise ValueError("non-finite attn_scores")
    b, h, sq, sk = scores.shape
    pq = (block - sq % block) % block
    pk = (block - sk % block) % block
    if pq or pk:
        scores = F.pad(scores, (0, pk, 0, pq), value=-math.inf)
    pooled = F.max_pool2d(scores, kernel_size=block, stride=block)
    if clamp is not None:
        fin = torch.isfinite(pooled)
        pooled = torch.where(fin, pooled.clamp(-clamp, clamp), pooled)
    nbq, nbk = pooled.shape[2], pooled.shape[3]
    flat = pooled.reshape(b, h, nbq * nbk)
    return F.softmax(flat / temperature if temperature != 1.0 else flat, dim=-1).reshape(b, h, nbq, nbk)


def gate_target_from_qk(q, k, block, temperature=1.0, clamp=None):
    """Gate target from Q, K via the training-scores path, one (b, h) at a time."""
    k, _ = _expand_kv(q, k, k)
    bsz, hq = q.shape[:2]
    outs = []
    for b in range(bsz):
        row = []
        for h in range(hq):
            sc = training_scores(q[b : b + 1, h : h + 1], k[b : b + 1, h : h + 1])
            row.append(gate_target(sc, block, temperature, clamp))
        outs.append(torch.cat(row, dim=1))
    return torch.cat(outs, dim=0)


_EPS = 1e-8


def gate_loss(soft: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    """KL(target || normalised gate), batchmean over B.

    Follows ``tasft/training/objectives.py:187-221``: ``g = soft / (sum soft + 1e-8)``
    over the flattened grid, ``kl_div(log(g + 1e-8), target, 'batchmean')`` which is
    ``sum target * (log target - log(g + 1e-8)) / B`` with ``0 log 0 = 0``.
    """
    b, h, nq, nk = soft.shape
    g = soft.reshape(b, h, nq * nk)
    g = g / (g.sum(dim=-1, keepdim=True) + _EPS)
    t = target.reshape(b, h, nq * nk)
    return F.kl_div(torch.log(g + _EPS), t, reduction="batchmean", log_target=False)


def sparsity_loss(soft: torch.Tensor, tau: float) -> torch.Tensor:
    """``(mean(soft) - tau)^2`` (``tasft/training/objectives.py:223-241``)."""
    return (soft.mean() - tau) ** 2
