"""The projection epilogue (tasft_qkv_rope_pool): head split + rotary + the gate's block
pooling in one pass, and the gate run from those means (pooled-input mode), against the
reference's _prepare_qkv / _apply_rotary_pos_emb restated in the oracle
(tasft/modules/tasft_attention.py:615-742, :872-908) and against AttnGate on the rotated
tensors."""
from __future__ import annotations

import pytest
import torch

import oracle as O
import tasft_b200 as T

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rope_tables(B, S, D, dtype, seed):
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2).float() / D))
    pos = torch.arange(S).float() + seed
    ang = torch.outer(pos, inv)
    emb = torch.cat([ang, ang], -1)
    cos, sin = emb.cos().to(dtype), emb.sin().to(dtype)
    return cos.expand(B, S, D).contiguous(), sin.expand(B, S, D).contiguous()


@pytest.mark.parametrize("dtype,B,S,Hq,Hk,D", [
    (torch.bfloat16, 2, 700, 8, 2, 128),
    (torch.float16, 1, 256, 4, 4, 64),
    (torch.float32, 1, 130, 4, 2, 64),
])
def test_epilogue_matches_reference_rotary_and_pooling(dtype, B, S, Hq, Hk, D):
    g = torch.Generator().manual_seed(S)
    ql = torch.randn(B, S, Hq * D, generator=g).to(dtype)
    kl = torch.randn(B, S, Hk * D, generator=g).to(dtype)
    vl = torch.randn(B, S, Hk * D, generator=g).to(dtype)
    cos, sin = _rope_tables(B, S, D, dtype, 3)
    q, k, v, pq, pk = T.qkv_rope_pool(ql.to(DEV), kl.to(DEV), vl.to(DEV), Hq, Hk, cos.to(DEV), sin.to(DEV), 64)
    rq = O.apply_rotary(ql.view(B, S, Hq, D).transpose(1, 2), cos, sin)
    rk = O.apply_rotary(kl.view(B, S, Hk, D).transpose(1, 2), cos, sin)
    assert torch.equal(q.cpu(), rq)  # same element-wise roundings
    assert torch.equal(k.cpu(), rk)
    assert torch.equal(v.cpu(), vl.view(B, S, Hk, D).transpose(1, 2))
    assert (pq.cpu() - O.pool_to_blocks(rq.float(), 64)).abs().max().item() <= 1e-6
    assert (pk.cpu() - O.pool_to_blocks(rk.float(), 64)).abs().max().item() <= 1e-6


def test_gate_from_pooled_means_equals_gate_on_tensors():
    torch.manual_seed(4)
    B, S, Hq, Hk, D = 2, 1000, 8, 2, 128
    ql = torch.randn(B, S, Hq * D, device=DEV).bfloat16()
    kl = torch.randn(B, S, Hk * D, device=DEV).bfloat16()
    vl = torch.randn(B, S, Hk * D, device=DEV).bfloat16()
    cos, sin = _rope_tables(1, S, D, torch.bfloat16, 0)
    q, k, _, pq, pk = T.qkv_rope_pool(ql, kl, vl, Hq, Hk, cos.to(DEV), sin.to(DEV), 64)
    gate = T.AttnGate(Hq, D).to(DEV)
    with torch.no_grad():
        gate.gate_proj_out.weight.mul_(40)
        a = gate(q, k)
    b = gate.forward_pooled(pq, pk, S, S)
    assert (a.soft_scores - b.soft_scores).abs().max().item() <= 1e-5
    hard, kept, _ = T.threshold_scores(b.soft_scores, gate.default_threshold, True)
    assert torch.equal(b.hard_mask, hard) and torch.equal(b.kept.idx, kept.idx)
    assert b.sparsity_ratio == pytest.approx(1.0 - b.hard_mask.float().mean().item())


def test_epilogue_larger_block_pooling():
    g = torch.Generator().manual_seed(9)
    B, S, Hq, Hk, D = 1, 300, 4, 2, 128
    ql, kl, vl = (torch.randn(B, S, h * D, generator=g).bfloat16() for h in (Hq, Hk, Hk))
    cos, sin = _rope_tables(B, S, D, torch.bfloat16, 1)
    q, k, v, pq, pk = T.qkv_rope_pool(ql.to(DEV), kl.to(DEV), vl.to(DEV), Hq, Hk, cos.to(DEV), sin.to(DEV), 128)
    rq = O.apply_rotary(ql.view(B, S, Hq, D).transpose(1, 2), cos, sin)
    assert torch.equal(q.cpu(), rq)
    assert (pq.cpu() - O.pool_to_blocks(rq.float(), 128)).abs().max().item() <= 1e-6


@pytest.mark.parametrize("case", ["fused_proj_shared_tables", "no_rope", "short_sequence"])
def test_epilogue_layouts(case):
    """q/k/v as column slices of one fused [B, S, (Hq + 2 Hk) * D] projection (token stride
    larger than the row), rotary tables shared over the batch, no rotary, S below a block."""
    B, S, Hq, Hk, D = (3, 200, 8, 2, 128) if case != "short_sequence" else (2, 40, 4, 1, 64)
    g = torch.Generator().manual_seed(11)
    fused = torch.randn(B, S, (Hq + 2 * Hk) * D, generator=g).bfloat16()
    ql, kl, vl = fused.split([Hq * D, Hk * D, Hk * D], dim=-1)
    cos, sin = _rope_tables(1, S, D, torch.bfloat16, 5)
    fd = fused.to(DEV)
    qd, kd, vd = fd.split([Hq * D, Hk * D, Hk * D], dim=-1)
    rope = case != "no_rope"
    q, k, v, pq, pk = T.qkv_rope_pool(qd, kd, vd, Hq, Hk, cos.to(DEV) if rope else None,
                                      sin.to(DEV) if rope else None, 64)
    xq = ql.reshape(B, S, Hq, D).transpose(1, 2)
    xk = kl.reshape(B, S, Hk, D).transpose(1, 2)
    rq = O.apply_rotary(xq, cos, sin) if rope else xq
    rk = O.apply_rotary(xk, cos, sin) if rope else xk
    assert torch.equal(q.cpu(), rq)
    assert torch.equal(k.cpu(), rk)
    assert torch.equal(v.cpu(), vl.reshape(B, S, Hk, D).transpose(1, 2))
    assert (pq.cpu() - O.pool_to_blocks(rq.float(), 64)).abs().max().item() <= 1e-6
    assert (pk.cpu() - O.pool_to_blocks(rk.float(), 64)).abs().max().item() <= 1e-6
