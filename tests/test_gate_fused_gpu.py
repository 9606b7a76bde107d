"""The fused pool + projection gate kernel (16-bit Q/K, D 64/128, hidden 32/64) against
the two-kernel path it replaces and against the oracle, including the pooled means the
training backward uses and the gradients through the gate."""
from __future__ import annotations

import pytest
import torch

import oracle as O
import tasft_b200 as T

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("dtype,D,hid,Hq,Hk,S", [
    (torch.bfloat16, 128, 32, 8, 2, 1000),
    (torch.bfloat16, 128, 64, 4, 4, 512),
    (torch.float16, 64, 32, 6, 2, 333),
    (torch.float16, 64, 64, 4, 1, 256),
])
def test_fused_gate_matches_unfused_and_oracle(dtype, D, hid, Hq, Hk, S, monkeypatch):
    torch.manual_seed(S)
    g = T.AttnGate(Hq, D, block_size=64, gate_hidden_dim=hid).to(DEV)
    with torch.no_grad():
        g.gate_proj_out.weight.mul_(40)  # spread the scores across tau
    q = torch.randn(2, Hq, S, D, dtype=dtype, device=DEV)
    k = torch.randn(2, Hk, S, D, dtype=dtype, device=DEV)
    fused = g(q, k)
    monkeypatch.setenv("TASFT_GATE_UNFUSED", "1")
    plain = g(q, k)
    monkeypatch.delenv("TASFT_GATE_UNFUSED")
    assert (fused.soft_scores - plain.soft_scores).abs().max().item() <= 1e-5
    # lists and masks are exactly those of the fused kernel's own scores
    hard, kept, num = T.threshold_scores(fused.soft_scores, g.default_threshold, True)
    assert torch.equal(fused.hard_mask, hard)
    assert torch.equal(fused.kept.idx, kept.idx) and torch.equal(fused.kept.cnt, kept.cnt)
    w = [p.detach().cpu() for p in (g.gate_proj_in.weight, g.gate_proj_in.bias, g.gate_proj_out.weight)]
    soft_ref, _, _ = O.gate_forward_gqa(q.float().cpu(), k.float().cpu(), *w, 64, g.default_threshold)
    assert (fused.soft_scores.cpu() - soft_ref).abs().max().item() <= 2e-5


def test_fused_gate_backward_matches_unfused(monkeypatch):
    torch.manual_seed(1)
    g = T.AttnGate(8, 128, block_size=64).to(DEV)
    q = torch.randn(1, 8, 768, 128, dtype=torch.bfloat16, device=DEV)
    k = torch.randn(1, 2, 768, 128, dtype=torch.bfloat16, device=DEV)
    tgt = T.gate_target_from_qk(q, k, 64)
    grads = []
    for unfused in (False, True):
        if unfused:
            monkeypatch.setenv("TASFT_GATE_UNFUSED", "1")
        g.zero_grad()
        out = g(q, k)
        total, _, _ = T.gate_objective(out.soft_scores, tgt)
        total.backward()
        grads.append([p.grad.clone() for p in g.parameters()])
    for a, b in zip(*grads):
        assert (a - b).abs().max().item() <= 1e-5 * max(1.0, b.abs().max().item())
