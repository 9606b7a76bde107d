"""The training-side drop-in on the GPU: ``TASFTObjective`` (gate target from a score
tensor, differentiable gate and sparsity losses, ``compute`` with Kahan accumulation),
the explicit ``DENSE_FALLBACK`` backend, the BASELINE CPU-runnable config (C1) end to end
in fp32, and the tensor-core gate target at D=128 against the oracle.

References: ``tasft/training/objectives.py:128-361``, ``tasft/kernels/block_sparse_fa.py:340-359``,
``tasft/modules/tasft_attention.py:220-290``. Checkers are the oracle (pinned to the
reference) and the reference-run golden fixtures.
"""
from __future__ import annotations

import math

import pytest
import torch

import oracle as O
import tasft_b200 as T
from tasft_b200 import masks as M
from tasft_b200.exceptions import NaNDetectedError
from tasft_b200.training import ObjectiveLossOutput, TASFTObjective, gate_target_from_scores

pytestmark = pytest.mark.gpu
DEV = "cuda"
FP32_ATOL = 1e-5
BF16_ATOL = 2e-2


def test_compute_gate_target_matches_reference_fixtures(golden):
    for case in golden["objective"]:
        got = TASFTObjective.compute_gate_target(case["scores"].to(DEV), case["block"])
        assert got.dtype == case["target"].dtype
        assert (got.cpu() - case["target"]).abs().max().item() <= 1e-6


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("Sq,Sk,block", [(1024, 1024, 64), (100, 130, 32), (256, 192, 128), (77, 77, 7)])
def test_gate_target_from_scores_matches_oracle(dtype, Sq, Sk, block):
    g = torch.Generator().manual_seed(Sq * 7 + block)
    B, H = 2, 3
    sc = (torch.randn(B, H, Sq, Sk, generator=g) * 4).to(dtype)
    if Sq == Sk:  # pre-softmax training scores carry -inf above the diagonal
        sc = sc + torch.triu(torch.full((Sq, Sk), float("-inf")), 1).to(dtype)
    got = gate_target_from_scores(sc.to(DEV), block, out_dtype=torch.float32)
    ref = O.gate_target(sc.float(), block)
    assert (got.cpu() - ref).abs().max().item() <= FP32_ATOL
    # the alternate target of TASFTAttention._compute_gate_target (T=2, clamp 50)
    got2 = gate_target_from_scores(sc.to(DEV), block, temperature=2.0, clamp=50.0, out_dtype=torch.float32)
    ref2 = O.gate_target(sc.float(), block, temperature=2.0, clamp=50.0)
    assert (got2.cpu() - ref2).abs().max().item() <= FP32_ATOL


def test_gate_target_from_scores_strided_view():
    # a non-contiguous view of a larger buffer (rows strided by 2): the scalar load path
    base = torch.randn(1, 2, 256, 2 * 256, device=DEV)
    sc = base[..., ::2]
    got = gate_target_from_scores(sc, 64, out_dtype=torch.float32)
    ref = O.gate_target(sc.float().cpu(), 64)
    assert (got.cpu() - ref).abs().max().item() <= FP32_ATOL


def test_gate_target_from_scores_rejects_nan_and_pos_inf_like_the_reference():
    sc = torch.randn(1, 1, 128, 128, device=DEV)
    sc[0, 0, 3, 5] = float("nan")
    with pytest.raises(NaNDetectedError, match="NaN=True, Inf=False"):
        TASFTObjective.compute_gate_target(sc, 64)
    sc[0, 0, 3, 5] = float("inf")
    with pytest.raises(NaNDetectedError, match="NaN=False, Inf=True"):
        TASFTObjective.compute_gate_target(sc, 64)
    sc[0, 0, 3, 5] = float("-inf")  # allowed: causal masking
    TASFTObjective.compute_gate_target(sc, 64)
    with pytest.raises(ValueError):
        TASFTObjective.compute_gate_target(sc, 0)


def _soft(B, H, nb, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.rand(B, H, nb, nb, generator=g) * 0.98 + 0.01


def test_gate_and_sparsity_losses_backpropagate_like_reference_autograd():
    B, H, nb = 2, 4, 16
    soft = _soft(B, H, nb, 3)
    tgt = O.gate_target(torch.randn(B, H, nb * 64, nb * 64) * 3, 64)
    # reference autograd on the CPU (the oracle restates objectives.py:187-241 with torch ops)
    s_ref = soft.clone().requires_grad_(True)
    kl_ref = O.gate_loss(s_ref, tgt)
    sp_ref = O.sparsity_loss(s_ref, 0.8)
    (kl_ref + 0.37 * sp_ref).backward()
    s = soft.to(DEV).requires_grad_(True)
    kl = TASFTObjective.compute_gate_loss(s, tgt.to(DEV))
    sp = TASFTObjective.compute_sparsity_loss(s, 0.8)
    (kl + 0.37 * sp).backward()
    assert abs(kl.item() - kl_ref.item()) <= 1e-5 * max(1.0, abs(kl_ref.item()))
    assert abs(sp.item() - sp_ref.item()) <= 1e-6
    assert (s.grad.cpu() - s_ref.grad).abs().max().item() <= 1e-5 * max(1.0, s_ref.grad.abs().max().item())


def test_objective_compute_matches_reference_formula_and_gradients():
    torch.manual_seed(5)
    B, H, nb, S, V = 1, 2, 8, 512, 64
    logits = torch.randn(B, S, V)
    labels = torch.randint(0, V, (B, S))
    labels[0, :7] = -100
    layers = [0, 3]
    soft = {i: _soft(B, H, nb, 10 + i) for i in layers}
    scores = {i: O.training_scores(torch.randn(B, H, S, 32), torch.randn(B, H, S, 32)) for i in layers}
    obj = TASFTObjective(lambda_gate=0.5, beta_sparse=0.1, tau_target=0.7)
    s_dev = {i: soft[i].to(DEV).requires_grad_(True) for i in layers}
    out = obj.compute(logits.to(DEV), labels.to(DEV), s_dev, {i: scores[i].to(DEV) for i in layers}, layers, 64)
    assert isinstance(out, ObjectiveLossOutput)
    out.total.backward()
    # reference formula (objectives.py:268-361) with the oracle's pieces and CPU autograd
    s_ref = {i: soft[i].clone().requires_grad_(True) for i in layers}
    task = torch.nn.functional.cross_entropy(logits[:, :-1].reshape(-1, V), labels[:, 1:].reshape(-1),
                                             ignore_index=-100)
    gate = sum(O.gate_loss(s_ref[i], O.gate_target(scores[i], 64)) for i in layers)
    sparse = sum(O.sparsity_loss(s_ref[i], 0.7) for i in layers)
    total = task + 0.5 * (gate + 0.1 * sparse)
    total.backward()
    assert abs(out.total.item() - total.item()) <= 1e-5 * max(1.0, abs(total.item()))
    assert abs(out.gate.item() - gate.item()) <= 1e-5 * max(1.0, abs(gate.item()))
    assert abs(out.sparse.item() - sparse.item()) <= 1e-6
    assert out.active_layers == layers and set(out.per_layer_gate_loss) == set(layers)
    for i in layers:
        assert (s_dev[i].grad.cpu() - s_ref[i].grad).abs().max().item() <= 1e-6
    # a ready target in place of the score tensor (the path that never forms it)
    tg = {i: O.gate_target(scores[i], 64).to(DEV) for i in layers}
    out2 = obj.compute(logits.to(DEV), labels.to(DEV), {i: soft[i].to(DEV) for i in layers}, tg, layers, 64)
    assert abs(out2.total.item() - total.item()) <= 1e-5 * max(1.0, abs(total.item()))


def test_objective_validation_matches_reference():
    for kw in [{"lambda_gate": 0.0}, {"lambda_gate": 11.0}, {"beta_sparse": -1.0}, {"tau_target": 1.0},
               {"label_smoothing": 1.0}]:
        with pytest.raises(ValueError):
            TASFTObjective(**kw)


def test_dense_fallback_backend_runs_full_causal_attention():
    g = torch.Generator().manual_seed(9)
    B, Hq, Hk, S, D = 1, 4, 2, 320, 64
    q, k, v = (torch.randn(B, h, S, D, generator=g).bfloat16() for h in (Hq, Hk, Hk))
    nb = math.ceil(S / 64)
    sparse_mask = torch.zeros(B, Hq, nb, nb, dtype=torch.bool)
    sparse_mask[..., 0] = True  # ignored by the dense backend, as in the reference
    bsfa = T.BlockSparseFlashAttention(backend=T.KernelBackend.DENSE_FALLBACK)
    assert bsfa.backend == T.KernelBackend.DENSE_FALLBACK
    out = bsfa.forward(q.to(DEV), k.to(DEV), v.to(DEV), sparse_mask.to(DEV))
    full = torch.ones(B, Hk, nb, nb, dtype=torch.bool).tril()
    ref = O.bsa_prefill_masked_dense(q, k, v, full, 64)
    assert (out.float().cpu() - ref.float()).abs().max().item() <= BF16_ATOL
    assert T.detect_kernels()[-1] == T.KernelBackend.DENSE_FALLBACK


def test_config1_fp32_layer_end_to_end():
    """fp32, B1, 8 heads MHA, S1024, D64, block 64, causal, gate hidden 64,
    mask = diagonal + top 20% of causal blocks by the random-init gate's scores. Gate and
    attention against the oracle at fp32 tolerance."""
    torch.manual_seed(0)
    B, H, S, D = 1, 8, 1024, 64
    q, k, v = (torch.randn(B, H, S, D) for _ in range(3))
    gate = T.AttnGate(H, D, block_size=64, gate_hidden_dim=64).to(DEV)
    go = gate(q.to(DEV), k.to(DEV))
    w = [p.detach().cpu() for p in (gate.gate_proj_in.weight, gate.gate_proj_in.bias, gate.gate_proj_out.weight)]
    soft_ref, _, _ = O.gate_forward_gqa(q, k, *w, 64, 0.5)
    assert (go.soft_scores.cpu() - soft_ref).abs().max().item() <= FP32_ATOL
    mask = M.diag_topk_mask(go.soft_scores, 0.2)
    out = T.BlockSparseFlashAttention(block_size=64).forward(q.to(DEV), k.to(DEV), v.to(DEV), mask)
    ref = O.bsa_prefill_masked_dense(q, k, v, mask.cpu(), 64)
    assert (out.cpu() - ref).abs().max().item() <= FP32_ATOL


def test_tensor_core_gate_target_d128_against_oracle():
    g = torch.Generator().manual_seed(31)
    B, Hq, Hk, S, D = 1, 4, 2, 1024, 128
    q = torch.randn(B, Hq, S, D, generator=g).bfloat16()
    k = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    got = T.gate_target_from_qk(q.to(DEV), k.to(DEV), 64)  # tcgen05 kernel (bf16, block 64)
    ref = O.gate_target_from_qk(q, k, 64)  # bf16 training scores, as the reference forms them
    assert (got.cpu() - ref.float()).abs().max().item() <= BF16_ATOL
    got2 = T.gate_target_from_qk(q.to(DEV), k.to(DEV), 64, temperature=2.0, clamp=50.0)
    ref2 = O.gate_target_from_qk(q, k, 64, temperature=2.0, clamp=50.0)
    assert (got2.cpu() - ref2.float()).abs().max().item() <= BF16_ATOL


@pytest.mark.parametrize("target", [0.0, 0.5, 0.8, 0.93, 1.0])
def test_calibrate_tau_exact_quantile(target):
    g = torch.Generator().manual_seed(int(target * 100))
    soft = torch.rand(2, 8, 64, 64, generator=g)
    soft = soft * torch.ones(64, 64).tril()  # causal zeros count, as in the reference's sparsity
    soft[0, 0, 5, :3] = 0.5  # ties
    tau, achieved = T.calibrate_tau(soft.to(DEV), target)
    n = soft.numel()
    keep = int(round((1 - target) * n))
    if keep == 0:
        assert tau == float("inf") and achieved == 1.0
        return
    ref_tau = torch.sort(soft.view(-1), descending=True).values[keep - 1].item()
    assert tau == ref_tau
    assert achieved == pytest.approx(1.0 - (soft >= ref_tau).sum().item() / n)
    assert achieved <= 1.0 - keep / n + 1e-12  # ties only ever keep more
    # the gate output's own sparsity as a device scalar, without a host sync
    gate = T.AttnGate(4, 64).to(DEV)
    out = gate(torch.randn(1, 4, 256, 64, device=DEV), torch.randn(1, 4, 256, 64, device=DEV))
    assert abs(out.sparsity_ratio_device.item() - out.sparsity_ratio) <= 1e-6
