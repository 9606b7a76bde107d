"""The fused training forward: attention output and gate target from one pass, never
forming the [B, H, S, S] scores (tasft_attention_train_fwd / training_attention), and the
reference's TASFTAttention training step running on it after patch(training=True).

References: tasft/modules/tasft_attention.py:363-468 (training forward),
tasft/training/objectives.py:128-185 (target), :268-361 (compute)."""
from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

import oracle as O
import tasft_b200 as T
from conftest import import_reference

pytestmark = pytest.mark.gpu
DEV = "cuda"
BF16_ATOL = 2e-2


@pytest.mark.parametrize("dtype,Hq,Hk,S,D", [
    (torch.bfloat16, 8, 2, 512, 128),
    (torch.bfloat16, 4, 4, 320, 64),    # MHA, ragged S
    (torch.float16, 4, 1, 384, 128),
    (torch.float32, 2, 1, 192, 64),     # CUDA-core fallback: prefill + target kernels
])
def test_training_attention_matches_oracle(dtype, Hq, Hk, S, D):
    g = torch.Generator().manual_seed(S + Hq)
    q = torch.randn(1, Hq, S, D, generator=g).to(dtype)
    k = torch.randn(1, Hk, S, D, generator=g).to(dtype)
    v = torch.randn(1, Hk, S, D, generator=g).to(dtype)
    out, tgt, bm = T.training_attention(q.to(DEV), k.to(DEV), v.to(DEV), 64, return_block_max=True)
    nb = math.ceil(S / 64)
    full = torch.ones(1, Hk, nb, nb, dtype=torch.bool).tril()
    ref = O.bsa_prefill_masked_dense(q, k, v, full, 64)
    tol = 1e-5 if dtype == torch.float32 else BF16_ATOL
    assert (out.float().cpu() - ref.float()).abs().max().item() <= tol
    # the target: against the reference's scores path restated, and against this library's
    # stand-alone target kernel (same rounding of the maxima)
    rt = O.gate_target_from_qk(q, k, 64)
    assert (tgt.cpu() - rt.float()).abs().max().item() <= (1e-5 if dtype == torch.float32 else BF16_ATOL)
    t2, bm2 = T.gate_target_from_qk(q.to(DEV), k.to(DEV), 64, return_block_max=True)
    fin = torch.isfinite(bm2)
    assert torch.equal(torch.isfinite(bm), fin)
    assert (bm[fin] - bm2[fin]).abs().max().item() <= 1e-2 * max(1.0, bm2[fin].abs().max().item())
    assert (tgt - t2).abs().max().item() <= 1e-3


def test_training_attention_gradients_match_dense_attention():
    g = torch.Generator().manual_seed(7)
    q, k, v = (torch.randn(1, h, 256, 64, generator=g).bfloat16().to(DEV) for h in (4, 2, 2))
    go = torch.randn(1, 4, 256, 64, generator=g).bfloat16().to(DEV)
    qa, ka, va = (t.clone().requires_grad_(True) for t in (q, k, v))
    out, _ = T.training_attention(qa, ka, va, 64)
    out.backward(go)
    qr, kr, vr = (t.float().clone().requires_grad_(True) for t in (q, k, v))
    ref = F.scaled_dot_product_attention(qr, kr.repeat_interleave(2, 1), vr.repeat_interleave(2, 1), is_causal=True)
    ref.backward(go.float())
    for a, b in ((qa, qr), (ka, kr), (va, vr)):
        assert (a.grad.float() - b.grad).abs().max().item() <= 5e-2 * max(1.0, b.grad.abs().max().item())


def test_reference_training_step_after_patch():
    import_reference()
    import tasft.modules.tasft_attention as R  # noqa: PLC0415
    from transformers import LlamaConfig, LlamaForCausalLM  # noqa: PLC0415

    # tasft.training's package init pulls the reference's logging stack (structlog), which this
    # image lacks, so the objective is this package's TASFTObjective directly (patch() would
    # rebind it in tasft.training.objectives / .trainer once those are imported)
    names = T.patch(training=True)
    assert "tasft.modules.tasft_attention.TASFTAttention._training_forward" in names
    try:
        cfg = LlamaConfig(hidden_size=512, intermediate_size=1024, num_attention_heads=8, num_key_value_heads=2,
                          head_dim=64, num_hidden_layers=1, vocab_size=128, max_position_embeddings=2048)
        torch.manual_seed(0)
        model = LlamaForCausalLM(cfg).to(device=DEV, dtype=torch.bfloat16)
        model.requires_grad_(False)
        layers = R.patch_model_attention(model, R.GateConfig(block_size=64, num_layers=1))
        layer = layers[0]
        layer.set_training_mode(True)
        ids = torch.randint(0, 128, (1, 256), device=DEV)
        out = model(input_ids=ids)
        target = layer._last_attn_weights
        assert target.shape == (1, 8, 4, 4)  # the gate target, not [B, H, S, S] scores
        # the same target from the layer's own q / k through the reference's score path
        with torch.no_grad():
            hidden = model.model.embed_tokens(ids)
            hidden = model.model.layers[0].input_layernorm(hidden)
            pos = torch.arange(256, device=DEV).unsqueeze(0)
            cos, sin = model.model.rotary_emb(hidden, pos)
            q, k, _, _ = layer._prepare_qkv(layer.base_attn, hidden, 1, 256, pos, (cos, sin), None)
        rt = O.gate_target(O.training_scores(q.cpu(), k.cpu()), 64)
        assert (target.cpu() - rt.float()).abs().max().item() <= BF16_ATOL
        obj = T.TASFTObjective(lambda_gate=0.5)
        loss = obj.compute(out.logits.float(), ids, {0: layer._last_gate_output.soft_scores}, {0: target}, [0], 64)
        loss.total.backward()
        assert layer.gate.gate_proj_in.weight.grad is not None
        assert torch.isfinite(layer.gate.gate_proj_in.weight.grad).all()
    finally:
        T.unpatch()
