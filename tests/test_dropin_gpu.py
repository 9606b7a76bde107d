"""The real drop-in path: the reference's own ``TASFTAttention`` layer, built by the
reference's ``patch_model_attention`` on a small Llama model, running its unmodified
``_inference_forward`` (``tasft/modules/tasft_attention.py:517-613``) after
``tasft_b200.patch()``.

That caller hands the kernel GQA-expanded K/V (``repeat_interleave`` at :725-729) and the
gate's per-q-head hard mask (:574-593), so this covers the kernel's MHA tiling with
Hk = Hq and per-q-head lists. The kernel call is recorded and checked against the oracle
on exactly the tensors the layer passed; the gate's scores against the oracle gate.

Needs the reference package importable (``$TASFT_REFERENCE`` or ``baseline/_ref``); skips
otherwise.
"""
from __future__ import annotations

import pytest
import torch

import oracle as O
import tasft_b200
from conftest import import_reference

pytestmark = pytest.mark.gpu
DEV = "cuda"
BF16_ATOL = 2e-2


@pytest.fixture()
def patched():
    import_reference()
    import tasft.modules.tasft_attention as R  # noqa: PLC0415

    tasft_b200.patch()
    try:
        yield R
    finally:
        tasft_b200.unpatch()


def _tiny_llama(S):
    from transformers import LlamaConfig, LlamaForCausalLM  # noqa: PLC0415

    cfg = LlamaConfig(hidden_size=512, intermediate_size=1024, num_attention_heads=8, num_key_value_heads=2,
                      head_dim=64, num_hidden_layers=2, vocab_size=256, max_position_embeddings=max(2048, S))
    torch.manual_seed(0)
    m = LlamaForCausalLM(cfg).to(device=DEV, dtype=torch.bfloat16).eval()
    m.requires_grad_(False)
    return m


def test_reference_tasft_attention_inference_forward_after_patch(patched, monkeypatch):
    R = patched
    S = 512
    model = _tiny_llama(S)
    layers = R.patch_model_attention(model, R.GateConfig(block_size=64, num_layers=2, default_threshold=0.5))
    assert all(isinstance(l.gate, tasft_b200.AttnGate) for l in layers.values())
    calls = []
    orig = tasft_b200.BlockSparseFlashAttention.forward

    def spy(self, q, k, v, block_mask, **kw):
        out = orig(self, q, k, v, block_mask, **kw)
        calls.append((q.detach().clone(), k.detach().clone(), v.detach().clone(), block_mask.clone(), out.clone()))
        return out

    monkeypatch.setattr(tasft_b200.BlockSparseFlashAttention, "forward", spy)
    ids = torch.randint(0, 256, (2, S), device=DEV, generator=torch.Generator(device=DEV).manual_seed(1))
    with torch.no_grad():
        logits = model(input_ids=ids).logits
    assert torch.isfinite(logits.float()).all()
    # both layers went through the sparse kernel (sparsity above min_sparsity_for_speedup)
    assert len(calls) == 2
    for li, (q, k, v, mask, out) in enumerate(calls):
        assert q.shape == k.shape == v.shape == (2, 8, S, 64)  # K/V expanded per q-head by the caller
        assert mask.shape == (2, 8, S // 64, S // 64) and mask.dtype == torch.bool
        ref = O.bsa_prefill_masked_dense(q.cpu(), k.cpu(), v.cpu(), mask.cpu(), 64)
        err = (out.float().cpu() - ref.float()).abs()
        assert err.max().item() <= BF16_ATOL, f"layer {li}"
        # the gate's fp32 scores and mask against the oracle gate on the same Q, K
        gate = layers[li].gate
        w = [p.detach().float().cpu() for p in (gate.gate_proj_in.weight, gate.gate_proj_in.bias,
                                                gate.gate_proj_out.weight)]
        soft_ref, hard_ref, _ = O.gate_forward_gqa(q.float().cpu(), k.float().cpu(), *w, 64, 0.5)
        go = layers[li]._last_gate_output
        assert (go.soft_scores.cpu() - soft_ref).abs().max().item() <= 1e-5
        same = go.hard_mask.cpu() == hard_ref
        # masks are bit-exact where the scores are not within rounding of tau
        near = (soft_ref - 0.5).abs() <= 1e-5
        assert bool((same | near).all())


def test_reference_layer_output_equals_masked_attention_then_o_proj(patched):
    R = patched
    S = 384
    model = _tiny_llama(S)
    layers = R.patch_model_attention(model, R.GateConfig(block_size=64, num_layers=1, default_threshold=0.5))
    layer = layers[0]
    hidden = torch.randn(1, S, 512, device=DEV, dtype=torch.bfloat16)
    pos = torch.arange(S, device=DEV).unsqueeze(0)
    cos, sin = model.model.rotary_emb(hidden, pos)
    with torch.no_grad():
        out, _ = layer(hidden, position_embeddings=(cos, sin))
        q, k, v, _ = layer._prepare_qkv(layer.base_attn, hidden, 1, S, pos, (cos, sin), None)
        mask = layer._last_gate_output.hard_mask
    attn = O.bsa_prefill_masked_dense(q.cpu(), k.cpu(), v.cpu(), mask.cpu(), 64)
    ref = layer.base_attn.o_proj(attn.to(DEV, torch.bfloat16).transpose(1, 2).reshape(1, S, 512))
    assert (out.float() - ref.float()).abs().max().item() <= 5e-2  # one bf16 projection after the 2e-2 attention
