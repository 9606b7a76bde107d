"""Pin the CPU oracle: reference known-answer tests and fixtures made by running the reference.

Known answers restated from the reference's own tests:
tests/unit/test_numerical_correctness.py:40-98 (pooling), :119-184 (gate target),
:196-238 (KL), :407-443 (sparsity loss), :714-721 (uniform target);
tests/unit/test_objectives.py:166-227 (4x4 target, -inf padding).
"""
from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

import oracle as O


class TestPoolingKAT:
    def test_arange_block4(self):
        q = torch.arange(1, 33, dtype=torch.float32).reshape(1, 1, 8, 4)
        exp = torch.tensor([[[[7.0, 8.0, 9.0, 10.0], [23.0, 24.0, 25.0, 26.0]]]])
        torch.testing.assert_close(O.pool_to_blocks(q, 4), exp, atol=1e-6, rtol=1e-6)

    def test_padding_counts_zeros(self):
        q = torch.ones(1, 1, 6, 2)
        exp = torch.tensor([[[[1.0, 1.0], [0.5, 0.5]]]])
        torch.testing.assert_close(O.pool_to_blocks(q, 4), exp, atol=1e-6, rtol=1e-6)

    def test_single_block(self):
        q = torch.tensor([[1.0, 2.0, 3.0], [4.0, 5.0, 6.0], [7.0, 8.0, 9.0], [10.0, 11.0, 12.0]])
        q = q.unsqueeze(0).unsqueeze(0).expand(1, 2, 4, 3)
        out = O.pool_to_blocks(q, 4)
        torch.testing.assert_close(out[0, 1, 0], torch.tensor([5.5, 6.5, 7.5]))


class TestGateTargetKAT:
    def test_8x8_block4(self):
        attn = torch.arange(1, 65, dtype=torch.float32).reshape(1, 1, 8, 8)
        t = O.gate_target(attn, 4)
        exp = F.softmax(torch.tensor([28.0, 32.0, 60.0, 64.0]), dim=-1).reshape(1, 1, 2, 2)
        torch.testing.assert_close(t, exp, atol=1e-6, rtol=1e-6)

    def test_4x4_block2(self):
        attn = torch.arange(1, 17, dtype=torch.float32).reshape(1, 1, 4, 4)
        exp = F.softmax(torch.tensor([6.0, 8.0, 14.0, 16.0]), dim=-1).reshape(1, 1, 2, 2)
        torch.testing.assert_close(O.gate_target(attn, 2), exp, atol=1e-6, rtol=1e-6)

    def test_causal_neg_inf(self):
        attn = torch.randn(1, 1, 8, 8)
        attn[0, 0][torch.triu(torch.ones(8, 8), diagonal=1).bool()] = float("-inf")
        t = O.gate_target(attn, 4)
        assert torch.isfinite(t).all() and abs(t.sum().item() - 1.0) < 1e-5

    def test_uniform(self):
        t = O.gate_target(torch.full((1, 1, 8, 8), 5.0), 4)
        torch.testing.assert_close(t, torch.full((1, 1, 2, 2), 0.25), atol=1e-5, rtol=1e-5)

    def test_ragged_padded_neg_inf(self):
        t = O.gate_target(torch.randn(1, 1, 5, 5), 4)
        assert t.shape == (1, 1, 2, 2) and torch.isfinite(t).all()

    def test_nan_raises(self):
        with pytest.raises(ValueError):
            O.gate_target(torch.tensor([[[[1.0, float("nan")], [3.0, 4.0]]]]), 1)


class TestLossKAT:
    def test_kl_matches_restatement(self):
        P = torch.tensor([0.1, 0.2, 0.7], dtype=torch.float64).reshape(1, 1, 1, 3)
        Qs = torch.tensor([0.3, 0.3, 0.4], dtype=torch.float64).reshape(1, 1, 1, 3)
        ref = sum(p * math.log(p / (q / (1.0 + 1e-8) + 1e-8)) for p, q in zip([0.1, 0.2, 0.7], [0.3, 0.3, 0.4]))
        assert O.gate_loss(Qs, P).item() == pytest.approx(ref, abs=1e-6)

    def test_kl_self_zero(self):
        P = torch.full((1, 1, 2, 2), 0.25, dtype=torch.float64)
        assert O.gate_loss(P, P).item() == pytest.approx(0.0, abs=1e-4)

    @pytest.mark.parametrize("val,tau,exp", [(0.8, 0.8, 0.0), (0.5, 0.8, 0.09), (1.0, 0.8, 0.04), (0.0, 0.5, 0.25)])
    def test_sparsity_points(self, val, tau, exp):
        assert O.sparsity_loss(torch.full((1, 1, 4, 4), val), tau).item() == pytest.approx(exp, abs=1e-6)


class TestAgainstReferenceRun:
    """Fixtures from tests/golden/make_golden.py (the reference run in the build container)."""

    def test_gate_forward_bit_exact(self, golden):
        for c in golden["gate"]:
            soft, hard, sp = O.gate_forward(c["q"], c["k"], c["w_in"], c["b_in"], c["w_out"], c["block"], c["tau"],
                                            c["causal"])
            assert torch.equal(soft, c["soft"]), c["dtype"]
            assert torch.equal(hard, c["hard"])
            assert sp == c["sparsity"]

    def test_pool_matches_reference(self, golden):
        for c in golden["gate"]:
            assert torch.equal(O.pool_to_blocks(c["q"], c["block"]), c["pooled_q"])

    def test_prefill_matches_reference_triton(self, golden):
        for c in golden["kernel"]:
            o1 = O.bsa_prefill_masked_dense(c["q"], c["k"], c["v"], c["mask"], c["block"], c["causal"])
            o2 = O.bsa_prefill_blockwise(c["q"], c["k"], c["v"], c["mask"], c["block"], c["causal"])
            assert (o1 - c["out"]).abs().max().item() < 1e-5
            assert (o2 - c["out"]).abs().max().item() < 1e-5

    def test_objectives_bit_exact(self, golden):
        for c in golden["objective"]:
            t = O.gate_target(c["scores"], c["block"])
            assert torch.equal(t, c["target"])
            assert torch.equal(O.gate_loss(c["soft"], t), c["kl"])
            assert torch.equal(O.sparsity_loss(c["soft"], 0.8), c["sparse"])


class TestOracleSelfConsistency:
    def test_kept_roundtrip(self):
        g = torch.Generator().manual_seed(0)
        m = torch.rand(2, 3, 9, 9, generator=g) < 0.4
        idx, cnt = O.kept_from_mask(m, causal=False)
        assert torch.equal(O.mask_from_kept(idx, cnt, 9), m)
        idx, cnt = O.kept_from_mask(m, causal=True)
        assert torch.equal(O.mask_from_kept(idx, cnt, 9), m & torch.ones(9, 9, dtype=torch.bool).tril())

    def test_gqa_prefill_equals_expanded(self):
        g = torch.Generator().manual_seed(1)
        q = torch.randn(1, 4, 130, 32, generator=g)
        k = torch.randn(1, 2, 130, 32, generator=g)
        v = torch.randn(1, 2, 130, 32, generator=g)
        mask = torch.rand(1, 2, 3, 3, generator=g) < 0.7
        a = O.bsa_prefill_masked_dense(q, k, v, mask, 64)
        b = O.bsa_prefill_masked_dense(q, k.repeat_interleave(2, 1), v.repeat_interleave(2, 1),
                                       mask.repeat_interleave(2, 1), 64)
        assert torch.equal(a, b)

    def test_decode_combine_equals_full(self):
        g = torch.Generator().manual_seed(2)
        B, Hq, Hk, L, D, blk = 2, 4, 2, 300, 16, 64
        q = torch.randn(B, Hq, D, generator=g)
        kc = torch.randn(B, Hk, L, D, generator=g)
        vc = torch.randn(B, Hk, L, D, generator=g)
        kv_len = torch.tensor([300, 170], dtype=torch.int32)
        nb = math.ceil(L / blk)
        idx = torch.arange(nb, dtype=torch.int32).expand(B, Hk, nb).contiguous()
        cnt = torch.full((B, Hk), nb, dtype=torch.int32)
        full = O.bsa_decode(q, kc, vc, kv_len, idx, cnt, blk)
        parts = []
        for lo, hi in [(0, 2), (2, nb)]:
            sub = torch.full_like(idx, -1)
            sub[..., : hi - lo] = idx[..., lo:hi]
            c = torch.full_like(cnt, hi - lo)
            parts.append(O.bsa_decode(q, kc, vc, kv_len, sub, c, blk, return_lse=True))
        o = torch.stack([p[0].float() for p in parts])
        m = torch.stack([p[1] for p in parts])
        l_ = torch.stack([p[2] for p in parts])
        torch.testing.assert_close(O.decode_combine(o, m, l_), full.float(), atol=1e-6, rtol=1e-5)
