"""Host-side logic on CPU: API validation (mirrors the reference's tests), no CPU fallback,
benchmark mask rules, and the reference drop-in patch."""
from __future__ import annotations

import math
import sys
from pathlib import Path

import pytest
import torch

import oracle as O
from conftest import import_reference
from tasft_b200 import AttnGate, BlockSparseFlashAttention, KernelBackend, KernelError, KeptBlocks, ValidationError
from tasft_b200 import masks as M


class TestBlockSparseCtor:
    """Mirrors tasft/tests/unit/test_kernel.py:133-161 (constructor validation)."""

    @pytest.mark.parametrize("bs", [16, 48, 256])
    def test_bad_block_size(self, bs):
        with pytest.raises(ValueError, match="block_size"):
            BlockSparseFlashAttention(block_size=bs)

    @pytest.mark.parametrize("ms", [-0.1, 1.5])
    def test_bad_min_sparsity(self, ms):
        with pytest.raises(ValueError, match="min_sparsity"):
            BlockSparseFlashAttention(min_sparsity_for_speedup=ms)

    def test_other_backends_rejected(self):
        with pytest.raises(KernelError):
            BlockSparseFlashAttention(backend=KernelBackend.TRITON)

    def test_speedup_model(self):
        assert BlockSparseFlashAttention.estimate_speedup(0.0) == pytest.approx(1.0)
        assert BlockSparseFlashAttention.estimate_speedup(0.9) == pytest.approx(1 / (1 - 0.9 * 0.98))

    def test_sparsity_stats(self):
        k = BlockSparseFlashAttention()
        m = torch.zeros(1, 2, 4, 4, dtype=torch.bool)
        m[..., 0] = True
        st = k.compute_sparsity_stats(m)
        assert st.total_blocks == 32 and st.active_blocks == 8 and st.sparsity_ratio == pytest.approx(0.75)

    def test_cpu_tensors_fail_loudly(self):
        k = BlockSparseFlashAttention()
        q = torch.randn(1, 2, 64, 64)
        with pytest.raises(KernelError, match="CUDA"):
            k.forward(q, q, q, torch.ones(1, 2, 1, 1, dtype=torch.bool))

    def test_shape_errors(self):
        k = BlockSparseFlashAttention()
        q = torch.randn(1, 2, 64, 64)
        with pytest.raises(KernelError):
            k.forward(q[0], q[0], q[0], torch.ones(1, 1))
        with pytest.raises(KernelError):
            k.forward(q, torch.randn(1, 3, 64, 64), torch.randn(1, 3, 64, 64), torch.ones(1, 2, 1, 1))


class TestAttnGateHost:
    """Mirrors tasft/tests/unit/test_attn_gate.py:51-110, :330-347, :404-440."""

    def test_defaults(self):
        g = AttnGate(num_heads=8, head_dim=128)
        assert g.gate_hidden_dim == 32 and g.block_size == 64 and g.is_causal
        assert set(dict(g.named_parameters())) == {"gate_proj_in.weight", "gate_proj_in.bias",
                                                   "gate_proj_out.weight"}
        assert g.num_parameters == 2 * 128 * 32 + 32 + 32

    @pytest.mark.parametrize("kw", [{"num_heads": 0, "head_dim": 4}, {"num_heads": 1, "head_dim": 0},
                                    {"num_heads": 1, "head_dim": 4, "block_size": 0},
                                    {"num_heads": 1, "head_dim": 4, "default_threshold": 1.5}])
    def test_invalid_ctor(self, kw):
        with pytest.raises(ValidationError):
            AttnGate(**kw)

    def test_state_dict_compatible_with_reference(self):
        import_reference()
        from tasft.modules.attn_gate import AttnGate as RefGate  # noqa: PLC0415
        ref = RefGate(4, 64, block_size=64)
        ours = AttnGate(4, 64, block_size=64)
        ours.load_state_dict(ref.state_dict())

    @pytest.mark.parametrize("q,k", [((2, 64, 16), (1, 2, 64, 16)), ((1, 2, 64, 16), (1, 2, 64))])
    def test_rank_errors(self, q, k):
        g = AttnGate(2, 16)
        with pytest.raises(ValidationError):
            g(torch.randn(*q), torch.randn(*k))

    def test_head_and_dim_errors(self):
        g = AttnGate(2, 16)
        with pytest.raises(ValidationError):
            g(torch.randn(1, 3, 64, 16), torch.randn(1, 3, 64, 16))
        with pytest.raises(ValidationError):
            g(torch.randn(1, 2, 64, 8), torch.randn(1, 2, 64, 8))
        with pytest.raises(ValidationError):
            g(torch.randn(1, 2, 0, 16), torch.randn(1, 2, 0, 16))

    def test_cpu_tensors_fail_loudly(self):
        g = AttnGate(2, 16)
        with pytest.raises(KernelError):
            g(torch.randn(1, 2, 64, 16), torch.randn(1, 2, 64, 16))


class TestMaskRules:
    def test_llama_prefill_count(self):
        nb = 64
        s = torch.rand(1, 1, nb, nb, generator=torch.Generator().manual_seed(0))
        m = M.prefill_mask(s, 0.2)
        assert int(m.sum()) == 424  # kept causal blocks per (b, head) at 80% sparsity
        assert bool(m[..., torch.arange(nb), torch.arange(nb)].all()) and bool(m[..., :, 0].all())
        assert not bool(m.triu(1).any())

    def test_qwen_prefill_count(self):
        nb = 512
        s = torch.rand(1, 1, nb, nb, generator=torch.Generator().manual_seed(0))
        assert int(M.prefill_mask(s, 0.1).sum()) == 13150

    def test_rule_is_a_row_threshold(self):
        s = torch.rand(2, 3, 16, 16, generator=torch.Generator().manual_seed(1))
        m = M.prefill_mask(s, 0.3)
        for b in range(2):
            for h in range(3):
                for i in range(2, 16):
                    kept = s[b, h, i, 1:i][m[b, h, i, 1:i]]
                    dropped = s[b, h, i, 1:i][~m[b, h, i, 1:i]]
                    if kept.numel() and dropped.numel():
                        assert kept.min() >= dropped.max()

    def test_decode_rule(self):
        s = torch.rand(3, 2, 128, generator=torch.Generator().manual_seed(2))
        nbv = torch.tensor([128, 100, 3])
        m = M.decode_mask(s, nbv, 0.2, 128)
        assert m[0].sum(-1).tolist() == [26, 26] and m[1].sum(-1).tolist() == [26, 26]
        assert m[2].sum(-1).tolist() == [3, 3]
        assert bool(m[:, :, 0].all()) and bool(m[1, :, 99].all()) and not bool(m[1, :, 100:].any())

    def test_lists_match_oracle(self):
        m = torch.rand(2, 2, 9, 9, generator=torch.Generator().manual_seed(3)) < 0.5
        a = M.lists_from_mask(m)
        b = O.kept_from_mask(m, causal=False)
        assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])

    def test_cpu_config_rule(self):
        s = torch.rand(1, 8, 16, 16, generator=torch.Generator().manual_seed(4))
        m = M.diag_topk_mask(s, 0.2)
        counts = m.sum(-1)[0, 0].tolist()
        assert counts == [max(1, int(round(0.2 * (i + 1)))) for i in range(16)]


def test_patch_into_reference():
    import_reference()
    import tasft_b200

    names = tasft_b200.patch()
    try:
        import tasft.kernels.block_sparse_fa as R  # noqa: PLC0415
        import tasft.modules.attn_gate as G  # noqa: PLC0415

        assert R.BlockSparseFlashAttention is tasft_b200.BlockSparseFlashAttention
        assert G.AttnGate is tasft_b200.AttnGate
        assert any("BlockSparseFlashAttention" in n for n in names)
    finally:
        tasft_b200.unpatch()
    import tasft.kernels.block_sparse_fa as R  # noqa: PLC0415

    assert R.BlockSparseFlashAttention is not tasft_b200.BlockSparseFlashAttention


def test_prefill_flops_accounting():
    nb = 64
    s = torch.rand(4, 8, nb, nb, generator=torch.Generator().manual_seed(5))
    m = M.prefill_mask(s, 0.2)
    flops = int(m.sum()) * 4 * 4 * 64 * 64 * 128  # x4 q-heads per kv-head
    assert math.isclose(flops / 1e9, 113.8, rel_tol=2e-3)


class TestNewEntryPointsFailLoudly:
    """The varlen prefill, paged decode and split-KV helpers reject bad input on the host
    (no CPU fallback: CPU tensors raise, shape errors raise before any launch)."""

    def test_varlen_shape_and_device_errors(self):
        kern = BlockSparseFlashAttention()
        q = torch.randn(100, 4, 64)
        cu = torch.tensor([0, 100], dtype=torch.int32)
        mask = torch.ones(1, 2, 2, 2, dtype=torch.bool)
        with pytest.raises(KernelError):
            kern.forward_varlen(q, torch.randn(100, 3, 64), torch.randn(100, 3, 64), cu, 100, mask)  # 4 % 3
        with pytest.raises(KernelError):
            kern.forward_varlen(q.unsqueeze(0), q, q, cu, 100, mask)  # not [T, H, D]
        with pytest.raises(KernelError, match="CUDA"):
            kern.forward_varlen(q, torch.randn(100, 2, 64), torch.randn(100, 2, 64), cu, 100, mask)

    def test_paged_decode_errors(self):
        import tasft_b200 as T  # noqa: PLC0415

        q = torch.randn(2, 8, 64)
        pages = torch.randn(10, 16, 2, 64)
        table = torch.zeros(2, 4, dtype=torch.int32)
        kept = KeptBlocks(torch.zeros(2, 2, 1, dtype=torch.int32), torch.ones(2, 2, dtype=torch.int32))
        with pytest.raises(KernelError, match="CUDA"):
            T.bsa_decode_paged(q, pages, pages, table, torch.full((2,), 64, dtype=torch.int32), kept)

    def test_split_kv_helpers_need_a_process_group_only_for_the_exchange(self):
        from tasft_b200 import shards as SH  # noqa: PLC0415

        # the planning helpers are plain host/tensor code
        assert SH.block_range(10, 0, 3) == (0, 4)
        kept = KeptBlocks(torch.tensor([[[0, 5, 9]]], dtype=torch.int32), torch.tensor([[3]], dtype=torch.int32))
        assert SH.local_kept(kept, 4, 10).idx.tolist() == [[[1, 5, -1]]]
