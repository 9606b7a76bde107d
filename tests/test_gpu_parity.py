"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle and the reference's
own outputs. Tolerances: masks and kept lists bit-exact from the
same fp32 scores; attention bf16 <= 2e-2 max-abs and 1e-2 relative (mean), fp32 <= 1e-5.
"""
from __future__ import annotations

import math

import pytest
import torch

import oracle as O
import tasft_b200 as T
from tasft_b200 import _lib as L
from tasft_b200 import masks as M

pytestmark = pytest.mark.gpu
DEV = "cuda"
BF16_ABS, BF16_REL, FP32_ABS = 2e-2, 1e-2, 1e-5


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float(), b.float()
    return ((a - b).abs().sum() / b.abs().sum().clamp_min(1e-30)).item()


def assert_bf16_close(out, ref):
    out = out.float().cpu()
    ref = ref.float().cpu()
    assert torch.isfinite(out).all()
    assert (out - ref).abs().max().item() <= BF16_ABS, (out - ref).abs().max().item()
    assert rel_err(out, ref) <= BF16_REL


# ---------------------------------------------------------------------------
# gate
# ---------------------------------------------------------------------------
class TestGate:
    def test_golden_reference_gate(self, golden):
        for c in golden["gate"]:
            g = T.AttnGate(c["H"], c["D"], block_size=c["block"], gate_hidden_dim=c["w_in"].shape[0],
                           default_threshold=c["tau"], is_causal=c["causal"]).to(DEV)
            with torch.no_grad():
                g.gate_proj_in.weight.copy_(c["w_in"])
                g.gate_proj_in.bias.copy_(c["b_in"])
                g.gate_proj_out.weight.copy_(c["w_out"])
            out = g(c["q"].to(DEV), c["k"].to(DEV))
            soft = out.soft_scores.cpu()
            ref = c["soft"].float()
            tol = 1e-5 if c["dtype"] == "torch.float32" else 1.2e-2
            assert (soft - ref).abs().max().item() <= tol, c["dtype"]
            # hard mask: identical except where the reference's score is within tol of tau
            near = (ref - c["tau"]).abs() <= tol
            assert torch.equal(out.hard_mask.cpu()[~near], c["hard"][~near])
            # the hard mask is exactly `soft >= tau` of our own scores
            assert torch.equal(out.hard_mask.cpu(), soft >= c["tau"])

    @pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
    def test_gqa_gate_matches_oracle(self, dtype):
        torch.manual_seed(0)
        B, Hq, Hk, S, D = 2, 8, 2, 300, 64
        g = T.AttnGate(Hq, D, block_size=64, default_threshold=0.5)
        with torch.no_grad():
            g.gate_proj_out.weight.mul_(50)
        q = torch.randn(B, Hq, S, D).to(dtype)
        k = torch.randn(B, Hk, S, D).to(dtype)
        soft_ref, _, _ = O.gate_forward_gqa(q.float(), k.float(), g.gate_proj_in.weight.detach(),
                                            g.gate_proj_in.bias.detach(), g.gate_proj_out.weight.detach(),
                                            64, 0.5)
        out = g.to(DEV)(q.to(DEV), k.to(DEV))
        assert (out.soft_scores.cpu() - soft_ref).abs().max().item() < 2e-5
        idx, cnt = O.kept_from_mask(out.hard_mask.cpu(), causal=True)
        assert torch.equal(out.kept.idx.cpu(), idx)
        assert torch.equal(out.kept.cnt.cpu(), cnt)
        assert out.sparsity_ratio == pytest.approx(1.0 - out.hard_mask.float().mean().item())

    def test_threshold_bit_exact(self):
        g = torch.Generator().manual_seed(3)
        soft = torch.rand(3, 5, 33, 33, generator=g)
        soft[..., 4] = 0.5  # exact ties at tau
        for tau in (0.0, 0.5, 0.73, 1.0):
            for causal in (False, True):
                hard, kept, num = T.threshold_scores(soft.to(DEV), tau, causal)
                ref_hard = soft >= tau  # the reference's comparison (attn_gate.py:475)
                assert torch.equal(hard.cpu(), ref_hard)
                idx, cnt = O.kept_from_mask(ref_hard, causal=causal)
                assert torch.equal(kept.idx.cpu(), idx) and torch.equal(kept.cnt.cpu(), cnt)
                assert int(num.item()) == int(ref_hard.sum())

    def test_mask_to_kept_bit_exact(self):
        m = torch.rand(2, 4, 70, 70, generator=torch.Generator().manual_seed(4)) < 0.3
        for causal in (False, True):
            kept = T.mask_to_kept(m.to(DEV), causal)
            idx, cnt = O.kept_from_mask(m, causal)
            assert torch.equal(kept.idx.cpu(), idx) and torch.equal(kept.cnt.cpu(), cnt)

    def test_decode_scoring_shapes(self):
        g = T.AttnGate(8, 128, block_size=64).to(DEV)
        q = torch.randn(2, 8, 1, 128, device=DEV, dtype=torch.bfloat16)
        k = torch.randn(2, 2, 1000, 128, device=DEV, dtype=torch.bfloat16)
        out = g(q, k)
        assert out.soft_scores.shape == (2, 8, 1, 16)
        ref, _, _ = O.gate_forward_gqa(q.float().cpu(), k.float().cpu(), g.gate_proj_in.weight.detach().cpu(),
                                       g.gate_proj_in.bias.detach().cpu(), g.gate_proj_out.weight.detach().cpu(),
                                       64, 0.5)
        assert (out.soft_scores.cpu() - ref).abs().max().item() < 2e-5


# ---------------------------------------------------------------------------
# prefill
# ---------------------------------------------------------------------------
def _prefill_case(B, Hq, Hk, S, D, dtype, density, seed, per_q_head=False, block=64):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, S, D, generator=g).to(dtype)
    k = torch.randn(B, Hk, S, D, generator=g).to(dtype)
    v = torch.randn(B, Hk, S, D, generator=g).to(dtype)
    nb = math.ceil(S / block)
    hm = Hq if per_q_head else Hk
    scores = torch.rand(B, hm, nb, nb, generator=g)
    mask = M.prefill_mask(scores, density)
    return q, k, v, mask


class TestPrefill:
    def test_golden_reference_triton_fp32(self, golden):
        for c in golden["kernel"]:
            k = T.BlockSparseFlashAttention(block_size=c["block"], min_sparsity_for_speedup=0.0)
            out = k.forward(c["q"].to(DEV), c["k"].to(DEV), c["v"].to(DEV), c["mask"].to(DEV), causal=c["causal"])
            assert (out.cpu() - c["out"]).abs().max().item() <= FP32_ABS

    @pytest.mark.parametrize("B,Hq,Hk,S,D,density,per_q", [
        (1, 4, 1, 512, 128, 0.3, False),   # GQA 4:1, D128
        (2, 8, 2, 700, 128, 0.25, False),  # ragged S
        (1, 7, 1, 384, 128, 0.4, False),   # GQA 7:1 (odd group)
        (1, 4, 4, 448, 64, 0.3, False),    # MHA D64: slots are q-block pairs
        (1, 4, 2, 512, 128, 0.3, True),    # per-q-head masks under GQA
        (2, 2, 2, 130, 64, 1.0, False),    # dense, tiny, ragged
        (1, 4, 1, 2048, 128, 0.6, False),  # long kept lists: deep ring reuse
        (1, 2, 2, 1536, 64, 1.0, False),   # dense MHA, 24 blocks per row
    ])
    def test_tc_bf16_vs_oracle(self, B, Hq, Hk, S, D, density, per_q):
        q, k, v, mask = _prefill_case(B, Hq, Hk, S, D, torch.bfloat16, density, seed=S + Hq, per_q_head=per_q)
        kern = T.BlockSparseFlashAttention(block_size=64)
        err = torch.zeros(1, dtype=torch.int32, device=DEV)
        out = kern.forward(q.to(DEV), k.to(DEV), v.to(DEV), mask.to(DEV), causal=True, err=err)
        ref = O.bsa_prefill_masked_dense(q, k, v, mask, 64, causal=True)
        assert int(err.item()) == 0
        assert_bf16_close(out, ref)

    @pytest.mark.parametrize("gain", [6.0, 20.0])
    def test_lazy_rescale_path(self, gain):
        """Large logits make the running max jump by > 2^8 (log2 units): O gets rescaled."""
        q, k, v, mask = _prefill_case(1, 4, 1, 1024, 128, torch.bfloat16, 0.5, seed=31)
        q = (q.float() * gain).to(torch.bfloat16)
        # make late blocks dominate so the max keeps growing along each row
        ramp = torch.linspace(0.2, 3.0, 1024).view(1, 1, 1024, 1)
        k = (k.float() * ramp).to(torch.bfloat16)
        out = T.BlockSparseFlashAttention().forward(q.to(DEV), k.to(DEV), v.to(DEV), mask.to(DEV))
        assert_bf16_close(out, O.bsa_prefill_masked_dense(q, k, v, mask, 64))

    @pytest.mark.parametrize("grid", ["1", "3"])
    def test_persistent_many_tiles_per_cta(self, grid, monkeypatch):
        """Cap the persistent grid so each CTA walks many tiles: the list/Q/O hand-offs
        between consecutive tiles of one CTA are exercised at a small size."""
        monkeypatch.setenv("TASFT_PREFILL_GRID", grid)
        q, k, v, mask = _prefill_case(2, 8, 2, 1024, 128, torch.bfloat16, 0.4, seed=41)
        err = torch.zeros(1, dtype=torch.int32, device=DEV)
        out = T.BlockSparseFlashAttention().forward(q.to(DEV), k.to(DEV), v.to(DEV), mask.to(DEV), err=err)
        assert int(err.item()) == 0
        assert_bf16_close(out, O.bsa_prefill_masked_dense(q, k, v, mask, 64))

    def test_run_to_run_deterministic(self):
        q, k, v, mask = _prefill_case(2, 8, 2, 2048, 128, torch.bfloat16, 0.3, seed=33)
        kern = T.BlockSparseFlashAttention()
        a = kern.forward(q.to(DEV), k.to(DEV), v.to(DEV), mask.to(DEV))
        b = kern.forward(q.to(DEV), k.to(DEV), v.to(DEV), mask.to(DEV))
        assert torch.equal(a, b)

    def test_tc_matches_simt(self):
        q, k, v, mask = _prefill_case(2, 8, 2, 1024, 128, torch.bfloat16, 0.2, seed=7)
        kern = T.BlockSparseFlashAttention(block_size=64)
        a = kern.forward(q.to(DEV), k.to(DEV), v.to(DEV), mask.to(DEV))
        kern.force_simt = True
        b = kern.forward(q.to(DEV), k.to(DEV), v.to(DEV), mask.to(DEV))
        assert (a.float() - b.float()).abs().max().item() <= BF16_ABS

    def test_fp16_and_noncausal(self):
        q, k, v, mask = _prefill_case(1, 4, 2, 320, 64, torch.float16, 0.5, seed=9)
        full = torch.rand(mask.shape, generator=torch.Generator().manual_seed(1)) < 0.5
        kern = T.BlockSparseFlashAttention(block_size=64)
        out = kern.forward(q.to(DEV), k.to(DEV), v.to(DEV), full.to(DEV), causal=False)
        ref = O.bsa_prefill_masked_dense(q, k, v, full, 64, causal=False)
        assert_bf16_close(out, ref)

    def test_empty_rows_give_zero(self):
        q, k, v, mask = _prefill_case(1, 4, 1, 256, 128, torch.bfloat16, 0.5, seed=11)
        mask[:, :, 2, :] = False
        out = T.BlockSparseFlashAttention().forward(q.to(DEV), k.to(DEV), v.to(DEV), mask.to(DEV))
        assert out[:, :, 128:192].abs().max().item() == 0.0
        assert_bf16_close(out, O.bsa_prefill_masked_dense(q, k, v, mask, 64))

    @pytest.mark.parametrize("block", [32, 128])
    def test_other_block_sizes_fp32(self, block):
        q, k, v, mask = _prefill_case(1, 2, 1, 300, 64, torch.float32, 0.5, seed=block, block=block)
        out = T.BlockSparseFlashAttention(block_size=block).forward(q.to(DEV), k.to(DEV), v.to(DEV),
                                                                    mask.to(DEV))
        ref = O.bsa_prefill_masked_dense(q, k, v, mask, block)
        assert (out.cpu() - ref).abs().max().item() <= FP32_ABS

    def test_kept_lists_input(self):
        q, k, v, mask = _prefill_case(1, 4, 1, 512, 128, torch.bfloat16, 0.3, seed=13)
        idx, cnt = M.lists_from_mask(mask)
        kern = T.BlockSparseFlashAttention()
        a = kern.forward(q.to(DEV), k.to(DEV), v.to(DEV), T.KeptBlocks(idx.to(DEV), cnt.to(DEV)))
        b = kern.forward(q.to(DEV), k.to(DEV), v.to(DEV), mask.to(DEV))
        assert torch.equal(a, b)

    def test_bad_index_sets_error_word(self):
        q, k, v, mask = _prefill_case(1, 2, 1, 256, 128, torch.bfloat16, 1.0, seed=15)
        idx, cnt = M.lists_from_mask(mask)
        idx[0, 0, 3, 0] = 99  # out of range: skipped, reported, never dereferenced
        err = torch.zeros(1, dtype=torch.int32, device=DEV)
        T.BlockSparseFlashAttention().forward(q.to(DEV), k.to(DEV), v.to(DEV),
                                              T.KeptBlocks(idx.to(DEV), cnt.to(DEV)), err=err)
        assert int(err.item()) & L.DEVERR_INDEX

    def test_llama_shape_sampled_heads(self):
        """Full C2 shape on the GPU; two (b, kv-head) groups checked against the oracle."""
        B, Hq, Hk, S, D = 4, 32, 8, 4096, 128
        g = torch.Generator(device=DEV).manual_seed(1236)
        q = torch.randn(B, Hq, S, D, device=DEV, dtype=torch.bfloat16, generator=g)
        k = torch.randn(B, Hk, S, D, device=DEV, dtype=torch.bfloat16, generator=g)
        v = torch.randn(B, Hk, S, D, device=DEV, dtype=torch.bfloat16, generator=g)
        scores = torch.rand(B, Hk, 64, 64, device=DEV, generator=g)
        mask = M.prefill_mask(scores, 0.2)
        out = T.BlockSparseFlashAttention().forward(q, k, v, mask)
        torch.cuda.synchronize()
        for b, hk in [(0, 0), (3, 7)]:
            sl = slice(hk * 4, hk * 4 + 4)
            ref = O.bsa_prefill_masked_dense(q[b:b + 1, sl].cpu(), k[b:b + 1, hk:hk + 1].cpu(),
                                             v[b:b + 1, hk:hk + 1].cpu(), mask[b:b + 1, hk:hk + 1].cpu(), 64)
            assert_bf16_close(out[b:b + 1, sl], ref)


# ---------------------------------------------------------------------------
# decode
# ---------------------------------------------------------------------------
def _decode_case(B, Hq, Hk, L_, D, dtype, density, seed, lens=None):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, D, generator=g).to(dtype)
    kc = torch.randn(B, Hk, L_, D, generator=g).to(dtype)
    vc = torch.randn(B, Hk, L_, D, generator=g).to(dtype)
    kv_len = torch.tensor(lens if lens is not None else [L_] * B, dtype=torch.int32)
    nb = math.ceil(L_ / 64)
    nbv = (kv_len + 63) // 64
    mask = M.decode_mask(torch.rand(B, Hk, nb, generator=g), nbv, density, nb)
    idx, cnt = M.lists_from_mask(mask)
    return q, kc, vc, kv_len, idx, cnt


class TestDecode:
    @pytest.mark.parametrize("splits", [1, 2, 3, 5])
    def test_splits_vs_oracle(self, splits):
        q, kc, vc, kv_len, idx, cnt = _decode_case(4, 8, 2, 1000, 128, torch.bfloat16, 0.3, 21,
                                                   lens=[1000, 999, 640, 65])
        ws = T.DecodeWorkspace(4, 8, 2, 128, 8, DEV)
        out = T.bsa_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), kv_len.to(DEV),
                           T.KeptBlocks(idx.to(DEV), cnt.to(DEV)), num_splits=splits, workspace=ws)
        ref = O.bsa_decode(q, kc, vc, kv_len, idx, cnt, 64)
        assert_bf16_close(out, ref)
        # a second call reuses the (self-resetting) tickets
        out2 = T.bsa_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), kv_len.to(DEV),
                            T.KeptBlocks(idx.to(DEV), cnt.to(DEV)), num_splits=splits, workspace=ws)
        assert torch.equal(out, out2)

    @pytest.mark.parametrize("splits,D,grp", [(24, 128, 7), (64, 128, 7), (40, 64, 8), (0, 128, 7)])
    def test_wide_splits_separate_merge(self, splits, D, grp):
        """More than 16 splits: the decode grid writes every split's partial and a merge
        kernel (launched behind it) combines them; one long sequence (the configs[3]
        shape at a smaller L), ragged lengths, splits with nothing kept, then the same
        call twice (partials are rewritten, no state carried over)."""
        B, Hk = 2, 4
        q, kc, vc, kv_len, idx, cnt = _decode_case(B, grp * Hk, Hk, 4096, D, torch.bfloat16, 0.1, 31,
                                                   lens=[4096, 2500])
        kept = T.KeptBlocks(idx.to(DEV), cnt.to(DEV))
        ws = T.DecodeWorkspace(B, grp * Hk, Hk, D, 64, DEV)
        run = lambda: T.bsa_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), kv_len.to(DEV), kept, num_splits=splits,
                                   workspace=ws)
        out = run()
        ref = O.bsa_decode(q, kc, vc, kv_len, idx, cnt, 64)
        assert_bf16_close(out, ref)
        assert torch.equal(out, run())
        # the merged (o, m, l) for a cross-GPU combine agree with the output
        po = torch.empty(B, grp * Hk, D, device=DEV)
        pm = torch.empty(B, grp * Hk, 2, device=DEV)
        T.bsa_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), kv_len.to(DEV), kept, num_splits=splits, workspace=ws,
                     partials=(po, pm))
        assert (po.bfloat16().float() - out.float()).abs().max().item() <= 1e-2

    def test_dynamic_claiming_more_items_than_ctas(self):
        """1536 work items > resident CTAs: items are claimed from the workspace counter,
        which must be back at zero for the next call."""
        q, kc, vc, kv_len, idx, cnt = _decode_case(64, 32, 8, 768, 128, torch.bfloat16, 0.5, 25)
        ws = T.DecodeWorkspace(64, 32, 8, 128, 3, DEV)
        kept = T.KeptBlocks(idx.to(DEV), cnt.to(DEV))
        outs = [T.bsa_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), kv_len.to(DEV), kept, num_splits=3, workspace=ws)
                for _ in range(3)]
        assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
        ref = O.bsa_decode(q[:4], kc[:4], vc[:4], kv_len[:4], idx[:4], cnt[:4], 64)
        assert_bf16_close(outs[0][:4], ref)
        assert int(ws.buf[: 64 * 8 * 4 + 8].view(torch.int32).abs().sum()) == 0  # tickets and counters reset

    @pytest.mark.parametrize("dtype,D,grp", [(torch.float32, 64, 4), (torch.float16, 128, 7), (torch.bfloat16, 64, 1)])
    def test_dtypes(self, dtype, D, grp):
        q, kc, vc, kv_len, idx, cnt = _decode_case(3, 2 * grp, 2, 520, D, dtype, 0.5, 22)
        out = T.bsa_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), kv_len.to(DEV),
                           T.KeptBlocks(idx.to(DEV), cnt.to(DEV)), num_splits=2)
        ref = O.bsa_decode(q, kc, vc, kv_len, idx, cnt, 64)
        if dtype == torch.float32:
            assert (out.cpu() - ref).abs().max().item() <= FP32_ABS
        else:
            assert_bf16_close(out, ref)

    def test_empty_lists(self):
        q, kc, vc, kv_len, idx, cnt = _decode_case(2, 4, 1, 256, 128, torch.bfloat16, 0.5, 23)
        cnt[1] = 0
        out = T.bsa_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), kv_len.to(DEV),
                           T.KeptBlocks(idx.to(DEV), cnt.to(DEV)), num_splits=2)
        assert out[1].abs().max().item() == 0.0
        assert_bf16_close(out, O.bsa_decode(q, kc, vc, kv_len, idx, cnt, 64))

    def test_partials_and_combine(self):
        """Split the kept lists in two halves (two 'GPUs'), combine the partials."""
        q, kc, vc, kv_len, idx, cnt = _decode_case(2, 8, 2, 2048, 128, torch.bfloat16, 0.4, 24)
        parts_o, parts_ml = [], []
        for half in range(2):
            sub = torch.full_like(idx, -1)
            c2 = torch.zeros_like(cnt)
            for b in range(2):
                for h in range(2):
                    n = int(cnt[b, h])
                    lo, hi = (0, n // 2) if half == 0 else (n // 2, n)
                    sub[b, h, : hi - lo] = idx[b, h, lo:hi]
                    c2[b, h] = hi - lo
            po = torch.empty(2, 8, 128, device=DEV)
            pm = torch.empty(2, 8, 2, device=DEV)
            T.bsa_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), kv_len.to(DEV),
                         T.KeptBlocks(sub.to(DEV), c2.to(DEV)), num_splits=2, partials=(po, pm))
            parts_o.append(po)
            parts_ml.append(pm)
        out = T.decode_combine(torch.stack(parts_o), torch.stack(parts_ml), torch.bfloat16)
        assert_bf16_close(out, O.bsa_decode(q, kc, vc, kv_len, idx, cnt, 64))


# ---------------------------------------------------------------------------
# gate target / losses / gate backward
# ---------------------------------------------------------------------------
class TestTarget:
    @pytest.mark.parametrize("dtype,S,Hq,Hk", [(torch.float32, 200, 2, 1), (torch.bfloat16, 512, 4, 2)])
    def test_target_vs_oracle(self, dtype, S, Hq, Hk):
        g = torch.Generator().manual_seed(S)
        q = torch.randn(1, Hq, S, 64, generator=g).to(dtype)
        k = torch.randn(1, Hk, S, 64, generator=g).to(dtype)
        tgt = T.gate_target_from_qk(q.to(DEV), k.to(DEV), 64)
        ref = O.gate_target_from_qk(q, k, 64)
        assert (tgt.cpu() - ref.float()).abs().max().item() <= (1e-5 if dtype == torch.float32 else 2e-2)

    @pytest.mark.parametrize("dtype,B,Hq,Hk,S,D", [
        (torch.bfloat16, 1, 4, 1, 448, 64),     # odd NB: last M tile has one q-block
        (torch.bfloat16, 2, 8, 2, 1000, 128),   # ragged S, GQA 4
        (torch.bfloat16, 1, 3, 3, 640, 128),    # MHA: one head per unit
        (torch.bfloat16, 1, 6, 2, 384, 64),     # GQA 3: a pair and a single head
        (torch.float16, 1, 4, 2, 512, 128),
        (torch.bfloat16, 1, 8, 2, 4096, 128),   # many units per CTA
    ])
    def test_tensor_core_block_max_matches_cuda_core(self, dtype, B, Hq, Hk, S, D):
        g = torch.Generator(device=DEV).manual_seed(S + Hq)
        q = torch.randn(B, Hq, S, D, device=DEV, generator=g).to(dtype)
        k = torch.randn(B, Hk, S, D, device=DEV, generator=g).to(dtype)
        t_tc, bm_tc = T.gate_target_from_qk(q, k, 64, return_block_max=True)
        t_ref, bm_ref = T.gate_target_from_qk(q, k, 64, return_block_max=True, force_simt=True)
        torch.cuda.synchronize()
        inf = torch.isinf(bm_ref)
        assert torch.equal(inf, torch.isinf(bm_tc))
        # fp32 accumulation in another order; bf16-emulated maxima may land one bf16 ulp apart
        assert (bm_tc[~inf] - bm_ref[~inf]).abs().max().item() <= 1e-2 * bm_ref[~inf].abs().max().item()
        assert (t_tc - t_ref).abs().max().item() <= 2e-2 * t_ref.max().item() + 1e-6

    def test_alternate_target(self):
        g = torch.Generator().manual_seed(5)
        q = torch.randn(1, 2, 256, 64, generator=g) * 3
        k = torch.randn(1, 2, 256, 64, generator=g) * 3
        tgt = T.gate_target_from_qk(q.to(DEV), k.to(DEV), 64, temperature=2.0, clamp=50.0)
        ref = O.gate_target_from_qk(q, k, 64, temperature=2.0, clamp=50.0)
        assert (tgt.cpu() - ref).abs().max().item() <= 1e-5

    def test_losses_vs_reference_fixtures(self, golden):
        for c in golden["objective"]:
            kl, sp, d = T.gate_losses(c["soft"].to(DEV), c["target"].to(DEV), 0.8, w_kl=1.0, w_sparse=0.5)
            assert kl.item() == pytest.approx(c["kl"].item(), rel=1e-4, abs=1e-6)
            assert sp.item() == pytest.approx(c["sparse"].item(), rel=1e-4, abs=1e-7)
            s = c["soft"].clone().double().requires_grad_(True)
            (O.gate_loss(s, c["target"].double()) + 0.5 * O.sparsity_loss(s, 0.8)).backward()
            torch.testing.assert_close(d.cpu().double(), s.grad, atol=1e-5, rtol=1e-3)

    def test_gate_backward_vs_autograd(self):
        torch.manual_seed(1)
        B, Hq, Hk, S, D = 2, 4, 2, 256, 64
        gate = T.AttnGate(Hq, D).to(DEV)
        with torch.no_grad():
            gate.gate_proj_out.weight.mul_(30)
        q = torch.randn(B, Hq, S, D, device=DEV, requires_grad=True)
        k = torch.randn(B, Hk, S, D, device=DEV, requires_grad=True)
        tgt = torch.softmax(torch.randn(B, Hq, 16, device=DEV), -1).view(B, Hq, 4, 4)
        out = gate(q, k)
        total, _, _ = T.gate_objective(out.soft_scores, tgt, 0.8, 1.0, 0.1)
        total.backward()
        # oracle: the reference gate maths under torch autograd, on CPU in fp64
        w_in = gate.gate_proj_in.weight.detach().cpu().double().requires_grad_(True)
        b_in = gate.gate_proj_in.bias.detach().cpu().double().requires_grad_(True)
        w_out = gate.gate_proj_out.weight.detach().cpu().double().requires_grad_(True)
        qc = q.detach().cpu().double().requires_grad_(True)
        kc = k.detach().cpu().double().requires_grad_(True)
        soft, _, _ = O.gate_forward_gqa(qc, kc, w_in, b_in, w_out, 64, 0.5)
        ref_total = O.gate_loss(soft, tgt.cpu().double()) + 0.1 * O.sparsity_loss(soft, 0.8)
        ref_total.backward()
        assert total.item() == pytest.approx(ref_total.item(), rel=1e-4)
        for ours, ref in [(gate.gate_proj_in.weight.grad, w_in.grad), (gate.gate_proj_in.bias.grad, b_in.grad),
                          (gate.gate_proj_out.weight.grad, w_out.grad), (q.grad, qc.grad), (k.grad, kc.grad)]:
            torch.testing.assert_close(ours.cpu().double(), ref, atol=1e-6, rtol=2e-3)
