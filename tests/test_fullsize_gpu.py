"""Parity at the BASELINE configs' full sizes, through properties that do not need the
CPU oracle to run at that size:

* prefill with every causal block kept equals dense causal GQA attention (C2 shape);
* long-context prefill (C4: S = 32768, 90% sparsity): sampled q-blocks against dense
  attention over exactly their kept keys, and every output inside the convex hull of V;
* decode with every block kept equals dense attention (C3 shape); C4 decode against a
  gather of its kept keys;
* gate target at the full C5 grid: tensor-core tile maxima equal the CUDA-core ones.
References here are torch fp32 on the GPU, used only as checkers.
"""
from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

import tasft_b200 as T
from tasft_b200 import masks as M

pytestmark = pytest.mark.gpu
DEV = "cuda"
BF16_ATOL = 2e-2  # bf16 output tolerance used across the suite


def _dense_causal(q, k, v):
    grp = q.shape[1] // k.shape[1]
    kk = k.float().repeat_interleave(grp, 1)
    vv = v.float().repeat_interleave(grp, 1)
    return F.scaled_dot_product_attention(q.float(), kk, vv, is_causal=True)


def test_prefill_all_kept_equals_dense_llama():
    B, Hq, Hk, S, D = 4, 32, 8, 4096, 128
    g = torch.Generator(device=DEV).manual_seed(21)
    q = torch.randn(B, Hq, S, D, device=DEV, generator=g).bfloat16()
    k = torch.randn(B, Hk, S, D, device=DEV, generator=g).bfloat16()
    v = torch.randn(B, Hk, S, D, device=DEV, generator=g).bfloat16()
    nb = S // 64
    mask = torch.ones(B, Hk, nb, nb, dtype=torch.bool, device=DEV).tril()
    out = T.BlockSparseFlashAttention().forward(q, k, v, mask)
    for b in range(B):  # per sequence keeps the fp32 reference's memory modest
        ref = _dense_causal(q[b:b + 1], k[b:b + 1], v[b:b + 1])
        assert (out[b:b + 1].float() - ref).abs().max().item() <= BF16_ATOL


def test_prefill_qwen_long_context_sampled_blocks():
    B, Hq, Hk, S, D = 1, 28, 4, 32768, 128
    g = torch.Generator(device=DEV).manual_seed(22)
    q = torch.randn(B, Hq, S, D, device=DEV, generator=g).bfloat16()
    k = torch.randn(B, Hk, S, D, device=DEV, generator=g).bfloat16()
    v = torch.randn(B, Hk, S, D, device=DEV, generator=g).bfloat16()
    nb = S // 64
    mask = M.prefill_mask(torch.rand(B, Hk, nb, nb, device=DEV, generator=g), 0.1)
    out = T.BlockSparseFlashAttention().forward(q, k, v, mask)
    torch.cuda.synchronize()
    # convex hull: every output coordinate lies within the range of its kv-head's V
    grp = Hq // Hk
    vmin = v.float().amin(dim=2).repeat_interleave(grp, 1)  # [B, Hq, D]
    vmax = v.float().amax(dim=2).repeat_interleave(grp, 1)
    o = out.float()
    assert (o >= vmin.unsqueeze(2) - BF16_ATOL).all() and (o <= vmax.unsqueeze(2) + BF16_ATOL).all()
    # sampled q-blocks against dense attention over exactly their kept keys
    scale = 1.0 / math.sqrt(D)
    for hq, i in [(0, 0), (5, 17), (13, 255), (27, 511)]:
        hk = hq // grp
        kept = mask[0, hk, i].nonzero().flatten()
        keys = (kept[:, None] * 64 + torch.arange(64, device=DEV)[None, :]).flatten()
        qi = q[0, hq, i * 64:(i + 1) * 64].float()
        s = (qi @ k[0, hk, keys].float().T) * scale
        qpos = torch.arange(i * 64, (i + 1) * 64, device=DEV)[:, None]
        s = s.masked_fill(keys[None, :] > qpos, float("-inf"))
        p = torch.softmax(s, dim=-1)
        # the kernel rounds p to bf16 before P.V, as the reference kernel does
        ref = p.bfloat16().float() @ v[0, hk, keys].float() / p.bfloat16().float().sum(-1, keepdim=True)
        assert (o[0, hq, i * 64:(i + 1) * 64] - ref).abs().max().item() <= BF16_ATOL


def test_decode_all_kept_equals_dense_llama():
    B, Hq, Hk, L, D = 64, 32, 8, 8192, 128
    g = torch.Generator(device=DEV).manual_seed(23)
    q = torch.randn(B, Hq, D, device=DEV, generator=g).bfloat16()
    kc = torch.randn(B, Hk, L, D, device=DEV, generator=g).bfloat16()
    vc = torch.randn(B, Hk, L, D, device=DEV, generator=g).bfloat16()
    kv_len = torch.full((B,), L, dtype=torch.int32, device=DEV)
    nb = L // 64
    idx = torch.arange(nb, device=DEV, dtype=torch.int32).expand(B, Hk, nb).contiguous()
    cnt = torch.full((B, Hk), nb, dtype=torch.int32, device=DEV)
    out = T.bsa_decode(q, kc, vc, kv_len, T.KeptBlocks(idx, cnt), 64).float()
    grp = Hq // Hk
    for b0 in range(0, B, 16):
        sl = slice(b0, b0 + 16)
        ref = F.scaled_dot_product_attention(q[sl].float().unsqueeze(2), kc[sl].float().repeat_interleave(grp, 1),
                                             vc[sl].float().repeat_interleave(grp, 1)).squeeze(2)
        assert (out[sl] - ref).abs().max().item() <= BF16_ATOL


def test_decode_qwen_long_context_vs_gathered_keys():
    B, Hq, Hk, L, D = 1, 28, 4, 32768, 128
    g = torch.Generator(device=DEV).manual_seed(24)
    q = torch.randn(B, Hq, D, device=DEV, generator=g).bfloat16()
    kc = torch.randn(B, Hk, L, D, device=DEV, generator=g).bfloat16()
    vc = torch.randn(B, Hk, L, D, device=DEV, generator=g).bfloat16()
    kv_len = torch.tensor([L - 100], dtype=torch.int32, device=DEV)
    nb = L // 64
    mask = M.decode_mask(torch.rand(B, Hk, nb, device=DEV, generator=g), (kv_len + 63) // 64, 0.1, nb)
    kept = T.KeptBlocks(*M.lists_from_mask(mask))
    out = T.bsa_decode(q, kc, vc, kv_len, kept).float()
    grp = Hq // Hk
    for hk in range(Hk):
        blocks = kept.idx[0, hk, : int(kept.cnt[0, hk])].long()
        keys = (blocks[:, None] * 64 + torch.arange(64, device=DEV)[None, :]).flatten()
        keys = keys[keys < int(kv_len[0])]
        s = (q[0, hk * grp:(hk + 1) * grp].float() @ kc[0, hk, keys].float().T) / math.sqrt(D)
        p = torch.softmax(s, dim=-1)
        ref = p.bfloat16().float() @ vc[0, hk, keys].float() / p.bfloat16().float().sum(-1, keepdim=True)
        assert (out[0, hk * grp:(hk + 1) * grp] - ref).abs().max().item() <= BF16_ATOL


def test_gate_target_full_c5_tensor_core_equals_cuda_core():
    B, Hq, Hk, S, D = 4, 32, 8, 4096, 128
    g = torch.Generator(device=DEV).manual_seed(25)
    q = torch.randn(B, Hq, S, D, device=DEV, generator=g).bfloat16()
    k = torch.randn(B, Hk, S, D, device=DEV, generator=g).bfloat16()
    t_tc, bm_tc = T.gate_target_from_qk(q, k, 64, return_block_max=True)
    t_cc, bm_cc = T.gate_target_from_qk(q, k, 64, return_block_max=True, force_simt=True)
    inf = torch.isinf(bm_cc)
    assert torch.equal(inf, torch.isinf(bm_tc))
    # fp32 sums in another order; the bf16-emulated maxima may land one bf16 ulp apart
    rel = ((bm_tc[~inf] - bm_cc[~inf]).abs() / bm_cc[~inf].abs().clamp_min(1.0)).max().item()
    assert rel <= 1e-2
    # each (b, h) target is a distribution over its NB x NB grid
    sums = t_tc.sum(dim=(-1, -2))
    assert torch.allclose(sums, torch.ones_like(sums), atol=1e-4)
    assert (t_tc - t_cc).abs().max().item() <= 2e-2 * t_cc.max().item() + 1e-6
