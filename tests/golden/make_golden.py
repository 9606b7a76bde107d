"""Generate the golden fixtures in this folder by running the REFERENCE implementation.

Run in the build container, where the reference checkout is importable:

    TASFT_REFERENCE=/path/to/tasft python tests/golden/make_golden.py

It imports the reference's own modules (``tasft.modules.attn_gate``,
``tasft.kernels.block_sparse_fa`` with ``TRITON_INTERPRET=1`` so its Triton kernel
runs on the CPU in fp32, and ``tasft/training/objectives.py`` loaded standalone because
``tasft.training``'s package init needs ``structlog``) and writes their outputs for
small seeded inputs to ``golden.pt``. The GPU box never runs this script; the tests
read only the committed ``golden.pt``.
"""
from __future__ import annotations

import importlib.util
import math
import os
import sys
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

import torch  # noqa: E402

HERE = Path(__file__).resolve().parent


def _load_reference(root: Path):
    sys.path.insert(0, str(root))
    from tasft.kernels import block_sparse_fa  # noqa: PLC0415
    from tasft.modules import attn_gate  # noqa: PLC0415

    spec = importlib.util.spec_from_file_location(
        "tasft_ref_objectives", root / "tasft" / "training" / "objectives.py"
    )
    obj = importlib.util.module_from_spec(spec)
    sys.modules["tasft_ref_objectives"] = obj  # slots dataclass needs the module registered
    spec.loader.exec_module(obj)
    return attn_gate, block_sparse_fa, obj


def _gate_cases(attn_gate):
    cases = []
    specs = [
        # (B, H, S, D, block, hidden, tau, causal, dtype, seed)
        (1, 2, 256, 32, 64, None, 0.5, True, torch.float32, 1),
        (2, 3, 200, 16, 32, 24, 0.499, True, torch.float32, 2),   # ragged last block
        (1, 2, 192, 64, 64, 64, 0.39, False, torch.float32, 3),   # non-causal
        (1, 4, 256, 64, 64, None, 0.5, True, torch.bfloat16, 4),  # bf16 module
        (1, 2, 130, 128, 128, None, 0.46, True, torch.float32, 5), # block 128, ragged
    ]
    for b, h, s, d, blk, hid, tau, causal, dt, seed in specs:
        torch.manual_seed(seed)
        gate = attn_gate.AttnGate(h, d, block_size=blk, gate_hidden_dim=hid,
                                  default_threshold=tau, is_causal=causal)
        # make scores spread out so the threshold is not tie-dominated
        with torch.no_grad():
            gate.gate_proj_out.weight.mul_(60.0)
        gate = gate.to(dt)
        g = torch.Generator().manual_seed(100 + seed)
        q = torch.randn(b, h, s, d, generator=g).to(dt)
        k = torch.randn(b, h, s, d, generator=g).to(dt)
        out = gate(q, k)
        cases.append({
            "B": b, "H": h, "S": s, "D": d, "block": blk, "tau": tau, "causal": causal,
            "dtype": str(dt), "q": q, "k": k,
            "w_in": gate.gate_proj_in.weight.detach().float().clone(),
            "b_in": gate.gate_proj_in.bias.detach().float().clone(),
            "w_out": gate.gate_proj_out.weight.detach().float().clone(),
            "pooled_q": gate._pool_to_blocks(q).detach().clone(),
            "soft": out.soft_scores.detach().clone(),
            "hard": out.hard_mask.clone(),
            "sparsity": float(out.sparsity_ratio),
        })
    return cases


def _kernel_cases(bsfa):
    cases = []
    specs = [
        # (B, H, S, D, block, causal, density, seed)
        (1, 2, 256, 64, 64, True, 0.5, 11),
        (1, 2, 200, 64, 64, True, 0.6, 12),   # ragged S
        (1, 1, 256, 128, 64, True, 0.4, 13),  # head_dim 128
        (1, 2, 192, 64, 64, False, 0.5, 14),  # non-causal
        (1, 1, 256, 64, 32, True, 0.5, 15),   # block 32
        (1, 1, 256, 64, 128, True, 1.0, 16),  # block 128, dense
    ]
    for b, h, s, d, blk, causal, dens, seed in specs:
        g = torch.Generator().manual_seed(seed)
        q = torch.randn(b, h, s, d, generator=g)
        k = torch.randn(b, h, s, d, generator=g)
        v = torch.randn(b, h, s, d, generator=g)
        nb = math.ceil(s / blk)
        mask = torch.rand(b, h, nb, nb, generator=g) < dens
        mask[..., 0] = True
        # one row with nothing kept -> zero output rows
        mask[0, 0, nb - 1, :] = False
        kern = bsfa.BlockSparseFlashAttention(block_size=blk, min_sparsity_for_speedup=0.0)
        out = kern._triton_forward(q, k, v, mask, causal)
        cases.append({"B": b, "H": h, "S": s, "D": d, "block": blk, "causal": causal,
                      "q": q, "k": k, "v": v, "mask": mask, "out": out.clone()})
    return cases


def _objective_cases(obj):
    T = obj.TASFTObjective
    cases = []
    for seed, (b, h, s, blk) in enumerate([(1, 2, 64, 8), (2, 1, 70, 16), (1, 3, 128, 32)]):
        g = torch.Generator().manual_seed(200 + seed)
        sc = torch.randn(b, h, s, s, generator=g) * 3.0
        sc = sc + torch.triu(torch.full((s, s), float("-inf")), diagonal=1)
        target = T.compute_gate_target(sc, blk)
        nb = target.shape[-1]
        soft = torch.rand(b, h, nb, nb, generator=g) * torch.ones(nb, nb).tril()
        cases.append({
            "scores": sc, "block": blk, "target": target, "soft": soft,
            "kl": T.compute_gate_loss(soft, target).clone(),
            "sparse": T.compute_sparsity_loss(soft, 0.8).clone(),
        })
    return cases


def main() -> None:
    if "TASFT_REFERENCE" not in os.environ:
        raise SystemExit("set TASFT_REFERENCE to the reference checkout (the folder holding tasft/)")
    root = Path(os.environ["TASFT_REFERENCE"])
    attn_gate, bsfa, obj = _load_reference(root)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    data = {
        "gate": _gate_cases(attn_gate),
        "kernel": _kernel_cases(bsfa),
        "objective": _objective_cases(obj),
        "generator": "tests/golden/make_golden.py (reference run in the build container)",
    }
    torch.save(data, HERE / "golden.pt")
    print("wrote", HERE / "golden.pt")


if __name__ == "__main__":
    main()
