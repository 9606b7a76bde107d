"""Benchmark: block-sparse prefill effective TFLOP/s (+ decode tok/s) at the Llama-3-8B
attention shape with 80% block sparsity, on N B200 GPUs (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: prefill bf16 B=4 (per GPU), 32 q-heads /
8 kv-heads, S=4096, D=128, block 64, causal, mask from the random-init AttnGate's fp32
scores (kv-head max, row rule of ``tasft_b200.masks.prefill_mask`` at density 0.2);
decode bf16 batch 64 (per GPU), KV 8192, 26 kept blocks per (sequence, kv-head).
Work is partitioned by batch, so N GPUs process N independent shards ("weak" scaling,
no data-path collective). Each timed step is bracketed by CUDA events on the launching
stream; L2 is flushed (a 256 MiB write) before every timed step, outside the events.

``value`` = kept-block FLOPs of all ranks / max-over-ranks device time of the step
``mask -> kept lists -> tcgen05 prefill``. ``e2e`` = the same metric through
``BlockSparseFlashAttention.forward`` with pinned host inputs (H2D q, k, v, mask and D2H
of the output inside the timed region; one call per sequence, copies and calls pipelined
on two streams; the unpipelined time is reported beside it). ``--impl reference`` times
the CPU oracle (the restatement of the reference kernel) on the host cores instead.

Also on the line: ``roofline`` (prefill kernel vs measured bf16 peak), ``decode``
(configs[2], HBM roofline; ``decode.paged`` the same over a 16-token paged cache),
``gate`` (mask build replayed from a CUDA graph, HBM roofline), ``gate_target``
(configs[4], tensor roofline), ``long_decode`` (configs[3] decode at KV 32768; with N > 1
the cache is split by position over the ranks and the partials are all-gathered and
merged), ``clocks`` (nvidia-smi sampled during the timed phases), ``cpu_baseline``.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "prefill effective TFLOP/s + decode tok/s, Llama-3-8B attn @80% sparsity"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
CFG = dict(B=4, Hq=32, Hk=8, S=4096, D=128, block=64, density=0.2)
DEC = dict(B=64, Hq=32, Hk=8, L=8192, D=128, block=64, density=0.2)
LONG = dict(B=1, Hq=28, Hk=4, L=32768, D=128, block=64, density=0.1)


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "src": "measured"}
    return {**PEAKS_FALLBACK, "src": "fallback"}


def load_traffic():
    p = ROOT / "profiles" / "traffic.json"
    return json.loads(p.read_text()) if p.exists() else {}


# ---------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi polled every 200 ms during the timed region (clocks + throttle reasons).

    One-shot queries from a thread: a long-running `nvidia-smi -lms` writing into a pipe
    is block-buffered and loses its samples when it is stopped.
    """

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.lines: list[str] = []
        self._stop = threading.Event()

    def __enter__(self):
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()
        return self

    def _run(self):
        while not self._stop.is_set():
            try:
                r = subprocess.run(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                    "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                self.lines.extend(ln.strip() for ln in r.stdout.splitlines() if ln.strip())
            except (OSError, subprocess.SubprocessError):
                return
            self._stop.wait(0.2)

    def __exit__(self, *exc):
        self._stop.set()
        self.t.join(timeout=10)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
def dist_setup(n_gpus: int):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import torch.distributed as dist  # noqa: PLC0415

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, ws, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist  # noqa: PLC0415

        dist.barrier()


def max_over_ranks(x: float, ws: int) -> float:
    if ws == 1:
        return x
    import torch.distributed as dist  # noqa: PLC0415

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, ws: int) -> float:
    if ws == 1:
        return x
    import torch.distributed as dist  # noqa: PLC0415

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ---------------------------------------------------------------------------
def make_prefill_inputs(seed: int, dev):
    import tasft_b200 as T  # noqa: PLC0415
    from tasft_b200 import masks as M  # noqa: PLC0415

    c = CFG
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(c["B"], c["Hq"], c["S"], c["D"], device=dev, dtype=torch.bfloat16, generator=g)
    k = torch.randn(c["B"], c["Hk"], c["S"], c["D"], device=dev, dtype=torch.bfloat16, generator=g)
    v = torch.randn(c["B"], c["Hk"], c["S"], c["D"], device=dev, dtype=torch.bfloat16, generator=g)
    torch.manual_seed(0)
    gate = T.AttnGate(c["Hq"], c["D"], block_size=c["block"]).to(dev)
    with torch.no_grad():
        out = gate(q, k)
    scores = M.group_max(out.soft_scores, c["Hk"])  # fp32, per kv-head
    mask = M.prefill_mask(scores, c["density"])      # [B, Hk, NB, NB]
    return q, k, v, mask, gate


def make_decode_inputs(seed: int, dev):
    import tasft_b200 as T  # noqa: PLC0415
    from tasft_b200 import masks as M  # noqa: PLC0415

    c = DEC
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(c["B"], c["Hq"], c["D"], device=dev, dtype=torch.bfloat16, generator=g)
    kc = torch.randn(c["B"], c["Hk"], c["L"], c["D"], device=dev, dtype=torch.bfloat16, generator=g)
    vc = torch.randn(c["B"], c["Hk"], c["L"], c["D"], device=dev, dtype=torch.bfloat16, generator=g)
    kv_len = torch.full((c["B"],), c["L"], dtype=torch.int32, device=dev)
    torch.manual_seed(0)
    gate = T.AttnGate(c["Hq"], c["D"], block_size=c["block"]).to(dev)
    with torch.no_grad():
        sc = gate(q.unsqueeze(2), kc).soft_scores[:, :, 0, :]  # query pooled with the 1-token padding
    nb = c["L"] // c["block"]
    mask = M.decode_mask(M.group_max(sc, c["Hk"]), (kv_len + 63) // 64, c["density"], nb)
    idx, cnt = M.lists_from_mask(mask)
    return q, kc, vc, kv_len, T.KeptBlocks(idx, cnt)


class L2Flush:
    def __init__(self, dev):
        self.buf = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    def __call__(self):
        self.buf.fill_(1.0)


def graphed(fn):
    """Capture ``fn`` (one step of device work) in a CUDA graph and return its replay: for
    short steps whose Python launch path would otherwise be timed instead of the kernels."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()  # first call outside capture: lazy set-up (function attributes, workspaces)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g.replay


def time_steps(fn, steps, warmup, flush, ws):
    for _ in range(warmup):
        flush()
        fn()
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    times = []
    for _ in range(steps):
        flush()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(st)
        fn()
        e1.record(st)
        times.append((e0, e1))
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in times]


# ---------------------------------------------------------------------------
def cpu_prefill_sample(budget_s: float = 10.0):
    """Oracle (reference restatement) on host cores: (b, kv-head) chunks of the C2 workload."""
    import oracle as O  # noqa: PLC0415  (CPU baseline leg)
    from tasft_b200 import masks as M  # noqa: PLC0415

    torch.set_num_threads(os.cpu_count() or 1)
    c = CFG
    grp = c["Hq"] // c["Hk"]
    g = torch.Generator().manual_seed(1234)
    nb = c["S"] // c["block"]
    q = torch.randn(1, grp, c["S"], c["D"], generator=g).to(torch.bfloat16)
    k = torch.randn(1, 1, c["S"], c["D"], generator=g).to(torch.bfloat16)
    v = torch.randn(1, 1, c["S"], c["D"], generator=g).to(torch.bfloat16)
    mask = M.prefill_mask(torch.rand(1, 1, nb, nb, generator=g), c["density"])
    flops_chunk = int(mask.sum()) * grp * 4 * c["block"] * c["block"] * c["D"]
    t0 = time.perf_counter()
    n = 0
    while True:
        O.bsa_prefill_masked_dense(q, k, v, mask, c["block"])
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": round(flops_chunk * n / dt / 1e12, 6), "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{n} x one (batch, kv-head) chunk = {grp} q-heads, S={c['S']}, D={c['D']}, "
                      f"{int(mask.sum())} kept blocks; oracle masked-dense restatement in bf16/fp32 "
                      f"(oracle/tasft_oracle.py:bsa_prefill_masked_dense), {dt:.1f} s"}


# ---------------------------------------------------------------------------
def bench_dropin(q, k, v, gate, kern, flush, ws, args, peaks):
    """Prefill in the form the reference callers use (tasft_attention.py:574-593, 725-729):
    K/V repeated per q-head (Hk = Hq) and the gate's per-q-head masks. Also the reference's
    own Triton kernel (block_sparse_fa.py:108-269) on the same inputs when the reference
    package is importable (baseline/_ref), on one GPU only."""
    import tasft_b200 as T  # noqa: PLC0415
    from tasft_b200 import masks as M  # noqa: PLC0415

    grp = CFG["Hq"] // CFG["Hk"]
    ke = k.repeat_interleave(grp, dim=1)
    ve = v.repeat_interleave(grp, dim=1)
    with torch.no_grad():
        sc = gate(q, ke).soft_scores  # per q-head fp32 scores over the expanded K
    mask_q = M.prefill_mask(sc, CFG["density"])  # [B, Hq, NB, NB]
    kept_q = T.mask_to_kept(mask_q, True)
    kept_blocks = int(mask_q.sum().item())
    flops = kept_blocks * 4 * CFG["block"] * CFG["block"] * CFG["D"]
    out = torch.empty_like(q)
    t_k = time_steps(lambda: kern.forward(q, ke, ve, kept_q, out=out), args.steps, args.warmup, flush, ws)
    t_f = time_steps(lambda: kern.forward(q, ke, ve, mask_q, out=out), args.steps, args.warmup, flush, ws)
    ms_k, ms_f = statistics.mean(t_k), statistics.mean(t_f)
    info = {"config": "BASELINE configs[1] as the reference callers pass it: K/V repeated to 32 heads, per-q-head "
                      "gate masks (prefill_mask at density 0.2 on each q-head's scores)",
            "kept_blocks": kept_blocks, "gflop": round(flops / 1e9, 3),
            "ms_kernel": round(ms_k, 4), "ms_forward": round(ms_f, 4),
            "tflops": round(flops / (ms_k * 1e-3) / 1e12, 2),
            "frac": round(flops / (ms_k * 1e-3) / 1e12 / peaks["bf16_tflops"], 4)}
    if ws == 1 and not args.no_triton:
        info["triton_ref"] = bench_triton_ref(q, ke, ve, mask_q, out, flops, ms_k, flush, args)
    del ke, ve
    return info


def bench_triton_ref(q, ke, ve, mask_q, ours_out, flops, ours_ms, flush, args):
    """The reference's Triton kernel JIT-compiled on this GPU, unmodified, through its own
    ``_triton_forward`` (launch incl. its host-side mask prep) and ``forward`` (adds the
    sparsity-stats host sync)."""
    ref_root = ROOT / "baseline" / "_ref"
    if not (ref_root / "tasft" / "__init__.py").exists():
        return {"unavailable": "reference package not installed in baseline/_ref"}
    try:
        if str(ref_root) not in sys.path:
            sys.path.insert(0, str(ref_root))
        from tasft.kernels.block_sparse_fa import BlockSparseFlashAttention as RefBSFA  # noqa: PLC0415
        from tasft.kernels.block_sparse_fa import KernelBackend as RefBackend  # noqa: PLC0415

        ref = RefBSFA(block_size=CFG["block"], backend=RefBackend.TRITON)
        o_ref = ref._triton_forward(q, ke, ve, mask_q, True)  # JIT compile
        torch.cuda.synchronize()
        err = (o_ref.float() - ours_out.float()).abs().max().item()
        steps = max(3, min(args.steps, 5))
        t_l = time_steps(lambda: ref._triton_forward(q, ke, ve, mask_q, True), steps, 3, flush, 1)
        t_f = time_steps(lambda: ref.forward(q, ke, ve, mask_q, causal=True), steps, 3, flush, 1)
        ms_l, ms_f = statistics.mean(t_l), statistics.mean(t_f)
        return {"ms_launch": round(ms_l, 4), "ms_forward": round(ms_f, 4),
                "tflops": round(flops / (ms_l * 1e-3) / 1e12, 2),
                "speedup_ours_vs_triton": round(ms_l / ours_ms, 2),
                "max_abs_diff_vs_ours": round(err, 5),
                "what": "unmodified reference _block_sparse_attn_fwd_kernel (Triton JIT on this B200) on the same "
                        "expanded K/V and per-q-head masks"}
    except Exception as e:  # noqa: BLE001 - record why the reference kernel did not run
        return {"unavailable": f"{type(e).__name__}: {str(e).splitlines()[0][:200]}"}


def bench_epilogue_gate(gate, flush, ws, args, peaks):
    """The inference flow with the projection epilogue (``qkv_rope_pool``: head split +
    rotary + the gate's block means in one pass over the q/k/v projection outputs) and the
    gate run from those means (``AttnGate.forward_pooled``): the gate no longer re-reads Q
    and K. Algorithmic bytes of the epilogue: read + write of q, k, v (+ cos/sin)."""
    import tasft_b200 as T  # noqa: PLC0415

    c = CFG
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(77)
    ql = torch.randn(c["B"], c["S"], c["Hq"] * c["D"], device=dev, dtype=torch.bfloat16, generator=g)
    kl = torch.randn(c["B"], c["S"], c["Hk"] * c["D"], device=dev, dtype=torch.bfloat16, generator=g)
    vl = torch.randn_like(kl)
    inv = 1.0 / (10000 ** (torch.arange(0, c["D"], 2, device=dev).float() / c["D"]))
    ang = torch.outer(torch.arange(c["S"], device=dev).float(), inv)
    emb = torch.cat([ang, ang], -1)
    cos, sin = emb.cos().bfloat16()[None], emb.sin().bfloat16()[None]
    res = {}

    def epi():
        res["o"] = T.qkv_rope_pool(ql, kl, vl, c["Hq"], c["Hk"], cos, sin, c["block"])

    # graph replay: the kernel alone, not the Python launch path (argument struct, output
    # allocation), which otherwise takes longer than the kernel
    t_e = time_steps(graphed(epi), args.steps, args.warmup, flush, ws)
    ms_e = statistics.mean(t_e)
    _, _, _, pq, pk = res["o"]
    nbytes = 2 * (ql.numel() + kl.numel() + vl.numel()) * 2 + 2 * cos.numel() * 2
    t_g = time_steps(graphed(lambda: gate.forward_pooled(pq, pk, c["S"], c["S"])), args.steps, args.warmup, flush, ws)
    ms_g = statistics.mean(t_g)
    return {"epilogue_ms": round(ms_e, 4),
            "epilogue_roofline": {"bound": "hbm", "achieved": round(nbytes / (ms_e * 1e-3) / 1e9, 1),
                                  "peak": peaks["hbm_gbs"], "unit": "GB/s",
                                  "frac": round(nbytes / (ms_e * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
                                  "traffic": load_traffic().get("epilogue"),
                                  "algorithmic": f"{nbytes / 1e6:.1f} MB (read + write of q, k, v; cos, sin)"},
            "gate_from_means_ms": round(ms_g, 4),
            "what": "qkv_rope_pool (tasft_qkv_rope_pool) on [B, S, H*D] projection outputs, then "
                    "AttnGate.forward_pooled (projection + pair kernels); both timed as CUDA graph replays"}


def bench_gate_train(q, k, flush, ws, args):
    """BASELINE configs[4] end to end: gate forward (autograd), target from Q and K, KL +
    sparsity loss, backward to the gate parameters. Times the whole step and the
    loss + backward part alone."""
    import tasft_b200 as T  # noqa: PLC0415

    torch.manual_seed(0)
    gate = T.AttnGate(CFG["Hq"], CFG["D"], block_size=CFG["block"]).to(q.device)

    def train_step():
        go = gate(q, k)
        tgt = T.gate_target_from_qk(q, k, CFG["block"])
        total, _, _ = T.gate_objective(go.soft_scores, tgt, 0.8, 1.0, 0.01)
        total.backward()

    t_all = time_steps(train_step, args.steps, args.warmup, flush, ws)
    st = torch.cuda.current_stream()
    bw = []
    for i in range(args.warmup + args.steps):
        go = gate(q, k)
        tgt = T.gate_target_from_qk(q, k, CFG["block"])
        flush()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        total, _, _ = T.gate_objective(go.soft_scores, tgt, 0.8, 1.0, 0.01)
        total.backward()
        e1.record(st)
        if i >= args.warmup:
            bw.append((e0, e1))
    torch.cuda.synchronize()
    ms_bw = statistics.mean(a.elapsed_time(b) for a, b in bw)
    return {"config": "BASELINE configs[4]: B=4, Hq=32, Hk=8, S=4096, D=128, gate hidden 32; NB=64",
            "ms_train_step": round(statistics.mean(t_all), 4), "ms_loss_and_backward": round(ms_bw, 4),
            "kernels": "gate mask build + target_tc + target_softmax + loss_rows/final/add + gate bwd (5 kernels)",
            "what": "AttnGate.forward (autograd) -> gate_target_from_qk -> gate_objective -> backward to "
                    "gate_proj_in/out"}


def bench_qwen_prefill(rank, ws, dev, flush, args, peaks):
    """BASELINE configs[3] prefill: B=1, Hq=28, Hk=4, S=32768, 90% block sparsity. With N
    ranks the q-blocks are cut into N ranges of equal kept work (``shards.qblock_ranges``);
    each rank computes its range (strong scaling, no exchange)."""
    import tasft_b200 as T  # noqa: PLC0415
    from tasft_b200 import masks as M  # noqa: PLC0415
    from tasft_b200 import shards as SH  # noqa: PLC0415

    c = dict(B=1, Hq=28, Hk=4, S=32768, D=128, block=64, density=0.1)
    g = torch.Generator(device=dev).manual_seed(4321)  # same inputs on every rank
    q = torch.randn(c["B"], c["Hq"], c["S"], c["D"], device=dev, dtype=torch.bfloat16, generator=g)
    k = torch.randn(c["B"], c["Hk"], c["S"], c["D"], device=dev, dtype=torch.bfloat16, generator=g)
    v = torch.randn(c["B"], c["Hk"], c["S"], c["D"], device=dev, dtype=torch.bfloat16, generator=g)
    torch.manual_seed(0)
    gate = T.AttnGate(c["Hq"], c["D"], block_size=c["block"]).to(dev)
    with torch.no_grad():
        sc = M.group_max(gate(q, k).soft_scores, c["Hk"])
    mask = M.prefill_mask(sc, c["density"])
    kept = T.mask_to_kept(mask, True)
    grp = c["Hq"] // c["Hk"]
    total_blocks = int(mask.sum().item())
    lo, hi = SH.qblock_ranges(kept, ws)[rank]
    mine = SH.restrict_qblocks(kept, lo, hi) if ws > 1 else kept
    my_blocks = int(mine.cnt.sum().item())
    kern = T.BlockSparseFlashAttention(block_size=c["block"])
    out = torch.empty_like(q)
    rng = (lo, hi) if ws > 1 else None  # the rank visits only its q-block window
    t = time_steps(lambda: kern.forward(q, k, v, mine, out=out, q_block_range=rng), args.steps, args.warmup, flush, ws)
    ms = statistics.mean(t)
    ms_max = max_over_ranks(ms, ws)
    unit = grp * 4 * c["block"] * c["block"] * c["D"]
    flops = total_blocks * unit
    info = {"config": "BASELINE configs[3] prefill: B=1, Hq=28, Hk=4, S=32768, D=128, block 64, causal, 90% block "
                      "sparsity (kv-head masks from the random-init gate)",
            "gflop": round(flops / 1e9, 2), "ms": round(ms_max, 4),
            "tflops": round(flops / (ms_max * 1e-3) / 1e12, 2),
            # of the measured peak of all the ranks' GPUs together
            "frac": round(flops / (ms_max * 1e-3) / 1e12 / (peaks["bf16_tflops"] * ws), 4),
            "split": f"q-block ranges of equal kept work over {ws} rank(s)" if ws > 1 else "one GPU",
            "scaling": "strong"}
    if ws > 1:
        info["rank_blocks_max_over_mean"] = round(max_over_ranks(float(my_blocks), ws) / (total_blocks / ws), 4)
    del q, k, v, out
    return info


def bench_strong_c2(q, k, v, mask, rank, ws, flush, args, peaks):
    """BASELINE configs[1] as ONE global B=4 layer split over the ranks by (sequence,
    kv-head) units, balanced by kept blocks (``shards.assign_units``): strong scaling."""
    import tasft_b200 as T  # noqa: PLC0415
    from tasft_b200 import shards as SH  # noqa: PLC0415

    kept = T.mask_to_kept(mask, True)
    w = SH.unit_weights(kept, CFG["Hk"])
    units = SH.assign_units(w, ws)[rank]
    qu, ku, vu, ku_kept = SH.unit_slices(q, k, v, kept, units)
    kern = T.BlockSparseFlashAttention(block_size=CFG["block"])
    out = torch.empty_like(qu)
    t = time_steps(lambda: kern.forward(qu, ku, vu, ku_kept, out=out), args.steps, args.warmup, flush, ws)
    ms_max = max_over_ranks(statistics.mean(t), ws)
    grp = CFG["Hq"] // CFG["Hk"]
    total_blocks = int(w.sum().item())
    flops = total_blocks * grp * 4 * CFG["block"] * CFG["block"] * CFG["D"]
    mine = float(sum(int(w[u]) for u in units))
    return {"config": "BASELINE configs[1], one global B=4 layer (32 sequence x kv-head units) split over the ranks",
            "units_per_rank": len(units), "ms": round(ms_max, 4),
            "tflops": round(flops / (ms_max * 1e-3) / 1e12, 2),
            "frac_of_one_gpu_peak_x_n": round(flops / (ms_max * 1e-3) / 1e12 / (peaks["bf16_tflops"] * ws), 4),
            "rank_blocks_max_over_mean": round(max_over_ranks(mine, ws) / (total_blocks / ws), 4),
            "scaling": "strong"}


# ---------------------------------------------------------------------------
def cpu_decode_sample(budget_s: float = 3.0):
    """Oracle decode (restated single-query masked attention) on host cores: a few
    sequences of the configs[2] workload."""
    import oracle as O  # noqa: PLC0415  (CPU baseline leg)
    from tasft_b200 import masks as M  # noqa: PLC0415

    torch.set_num_threads(os.cpu_count() or 1)
    c = DEC
    nseq = 2
    g = torch.Generator().manual_seed(77)
    q = torch.randn(nseq, c["Hq"], c["D"], generator=g).bfloat16()
    kc = torch.randn(nseq, c["Hk"], c["L"], c["D"], generator=g).bfloat16()
    vc = torch.randn(nseq, c["Hk"], c["L"], c["D"], generator=g).bfloat16()
    kv_len = torch.full((nseq,), c["L"], dtype=torch.int32)
    nb = c["L"] // c["block"]
    idx, cnt = M.lists_from_mask(M.decode_mask(torch.rand(nseq, c["Hk"], nb, generator=g), kv_len // 64,
                                               c["density"], nb))
    t0 = time.perf_counter()
    n = 0
    while True:
        O.bsa_decode(q, kc, vc, kv_len, idx, cnt, c["block"])
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": round(nseq * n / dt, 2), "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{n} x {nseq} sequences of configs[2] (KV 8192, 26 kept blocks per kv-head); "
                      f"oracle/tasft_oracle.py:bsa_decode, {dt:.1f} s"}


def cpu_gate_sample(budget_s: float = 3.0):
    """Oracle AttnGate.forward (fp32, attn_gate.py:377-485) on one (sequence, kv-group)
    chunk of the configs[1] workload; rate in algorithmic bytes (bf16 |Q| + |K|) per s."""
    import oracle as O  # noqa: PLC0415  (CPU baseline leg)

    torch.set_num_threads(os.cpu_count() or 1)
    c = CFG
    grp = c["Hq"] // c["Hk"]
    g = torch.Generator().manual_seed(78)
    q = torch.randn(1, grp, c["S"], c["D"], generator=g)
    k = torch.randn(1, 1, c["S"], c["D"], generator=g)
    hid = max(32, c["D"] // 4)
    w_in = torch.randn(hid, 2 * c["D"], generator=g) * 0.05
    b_in = torch.zeros(hid)
    w_out = torch.randn(1, hid, generator=g) * 0.01
    t0 = time.perf_counter()
    n = 0
    while True:
        O.gate_forward_gqa(q, k, w_in, b_in, w_out, c["block"], 0.5)
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    nbytes = (q.numel() + k.numel()) * 2
    return {"value": round(nbytes * n / dt / 1e9, 4), "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{n} x one (sequence, kv-head group) chunk: 4 q-heads + 1 kv-head, S=4096, D=128, fp32; "
                      f"oracle/tasft_oracle.py:gate_forward_gqa, {dt:.1f} s"}


def cpu_target_sample(budget_s: float = 3.0):
    """Oracle gate target (bf16 training scores, max-pool, softmax; tasft_attention.py:427-443 +
    objectives.py:128-185) for single heads of the configs[4] workload."""
    import oracle as O  # noqa: PLC0415  (CPU baseline leg)

    torch.set_num_threads(os.cpu_count() or 1)
    c = CFG
    g = torch.Generator().manual_seed(79)
    q = torch.randn(1, 1, c["S"], c["D"], generator=g).bfloat16()
    k = torch.randn(1, 1, c["S"], c["D"], generator=g).bfloat16()
    nb = c["S"] // c["block"]
    flop = nb * (nb + 1) // 2 * 2 * c["block"] * c["block"] * c["D"]
    t0 = time.perf_counter()
    n = 0
    while True:
        O.gate_target_from_qk(q, k, c["block"])
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": round(flop * n / dt / 1e12, 6), "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{n} x one head (S=4096, D=128, bf16 scores); oracle/tasft_oracle.py:gate_target_from_qk, "
                      f"{dt:.1f} s"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    budget = 3.0
    for _ in range(max(args.warmup, 0)):
        cpu_prefill_sample(budget_s=0.0)
    vals = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        vals.append(cpu_prefill_sample(budget_s=budget))
    wall = time.perf_counter() - t0
    v = statistics.median([x["value"] for x in vals])
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(wall / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "llama3-8b attention prefill, B=4 Hq=32 Hk=8 S=4096 D=128 block=64, 80% sparsity "
                               "(CPU sample: one (batch, kv-head) chunk per step)", "model": "llama3-8b-attn"},
        "cpu_baseline": {**vals[0], "value": v},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


# ---------------------------------------------------------------------------
def run_ours(args):
    import tasft_b200 as T  # noqa: PLC0415
    from tasft_b200 import _lib as L  # noqa: PLC0415

    rank, ws, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local if ws > 1 else 0)
    peaks = load_peaks()
    traffic = load_traffic()
    flush = L2Flush(dev)
    kern = T.BlockSparseFlashAttention(block_size=CFG["block"])

    # ---------------- prefill (value) ----------------
    q, k, v, mask, _gate = make_prefill_inputs(1234 + 2 + 1000 * rank, dev)
    kept_blocks = int(mask.sum().item())
    grp = CFG["Hq"] // CFG["Hk"]
    flops = kept_blocks * grp * 4 * CFG["block"] * CFG["block"] * CFG["D"]
    out = torch.empty_like(q)

    def step():
        kern.forward(q, k, v, mask, out=out)

    clk = ClockSampler(local).__enter__()  # sampled across all timed phases
    n0 = L.launch_count()
    t_step = time_steps(step, args.steps, args.warmup, flush, ws)
    launches = (L.launch_count() - n0) // (args.steps + args.warmup)
    ms = statistics.mean(t_step)
    ms_max = max_over_ranks(ms, ws)
    total_flops = sum_over_ranks(float(flops), ws)
    value = total_flops / (ms_max * 1e-3) / 1e12

    # kernel-only roofline: prefill kernel on prebuilt kept lists
    kept = T.mask_to_kept(mask, True)
    t_kern = time_steps(lambda: kern.forward(q, k, v, kept, out=out), args.steps, args.warmup, flush, ws)
    ms_k = statistics.mean(t_kern)
    achieved = flops / (ms_k * 1e-3) / 1e12
    tr = traffic.get("prefill")
    roofline = {"bound": "tensor", "achieved": round(achieved, 2), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                "frac": round(achieved / peaks["bf16_tflops"], 4), "traffic": tr,
                "peak_src": f"bf16 burst, {peaks['src']}", "kernel": "bsa_prefill_tc_kernel",
                "algorithmic": f"{flops / 1e9:.2f} GFLOP per launch (kept blocks x 4*64*64*128 x 4 q-heads)",
                "ms_per_launch": round(ms_k, 4)}

    # ---------------- gate mask build (HBM-bound: reads Q and K once) ----------------
    def gstep():
        with torch.no_grad():
            _gate(q, k)

    # device time of the gate's kernels: the step replayed from a CUDA graph (its Python
    # launch path takes longer than its ~50 us of kernels)
    t_gate = time_steps(graphed(gstep), args.steps, args.warmup, flush, ws)
    ms_g = statistics.mean(t_gate)
    gbytes = (q.numel() + k.numel()) * 2
    gate_info = {"ms_per_step": round(ms_g, 4), "timing": "CUDA graph replay of AttnGate.forward",
                 "kernels": "gate_pool_project_fused_kernel + gate_pair_slab_kernel",
                 "roofline": {"bound": "hbm", "achieved": round(gbytes / (ms_g * 1e-3) / 1e9, 1),
                              "peak": peaks["hbm_gbs"], "unit": "GB/s",
                              "frac": round(gbytes / (ms_g * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
                              "traffic": traffic.get("gate"),
                              "algorithmic": f"{gbytes / 1e6:.1f} MB per step (|Q| + |K|)"}}

    # ---------------- projection epilogue + gate from its block means ----------------
    gate_info["pooled_path"] = bench_epilogue_gate(_gate, flush, ws, args, peaks)

    # ---------------- training gate target (tensor-core bound: causal Q K^T tiles) ----------------
    def tstep():
        T.gate_target_from_qk(q, k, CFG["block"])

    t_tgt = time_steps(tstep, args.steps, args.warmup, flush, ws)
    ms_t = statistics.mean(t_tgt)
    nb = CFG["S"] // CFG["block"]
    tflop = nb * (nb + 1) // 2 * 2 * CFG["block"] * CFG["block"] * CFG["D"] * CFG["B"] * CFG["Hq"]
    t_ach = tflop / (ms_t * 1e-3) / 1e12
    target_info = {"ms_per_step": round(ms_t, 4), "kernels": "target_tc_kernel + target_softmax_kernel",
                   "config": "BASELINE configs[4]: gate target at the prefill shape (B=4, Hq=32, Hk=8, S=4096, D=128)",
                   "roofline": {"bound": "tensor", "achieved": round(t_ach, 2), "peak": peaks["bf16_tflops"],
                                "unit": "TFLOP/s", "frac": round(t_ach / peaks["bf16_tflops"], 4),
                                "traffic": traffic.get("target"), "peak_src": f"bf16 burst, {peaks['src']}",
                                "algorithmic": f"{tflop / 1e9:.1f} GFLOP per step (causal 64x64 tiles x 2*64*64*128 "
                                               "x B x Hq)"}}

    # ---------------- drop-in form, reference Triton kernel, gate training step, strong C2 ----------------
    dropin = bench_dropin(q, k, v, _gate, kern, flush, ws, args, peaks)
    gate_train = bench_gate_train(q, k, flush, ws, args)
    strong_c2 = bench_strong_c2(q, k, v, mask, rank, ws, flush, args, peaks) if ws > 1 else None

    # ---------------- e2e through the public API with host buffers ----------------
    qh = q.cpu().pin_memory()
    kh = k.cpu().pin_memory()
    vh = v.cpu().pin_memory()
    mh = mask.cpu().pin_memory()
    oh = torch.empty(q.shape, dtype=q.dtype).pin_memory()

    def step_e2e():
        qd = qh.to(dev, non_blocking=True)
        kd = kh.to(dev, non_blocking=True)
        vd = vh.to(dev, non_blocking=True)
        md = mh.to(dev, non_blocking=True)
        o = kern.forward(qd, kd, vd, md)
        oh.copy_(o, non_blocking=True)

    # the same calls pipelined over the batch on two streams: H2D of sequence b + 1, the
    # kernels of b and D2H of b - 1 overlap (copy engines run both directions at once)
    main = torch.cuda.current_stream()
    lanes = [torch.cuda.Stream() for _ in range(2)]
    slots = [(torch.empty_like(q[:1]), torch.empty_like(k[:1]), torch.empty_like(v[:1]),
              torch.empty_like(mask[:1])) for _ in range(2)]

    def step_e2e_pipe():
        for s_ in lanes:
            s_.wait_stream(main)
        for bi in range(qh.shape[0]):
            s_ = lanes[bi % 2]
            qd, kd, vd, md = slots[bi % 2]
            with torch.cuda.stream(s_):
                qd.copy_(qh[bi:bi + 1], non_blocking=True)
                kd.copy_(kh[bi:bi + 1], non_blocking=True)
                vd.copy_(vh[bi:bi + 1], non_blocking=True)
                md.copy_(mh[bi:bi + 1], non_blocking=True)
                o = kern.forward(qd, kd, vd, md)
                oh[bi:bi + 1].copy_(o, non_blocking=True)
        for s_ in lanes:
            main.wait_stream(s_)

    e2e_steps = max(3, min(args.steps, 10))
    t_e2e_serial = time_steps(step_e2e, e2e_steps, max(args.warmup, 3), flush, ws)
    ms_e2e_serial = max_over_ranks(statistics.mean(t_e2e_serial), ws)
    t_e2e = time_steps(step_e2e_pipe, e2e_steps, max(args.warmup, 3), flush, ws)
    ms_e2e = max_over_ranks(statistics.mean(t_e2e), ws)
    h2d = qh.numel() * 2 + kh.numel() * 2 + vh.numel() * 2 + mh.numel()
    d2h = oh.numel() * 2
    del qh, kh, vh, oh, mh, q, k, v, out, kept, slots

    # ---------------- decode ----------------
    qd, kc, vc, kv_len, dkept = make_decode_inputs(1234 + 3 + 1000 * rank, dev)
    mean_kept = float(dkept.cnt.float().mean().item())
    splits = T.decode.default_splits(DEC["B"], DEC["Hk"], mean_kept)
    wsp = T.DecodeWorkspace(DEC["B"], DEC["Hq"], DEC["Hk"], DEC["D"], max(splits, 1), dev)
    od = torch.empty_like(qd)

    def dstep():
        T.bsa_decode(qd, kc, vc, kv_len, dkept, DEC["block"], num_splits=splits, workspace=wsp, out=od)

    t_dec = time_steps(dstep, args.steps, args.warmup, flush, ws)

    # the same decode over a paged cache (vLLM flash layout, 16-token pages, shuffled pool)
    pg = 16
    mp = DEC["L"] // pg
    gperm = torch.Generator(device=dev).manual_seed(99)
    table = torch.randperm(DEC["B"] * mp, device=dev, generator=gperm).to(torch.int32).view(DEC["B"], mp)
    kpg = torch.empty(DEC["B"] * mp, pg, DEC["Hk"], DEC["D"], device=dev, dtype=kc.dtype)
    vpg = torch.empty_like(kpg)
    kpg[table.flatten().long()] = kc.view(DEC["B"], DEC["Hk"], mp, pg, DEC["D"]).permute(0, 2, 3, 1, 4).reshape(
        -1, pg, DEC["Hk"], DEC["D"])
    vpg[table.flatten().long()] = vc.view(DEC["B"], DEC["Hk"], mp, pg, DEC["D"]).permute(0, 2, 3, 1, 4).reshape(
        -1, pg, DEC["Hk"], DEC["D"])

    def pstep():
        T.bsa_decode_paged(qd, kpg, vpg, table, kv_len, dkept, DEC["block"], num_splits=splits, workspace=wsp, out=od)

    t_pag = time_steps(pstep, args.steps, args.warmup, flush, ws)
    del kpg, vpg
    clk.__exit__(None, None, None)
    ms_d = statistics.mean(t_dec)
    ms_d_max = max_over_ranks(ms_d, ws)
    kept_dec = int(dkept.cnt.sum().item())
    dbytes = kept_dec * 2 * DEC["block"] * DEC["D"] * 2 + qd.numel() * 2 * 2
    gbs = dbytes / (ms_d * 1e-3) / 1e9
    tok_s = sum_over_ranks(DEC["B"], ws) / (ms_d_max * 1e-3)
    decode = {"tok_s": round(tok_s, 1), "ms_per_step": round(ms_d_max, 4), "splits": splits,
              "kept_blocks_per_seq_head": round(mean_kept, 2),
              "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                           "frac": round(gbs / peaks["hbm_gbs"], 4), "traffic": traffic.get("decode"),
                           "peak_src": peaks["src"], "kernel": "bsa_decode_mma_kernel",
                           "algorithmic": f"{dbytes / 1e6:.1f} MB per launch (kept K+V blocks + q + out)"}}
    ms_p = statistics.mean(t_pag)
    decode["paged"] = {"page_size": pg, "layout": "[pages, page_size, Hk, D] + block table (vLLM flash layout)",
                       "ms_per_step": round(max_over_ranks(ms_p, ws), 4),
                       "achieved_gbs": round(dbytes / (ms_p * 1e-3) / 1e9, 1),
                       "frac": round(dbytes / (ms_p * 1e-3) / 1e9 / peaks["hbm_gbs"], 4)}

    # ---------------- long-context decode: cache split by position over ranks ----------------
    from tasft_b200 import masks as M  # noqa: PLC0415
    from tasft_b200 import shards as SH  # noqa: PLC0415

    lc = LONG
    g = torch.Generator(device=dev).manual_seed(1234 + 4)  # same cache and lists on every rank
    ql = torch.randn(lc["B"], lc["Hq"], lc["D"], device=dev, dtype=torch.bfloat16, generator=g)
    nbl = lc["L"] // lc["block"]
    lo, hi = SH.block_range(nbl, rank, ws)
    kl_full = torch.randn(lc["B"], lc["Hk"], lc["L"], lc["D"], device=dev, dtype=torch.bfloat16, generator=g)
    vl_full = torch.randn_like(kl_full)
    kl_loc = kl_full[:, :, lo * lc["block"]: hi * lc["block"]].contiguous()
    vl_loc = vl_full[:, :, lo * lc["block"]: hi * lc["block"]].contiguous()
    kvl = torch.full((lc["B"],), lc["L"], dtype=torch.int32, device=dev)
    lmask = M.decode_mask(torch.rand(lc["B"], lc["Hk"], nbl, device=dev, generator=g), (kvl + 63) // 64,
                          lc["density"], nbl)
    lkept = T.KeptBlocks(*M.lists_from_mask(lmask))
    long_extra = {}
    if ws > 1:
        # the step (local decode over this rank's KV range + merge of all ranks' partials over
        # peer memory) replayed from a CUDA graph: no NCCL call and no host work per token
        dec = SH.SplitKVDecoder(lc["B"], lc["Hq"], lc["Hk"], lc["D"], dev, exchange="peer")
        lloc = dec.local(lkept, lo, hi - lo)
        lstep = graphed(lambda: dec(ql, kl_loc, vl_loc, kvl, lkept, lo, local=lloc))
        ltiming = ("CUDA graph replay (local split decode whose merge kernel pushes the rank's rows to every "
                   "rank over peer memory and merges them: tasft_bsa_decode_peer_fwd)")
        # the NCCL all-gather + combine path, eager, for comparison
        dec_n = SH.SplitKVDecoder(lc["B"], lc["Hq"], lc["Hk"], lc["D"], dev, exchange="nccl")
        t_n = time_steps(lambda: dec_n(ql, kl_loc, vl_loc, kvl, lkept, lo, local=lloc), args.steps, args.warmup,
                         flush, ws)
        long_extra["ms_per_token_nccl_eager"] = round(max_over_ranks(statistics.mean(t_n), ws), 4)
        # where the step's time goes: this rank's local split decode alone (graph replay)
        t_loc = time_steps(graphed(lambda: T.bsa_decode(ql, kl_loc, vl_loc, kvl, lloc, lc["block"], workspace=dec.ws,
                                                         partials=(dec.po, dec.pm), kv_offset=lo * lc["block"])),
                           args.steps, args.warmup, flush, ws)
        long_extra["ms_local_decode_only"] = round(max_over_ranks(statistics.mean(t_loc), ws), 4)
        # and the stand-alone peer-memory merge kernel (tasft_peer_combine) alone, for comparison
        # (every rank replays it, so the ranks still meet)
        t_mrg = time_steps(graphed(lambda: dec.peer(dec.po, dec.pm, dec.out)), args.steps, args.warmup, flush, ws)
        long_extra["ms_merge_only"] = round(max_over_ranks(statistics.mean(t_mrg), ws), 4)
    else:
        # one GPU: the step replayed from a CUDA graph, as a serving loop would run it (its
        # Python launch path takes longer than the ~20 us of kernels)
        lws = T.DecodeWorkspace(lc["B"], lc["Hq"], lc["Hk"], lc["D"], 64, dev)  # kept across steps
        lstep = graphed(lambda: T.bsa_decode(ql, kl_loc, vl_loc, kvl, lkept, lc["block"], workspace=lws))
        ltiming = "CUDA graph replay"
    t_long = time_steps(lstep, args.steps, args.warmup, flush, ws)
    ms_l = max_over_ranks(statistics.mean(t_long), ws)
    # a serving loop's view: 50 steps back to back (no flush between them; the kept K/V of a
    # step, 6.7 MB, stays in L2, so this is the latency floor, not the bench value)
    barrier(ws)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(50):
        lstep()
    e1.record()
    torch.cuda.synchronize()
    long_extra["ms_per_token_back_to_back"] = round(max_over_ranks(e0.elapsed_time(e1) / 50, ws), 4)
    if ws > 1:
        # parity: the merged token against a one-rank decode of the whole cache, on every rank
        lstep()
        ref = T.bsa_decode(ql, kl_full, vl_full, kvl, lkept, lc["block"])
        err = (dec.out.float() - ref.float()).abs().max().item()
        long_extra["max_abs_err_vs_one_rank"] = round(max_over_ranks(err, ws), 6)
        long_extra["device_err_word"] = int(max_over_ranks(float(dec.peer.err.item()), ws))
        barrier(ws)
        dec.peer.close()
    long_decode = {"config": "BASELINE configs[3] decode: B=1, Hq=28, Hk=4, KV=32768, D=128, 90% block sparsity "
                             f"({int(lkept.cnt.float().mean().item())} of {nbl} blocks kept per kv-head)",
                   "split": f"KV positions over {ws} rank(s); partials merged over peer memory (CUDA IPC)"
                            if ws > 1 else "one GPU",
                   "scaling": "strong", "ms_per_token": round(ms_l, 4),
                   "timing": ltiming,
                   "tok_s": round(lc["B"] / (ms_l * 1e-3), 1), **long_extra}
    del kl_loc, vl_loc, kl_full, vl_full

    qwen_prefill = bench_qwen_prefill(rank, ws, dev, flush, args, peaks)

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        cpu = cpu_prefill_sample(budget_s=args.cpu_budget)
        decode["cpu_baseline"] = cpu_decode_sample()
        gate_info["cpu_baseline"] = cpu_gate_sample()
        target_info["cpu_baseline"] = cpu_target_sample()

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "llama3-8b attention prefill (BASELINE configs[1]): B=4 per GPU, Hq=32, Hk=8, "
                                   "S=4096, D=128, block=64, causal, 80% block sparsity (kv-head masks from the "
                                   "random-init AttnGate's fp32 scores); decode configs[2] alongside",
                       "model": "llama3-8b-attn", "global_batch": CFG["B"] * ws, "seq_len": CFG["S"],
                       "parallelism": f"dp{ws} (batch shards, no collective)",
                       "l2": "flushed (256 MiB write) before every timed step",
                       "kept_blocks_per_gpu": kept_blocks, "gflop_per_gpu_step": round(flops / 1e9, 3)},
            "roofline": roofline,
            "e2e": {"value": round(total_flops / (ms_e2e * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(ms_e2e, 3),
                    "api": "tasft_b200.BlockSparseFlashAttention.forward(q, k, v, bool mask) from pinned host, "
                           "one call per sequence, copies and calls pipelined on two streams",
                    "ms_per_step_unpipelined": round(ms_e2e_serial, 3)},
            "decode": decode,
            "gate": gate_info,
            "gate_target": target_info,
            "long_decode": long_decode,
            "prefill_dropin": dropin,
            "qwen_prefill": qwen_prefill,
            "gate_train": gate_train,
            "gpu_launches": launches * args.steps,
            "gpu_launches_per_step": launches,
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
        }
        if strong_c2 is not None:
            line["strong_c2"] = strong_c2
        print(json.dumps(line))
    if ws > 1:
        import torch.distributed as dist  # noqa: PLC0415

        dist.destroy_process_group()


def run_only(args):
    """Launch one kernel family `--steps` times on the bench workload (for ncu captures)."""
    import tasft_b200 as T  # noqa: PLC0415

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if args.only == "epilogue":  # qkv_rope_pool on the C2 projection outputs
        c = CFG
        g = torch.Generator(device=dev).manual_seed(77)
        ql = torch.randn(c["B"], c["S"], c["Hq"] * c["D"], device=dev, dtype=torch.bfloat16, generator=g)
        kl = torch.randn(c["B"], c["S"], c["Hk"] * c["D"], device=dev, dtype=torch.bfloat16, generator=g)
        vl = torch.randn_like(kl)
        inv = 1.0 / (10000 ** (torch.arange(0, c["D"], 2, device=dev).float() / c["D"]))
        emb = torch.cat([torch.outer(torch.arange(c["S"], device=dev).float(), inv)] * 2, -1)
        cos, sin = emb.cos().bfloat16()[None], emb.sin().bfloat16()[None]
        for _ in range(args.steps):
            T.qkv_rope_pool(ql, kl, vl, c["Hq"], c["Hk"], cos, sin, c["block"])
        torch.cuda.synchronize()
        print(f"{args.only}: {args.steps} launches ok")
        return
    if args.only == "long_decode":  # configs[3] decode on one GPU: wide splits + merge kernel
        from tasft_b200 import masks as M  # noqa: PLC0415

        lc = LONG
        g = torch.Generator(device=dev).manual_seed(1234 + 4)
        ql = torch.randn(lc["B"], lc["Hq"], lc["D"], device=dev, dtype=torch.bfloat16, generator=g)
        kl = torch.randn(lc["B"], lc["Hk"], lc["L"], lc["D"], device=dev, dtype=torch.bfloat16, generator=g)
        vl = torch.randn_like(kl)
        nbl = lc["L"] // lc["block"]
        kvl = torch.full((lc["B"],), lc["L"], dtype=torch.int32, device=dev)
        lmask = M.decode_mask(torch.rand(lc["B"], lc["Hk"], nbl, device=dev, generator=g), (kvl + 63) // 64,
                              lc["density"], nbl)
        lkept = T.KeptBlocks(*M.lists_from_mask(lmask))
        lws = T.DecodeWorkspace(lc["B"], lc["Hq"], lc["Hk"], lc["D"], 64, dev)
        for _ in range(args.steps):
            T.bsa_decode(ql, kl, vl, kvl, lkept, lc["block"], workspace=lws)
        torch.cuda.synchronize()
        print(f"{args.only}: {args.steps} launches ok")
        return
    if args.only in ("decode", "paged"):
        qd, kc, vc, kv_len, kept = make_decode_inputs(1237, dev)
        splits = T.decode.default_splits(DEC["B"], DEC["Hk"], float(kept.cnt.float().mean().item()))
        wsp = T.DecodeWorkspace(DEC["B"], DEC["Hq"], DEC["Hk"], DEC["D"], splits, dev)
        if args.only == "paged":  # the same cache as 16-token pages in a shuffled pool
            pg, mp = 16, DEC["L"] // 16
            table = torch.randperm(DEC["B"] * mp, device=dev).to(torch.int32).view(DEC["B"], mp)
            kp = torch.empty(DEC["B"] * mp, pg, DEC["Hk"], DEC["D"], device=dev, dtype=kc.dtype)
            vp = torch.empty_like(kp)
            shape = (-1, pg, DEC["Hk"], DEC["D"])
            kp[table.flatten().long()] = kc.view(DEC["B"], DEC["Hk"], mp, pg, DEC["D"]).permute(0, 2, 3, 1, 4).reshape(shape)
            vp[table.flatten().long()] = vc.view(DEC["B"], DEC["Hk"], mp, pg, DEC["D"]).permute(0, 2, 3, 1, 4).reshape(shape)
            del kc, vc
        for _ in range(args.steps):
            if args.only == "paged":
                T.bsa_decode_paged(qd, kp, vp, table, kv_len, kept, DEC["block"], num_splits=splits, workspace=wsp)
            else:
                T.bsa_decode(qd, kc, vc, kv_len, kept, DEC["block"], num_splits=splits, workspace=wsp)
    else:
        q, k, v, mask, gate = make_prefill_inputs(1236, dev)
        kern = T.BlockSparseFlashAttention(block_size=CFG["block"])
        kept = T.mask_to_kept(mask, True)
        for _ in range(args.steps):
            if args.only == "prefill":
                kern.forward(q, k, v, kept)
            elif args.only == "gate":
                with torch.no_grad():
                    gate(q, k)
            else:
                T.gate_target_from_qk(q, k, CFG["block"])
    torch.cuda.synchronize()
    print(f"{args.only}: {args.steps} launches ok")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-triton", action="store_true", help="skip timing the reference Triton kernel")
    ap.add_argument("--only", choices=["prefill", "decode", "paged", "gate", "target", "epilogue", "long_decode"],
                    help="profiling driver: run `--steps` launches of one kernel family, print nothing else")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.only:
        run_only(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
