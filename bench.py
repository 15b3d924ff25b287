"""Benchmark of the fused layer-op hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg2|cfg3|cfg5] [--legs cfg3,cfg4,cfg5|none]

A step is one pass of the hot path over one batch: the fused-op sequence of
one Cosmos-Predict2-2B denoiser forward at 1024x1024 (config 2: B=1,
S=4096, D=2048, 16 heads x 128; 1 adaln + 28 x [qkv_norm_rope,
residual_adaln, head_norm, residual_adaln, residual_adaln] + the final
residual_adaln = 141 launches), in the call order of the reference's
forward_fused (src/model.py:339-376).  ``--workload cfg3`` runs the FP8
forward sequence (forward_fp8, model.py:403-473) at B=2.

Every call reads its own freshly generated input buffers (the step's working
set is several GB, far above the 126 MB L2), so no input is served from L2
by an earlier call; between steps the same holds.  Every call's outputs stay
referenced until the graph is captured, so every call writes its own
addresses too (no output can be overwritten while still dirty in L2).  The
step is captured in a CUDA graph and launched with programmatic dependent
launch.

The same line carries the other configurations as sub-objects (`legs`):
cfg3, the FP8 forward step at B=2 (forward_fp8, model.py:403-473); cfg4,
the LoRA backward step (the backward ops of the config-2 forward in reverse
order, B=1); cfg5: 32 sequences of 4096 tokens sharded
over the ranks (strong scaling), running the FP8 forward step.

value: algorithmic HBM bytes of all ranks' steps / max-over-ranks device
time (CUDA events), in GB/s.  e2e: the same metric through the public API
with pinned host buffers, host<->device copies inside the timed region.
roofline: the dominant kernel (residual_adaln): the step's 84 launches of it
replayed alone back to back, CUDA events around the replays; the isolated
per-launch time (events around each launch, no overlap) is reported beside it.
cpu_baseline: the reference's unfused torch fp32 eager composition on the
host cores (rank 0, N=1), on a bounded sample of the config-2 step (the
same shapes as our arm), with the config-1 figure beside it.

Multi-GPU: one process per GPU (torchrun), each rank runs the same per-rank
workload on its own sequences (weak scaling); no collective on the data path.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from anima_flat_b200 import workload as W  # noqa: E402
from anima_flat_b200.shard import max_over_ranks, shard_sequences  # noqa: E402

METRIC = "fused AdaLN/RMSNorm/RoPE HBM GB/s"
FALLBACK_HBM_GBS = 6650.0


# ----------------------------------------------------------------- helpers --
def peak_hbm() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback (profiling recipe, 6.65 TB/s)"


def ncu_traffic(kernel_key: str):
    """dram bytes per launch of the dominant kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "ncu_traffic.json"
    try:
        return json.loads(p.read_text())[kernel_key]
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clocks/throttle sampling while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        rows = [r.split(",") for r in out.strip().splitlines() if r.count(",") >= 8]
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        loaded = [v for v in sm if v > 0]
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


def dist_info():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ------------------------------------------------------------- the step --
class Step:
    """Inputs, outputs and launch order of one forward's fused-op sequence."""

    def __init__(self, shape: W.Shape, fp8: bool, device, seed: int, distinct: bool = True):
        import anima_flat_b200 as afb

        self.afb = afb
        self.s = shape
        self.fp8 = fp8
        self.calls = W.fp8_forward_calls(shape) if fp8 else W.bf16_forward_calls(shape)
        self.bytes = W.step_bytes(self.calls, shape)
        s = shape
        g = torch.Generator(device=device).manual_seed(seed)
        bf = torch.bfloat16

        def act(*dims):
            return torch.randn(*dims, generator=g, device=device, dtype=torch.float32).to(bf)

        B, S, D, H, hd, L = s.batch, s.seq, s.dim, s.heads, s.head_dim, s.layers
        self.mod = (torch.randn(L, 3, 3, B, D, generator=g, device=device) * 0.1).to(bf)
        self.mod[:, :, 1] += 1.0
        self.fin = (torch.randn(B, 2 * D, generator=g, device=device) * 0.1).to(bf)
        side = int(round(S ** 0.5))
        self.cos, self.sin = afb.rope_tables(side, S // side, hd, device, (4.0, 4.0))
        self.qw = [1.0 + 0.02 * torch.randn(hd, generator=g, device=device) for _ in range(L)]
        self.kw = [1.0 + 0.02 * torch.randn(hd, generator=g, device=device) for _ in range(L)]
        self.xw = [1.0 + 0.02 * torch.randn(hd, generator=g, device=device) for _ in range(L)]
        # Distinct inputs per call: the residual stream too, so that no call reads
        # data a previous call left in L2.  With distinct=False (workloads whose
        # tensors are each far larger than L2) two input sets alternate.
        nset = L if distinct else 2
        self.z0 = act(B, S, D)
        self.qkv = [act(B, S, 3 * H * hd) for _ in range(nset)]
        self.sub = [[act(B, S, D) for _ in range(3)] for _ in range(nset)]   # o1, o2, mlp out
        self.res = [[act(B, S, D) for _ in range(3)] for _ in range(nset)]
        self.xq = [act(B, S, D) for _ in range(nset)]
        if fp8:
            self.attn = [[act(B, S, D) for _ in range(2)] for _ in range(nset)]
            self.up = [act(B, S, s.mlp) for _ in range(nset)]
        if not distinct:
            for name in ("qkv", "sub", "res", "xq") + (("attn", "up") if fp8 else ()):
                lst = getattr(self, name)
                setattr(self, name, [lst[i % 2] for i in range(L)])
        self.timed = "residual_adaln_fp8" if fp8 else "residual_adaln"
        self.timed_hook = None  # called around launches of self.timed when instrumenting
        self.only = None  # run only the launches of this op (roofline timing)
        self.keep = None  # a list: every call's outputs are appended (kept referenced)

    def _op(self, name, fn, *a, **kw):
        if self.only is not None and name != self.only:
            return None
        hook = self.timed_hook if name == self.timed else None
        if hook is not None:
            hook(True)
        out = fn(*a, **kw)
        if hook is not None:
            hook(False)
        if self.keep is not None:
            self.keep.append(out)
        return out

    def block_mods(self, l: int, j: int):
        """(gate, shift, scale) of sub-layer j of block l (model.py:317-336, 375)."""
        mod, s = self.mod, self.s
        if j < 2:
            return mod[l, j, 2], mod[l, j + 1, 0], mod[l, j + 1, 1]
        if l + 1 < s.layers:
            return mod[l, 2, 2], mod[l + 1, 0, 0], mod[l + 1, 0, 1]
        shift, scale = self.fin.chunk(2, dim=-1)
        return mod[-1, 2, 2], shift, scale + 1

    def run(self):
        """One forward's op sequence (model.py:366-375 or :434-472)."""
        afb, s, mod, op = self.afb, self.s, self.mod, self._op
        H = s.heads
        with torch.no_grad():
            if not self.fp8:
                op("adaln", afb.adaln, self.z0, mod[0, 0, 0], mod[0, 0, 1])
                for l in range(s.layers):
                    op("qkv_norm_rope", afb.qkv_norm_rope, self.qkv[l], self.qw[l], self.kw[l],
                       self.cos, self.sin, H)
                    op("residual_adaln", afb.residual_adaln, self.sub[l][0], self.res[l][0],
                       *self.block_mods(l, 0))
                    op("head_norm", afb.head_norm, self.xq[l], self.xw[l], H)
                    op("residual_adaln", afb.residual_adaln, self.sub[l][1], self.res[l][1],
                       *self.block_mods(l, 1))
                    if l + 1 < s.layers:
                        op("residual_adaln", afb.residual_adaln, self.sub[l][2], self.res[l][2],
                           *self.block_mods(l, 2))
            else:
                op("adaln_fp8", afb.adaln_fp8, self.z0, mod[0, 0, 0], mod[0, 0, 1])
                for l in range(s.layers):
                    op("qkv_norm_rope", afb.qkv_norm_rope, self.qkv[l], self.qw[l], self.kw[l],
                       self.cos, self.sin, H)
                    op("rowquant", afb.rowquant, self.attn[l][0])
                    op("residual_adaln_fp8", afb.residual_adaln_fp8, self.sub[l][0], self.res[l][0],
                       *self.block_mods(l, 0))
                    op("head_norm", afb.head_norm, self.xq[l], self.xw[l], H)
                    op("rowquant", afb.rowquant, self.attn[l][1])
                    op("residual_adaln_fp8", afb.residual_adaln_fp8, self.sub[l][1], self.res[l][1],
                       *self.block_mods(l, 1))
                    op("rowquant_gelu", afb.rowquant, self.up[l], gelu=True)
                    if l + 1 < s.layers:
                        op("residual_adaln_fp8", afb.residual_adaln_fp8, self.sub[l][2],
                           self.res[l][2], *self.block_mods(l, 2))
            L = s.layers - 1
            op("residual_adaln", afb.residual_adaln, self.sub[L][2], self.res[L][2],
               *self.block_mods(L, 2))


class BwdStep:
    """Inputs and launch order of the LoRA backward's fused-op sequence (config
    4): the backward ops of the config-2 forward in reverse call order, 84
    residual_adaln_bwd + 28 head_norm_bwd + 28 qkv_norm_rope_bwd + 1
    adaln_bwd, each on its own freshly generated inputs (upstream grads
    N(0, 1e-2), activations N(0, 1))."""

    def __init__(self, shape: W.Shape, device, seed: int):
        import anima_flat_b200 as afb

        self.afb = afb
        self.s = s = shape
        self.calls = list(reversed(["adaln_bwd" if c == "adaln" else c + "_bwd"
                                    for c in W.bf16_forward_calls(s)]))
        self.bytes = W.step_bytes(self.calls, s)
        g = torch.Generator(device=device).manual_seed(seed)
        bf = torch.bfloat16
        B, S, D, H, hd = s.batch, s.seq, s.dim, s.heads, s.head_dim

        def act(*dims, std=1.0):
            return (torch.randn(*dims, generator=g, device=device) * std).to(bf)

        vec = lambda: (0.1 * torch.randn(B, D, generator=g, device=device)).to(bf)
        side = int(round(S ** 0.5))
        self.cos, self.sin = afb.rope_tables(side, S // side, hd, device, (4.0, 4.0))
        self.w = 1.0 + 0.02 * torch.randn(hd, generator=g, device=device)
        self.args = []
        for c in self.calls:
            if c == "residual_adaln_bwd":
                self.args.append((act(B, S, D, std=1e-2), act(B, S, D, std=1e-2), act(B, S, D),
                                  act(B, S, D), vec(), vec() + 1, 1e-6))
            elif c == "adaln_bwd":
                self.args.append((act(B, S, D, std=1e-2), act(B, S, D), vec() + 1, 1e-6))
            elif c == "qkv_norm_rope_bwd":
                self.args.append((act(B, S, 3 * H * hd), act(B, S, H, hd, std=1e-2),
                                  act(B, S, H, hd, std=1e-2), act(B, S, H, hd, std=1e-2), self.w,
                                  self.w, self.cos, self.sin, H, 1e-5))
            else:  # head_norm_bwd
                self.args.append((act(B, S, H * hd), act(B, S, H, hd, std=1e-2), self.w, H, 1e-5))
        self.keep = None
        self.only = None

    def run(self):
        ops = torch.ops.anima_flat_b200
        with torch.no_grad():
            for c, a in zip(self.calls, self.args):
                if self.only is not None and c != self.only:
                    continue
                out = getattr(ops, c)(*a)
                if self.keep is not None:
                    self.keep.append(out)


def capture(step, only: str | None = None, keep_outputs: bool = False):
    """CUDA graph of one step (its outputs live in the graph's memory pool);
    with `only`, just that op's launches of the step.  With keep_outputs,
    every call's outputs stay referenced until the capture ends, so no call
    reuses another's output memory inside the graph."""
    step.only = only
    try:
        return _capture(step, keep_outputs)
    finally:
        step.only = None


def _capture(step, keep_outputs: bool = False):
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            step.run()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    step.keep = [] if keep_outputs else None
    try:
        with torch.cuda.graph(g):
            step.run()
    finally:
        step.keep = None  # the graph's pool keeps the memory for its replays
    torch.cuda.synchronize()
    return g


def time_replays(g, steps: int, warmup: int, barrier, device, clocks: "ClockSampler | None" = None) -> float:
    """ms of `steps` back-to-back replays of graph g after `warmup` replays:
    CUDA events on the current stream between barriers and synchronizes,
    max over ranks."""
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    if clocks is not None:
        clocks.start()
        time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        g.replay()
    t1.record()
    torch.cuda.synchronize()
    barrier()
    return max_over_ranks(t0.elapsed_time(t1), device)


def instrumented_capture(step: Step):
    """A copy of the step graph with external events around every residual_adaln."""
    events: list[tuple[torch.cuda.Event, torch.cuda.Event]] = []
    pending: list[torch.cuda.Event] = []

    def hook(before: bool):
        if before:
            ev = torch.cuda.Event(enable_timing=True, external=True)
            ev.record()
            pending.append(ev)
        else:
            ev = torch.cuda.Event(enable_timing=True, external=True)
            ev.record()
            events.append((pending.pop(), ev))

    from anima_flat_b200 import _lib

    step.timed_hook = hook
    pdl = _lib.load().afb_get_pdl()
    _lib.set_pdl(False)  # time each launch on its own, without overlap
    try:
        g = capture(step)
    finally:
        step.timed_hook = None
        _lib.set_pdl(bool(pdl))
    # events from the warm-up runs inside capture() are discarded
    return g, events[-step.calls.count(step.timed):]


# ------------------------------------------------------------ our arm --
LEG_DESC = {
    "cfg3": "FP8 forward step (forward_fp8, model.py:403-473) at CFG batch 2 per rank",
    "cfg4": "LoRA backward step at batch 1 per rank: 84 residual_adaln_bwd + 28 head_norm_bwd "
            "+ 28 qkv_norm_rope_bwd + 1 adaln_bwd, reverse forward order",
    "cfg5": "32 sequences x 4096 tokens (batch 16 with CFG) sharded by sequence over the ranks "
            "(strong scaling), FP8 forward step (the config-2 op set with FP8 quantisation)",
}


def run_leg(name: str, args, world, rank, device, barrier) -> dict:
    """One extra configuration: its step captured in a graph and timed like
    the headline (K replays after W, CUDA events, max over ranks)."""
    keep = True
    if name == "cfg3":
        shape = W.Shape(batch=2)
        step = Step(shape, fp8=True, device=device, seed=2345 + rank)
        rows, nbytes = shape.rows * world, step.bytes * world
    elif name == "cfg4":
        shape = W.Shape(batch=1)
        step = BwdStep(shape, device=device, seed=3456 + rank)
        rows, nbytes = shape.rows * world, step.bytes * world
    else:  # cfg5: this rank's sequences of 32
        seqs = shard_sequences(32, world, rank)
        shape = W.Shape(batch=len(seqs))
        # Two input sets alternate: every tensor (537 MB per activation at
        # batch 32) is far larger than L2, and so are the outputs, which are
        # not kept: no call can find another's data in L2.
        step = Step(shape, fp8=True, device=device, seed=4567 + rank, distinct=False)
        full = W.Shape(batch=32)
        rows, nbytes = full.rows, W.step_bytes(W.fp8_forward_calls(full), full)
        keep = False
    steps = max(1, min(args.steps, args.leg_steps))
    g = capture(step, keep_outputs=keep)
    ms = time_replays(g, steps, min(args.warmup, 3), barrier, device)
    del g
    launches = len(step.calls) * (2 if name == "cfg4" else 1)
    peak, _ = peak_hbm()
    gbs = nbytes * steps / (ms * 1e-3) / 1e9
    out = {
        "workload": LEG_DESC[name],
        "batch_per_rank": shape.batch,
        "rows": rows,
        "ops_per_step": len(step.calls),
        "steps": steps,
        "ms_per_step": round(ms / steps, 4),
        "gbs": round(gbs, 1),
        "mrows_per_s": round(rows * steps / (ms * 1e-3) / 1e6, 3),
        "frac_of_hbm_peak": round(gbs / world / peak, 4),
        "bytes_per_step": nbytes,
        "scaling": "strong" if name == "cfg5" else "weak",
        "outputs_kept": keep,
    }
    if name == "cfg4":
        out["gpu_launches_per_step"] = launches
    del step
    torch.cuda.empty_cache()
    return out


def run_ours(args, world, rank, local):
    import anima_flat_b200 as afb  # noqa: F401
    from anima_flat_b200 import _lib

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    _lib.set_pdl(not args.no_pdl)

    def barrier():
        if world > 1:
            torch.distributed.barrier(device_ids=[local])

    if args.workload == "cfg5":
        # config 5 alone: 32 sequences (batch 16 with CFG) sharded over the ranks
        seqs = shard_sequences(32, world, rank)
        shape = W.Shape(batch=len(seqs))
        step = Step(shape, fp8=True, device=device, seed=1234 + rank, distinct=False)
    else:
        shape = W.Shape(batch=2 if args.workload == "cfg3" else 1)
        step = Step(shape, fp8=args.workload == "cfg3", device=device, seed=1234 + rank)
    n_launch = len(step.calls)
    keep = args.workload != "cfg5"

    g = capture(step, keep_outputs=keep)
    sampler = ClockSampler(local)
    ms = time_replays(g, args.steps, args.warmup, barrier, device, clocks=sampler)
    clocks = sampler.stop()
    del g
    scaling = "strong" if args.workload == "cfg5" else "weak"
    if scaling == "strong":
        full = W.Shape(batch=32)
        total_bytes = W.step_bytes(W.fp8_forward_calls(full), full) * args.steps
        rows_total = 32 * shape.seq * args.steps
    else:
        total_bytes = step.bytes * world * args.steps
        rows_total = shape.rows * world * args.steps
    value = total_bytes / (ms * 1e-3) / 1e9
    recycled = None
    if keep:
        # the same step with the outputs recycled by the graph's pool (every
        # call's inputs still distinct), for comparison
        g = capture(step, keep_outputs=False)
        ms_r = time_replays(g, args.steps, args.warmup, barrier, device)
        del g
        recycled = {"ms_per_step": round(ms_r / args.steps, 4),
                    "value": round(total_bytes / (ms_r * 1e-3) / 1e9, 1)}

    # --- dominant kernel: the step's launches of it alone, back to back ---
    dominant = step.timed
    n_dom = step.calls.count(dominant)
    g2 = capture(step, only=dominant, keep_outputs=keep)
    avg_ms = time_replays(g2, args.steps, args.warmup, barrier, device) / (args.steps * n_dom)
    del g2
    # and each launch on its own (events around every launch, no overlap)
    g3, evs = instrumented_capture(step)
    per_launch = []
    for _ in range(max(3, args.warmup)):
        g3.replay()
    torch.cuda.synchronize()
    for _ in range(min(args.steps, 10)):
        g3.replay()
        torch.cuda.synchronize()
        per_launch += [a.elapsed_time(b) for a, b in evs]
    del g3
    iso_ms = sorted(per_launch)[len(per_launch) // 2]
    dom_bytes = W.call_bytes(dominant, shape)
    achieved = dom_bytes / (avg_ms * 1e-3) / 1e9
    peak, peak_src = peak_hbm()
    traffic = ncu_traffic(f"{dominant}_{args.workload}")

    # --- end to end through the public API with host buffers --------------
    e2e = run_e2e(step, shape, args, world, device, barrier)
    del step
    torch.cuda.empty_cache()

    # --- the other configurations, in the same run -------------------------
    legs = {}
    if args.workload == "cfg2" and args.legs != "none":
        for name in args.legs.split(","):
            legs[name] = run_leg(name, args, world, rank, device, barrier)

    line = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": scaling,
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.1) modulation; no dataset needed)",
        "config": {
            "workload": {
                "cfg2": "cfg2: Cosmos-Predict2-2B BF16 forward fused-op sequence (forward_fused), "
                        "1024x1024, 28 blocks, 141 launches",
                "cfg3": "cfg3: Cosmos-Predict2-2B FP8 forward fused-op sequence (forward_fp8) with "
                        f"CFG batch 2, {n_launch} launches",
                "cfg5": "cfg5: the FP8 forward op sequence over 32 sequences x 4096 tokens (batch 16 "
                        "with CFG), sequences sharded over the GPUs",
            }[args.workload],
            "global_batch": shape.batch * world if scaling == "weak" else 32,
            "seq_len": shape.seq,
            "rows_per_gpu": shape.rows,
            "dim": shape.dim,
            "heads": shape.heads,
            "head_dim": shape.head_dim,
            "parallelism": f"rows sharded by sequence over {world} GPU(s); no collective on the hot path",
            "l2": "inputs larger than L2: every call reads distinct buffers "
                  f"({total_bytes / args.steps / 1e9 / (world if scaling == 'weak' else 1):.2f} GB of "
                  "algorithmic traffic per step per GPU)"
                  + ("; every call's outputs kept, so every call writes distinct buffers" if keep else ""),
            "cuda_graph": True,
            "pdl": not args.no_pdl,
        },
        "mrows_per_s": round(rows_total / (ms * 1e-3) / 1e6, 3),
        "pct_of_hbm_peak": round(100.0 * value / world / peak, 1),
        "pct_of_spec_8tbs": round(100.0 * value / world / 8000.0, 1),
        "gpu_launches": n_launch * args.steps,
        "roofline": {
            "kernel": f"{dominant} (adaln_fwd_kernel)",
            "bound": "hbm",
            "achieved": round(achieved, 1),
            "peak": peak,
            "peak_source": peak_src,
            "unit": "GB/s",
            "frac": round(achieved / peak, 4),
            "traffic": traffic,
            "bytes_per_launch": dom_bytes,
            "avg_launch_us": round(avg_ms * 1e3, 3),
            "launches_timed": args.steps * n_dom,
            "timing": "the step's launches of this kernel alone, back to back (PDL), CUDA events "
                      "around K graph replays",
            "isolated_launch_us_median": round(iso_ms * 1e3, 3),
            "isolated_frac": round(dom_bytes / (iso_ms * 1e-3) / 1e9 / peak, 4),
        },
        "clocks": clocks,
        "e2e": e2e,
    }
    if recycled is not None:
        line["outputs_recycled"] = recycled
    if legs:
        line["legs"] = legs
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(budget_s=args.cpu_seconds)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier(device_ids=[local])
        torch.distributed.destroy_process_group()


def bind_numa(device) -> dict:
    """Bind this process to the host CPUs of the GPU's NUMA node (read from
    sysfs), so that pinned host buffers allocated afterwards are local to the
    GPU's PCIe root.  Returns what was done."""
    try:
        p = torch.cuda.get_device_properties(device)
        bdf = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        node = int(Path(f"/sys/bus/pci/devices/{bdf}/numa_node").read_text().strip())
        if node < 0:
            return {"numa_node": None, "bound": False, "pci": bdf}
        cpus = set()
        for part in Path(f"/sys/devices/system/node/node{node}/cpulist").read_text().strip().split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        os.sched_setaffinity(0, cpus)
        return {"numa_node": node, "bound": True, "cpus": len(cpus), "pci": bdf}
    except Exception as e:  # no sysfs entry (containers): run unbound
        return {"numa_node": None, "bound": False, "why": type(e).__name__}


def copy_rates(device, nbytes: int = 256 << 20) -> dict:
    """This rank's host-to-device and device-to-host copy bandwidth from
    pinned memory (GB/s, CUDA events, best of 3), each direction on its own;
    with several ranks, every rank copies at the same time, so the figures
    show what each rank gets of the shared host links."""
    h = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    d = torch.empty(nbytes, dtype=torch.uint8, device=device)
    out = {}
    for name, dst, src in (("h2d_gbs", d, h), ("d2h_gbs", h, d)):
        best = 0.0
        for _ in range(3):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            dst.copy_(src, non_blocking=True)
            b.record()
            torch.cuda.synchronize()
            best = max(best, nbytes / (a.elapsed_time(b) * 1e-3) / 1e9)
        out[name] = round(best, 1)
    del h, d
    return out


def run_e2e(step: Step, shape: W.Shape, args, world, device, barrier) -> dict:
    """The same op sequence through the public API with host buffers: each
    call's fresh inputs are copied from pinned host memory, each output is
    copied back to pinned host memory, all inside the timed region.

    The copies and the kernels run on three streams, as a host-side caller
    would pipeline them: host-to-device copies on one, the ops on the
    current stream, device-to-host copies on a third.  An op waits for its
    input copy (event); its output's copy waits for the op.  Inputs rotate
    over a ring of RING device buffers, and a copy into a buffer waits until
    the op that last read it has run, so no input is overwritten early.  The
    two copy directions overlap each other and the kernels (PCIe is full
    duplex)."""
    afb = step.afb
    s = shape
    H = s.heads
    B, S, D = s.batch, s.seq, s.dim
    RING = 3
    all_cpus = os.sched_getaffinity(0)
    numa = bind_numa(device)  # before any pinned allocation
    pin = lambda *d: torch.empty(*d, dtype=torch.bfloat16).pin_memory()
    h_qkv, h_act = pin(B, S, 3 * D), pin(B, S, D)
    h_act.copy_(step.sub[0][0].cpu())
    h_qkv.copy_(step.qkv[0].cpu())
    h_out = pin(B, S, D)
    d_qkv = [torch.empty(B, S, 3 * D, dtype=torch.bfloat16, device=device) for _ in range(RING)]
    d_x = [torch.empty(B, S, D, dtype=torch.bfloat16, device=device) for _ in range(RING)]
    nbytes = lambda t: t.numel() * t.element_size()
    comp = torch.cuda.current_stream(device)
    s_in = torch.cuda.Stream(device)
    s_out = torch.cuda.Stream(device)
    # free[kind][slot]: recorded on the compute stream after the op that read the slot
    free = {"x": [None] * RING, "qkv": [None] * RING}
    cursor = {"x": 0, "qkv": 0}

    def load(kind, host):
        """Copy `host` into the next ring buffer of `kind` on the copy-in
        stream; the compute stream waits for it.  Returns the buffer."""
        k = cursor[kind]
        cursor[kind] = (k + 1) % RING
        buf = (d_x if kind == "x" else d_qkv)[k]
        with torch.cuda.stream(s_in):
            if free[kind][k] is not None:
                s_in.wait_event(free[kind][k])
            buf.copy_(host, non_blocking=True)
            ready = torch.cuda.Event()
            ready.record(s_in)
        comp.wait_event(ready)
        return buf, k

    def release(kind, k):
        ev = torch.cuda.Event()
        ev.record(comp)
        free[kind][k] = ev

    def store(*outs):
        """Copy the op's outputs back on the copy-out stream, after the op."""
        done = torch.cuda.Event()
        done.record(comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(done)
            for o in outs:
                h_out.view(-1)[: o.numel()].copy_(o.reshape(-1), non_blocking=True)
                o.record_stream(s_out)
        return sum(nbytes(o) for o in outs)

    def run_once():
        h2d = d2h = 0
        mod = step.mod
        with torch.no_grad():
            x, k = load("x", h_act)
            h2d += nbytes(h_act)
            z = x.clone()
            hid = afb.adaln(z, mod[0, 0, 0], mod[0, 0, 1])
            release("x", k)
            d2h += store(hid)
            for l in range(s.layers):
                qkv, kq = load("qkv", h_qkv)
                h2d += nbytes(h_qkv)
                q, kk, _ = afb.qkv_norm_rope(qkv, step.qw[l], step.kw[l], step.cos, step.sin, H)
                release("qkv", kq)
                d2h += store(q, kk)
                for j in range(3):
                    if j == 1:
                        xq, k = load("x", h_act)
                        h2d += nbytes(h_act)
                        y = afb.head_norm(xq, step.xw[l], H)
                        release("x", k)
                        d2h += store(y)
                    x, k = load("x", h_act)
                    h2d += nbytes(h_act)
                    hid, z = afb.residual_adaln(x, z, *step.block_mods(l, j))
                    release("x", k)
                    d2h += store(hid)
            d2h += store(z)
        return h2d, d2h

    def join():
        comp.wait_stream(s_in)
        comp.wait_stream(s_out)

    for _ in range(2):
        run_once()
    join()
    torch.cuda.synchronize()
    n = max(1, min(args.steps, args.e2e_steps))
    barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(comp)
    s_in.wait_stream(comp)   # no copy starts before the timed region
    s_out.wait_stream(comp)
    for _ in range(n):
        h2d, d2h = run_once()
    join()                   # the region ends after the last copy of either direction
    b.record(comp)
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(a.elapsed_time(b), device)
    rates = copy_rates(device)  # after the timed region
    os.sched_setaffinity(0, all_cpus)  # the CPU baseline runs on every host thread
    calls = W.bf16_forward_calls(s)
    val = W.step_bytes(calls, s) * world * n / (ms * 1e-3) / 1e9
    return {"value": round(val, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "steps": n, "ms_per_step": round(ms / n, 3),
            "numa": numa, "copy_rates_this_rank": rates,
            "path": "anima_flat_b200 public API (torch custom ops -> C ABI), pinned host buffers; "
                    f"host-to-device copies, kernels and device-to-host copies on three streams, "
                    f"ordered by events, inputs in a ring of {RING} device buffers"}


# -------------------------------------------------- CPU baseline / reference --
def cpu_sequence(shape: W.Shape, seed: int = 0):
    """The reference's unfused torch fp32 eager composition of the step's ops
    on the host cores (oracle/formulation.py)."""
    from oracle import formulation as Fm

    from anima_flat_b200.tables import rope_tables

    s = shape
    g = torch.Generator().manual_seed(seed)
    bf = torch.bfloat16
    act = lambda *d: torch.randn(*d, generator=g).to(bf)
    B, S, D, H, hd = s.batch, s.seq, s.dim, s.heads, s.head_dim
    side = int(round(S ** 0.5))
    cos, sin = rope_tables(side, S // side, hd, "cpu", (4.0, 4.0))
    mod = (torch.randn(3, 3, B, D, generator=g) * 0.1).to(bf)
    mod[:, 1] += 1.0
    w = 1.0 + 0.02 * torch.randn(hd, generator=g)
    z0, qkv, x, xq = act(B, S, D), act(B, S, 3 * D), act(B, S, D), act(B, S, D)

    def run():
        z = z0
        Fm.adaln(z, mod[0, 0], mod[0, 1])
        for l in range(s.layers):
            Fm.qkv_norm_rope(qkv, w, w, cos, sin, H)
            _, z = Fm.residual_adaln(x, z, mod[0, 2], mod[1, 0], mod[1, 1])
            Fm.head_norm(xq, w, H)
            _, z = Fm.residual_adaln(x, z, mod[1, 2], mod[2, 0], mod[2, 1])
            _, z = Fm.residual_adaln(x, z, mod[2, 2], mod[0, 0], mod[0, 1])

    return run, W.step_bytes(W.bf16_forward_calls(s), s)


def _cpu_rate(shape: W.Shape, budget_s: float, max_steps: int = 1000):
    """Steps of the CPU composition at `shape` within about budget_s seconds
    (at least one after a warm-up step): (steps, seconds, bytes per step)."""
    run, nbytes = cpu_sequence(shape)
    run()
    n, t0 = 0, time.perf_counter()
    while True:
        run()
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s or n >= max_steps:
            return n, el, nbytes


def cpu_baseline(budget_s: float = 12.0) -> dict:
    """The config-2 step (the shapes our arm runs) on all host threads, for a
    bounded number of steps, and the config-1 shapes beside it."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    n, el, nbytes = _cpu_rate(W.Shape(), budget_s)
    n1, el1, nbytes1 = _cpu_rate(W.Shape(seq=256), max(1.0, budget_s / 4))
    return {"value": round(nbytes * n / el / 1e9, 3), "unit": "GB/s", "cores": threads,
            "kind": "port",
            "sample": (f"{n} steps of the config-2 op sequence (141 ops, B=1, S=4096, D=2048, "
                       "16x128 heads; the same shapes and byte model as our arm), torch fp32 eager "
                       "composition (oracle/formulation.py)"),
            "seconds": round(el, 2),
            "same_config": True,
            "cfg1": {"value": round(nbytes1 * n1 / el1 / 1e9, 3), "unit": "GB/s",
                     "sample": f"{n1} steps of the same op sequence at config-1 shapes (S=256)",
                     "seconds": round(el1, 2)}}


def run_reference(args, world, rank):
    """The reference arm: the unfused PyTorch-eager fp32 composition the task
    names as the reference's CPU path (the reference ships no CPU kernels),
    on the host cores, rank 0 only."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    shape = W.Shape()  # config 2: the shapes our arm runs
    run, nbytes = cpu_sequence(shape)
    for _ in range(min(args.warmup, 1)):  # a CPU step needs no more warm-up than one step
        run()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        run()
    el = time.perf_counter() - t0
    value = nbytes * args.steps / el / 1e9
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 3),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(el * 1e3 / args.steps, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp32",
        "data": "synthetic (seeded)",
        "config": {"workload": "cfg2: Cosmos-Predict2-2B forward fused-op sequence (141 ops), "
                               "1024x1024, B=1, S=4096, D=2048, 16x128 heads, on the host cores",
                   "global_batch": 1, "seq_len": 4096, "parallelism": "host threads"},
        "mrows_per_s": round(shape.rows * args.steps / el / 1e6, 4),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads,
                         "kind": "port",
                         "sample": f"{args.steps} steps of the config-2 op sequence, torch fp32 "
                                   "eager composition of the reference's formulas "
                                   "(oracle/formulation.py), config-2 shapes"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------- per-op table --
PER_OPS = ["residual_adaln", "adaln", "qkv_norm_rope", "head_norm", "residual_adaln_fp8",
           "adaln_fp8", "rowquant", "rowquant_gelu", "residual_adaln_bwd", "adaln_bwd",
           "qkv_norm_rope_bwd", "head_norm_bwd", "ctx_scale", "ctx_scale_bwd", "ctx_scale_rowquant",
           "rms_silu", "add_rms_silu", "shuffle_rms_silu", "rms_silu_bwd"]


def between_gemms(fn, sets, n: int, rows: int, dim: int, device) -> float:
    """The op's marginal time where the model runs it: every launch follows a
    bf16 GEMM of the model's projection shape ([rows, dim] x [dim, dim],
    src/model.py:297-337), as the GEMMs and attention surround these ops in
    a forward pass.  Two graphs, n x [GEMM, op] and n x [GEMM], CUDA events
    around each replay; returns (t_both - t_gemm) / n in microseconds."""
    g = torch.Generator(device=device).manual_seed(11)
    a = torch.randn(rows, dim, generator=g, device=device).to(torch.bfloat16)
    w = torch.randn(dim, dim, generator=g, device=device).to(torch.bfloat16)
    outs = [torch.empty(rows, dim, dtype=torch.bfloat16, device=device) for _ in range(2)]
    nbuf = len(sets)

    def timed(with_op: bool) -> float:
        with torch.no_grad():
            for i in range(3):
                torch.matmul(a, w, out=outs[i % 2])
                if with_op:
                    fn(*sets[i % nbuf])
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for i in range(n):
                    torch.matmul(a, w, out=outs[i % 2])
                    if with_op:
                        fn(*sets[i % nbuf])
            graph.replay()
            torch.cuda.synchronize()
            best = float("inf")
            for _ in range(3):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                graph.replay()
                e1.record()
                torch.cuda.synchronize()
                best = min(best, e0.elapsed_time(e1))
            del graph
        return best

    return (timed(True) - timed(False)) * 1e3 / n


def run_per_op(args):
    """Each op alone at its config shape (config 2 for the bf16 ops, config 3
    B=2 for the FP8 ops), inputs rotated over enough buffers to exceed 2x L2.
    Prints one JSON line per op: stream time (back-to-back launches with PDL,
    total / n) and isolated time (CUDA events around each launch)."""
    import anima_flat_b200 as afb
    from anima_flat_b200 import _lib

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    _lib.set_pdl(not args.no_pdl)
    peak, peak_src = peak_hbm()
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    names = PER_OPS if args.op == "all" else args.op.split(",")
    for name in names:
        fp8 = name in ("residual_adaln_fp8", "adaln_fp8", "rowquant", "rowquant_gelu", "ctx_scale_rowquant")
        s = W.Shape(batch=args.op_batch or (2 if fp8 else 1))
        B, S, D, H, hd = s.batch, s.seq, s.dim, s.heads, s.head_dim
        g = torch.Generator(device=device).manual_seed(7)
        act = lambda *d: torch.randn(*d, generator=g, device=device).to(torch.bfloat16)
        vec = lambda: (0.1 * torch.randn(B, D, generator=g, device=device)).to(torch.bfloat16)
        cos, sin = afb.rope_tables(64, 64, hd, device, (4.0, 4.0))
        w = 1.0 + 0.02 * torch.randn(hd, generator=g, device=device)
        nbytes = W.call_bytes(name, s)
        nbuf = max(2, int(2 * l2 // max(1, nbytes)) + 1)
        if name in ("residual_adaln", "residual_adaln_fp8"):
            sets = [(act(B, S, D), act(B, S, D), vec(), vec(), vec() + 1) for _ in range(nbuf)]
            fn = afb.residual_adaln if name == "residual_adaln" else afb.residual_adaln_fp8
        elif name in ("adaln", "adaln_fp8"):
            sets = [(act(B, S, D), vec(), vec() + 1) for _ in range(nbuf)]
            fn = afb.adaln if name == "adaln" else afb.adaln_fp8
        elif name == "qkv_norm_rope":
            sets = [(act(B, S, 3 * H * hd), w, w, cos, sin, H) for _ in range(nbuf)]
            fn = afb.qkv_norm_rope
        elif name == "head_norm":
            sets = [(act(B, S, H * hd), w, H) for _ in range(nbuf)]
            fn = afb.head_norm
        elif name == "residual_adaln_bwd":   # config 4 shapes (B=1), grads N(0, 1e-2)
            ops = torch.ops.anima_flat_b200
            sets = [(act(B, S, D) * 0.01, act(B, S, D) * 0.01, act(B, S, D), act(B, S, D), vec(),
                     vec() + 1, 1e-6) for _ in range(nbuf)]
            fn = ops.residual_adaln_bwd
        elif name == "adaln_bwd":
            ops = torch.ops.anima_flat_b200
            sets = [(act(B, S, D) * 0.01, act(B, S, D), vec() + 1, 1e-6) for _ in range(nbuf)]
            fn = ops.adaln_bwd
        elif name == "qkv_norm_rope_bwd":
            ops = torch.ops.anima_flat_b200
            sets = [(act(B, S, 3 * H * hd), act(B, S, H, hd) * 0.01, act(B, S, H, hd) * 0.01,
                     act(B, S, H, hd) * 0.01, w, w, cos, sin, H, 1e-5) for _ in range(nbuf)]
            fn = ops.qkv_norm_rope_bwd
        elif name == "head_norm_bwd":
            ops = torch.ops.anima_flat_b200
            sets = [(act(B, S, H * hd), act(B, S, H, hd) * 0.01, w, H, 1e-5) for _ in range(nbuf)]
            fn = ops.head_norm_bwd
        elif name in ("rms_silu", "add_rms_silu", "shuffle_rms_silu", "rms_silu_bwd"):
            # the VAE decoder's last stage at 1024x1024: [1, 1024, 1024, 96]
            Cv, side = W.VAE_C, 1024
            gam = 1.0 + 0.1 * torch.randn(Cv, generator=g, device=device)
            if name == "rms_silu":
                sets = [(act(1, side, side, Cv), gam) for _ in range(nbuf)]
                fn = afb.rms_silu
            elif name == "add_rms_silu":
                sets = [(act(1, side, side, Cv), act(1, side, side, Cv), gam) for _ in range(nbuf)]
                fn = afb.add_rms_silu
            elif name == "shuffle_rms_silu":
                sets = [(act(1, side // 2, side // 2, 4 * Cv), gam) for _ in range(nbuf)]
                fn = afb.shuffle_rms_silu
            else:
                ops = torch.ops.anima_flat_b200
                sets = [(act(1, side, side, Cv), gam, act(1, side, side, Cv) * 0.01,
                         act(1, side, side, Cv) * 0.01, False) for _ in range(nbuf)]
                fn = ops.rms_silu_bwd
        elif name in ("ctx_scale", "ctx_scale_bwd", "ctx_scale_rowquant"):
            # cross-attention output: config 2 for the bf16 ops, config 3 (B=2) for the FP8 one
            lse = lambda: 2.0 + 4.0 * torch.randn(B, H, S, generator=g, device=device)
            lnp = torch.full((B,), 4.0, device=device)
            if name == "ctx_scale_rowquant":
                sets = [(act(B, S, H, hd), lse(), lnp) for _ in range(nbuf)]
                fn = afb.ctx_scale_rowquant
            elif name == "ctx_scale":
                sets = [(act(B, S, H, hd), lse(), lnp) for _ in range(nbuf)]
                fn = afb.ctx_scale
            else:
                ops = torch.ops.anima_flat_b200
                sets = [(act(B, S, H, hd), lse(), lnp, act(B, S, H, hd) * 0.01) for _ in range(nbuf)]
                fn = ops.ctx_scale_bwd
        else:
            K = s.mlp if name == "rowquant_gelu" else D
            sets = [(act(B, S, K),) for _ in range(nbuf)]
            fn = (lambda x: afb.rowquant(x, gelu=True)) if name == "rowquant_gelu" else afb.rowquant
        n = max(args.steps, nbuf)
        with torch.no_grad():
            # stream: n launches back to back, captured in a graph
            for i in range(max(args.warmup, 3)):
                fn(*sets[i % nbuf])
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for i in range(n):
                    fn(*sets[i % nbuf])
            graph.replay()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            graph.replay()
            b.record()
            torch.cuda.synchronize()
            us_stream = a.elapsed_time(b) * 1e3 / n
            del graph
            # isolated: external events around each launch inside a graph
            # (no host gaps), PDL off so launches do not overlap
            _lib.set_pdl(False)
            ev = [(torch.cuda.Event(enable_timing=True, external=True),
                   torch.cuda.Event(enable_timing=True, external=True)) for _ in range(n)]
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for i in range(n):
                    ev[i][0].record()
                    fn(*sets[i % nbuf])
                    ev[i][1].record()
            _lib.set_pdl(not args.no_pdl)
            graph.replay()
            torch.cuda.synchronize()
            graph.replay()
            torch.cuda.synchronize()
            iso = sorted(x.elapsed_time(y) * 1e3 for x, y in ev)
            us_iso = iso[len(iso) // 2]
            del graph
            between = between_gemms(fn, sets, n, B * S, D, device) if args.between_gemms else None
        shape = ({"batch": 1, "height": 1024, "width": 1024, "channels": W.VAE_C} if "rms_silu" in name
                 else {"batch": B, "seq": S, "dim": D, "heads": H, "head_dim": hd})
        print(json.dumps({
            "op": name, "shape": shape,
            "bytes_per_launch": nbytes, "launches": n, "buffers": nbuf,
            "us_stream": round(us_stream, 3), "gbs_stream": round(nbytes / us_stream / 1e3, 1),
            "frac_stream": round(nbytes / us_stream / 1e3 / peak, 4),
            "us_isolated_median": round(us_iso, 3), "gbs_isolated": round(nbytes / us_iso / 1e3, 1),
            "frac_isolated": round(nbytes / us_iso / 1e3 / peak, 4),
            **({"us_between_gemms": round(between, 3),
                "frac_between_gemms": round(nbytes / between / 1e3 / peak, 4)} if between else {}),
            "peak_gbs": peak, "peak_source": peak_src, "pdl": not args.no_pdl}), flush=True)
        del sets
        torch.cuda.empty_cache()


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["cfg2", "cfg3", "cfg5"], default="cfg2")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--legs", default="cfg3,cfg4,cfg5",
                    help="extra configurations timed in the same run: comma-separated or 'none'")
    ap.add_argument("--leg-steps", type=int, default=20, help="at most this many timed steps per leg")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-pdl", action="store_true")
    ap.add_argument("--op", default=None,
                    help="per-op table instead of the step: 'all' or comma-separated op names")
    ap.add_argument("--between-gemms", action="store_true",
                    help="with --op: also time each op where every launch follows a model-shaped GEMM")
    ap.add_argument("--op-batch", type=int, default=0,
                    help="batch of the per-op shapes (default: the op's config, 1 or 2)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_info()
    if args.op:
        run_per_op(args)
        return
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    run_ours(args, world, rank, local)


if __name__ == "__main__":
    main()
