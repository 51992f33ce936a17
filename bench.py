#!/usr/bin/env python3
"""Benchmark of the sparse-attention hot path on B200.

Default workload: one CogVideoX-2B attention layer,
B=2, H=30, S=17776 (226 text + 13x30x45 video), D=64, bf16, 128x128 blocks,
top-10% blocks by mean-pooled score (k = 14 of 139) with text rows/columns
dense.  One step = block selection (mean-pool -> fp64 score -> top-k -> CSR)
+ block-sparse attention over the live blocks, inputs resident in HBM.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

N > 1 runs under torchrun, one rank per GPU, on ONE layer: its 30 heads
are split over the ranks (15/15, 8/8/7/7, 4,4,4,4,4,4,3,3), B = 2 on each,
with no collective on the data path (strong scaling; ``value`` = the
layer's live FLOP / the slowest rank's time).  A weak-scaling number (a
whole layer per rank) is reported beside it.  Times are CUDA-event times on
the launching stream, max over ranks; the timed steps replay the selection
and the attention as two CUDA graphs captured from the same calls, so host
load on a shared machine cannot leave the GPU idle inside the timed region.  At one GPU q/k/v/o are 136 MB each
(larger than the 126 MB L2), so no L2 flush is needed between steps.

At N = 1 the reference's own Triton kernels (installed unmodified in
``baseline/_ref``) are timed beside this package's kernels on the same
inputs and their outputs compared (``reference_triton``).  After every
timed region the GPU's sticky status flags are read; a run that set any is
marked ``failed``.

``e2e`` is the same metric through the public processor
(``special_attentions.block_mask_attn.BlockSparseAttention``) with pinned
host buffers: every step copies q, k, v in and the output out, in a
pipelined serving loop (copy-in, compute and copy-out on three streams with
double-buffered device buffers); the serial one-stream time is reported
beside it as ``ms_per_step_serial``.

Rank 0 prints ONE JSON line (see the keys below).  ``--impl reference``
times the reference's PyTorch masked-attention path (query-chunked boolean
mask SDPA, restated in ``oracle/attention.py``) on the host CPU cores.
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

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "ms per attention layer & effective TFLOP/s at S=17776,H=30,D=64, 10% blocks; ms/merge"
UNIT = "TFLOP/s"
FALLBACK_PEAKS = {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0}


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


def profile_traffic(name: str):
    """DRAM bytes per launch recorded from an ncu capture in profiles/<name>.md
    (a line `traffic_bytes_per_launch: N`), or None."""
    p = ROOT / "profiles" / f"{name}.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_uuid: str):
        self.samples = []
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", gpu_uuid, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), line.strip()))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0: float, t1: float):
        rows = []
        for ts, line in self.samples:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8:
                continue
            rows.append((ts, parts))
        win = [r for r in rows if t0 <= r[0] <= t1]
        if len(win) < 3:
            win = rows
        if not win:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(p[0]) for _, p in win if num(p[0]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, p in win for i in range(4) if p[4 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": num(win[0][1][1]), "reasons": reasons, "samples": len(win),
                "power_w_max": max((num(p[2]) or 0.0) for _, p in win)}


def init_dist():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        # rank 0's stdout carries exactly one JSON line: NCCL's own log lines go to stderr
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        torch.cuda.set_device(local)
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def allreduce(x: float, op: str, world: int):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# --------------------------------------------------------------------------- workloads

def c2_setup(device, rank, seed=1234):
    """The config-2 layer's q, k, v [2, 30, 17776, 64] bf16 on the CPU (one
    seeded layer, the same on every rank) and its selection parameters."""
    import torch

    from sparseattnfunctions_b200 import workloads
    from sparseattnfunctions_b200.geometry import COGVIDEOX_2B as geo

    B, H, D, bs, density = 2, 30, 64, 128, 0.10
    q, k, v = workloads.video_qkv(geo, B=B, H=H, D=D, dtype=torch.bfloat16, seed=seed)
    nb = geo.num_blocks(bs)
    cfg = dict(B=B, H=H, S=geo.seq_len, D=D, block=bs, density=density, topk=math.ceil(density * nb),
               text_blocks=geo.text_blocks(bs), geo=geo)
    return (q, k, v), cfg


def device_status(local):
    """Reads and clears this GPU's sticky status flags (a wait that ran out,
    an index that was skipped) after a timed region."""
    from sparseattnfunctions_b200 import _lib

    return int(_lib.read_device_status(local, clear=True))


def time_layer(step, stream, steps, world):
    """Times `steps` calls of `step` (CUDA events on `stream`, barrier and
    synchronize on both sides); returns (elapsed ms max over ranks, per-step
    [select, attention] ms of this rank)."""
    import torch

    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    t_start.record(stream)
    for i in range(steps):
        step(ev[i])
    t_end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    elapsed = t_start.elapsed_time(t_end)
    sel_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / steps
    att_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / steps
    return allreduce(elapsed, "max", world), sel_ms, att_ms


def cpu_masked_baseline(qkv_cpu, mask_cpu, cfg, budget_s=12.0, threads=None):
    """Times the reference's PyTorch masked path (oracle restatement) on the
    host CPU over whole heads until ``budget_s`` elapses; returns
    (TFLOP/s on the live-block FLOP of the heads done, heads done, seconds)."""
    import torch

    from oracle import attention as oatt

    if threads:
        torch.set_num_threads(threads)
    q, k, v = qkv_cpu
    B, H, S, D = q.shape
    bs = cfg["block"]
    rows = torch.full((mask_cpu.shape[2],), float(bs), dtype=torch.float64)
    rows[-1] = S - (mask_cpu.shape[2] - 1) * bs
    cols = torch.full((mask_cpu.shape[3],), float(bs), dtype=torch.float64)
    cols[-1] = S - (mask_cpu.shape[3] - 1) * bs
    flops, done = 0.0, 0
    t0 = time.perf_counter()
    for g in range(B * H):
        b, h = divmod(g, H)
        oatt.masked_sdpa_cpu(q, k, v, mask_cpu, 1.0 / math.sqrt(D), bs, bs, q_chunk=2048, heads=[g])
        flops += float(4.0 * D * torch.einsum("ij,i,j->", mask_cpu[b, h].double(), rows, cols))
        done += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    return flops / dt / 1e12, done, dt


# --------------------------------------------------------------------------- arms

def run_saf(args, world, rank, local):
    import torch

    from sparseattnfunctions_b200 import kernels
    from sparseattnfunctions_b200.special_attentions.block_mask_attn import BlockSparseAttention

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    (q_full, k_full, v_full), cfg = c2_setup(dev, rank)
    # strong scaling: the one layer's 30 heads split over the ranks
    # (15/15, 8/8/7/7, 4,4,4,4,4,4,3,3); B = 2 on every rank
    off = kernels.head_split(cfg["H"], world)
    h0, h1 = off[rank], off[rank + 1]
    q_c, k_c, v_c = (t[:, h0:h1].contiguous() for t in (q_full, k_full, v_full))
    q, k, v = q_c.to(dev), k_c.to(dev), v_c.to(dev)
    out = torch.empty_like(q)
    bs, D = cfg["block"], cfg["D"]
    scale = 1.0 / math.sqrt(D)
    sel_kw = dict(block_m=bs, block_n=bs, topk=cfg["topk"], text_blocks_q=cfg["text_blocks"],
                  text_blocks_k=cfg["text_blocks"])
    stream = torch.cuda.current_stream(dev)

    def make_step(qq, kk, vv, oo, holder):
        def step(ev):
            ev[0].record(stream)
            holder[0] = kernels.pool_topk(qq, kk, **sel_kw)
            ev[1].record(stream)
            kernels.bsa_fwd(qq, kk, vv, holder[0], scale, out=oo)
            ev[2].record(stream)
        return step

    def make_graph_step(qq, kk, vv, oo, holder):
        """The same two launches sequences captured as CUDA graphs (selection,
        attention), replayed on the stream: the host enqueues a step in a few
        microseconds, so a busy or descheduled host never leaves the GPU idle
        inside the timed region."""
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(2):
                holder[0] = kernels.pool_topk(qq, kk, **sel_kw)
                kernels.bsa_fwd(qq, kk, vv, holder[0], scale, out=oo)
        stream.wait_stream(side)
        torch.cuda.synchronize()
        g_sel, g_att = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_sel):
            holder[0] = kernels.pool_topk(qq, kk, **sel_kw)
        with torch.cuda.graph(g_att):
            kernels.bsa_fwd(qq, kk, vv, holder[0], scale, out=oo)
        torch.cuda.synchronize()
        holder.append((g_sel, g_att))  # keep the graphs alive

        def step(ev):
            ev[0].record(stream)
            g_sel.replay()
            ev[1].record(stream)
            g_att.replay()
            ev[2].record(stream)
        return step

    held = [None]
    dummy = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(3))]
    for _ in range(args.warmup):
        make_step(q, k, v, out, held)(dummy[0])
    torch.cuda.synchronize()
    step = make_graph_step(q, k, v, out, held)
    for _ in range(args.warmup):
        step(dummy[0])
    torch.cuda.synchronize()
    csr = held[0]
    live_flops = float(csr.live_flops(cfg["S"], cfg["S"], D))
    dense_flops = 4.0 * cfg["B"] * cfg["H"] * cfg["S"] ** 2 * D
    nnz = allreduce(float(csr.nnz_per_head().sum()), "sum", world)
    # pooling (q and k in one launch), score + top-k, CSR compaction, attention;
    # the attention's split counters are cleared by a memset node, not a kernel
    launches_per_step = 4

    uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    sampler = ClockSampler(uuid)
    time.sleep(0.3)
    w0 = time.time()
    max_elapsed, sel_ms, att_ms = time_layer(step, stream, args.steps, world)
    w1 = time.time()
    sampler.stop()
    status = {"layer": device_status(local)}
    total_flops = allreduce(live_flops, "sum", world)
    ms_per_step = max_elapsed / args.steps
    value = total_flops / (ms_per_step * 1e-3) / 1e12

    # weak scaling beside it: every rank runs a whole layer (all 30 heads)
    weak = None
    if world > 1:
        qf, kf, vf = q_full.to(dev), k_full.to(dev), v_full.to(dev)
        of = torch.empty_like(qf)
        wheld = [None]
        wstep = make_graph_step(qf, kf, vf, of, wheld)
        for _ in range(3):
            wstep(dummy[0])
        torch.cuda.synchronize()
        wflops = allreduce(float(wheld[0].live_flops(cfg["S"], cfg["S"], D)), "sum", world)
        n_weak = max(3, min(args.steps, 20))
        w_el, _, _ = time_layer(wstep, stream, n_weak, world)
        weak = {"workload": "every rank runs a whole config-2 layer (30 heads)",
                "value": round(wflops / (w_el / n_weak * 1e-3) / 1e12, 2), "unit": UNIT,
                "ms_per_step": round(w_el / n_weak, 4), "steps": n_weak}
        status["weak"] = device_status(local)
        del qf, kf, vf, of, wheld

    # ---- end to end through the public processor, host buffers
    proc = BlockSparseAttention(block_size=bs, density=cfg["density"], geometry=cfg["geo"])
    hq, hk, hv = (t.pin_memory() for t in (q_c, k_c, v_c))
    ho = torch.empty_like(hq).pin_memory()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    e2e_steps = max(1, min(args.steps, args.e2e_steps))

    def e2e_step():
        dq.copy_(hq, non_blocking=True)
        dk.copy_(hk, non_blocking=True)
        dv.copy_(hv, non_blocking=True)
        o = proc(dq, dk, dv)
        ho.copy_(o, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_serial_ms = allreduce(e0.elapsed_time(e1), "max", world) / e2e_steps
    ok_e2e = torch.equal(ho, out.cpu())

    # Pipelined serving loop: step i's host->device copies (copy-in stream)
    # overlap step i-1's compute and step i-2's device->host copy (copy-out
    # stream); device input and output buffers are double-buffered.  Every
    # step still moves its full inputs in and its output out.
    cin, cout = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    bufs = [tuple(torch.empty_like(t) for t in (q, k, v)) for _ in range(2)]
    obufs = [torch.empty_like(out) for _ in range(2)]
    ho2 = torch.empty_like(hq).pin_memory()

    def e2e_pipelined(n):
        in_free = [None, None]   # compute done with input buffer b
        out_free = [None, None]  # copy-out done with output buffer b
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(cin)
        for i in range(n):
            b = i % 2
            with torch.cuda.stream(cin):
                if in_free[b] is not None:
                    cin.wait_event(in_free[b])
                for d, h in zip(bufs[b], (hq, hk, hv)):
                    d.copy_(h, non_blocking=True)
                landed = torch.cuda.Event()
                landed.record(cin)
            stream.wait_event(landed)
            if out_free[b] is not None:
                stream.wait_event(out_free[b])
            proc(*bufs[b], out=obufs[b])
            computed = torch.cuda.Event()
            computed.record(stream)
            in_free[b] = computed
            with torch.cuda.stream(cout):
                cout.wait_event(computed)
                ho2.copy_(obufs[b], non_blocking=True)
                out_free[b] = torch.cuda.Event()
                out_free[b].record(cout)
        t1.record(cout)
        return t0, t1

    e2e_pipelined(2)
    torch.cuda.synchronize()
    barrier(world)
    t0, t1 = e2e_pipelined(e2e_steps)
    torch.cuda.synchronize()
    e2e_ms = allreduce(t0.elapsed_time(t1), "max", world) / e2e_steps
    e2e_val = total_flops / (e2e_ms * 1e-3) / 1e12
    h2d = int(allreduce(float(3 * q.numel() * q.element_size()), "sum", world))
    d2h = int(allreduce(float(out.numel() * out.element_size()), "sum", world))
    ok_e2e = ok_e2e and torch.equal(ho2, out.cpu())
    status["e2e"] = device_status(local)

    # ---- roofline of the dominant kernel (attention) and of the selection pass
    peaks, peak_kind = load_peaks()
    att_tflops = live_flops / (att_ms * 1e-3) / 1e12
    peak = peaks["bf16_tflops"]
    sel_bytes = 2 * q.numel() * q.element_size()
    sel_gbs = sel_bytes / (sel_ms * 1e-3) / 1e9
    traffic = profile_traffic("bsa_fwd_sm100_c2")
    if traffic is not None and world > 1:
        traffic = traffic * (h1 - h0) / cfg["H"]  # the capture covers all 30 heads
    clocks = sampler.summary(w0, w1)
    flags = allreduce(float(sum(status.values())), "sum", world)

    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded smooth field + noise, CogVideoX-2B shapes)",
            "config": {"workload": "config2: one CogVideoX-2B attention layer, select + block-sparse attention",
                       "B": cfg["B"], "H": cfg["H"], "S": cfg["S"], "D": D, "block": bs,
                       "density": cfg["density"], "topk": cfg["topk"],
                       "text_blocks_dense": cfg["text_blocks"], "live_blocks_per_layer": int(nnz),
                       "live_fraction": round(nnz / (cfg["B"] * cfg["H"] * csr.nbq * csr.nbk), 4),
                       "live_tflop_per_layer": round(total_flops / 1e12, 4),
                       "l2": "inputs larger than L2 (q/k/v/o 136 MB each at one GPU), no flush",
                       "parallelism": f"heads split over {world} GPU(s): {[off[i + 1] - off[i] for i in range(world)]}"
                                      ", B=2 on each, no collective"},
            "ms_per_layer": round(ms_per_step, 4),
            "dense_equiv_tflops": round(dense_flops / (ms_per_step * 1e-3) / 1e12, 1),
            "kernels_ms": {"select": round(sel_ms, 4), "attention": round(att_ms, 4)},
            "select_hbm": {"bytes": sel_bytes, "gbs": round(sel_gbs, 1),
                           "frac": round(sel_gbs / peaks["hbm_gbs"], 3)},
            "clocks": clocks,
            "device_status": {"flags": int(flags), "checked_after": sorted(status)},
            "e2e": {"value": round(e2e_val, 3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 3), "steps": e2e_steps,
                    "pipelined": "copy-in / compute / copy-out on three streams, double-buffered",
                    "ms_per_step_serial": round(e2e_serial_ms, 3),
                    "api": "special_attentions.block_mask_attn.BlockSparseAttention.__call__",
                    "matches_device_result": ok_e2e},
            "gpu_launches": launches_per_step * args.steps,
            "roofline": {"bound": "tensor", "kernel": "bsa_fwd_sm100_kernel<128,false,true>",
                         "achieved": round(att_tflops, 1), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(att_tflops / peak, 3),
                         "frac_sustained": round(att_tflops / peaks.get("bf16_tflops_sustained", peak), 3),
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json bf16_tflops burst)",
                         "traffic": traffic,
                         "algorithmic_flop_per_launch": live_flops,
                         "rank": 0},
        }
        if weak is not None:
            line["weak_scaling"] = weak
        if flags:
            line["failed"] = "device status flags set after a timed region: results not valid"
    if world == 1 and not args.no_reference_kernel:
        ref = bench_reference_kernels(args, dev, q, k, v, out, csr, cfg)
        if line is not None:
            line["reference_triton"] = ref
    subs = [("pool", args.no_pool, lambda: bench_pool(args, dev, world, q, k, v)),
            ("merge", args.no_merge, lambda: bench_merge(args, dev, world, rank)),
            ("combined", args.no_combined, lambda: bench_combined(args, dev, world, rank)),
            ("long", args.no_long, lambda: bench_long(args, dev, world, rank)),
            ("local_global", args.no_local_global, lambda: bench_local_global(args, dev, world, q, k, v))]
    for name, skip, fn in subs:
        if skip:
            continue
        sub = fn()
        sub_flags = int(allreduce(float(device_status(local)), "sum", world))
        if line is not None:
            sub["device_status"] = sub_flags
            if sub_flags:
                sub["failed"] = "device status flags set after the timed region: results not valid"
            line[name] = sub
    return line, (q_c, k_c, v_c), csr, cfg


def bench_reference_kernels(args, dev, q, k, v, out, csr, cfg):
    """The reference's own Triton kernels, installed unmodified in
    baseline/_ref, on this GPU: the kernel-level bar and a parity check
    against this package's kernels on the same inputs.

    * block_sparse_triton_fn (block_sparse_attn_kernel.py:293) on the
      config-2 layer with the same live tokens as this run's block list (each
      selected 128-block is the 2 x 2 64-blocks the reference kernel takes):
      time, TFLOP/s on the same live FLOP, and max |difference| from this
      package's output.
    * the same at config 1 (B1 H2 S2048 fp32, 64-blocks, top-8 with the
      diagonal): max |difference| from this package's fp32 kernel (the
      reference's fp32 dots run as TF32).
    * attn_with_pooling (attn_pooling_kernel.py:289; 64-blocks, its
      BLOCK_N <= HEAD_DIM limit) on the first 17728 tokens (277 whole
      blocks: its block pointers are not bounds-checked): time, and max
      |difference| of the output and of the pooled map from saf_bsa_fwd_pool.
    """
    import torch

    from baseline import reference_kernels as rk
    from sparseattnfunctions_b200 import kernels, workloads

    if not rk.available():
        return {"unavailable": "the reference is not installed in baseline/_ref"}
    try:
        bsk = rk.load("block_sparse_attn_kernel")
    except Exception as e:  # noqa: BLE001 - report why the bar is missing
        return {"unavailable": f"reference import failed: {type(e).__name__}: {e}"}
    stream = torch.cuda.current_stream(dev)
    res = {"source": "baseline/_ref/utils (pip-installed reference, unmodified)"}

    def timed(fn, n):
        fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    S, D = cfg["S"], cfg["D"]
    nb64 = math.ceil(S / 64)
    m64 = csr.to_dense().repeat_interleave(2, dim=-2).repeat_interleave(2, dim=-1)[..., :nb64, :nb64]
    m64 = m64.contiguous()
    live = float(csr.live_flops(S, S, D))
    try:
        ref_out = torch.empty_like(q)
        ms = timed(lambda: ref_out.copy_(bsk.block_sparse_triton_fn(q, k, v, m64, 0.125)), 3)
        ours = timed(lambda: kernels.bsa_fwd(q, k, v, csr, 0.125, out=out), 3)
        diff = (ref_out.float() - out.float()).abs()
        res["config2"] = {
            "ms": round(ms, 4), "tflops": round(live / (ms * 1e-3) / 1e12, 1),
            "saf_ms": round(ours, 4), "speedup": round(ms / ours, 2),
            "max_abs_diff_vs_saf": float(torch.nan_to_num(diff, nan=float("inf")).max()),
            "nan_rows_match": bool(torch.equal(ref_out.isnan(), out.isnan())),
            "mask": "the run's 128-block selection as 64 x 64 blocks"}
        del ref_out
    except Exception as e:  # noqa: BLE001
        res["config2"] = {"unavailable": f"{type(e).__name__}: {e}"}

    try:
        q1, k1, v1 = (t.to(dev) for t in workloads.config1_qkv())
        c1 = kernels.pool_topk(q1, k1, block_m=64, block_n=64, topk=8, force_diag=True,
                               forced_inside_topk=True)
        o1 = kernels.bsa_fwd(q1, k1, v1, c1, 0.125)
        r1 = bsk.block_sparse_triton_fn(q1, k1, v1, c1.to_dense().contiguous(), 0.125)
        torch.cuda.synchronize()
        res["config1"] = {"max_abs_diff_vs_saf": float((r1 - o1).abs().max()), "dtype": "fp32",
                          "note": "reference fp32 tl.dot runs as TF32"}
    except Exception as e:  # noqa: BLE001
        res["config1"] = {"unavailable": f"{type(e).__name__}: {e}"}

    try:
        pk = rk.load("attn_pooling_kernel")
        Sp = (S // 64) * 64
        qp, kp, vp = (t[:, :, :Sp] for t in (q, k, v))
        nbp = Sp // 64
        dense = kernels.mask_to_csr(torch.ones(q.shape[0], q.shape[1], nbp, nbp, dtype=torch.bool, device=dev),
                                    64, 64)
        holder = {}

        def ref_pool():
            holder["o"], holder["p"] = pk.attn_with_pooling(qp, kp, vp, False, 0.125, 64)

        ms_ref = timed(ref_pool, 2)
        o_s, p_s = kernels.bsa_fwd_pool(qp, kp, vp, dense, 0.125, pool_block=64)
        ms_saf = timed(lambda: kernels.bsa_fwd_pool(qp, kp, vp, dense, 0.125, pool_block=64), 2)
        torch.cuda.synchronize()
        flop = 4.0 * q.shape[0] * q.shape[1] * Sp * Sp * D
        res["attn_with_pooling"] = {
            "S": Sp, "block": 64, "ms": round(ms_ref, 3), "tflops": round(flop / (ms_ref * 1e-3) / 1e12, 1),
            "saf_ms": round(ms_saf, 3), "speedup": round(ms_ref / ms_saf, 2),
            "max_abs_diff_out": float((holder["o"].float() - o_s.float()).abs().max()),
            "max_abs_diff_pool": float((holder["p"].float() - p_s).abs().max()),
            "note": "reference casts bf16 to fp32 (TF32 dots) and stores the map in bf16"}
        del holder
    except Exception as e:  # noqa: BLE001
        res["attn_with_pooling"] = {"unavailable": f"{type(e).__name__}: {e}"}
    torch.cuda.synchronize()
    res["device_status"] = device_status(dev.index)
    return res


def bench_pool(args, dev, world, q, k, v):
    """Attention with the pooled attention map (attn_pooling_kernel.py, the
    warm-up path): dense attention over the config-2 layer with and without
    the pooled map [B, H, 139, 139]."""
    import torch

    from sparseattnfunctions_b200 import kernels

    B, H, S, D = q.shape
    nb = math.ceil(S / 128)
    csr = kernels.mask_to_csr(torch.ones(B, H, nb, nb, dtype=torch.bool, device=dev), 128, 128)
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream(dev)
    n = 3

    def timed(fn):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return allreduce(e0.elapsed_time(e1) / n, "max", world)

    ms_dense = timed(lambda: kernels.bsa_fwd(q, k, v, csr, 0.125, out=out))
    ms_pool = timed(lambda: kernels.bsa_fwd_pool(q, k, v, csr, 0.125, out=out))
    # comparison bar only (a library kernel, not this package's path): torch's
    # dense scaled-dot-product attention at the same shape
    import torch.nn.functional as F
    ms_sdpa = timed(lambda: F.scaled_dot_product_attention(q, k, v, scale=0.125))
    flop = 4.0 * B * H * S * S * D
    return {"workload": "dense attention over the config-2 layer (B=2, H=30, S=17776, D=64, bf16) with the "
                        "pooled 128-block attention map (attn_with_pooling)",
            "ms_dense": round(ms_dense, 4), "ms_dense_with_pool": round(ms_pool, 4),
            "pool_overhead": round(ms_pool / ms_dense - 1.0, 4),
            "dense_tflops": round(flop / (ms_dense * 1e-3) / 1e12, 1),
            "torch_sdpa_dense_ms": round(ms_sdpa, 4),
            "torch_sdpa_dense_tflops": round(flop / (ms_sdpa * 1e-3) / 1e12, 1), "steps": n}


def bench_local_global(args, dev, world, q, k, v):
    """LocalGlobalAttention (LocalGlobalAttention.py:183-259) on the config-2
    layer: dense text + frame-0 rows, 18 patches x 2 batches over their
    window + probe keys (7073 per list), the probe of 1280 sampled rows
    every update_gap calls."""
    import torch

    from sparseattnfunctions_b200 import kernels
    from sparseattnfunctions_b200.special_attentions import LocalGlobalAttention as lga

    B, H, S, D = q.shape
    stream = torch.cuda.current_stream(dev)
    obj = lga.LocalGlobalAttention()
    lga.counter = 0
    obj(q, k, v)  # builds the window lists and the first probe
    n = 5

    def timed(fn):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return allreduce(e0.elapsed_time(e1) / n, "max", world)

    def forward_no_probe():
        lga.counter = 1 << 30  # keep the current probe keys
        obj(q, k, v)

    ms_fwd = timed(forward_no_probe)
    qv = obj.slice_video(q)
    ms_probe = timed(lambda: obj.probe._probe(qv, k))
    dense = lga.TEXT_LEN + 1350
    out = torch.empty_like(q)
    ms_dense = timed(lambda: obj.attention_text(q[:, :, :dense], k, v, out=out[:, :, :dense]))
    keys, src = obj.patch_keys(qv, k)
    lga.counter = 1 << 30
    qp = obj.transform_q(q)
    # the patch attention with the listed k / v rows gathered inside the kernel
    ms_patch = timed(lambda: kernels.bsa_fwd_keys(qp, k, v, keys, src, 1.0 / math.sqrt(D)))
    # for comparison: the gathered copies the reference builds, and attention over them
    kidx = obj.key_lists(qv, k)
    lga.counter = 1 << 30
    ms_gather_kv = timed(lambda: (kernels.gather_rows(k, kidx), kernels.gather_rows(v, kidx)))
    kp, vp = kernels.gather_rows(k, kidx), kernels.gather_rows(v, kidx)
    ms_patch_gathered = timed(lambda: obj.attention_video(qp, kp, vp))
    del kp, vp
    L = keys.shape[1]
    flop_dense = 4.0 * B * H * dense * S * D
    flop_patch = 4.0 * keys.shape[0] * H * qp.shape[2] * L * D
    flop_probe = 2 * 2.0 * B * H * 1280 * S * D
    gather_bytes = 2 * 2 * kidx.numel() * H * D * 2  # k and v rows read and written
    return {"workload": "LocalGlobalAttention on the config-2 layer (B=2, H=30, S=17776, D=64, bf16): dense "
                        f"{dense} rows, 36 patch lists of {L} keys, probe of 1280 rows every 5 calls",
            "ms_forward": round(ms_fwd, 4), "ms_probe": round(ms_probe, 4),
            "ms_per_call_with_probe_every_5": round(ms_fwd + ms_probe / 5, 4),
            "ms_dense_rows": round(ms_dense, 4), "ms_patch_attention_key_lists": round(ms_patch, 4),
            "ms_gather_kv_copies": round(ms_gather_kv, 4),
            "ms_patch_attention_on_copies": round(ms_patch_gathered, 4),
            "dense_rows_tflops": round(flop_dense / (ms_dense * 1e-3) / 1e12, 1),
            "patch_attention_tflops": round(flop_patch / (ms_patch * 1e-3) / 1e12, 1),
            "probe_qk_tflops": round(flop_probe / (ms_probe * 1e-3) / 1e12, 1),
            "gather_kv_gbs": round(gather_bytes / (ms_gather_kv * 1e-3) / 1e9, 1), "steps": n}


def bench_merge(args, dev, world, rank):
    """ToMe on CogVideoX-2B hidden states [2, 17550, 1920]
    bf16, alternate split (src even / dst odd), r = 4000; then dense
    attention (H = 30, D = 64) over the 226 text + 13550 merged tokens with
    the log(size) bias, and unmerge.  'ms/merge' = match + merge."""
    import torch

    from sparseattnfunctions_b200 import kernels, workloads
    from sparseattnfunctions_b200.geometry import COGVIDEOX_2B as geo
    from sparseattnfunctions_b200.special_attentions.utils.merge_unmerge import alternate_split

    B, C, r, H, D, T = 2, 1920, 4000, 30, 64, geo.text_len
    N = geo.video_len
    x = workloads.video_hidden(geo, B=B, C=C, seed=4321 + rank).to(dev)
    g = torch.Generator().manual_seed(77 + rank)
    text = torch.randn(B, T, C, generator=g).to(torch.bfloat16).to(dev)
    xt = torch.cat([text, x], dim=1)
    a_idx, b_idx = alternate_split(N, dev)
    L = T + (a_idx.numel() - r) + b_idx.numel()
    nb = math.ceil(L / 128)
    csr = kernels.mask_to_csr(torch.ones(B, H, nb, nb, dtype=torch.bool, device=dev), 128, 128)
    stream = torch.cuda.current_stream(dev)
    n = max(3, min(args.merge_steps, args.steps))

    # outputs allocated once: the timed loop makes no allocation
    merged = torch.empty(B, L, C, dtype=xt.dtype, device=dev)
    o_rows = torch.empty(B, L, C, dtype=xt.dtype, device=dev)  # [B, L, H*D]: heads side by side
    y = torch.empty(B, T + N, C, dtype=xt.dtype, device=dev)
    bias = torch.zeros(B * H, L, dtype=torch.float32, device=dev)

    def one(ev):
        ev[0].record(stream)
        plan = kernels.tome_match(x, a_idx, b_idx, r)
        ev[1].record(stream)
        kernels.tome_merge(xt, plan, text_len=T, out=merged)
        ev[2].record(stream)
        qkv = merged.view(B, L, H, D).transpose(1, 2)
        bias.view(B, H, L)[:, :, L - plan.Nd:] = plan.log_count[:, None, :]
        ev[3].record(stream)
        kernels.bsa_fwd(qkv, qkv, qkv, csr, 1.0 / math.sqrt(D), kv_bias=bias,
                        out=o_rows.view(B, L, H, D).transpose(1, 2))
        ev[4].record(stream)
        kernels.tome_unmerge(o_rows, plan, text_len=T, out=y)
        ev[5].record(stream)
        return plan, y

    mk = lambda: [torch.cuda.Event(enable_timing=True) for _ in range(6)]
    for _ in range(2):
        one(mk())
    torch.cuda.synchronize()
    evs = [mk() for _ in range(n)]
    barrier(world)
    for e in evs:
        plan, _ = one(e)
    torch.cuda.synchronize()
    avg = lambda a, b: sum(e[a].elapsed_time(e[b]) for e in evs) / n
    m_match, m_merge, m_attn, m_unmerge = avg(0, 1), avg(1, 2), avg(3, 4), avg(4, 5)
    m_match = allreduce(m_match, "max", world)
    m_merge = allreduce(m_merge, "max", world)
    gemm_flop = 2.0 * B * a_idx.numel() * b_idx.numel() * C
    attn_flop = 4.0 * B * H * L * L * D
    merge_bytes = (B * N * C + B * (L - T) * C) * 2
    peaks, kind = load_peaks()
    return {
        "workload": "config3: ToMe r=4000 on [2,17550,1920] bf16 (alternate split), dense attention "
                    "over 226+13550 tokens, unmerge",
        "ms_per_merge": round(m_match + m_merge, 4), "ms_match": round(m_match, 4),
        "ms_merge": round(m_merge, 4), "ms_attention_merged": round(m_attn, 4),
        "ms_unmerge": round(m_unmerge, 4), "steps": n,
        "match_gemm_tflops": round(gemm_flop / (m_match * 1e-3) / 1e12, 1),
        "match_gemm_frac": round(gemm_flop / (m_match * 1e-3) / 1e12 / peaks["bf16_tflops"], 3),
        "merge_gbs": round(merge_bytes / (m_merge * 1e-3) / 1e9, 1),
        "attention_merged_tflops": round(attn_flop / (m_attn * 1e-3) / 1e12, 1),
        "merged_tokens": L, "max_merged_size": int(plan.counter.max()),
    }


def bench_combined(args, dev, world, rank):
    """combined attention (ToMe r = 4000 per (b, h) on the
    [k, |k|, v, |v|] metric -> top-15% block selection on the merged
    sequence -> block-sparse attention with the log(size) bias -> unmerge)
    in all 30 layers of a random-init CogVideoX-2B-shaped block stack
    (hidden 1920 = 30 heads x 64, B = 2, S = 17776, bf16).  Each layer
    projects the hidden state to q / k / v (cuBLAS, outside the timed
    region), calls the processor (timed with CUDA events), projects the
    output back and adds it to the residual stream.  Reported: attention ms
    per denoising step (sum over the 30 layers)."""
    import torch

    from sparseattnfunctions_b200 import workloads
    from sparseattnfunctions_b200.geometry import COGVIDEOX_2B as geo
    from sparseattnfunctions_b200.special_attentions.combined_attn import CombinedAttn

    B, C, H, D, layers, T = 2, 1920, 30, 64, 30, geo.text_len
    S = geo.seq_len
    g = torch.Generator().manual_seed(99 + rank)
    text = torch.randn(B, T, C, generator=g).to(torch.bfloat16)
    x0 = torch.cat([text, workloads.video_hidden(geo, B=B, C=C, seed=5151 + rank)], dim=1).to(dev)
    gd = torch.Generator(device=dev).manual_seed(2024 + rank)
    w_qkv = [torch.randn(C, 3 * C, generator=gd, device=dev, dtype=torch.bfloat16) / math.sqrt(C)
             for _ in range(layers)]
    w_o = [torch.randn(C, C, generator=gd, device=dev, dtype=torch.bfloat16) * (0.5 / math.sqrt(C))
           for _ in range(layers)]
    attn = CombinedAttn(warmup_epoch=0, layer_num=layers, density=0.15, block_size=128, full_merge=True)
    stream = torch.cuda.current_stream(dev)

    def one_step(evs, flops=None):
        x = x0.clone()
        for l in range(layers):
            qkv = (x @ w_qkv[l]).view(B, S, 3, H, D).permute(2, 0, 3, 1, 4).contiguous()
            q, k, v = qkv[0], qkv[1], qkv[2]
            evs[l][0].record(stream)
            o = attn(q, k, v)
            evs[l][1].record(stream)
            if flops is not None:
                L = attn._layers[l].merge_fn.plan.merged_len + T
                flops.append(attn.last_csr.live_flops(L, L, D))
            x = x + o.transpose(1, 2).reshape(B, S, C) @ w_o[l]
        return x

    mk = lambda: [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(layers)]
    flops = []
    one_step(mk(), flops)  # warm-up step (also builds every layer's plan once)
    torch.cuda.synchronize()
    live = float(sum(float(f) for f in flops))
    n = max(1, args.combined_steps)
    runs = [mk() for _ in range(n)]
    barrier(world)
    for evs in runs:
        one_step(evs)
    torch.cuda.synchronize()
    per_step = [sum(a.elapsed_time(b) for a, b in evs) for evs in runs]
    ms = allreduce(statistics.mean(per_step), "max", world)
    return {
        "workload": "config4: CombinedAttn (ToMe r=4000 per (b,h), 15% blocks of 128 on the merged "
                    "sequence, log-size bias, unmerge) in 30 layers, B=2, S=17776, H=30, D=64, bf16; "
                    "random-init 1920-wide projections outside the timed region",
        "ms_attention_per_step": round(ms, 3), "ms_per_layer": round(ms / layers, 4), "steps": n,
        "merged_len": int(attn._layers[0].merge_fn.plan.merged_len + T),
        "live_tflop_per_step": round(live / 1e12, 4),
        "effective_tflops": round(live / (ms * 1e-3) / 1e12, 1),
    }


def bench_long(args, dev, world, rank):
    """long video (25 x 30 x 45 + 226 text, S = 33976),
    B = 2, H = 30, D = 64, bf16, 10% of 128-blocks.  Every rank holds a
    sequence shard [B, S/N, H, D] of q / k / v; UlyssesAttention packs it,
    exchanges it with NCCL all-to-alls (heads split 4,4,4,4,4,4,3,3 at N = 8,
    sent in head chunks whose exchanges overlap the previous chunk's compute),
    selects blocks and runs the block-sparse kernel on its heads, and sends
    the output rows back.  Strong scaling: the layer is fixed, N GPUs share
    it."""
    import torch

    from sparseattnfunctions_b200 import kernels, workloads
    from sparseattnfunctions_b200.geometry import COGVIDEOX_2B_LONG as geo
    from sparseattnfunctions_b200.special_attentions.block_mask_attn import BlockSparseAttention
    from sparseattnfunctions_b200.ulysses import UlyssesAttention

    B, H, D, S = 2, 30, 64, geo.seq_len
    lens = [S // world + (1 if r < S % world else 0) for r in range(world)]
    at = sum(lens[:rank])
    full = workloads.video_qkv(geo, B=B, H=H, D=D, dtype=torch.bfloat16, seed=777)
    q, k, v = (t.transpose(1, 2)[:, at:at + lens[rank]].contiguous().to(dev) for t in full)
    del full
    inner = BlockSparseAttention(block_size=128, density=0.10, geometry=geo)
    live_acc, counting = [0.0], [True]

    def counted(qh, kh, vh, out=None):  # live FLOP of every head chunk (warm-up calls only)
        res = inner(qh, kh, vh, out=out)
        if counting[0]:
            live_acc[0] += float(inner.last_csr.live_flops(S, S, D))
        return res

    ua = UlyssesAttention(counted, heads=H, seq_lens=lens, chunks=args.ulysses_chunks)
    stream = torch.cuda.current_stream(dev)
    for _ in range(3):
        live_acc[0] = 0.0
        ua(q, k, v)
    torch.cuda.synchronize()
    h = ua.local_heads
    live = live_acc[0] if h > 0 else 0.0
    counting[0] = False
    live_total = allreduce(live, "sum", world)
    n = max(3, min(args.long_steps, args.steps))
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
    barrier(world)
    for e in evs:
        e[0].record(stream)
        ua(q, k, v)
        e[1].record(stream)
    torch.cuda.synchronize()
    ms = allreduce(statistics.mean(a.elapsed_time(b) for a, b in evs), "max", world)
    # the same attention on the rank's heads without the exchange
    grid = torch.empty(S, B, 3, max(h, 1), D, dtype=torch.bfloat16, device=dev)
    qh, kh, vh = (grid[:, :, t, :h].permute(1, 2, 0, 3) for t in range(3))
    aev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
    if h > 0:
        torch.manual_seed(5)
        grid.normal_()
        for _ in range(2):
            inner(qh, kh, vh)
        for e in aev:
            e[0].record(stream)
            inner(qh, kh, vh)
            e[1].record(stream)
        torch.cuda.synchronize()
        ms_attn_local = statistics.mean(a.elapsed_time(b) for a, b in aev)
    else:
        ms_attn_local = 0.0
    ms_attn = allreduce(ms_attn_local, "max", world)
    a2a_bytes = 2 * (B * lens[rank] * 3 * H * D + B * lens[rank] * H * D) * (world - 1) / max(world, 1)
    return {
        "workload": "config5: S=33976 (25x30x45 + 226 text), B=2, H=30, D=64, bf16, 10% of 128-blocks; "
                    f"sequence-sharded over {world} GPU(s), Ulysses all-to-all (NCCL) to "
                    f"{kernels.head_split(H, world)} head ranges and back, "
                    f"in {len(ua.plan) if world > 1 else 1} pipelined head chunk(s)",
        "ms_per_layer": round(ms, 4), "ms_attention_only": round(ms_attn, 4),
        "live_tflop": round(live_total / 1e12, 4),
        "effective_tflops": round(live_total / (ms * 1e-3) / 1e12, 1),
        "a2a_bytes_per_rank": int(a2a_bytes), "scaling": "strong", "steps": n,
    }


def run_reference(args, world, rank):
    """Reference arm: the reference's PyTorch masked path on the host CPU."""
    import torch

    if rank != 0:
        return None
    from oracle import selection as osel

    (q, k, v), cfg = c2_setup("cpu", 0)
    bs = cfg["block"]
    mask, _ = osel.select_blocks(q, k, bs, bs, cfg["topk"], cfg["text_blocks"], cfg["text_blocks"])
    mask = torch.from_numpy(mask)
    threads = os.cpu_count()
    torch.set_num_threads(threads)
    heads_per_step = max(1, args.ref_heads)
    vals = []
    t_all = 0.0
    for i in range(args.warmup + args.steps):
        g0 = (i * heads_per_step) % (cfg["B"] * cfg["H"])
        sub = [g0 + j for j in range(heads_per_step) if g0 + j < cfg["B"] * cfg["H"]]
        qs, ks, vs_ = q, k, v
        t0 = time.perf_counter()
        from oracle import attention as oatt
        oatt.masked_sdpa_cpu(qs, ks, vs_, mask, 1.0 / math.sqrt(cfg["D"]), bs, bs, q_chunk=2048,
                             heads=sub)
        dt = time.perf_counter() - t0
        rows = torch.full((mask.shape[2],), float(bs), dtype=torch.float64)
        rows[-1] = cfg["S"] - (mask.shape[2] - 1) * bs
        fl = sum(float(4.0 * cfg["D"] * torch.einsum("ij,i,j->", mask[g // cfg["H"], g % cfg["H"]].double(),
                                                     rows, rows)) for g in sub)
        if i >= args.warmup:
            vals.append(fl / dt / 1e12)
            t_all += dt
    value = statistics.median(vals)
    sample = f"{heads_per_step} of 60 (b,h) heads per step, query chunks of 2048, bf16 masked SDPA"
    return {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000 * t_all / max(1, args.steps), 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded smooth field + noise, CogVideoX-2B shapes)",
        "config": {"workload": "config2: CogVideoX-2B attention layer (reference masked path, CPU)",
                   "B": cfg["B"], "H": cfg["H"], "S": cfg["S"], "D": cfg["D"], "block": bs,
                   "density": cfg["density"], "topk": cfg["topk"]},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def _json_out():
    """The real stdout, kept for the one JSON line; file descriptor 1 is
    pointed at stderr so that anything native code prints there (NCCL's
    version banner, library messages) cannot mix into the result."""
    sys.stdout.flush()
    out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    return out


def main():
    out = _json_out()
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["saf", "reference"], default="saf")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--ref-heads", type=int, default=1, help="heads per step of the reference arm")
    ap.add_argument("--cpu-budget", type=float, default=12.0, help="seconds of CPU baseline work")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-merge", action="store_true", help="skip the config-3 ToMe sub-benchmark")
    ap.add_argument("--no-pool", action="store_true", help="skip the attention-with-pooling sub-benchmark")
    ap.add_argument("--merge-steps", type=int, default=20)
    ap.add_argument("--no-combined", action="store_true", help="skip the config-4 combined sub-benchmark")
    ap.add_argument("--combined-steps", type=int, default=2)
    ap.add_argument("--no-long", action="store_true", help="skip the config-5 sequence-sharded sub-benchmark")
    ap.add_argument("--long-steps", type=int, default=10)
    ap.add_argument("--ulysses-chunks", type=int, default=3,
                    help="head chunks of the config-5 exchange pipeline (1: one exchange each way)")
    ap.add_argument("--no-local-global", action="store_true", help="skip the LocalGlobalAttention sub-benchmark")
    ap.add_argument("--no-reference-kernel", action="store_true",
                    help="skip timing the reference's own Triton kernels (baseline/_ref) at N=1")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    world, rank, local = init_dist() if args.impl == "saf" else (
        int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0)
    if args.impl == "reference":
        line = run_reference(args, world, rank)
        if line is not None:
            print(json.dumps(line), file=out, flush=True)
        return

    line, qkv_cpu, csr, cfg = run_saf(args, world, rank, local)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        mask_cpu = csr.to_dense().cpu()
        val, heads, secs = cpu_masked_baseline(qkv_cpu, mask_cpu, cfg, budget_s=args.cpu_budget)
        import torch
        line["cpu_baseline"] = {"value": round(val, 5), "unit": UNIT, "cores": torch.get_num_threads(),
                                "kind": "port",
                                "sample": f"{heads} of 60 (b,h) heads of config 2 in {secs:.1f} s: "
                                          "query-chunked (2048) bf16 masked SDPA, same block mask"}
    if rank == 0:
        print(json.dumps(line), file=out, flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
