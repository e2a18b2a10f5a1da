#!/usr/bin/env python
"""Benchmark of the SeedVR2 windowed MM-attention path on B200.

One step = the attention stage of one DiT Euler step at 720p: 32 window-
attention layers (16 plain + 16 shifted windows; block parity as in the
reference's export) over the 6x45x80 = 21,600-token grid, 20 heads x 128,
58 text tokens. Each layer is the fused prologue (QK-RMSNorm + MM-RoPE, fp16
packing), the tcgen05 window-attention kernel and the text-mean kernel.

value     = algorithmic attention FLOPs of all ranks / max-over-ranks device
            time of the timed steps (CUDA events), inputs resident in HBM.
e2e       = same metric through the layer's host-buffer C-ABI call
            (s2_attention_layer_forward_host): pinned host QKV in, host
            outputs back, copies inside the timed region.
roofline  = the attention kernel alone: FLOPs per launch / mean launch time
            (events around each launch inside the timed region).
cpu_baseline / --impl reference: the reference's own CPU attention()
            (oracle/_ref, built from the reference sources) on a bounded
            sample of the same workload, on this host's cores.
euler_step: the second half of the metric -- one full DiT Euler step
            at 720p (33-channel 6x90x160 latent, 58 text
            tokens x 5120, 32 blocks of dim 2560 / 20 heads / SwiGLU 6912,
            random-init weights) through s2_dit_euler_step, replayed as a
            CUDA graph; device ms per step, the same through the host-buffer
            call (e2e), GEMM throughput, clocks. At N > 1 the ONE step is
            sharded by window over the ranks (strong scaling, max over ranks).
vae_attention (N = 1): the VAE mid-block attention layer at config 4
            (C 512, 6 frames of 90x160) through s2_vae_attention_forward.

config3 (all N): BASELINE config 3, the 1080p x 45f ragged stress test
            (12x67x120 = 96,480 tokens, 100 plain / 125 shifted windows):
            one plain and one shifted attention layer per step through the
            layer objects, sharded by window across the ranks at N > 1.
vae_layers (N = 1): the VAE's GroupNorm, space-time shuffle and 3x3x3
            Conv3D at the config-4 latent (512 channels, 6 x 90 x 160).

Multi-GPU (torchrun): ONE clip's windows are split across the ranks (LPT by
S_w^2, the north star's window sharding) and the text partial sums are
all-reduced over NCCL after every layer: strong scaling of the headline
stage, the config-3 stage and the Euler step. --weak instead gives each rank
its own clip (weak scaling, no data-path collective).
"""
from __future__ import annotations

import argparse
import contextlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "seedvr2-ncnn-valkan_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

METRIC = "window-attn TFLOP/s (% tcgen05 peak); DiT Euler-step ms at 1/2/4/8 B200 vs CPU ref"
UNIT = "TFLOP/s"
FALLBACK_PEAKS = {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


def profile_traffic(name):
    """DRAM bytes per launch recorded in a committed ncu summary (profiles/)."""
    p = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("dram_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


@contextlib.contextmanager
def nvtx_range(torch, name):
    """An NVTX push/pop range around a warm-up phase, so that a profiler can
    select it (`ncu --nvtx --nvtx-include "<name>/"`)."""
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def preroll_steps(step_ms, dist, dev, target_ms=400.0):
    """Untimed steps of the same work run inside the clock sampler before the
    timed region, so that a short timed region still has clock samples taken
    under load; the same count on every rank (the steps hold collectives)."""
    import torch
    n = torch.tensor([float(max(1, int(np.ceil(target_ms / max(step_ms, 1e-3)))))], dtype=torch.float64,
                     device=dev)
    if dist:
        dist.all_reduce(n, op=dist.ReduceOp.MAX)
    return int(min(n.item(), 1000))


class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev = self._physical(device_index)
        self.proc = None
        self.lines = []

    @staticmethod
    def _physical(index):
        """nvidia-smi ignores CUDA_VISIBLE_DEVICES: map the process's device
        index to the physical index (or UUID) it names."""
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "").strip()
        if vis:
            ids = [v.strip() for v in vis.split(",") if v.strip()]
            if 0 <= index < len(ids):
                return ids[index]
        return str(index)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.dev)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            # nvidia-smi takes a moment to start: wait for its first sample so a
            # short timed region is still sampled
            t0 = time.time()
            while not self.lines and self.proc.poll() is None and time.time() - t0 < 5.0:
                time.sleep(0.02)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        # the first sample is taken before the work starts (the sampler waits for it)
        for ln in self.lines[1:]:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------- CPU reference


def cpu_reference_sample(grid, text_len, heads_total, seed=666):
    """Times the reference's own attention() (oracle/_ref) on one head per host
    core (at most all heads) of the plain 720p layer. Returns a dict."""
    import oracle
    from s2b200 import synth
    ref = oracle.ref()
    kind = "reference"
    if ref is None:
        ref, kind = oracle.port(), "port"
    cores = os.cpu_count() or 1
    heads = max(1, min(heads_total, cores))
    vid, txt, gam, fr = synth.layer_inputs(grid, heads=heads_total, text_len=text_len, seed=seed)
    wins = ref.make_windows(*grid, 0)
    flops = synth.attention_flops(wins, text_len, heads)
    t0 = time.perf_counter()
    if kind == "reference":
        ref.attention(vid, txt, grid, heads_total, list(gam), fr, 0, head_count=heads, threads=heads)
    else:
        ref.window_attention(vid, txt, grid, heads_total, list(gam), fr, 0, heads_range=(0, heads), threads=heads)
    dt = time.perf_counter() - t0
    return {"value": flops / dt / 1e12, "unit": UNIT, "cores": heads, "kind": kind, "seconds": dt,
            "sample": f"plain-window layer of the {grid[0]}x{grid[1]}x{grid[2]} grid, heads 0..{heads - 1} of "
                      f"{heads_total} (one head per thread, {heads} threads of {cores} host cores), "
                      f"{flops / 1e9:.1f} GFLOP algorithmic"}


def cpu_euler_estimate(seed=666):
    """The reference's own CPU code for the config-2 Euler step, estimated from
    two timed blocks: oracle/_ref's SeedVR2DiTBlock::forward (the reference's
    source compiled against the ncnn shim, whose InnerProduct is this
    repository's fp32 GEMM, not ncnn's) for one plain and one shifted block on
    all host cores, times 16 each (the step's 16 plain + 16 shifted blocks; the
    DiT heads are < 1 % and left out). The reference's attention() alone on
    the same two layers is timed beside it, so that the part of the estimate
    that is the reference's own arithmetic is stated separately."""
    import oracle
    from s2b200 import synth
    ref = oracle.ref()
    if ref is None:
        return {"unavailable": "oracle/_ref (the reference build) is not present"}
    grid, dim, heads, mlp = synth.GRIDS["cfg2"], 2560, 20, 6912
    cores = os.cpu_count() or 1
    vid, txt, emb = synth.block_activations(grid, dim, seed=seed)
    qv, qt, gam, fr = synth.layer_inputs(grid, heads=heads, seed=seed)
    out = {"cores": cores, "kind": "reference", "extrapolated": True}
    for name, idx, shifted in (("plain", 0, 0), ("shifted", 1, 1)):
        w = synth.block_weights(dim, heads, mlp, shared=False, seed=100 + idx)
        params = dict(block_index=idx, shared=False, last=False, shifted=bool(shifted), dim=dim, heads=heads,
                      head_dim=128, mlp_hidden=mlp, eps=1e-5)
        t0 = time.perf_counter()
        ref.block_forward(params, w, vid, txt, emb, grid, threads=cores)
        out[f"block_{name}_s"] = time.perf_counter() - t0
        del w
        t0 = time.perf_counter()
        ref.attention(qv, qt, grid, heads, list(gam), fr, shifted, threads=cores)
        out[f"attention_{name}_s"] = time.perf_counter() - t0
    out["ms_per_step"] = 16e3 * (out["block_plain_s"] + out["block_shifted_s"])
    out["attention_ms_per_step"] = 16e3 * (out["attention_plain_s"] + out["attention_shifted_s"])
    out["sample"] = ("blocks 0 (plain) and 1 (shifted) of the config-2 step through the reference's block code, "
                     f"{cores} threads; step = 16 x (plain + shifted)")
    return out


def run_reference_arm(args, rank):
    if rank != 0:
        return
    from s2b200 import synth
    grid = synth.GRIDS["cfg2"]
    vals = []
    last = None
    for i in range(args.warmup + args.steps):
        r = cpu_reference_sample(grid, 58, 20)
        if i >= args.warmup:
            vals.append(r["value"])
        last = r
    v = float(statistics.mean(vals)) if vals else last["value"]
    secs = last["seconds"]
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": secs * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32/f64 (reference CPU)", "data": "synthetic",
            "config": workload_config(args),
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": last["cores"], "kind": last["kind"],
                             "sample": last["sample"]},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------- GPU arm


def workload_config(args):
    return {"workload": "720p DiT-step attention stage: 32 MM window-attention layers (16 plain + 16 shifted), "
                        "token grid 6x45x80 = 21,600, 20 heads x 128, 58 text tokens, reference window rule "
                        "(2x15x27: 27 plain / 64 shifted windows)" if not args.override else
                        "720p DiT-step attention stage with BASELINE.json's 6x15x20 window override",
            "layers_per_step": 32, "grid": [6, 45, 80], "heads": 20, "head_dim": 128, "text_len": 58,
            "mode": args.mode, "io": "fp16 QKV in, fp16 out" if args.mode == "f16" else "fp16 QKV in, bf16 out",
            "l2": "no flush: every layer reads a distinct >L2 input (332 MB QKV, 356 MB packed Q/K/V)",
            "sharding": "window-sharded single clip + per-layer NCCL text all-reduce, overlapped with the next "
                        "layer (strong)" if args.shard else
                        "one clip per rank (weak)"}


def run_ours(args, rank, world, local_rank):
    import torch

    import s2b200
    from s2b200 import synth

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    rc = s2b200.device_check(local_rank)
    if rc != 0:
        raise RuntimeError(s2b200.last_error())
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)

    grid = synth.GRIDS["cfg2"]
    T, H, W = grid
    heads, Lt, dim = 20, 58, 2560
    mode = s2b200.MODE_F16 if args.mode == "f16" else s2b200.MODE_BF16_REF
    override = synth.OVERRIDES["cfg2"] if args.override else (0, 0, 0)
    stream = torch.cuda.current_stream()

    # plans: plain (shifted=0) and shifted layers
    plans = []
    for shifted in (0, 1):
        wins = s2b200.make_windows(T, H, W, shifted, override)
        ids = np.arange(len(wins))
        if args.shard and world > 1:
            ids = s2b200.shard_windows(wins, Lt, world)[rank]
        local = wins[ids]
        cu, rows = s2b200.build_varlen(T, H, W, local, Lt)
        work = s2b200.plan_work(cu)
        max_pos = int(rows[:, 1:].max()) + 1
        plans.append(dict(
            shifted=shifted, n_total=len(wins), n_local=len(local), flops=synth.attention_flops(local, Lt, heads),
            cu=torch.from_numpy(cu).to(dev), rows=torch.from_numpy(rows.copy()).to(dev),
            work=torch.from_numpy(work).to(dev), n_rows=rows.shape[0], max_pos=max_pos))

    vid_np, txt_np, gam, fr = synth.layer_inputs(grid, heads=heads, text_len=Lt, seed=666 + rank)
    gam_d = torch.from_numpy(gam).to(dev)
    fr_d = torch.from_numpy(fr).to(dev)
    for p in plans:
        p["tab"] = s2b200.rope_table(fr_d, p["max_pos"])
    # 4 distinct QKV inputs (2 per layer kind), each 332 MB fp16 > L2
    base_v = torch.from_numpy(vid_np).to(dev, torch.float16)
    base_t = torch.from_numpy(txt_np).to(dev, torch.float16)
    inputs = []
    for i in range(4):
        g = torch.Generator(device=dev).manual_seed(1000 * rank + i)
        noise = (torch.randn(base_v.shape, device=dev, generator=g, dtype=torch.float32) * 0.01).to(torch.float16)
        inputs.append((base_v + noise, base_t.clone()))
    del base_v
    out_dtype = s2b200.mode_dtype(mode)
    n_rows_max = max(p["n_rows"] for p in plans)
    ws = [torch.empty((heads, n_rows_max, 128), dtype=torch.float16, device=dev) for _ in range(3)]
    vid_out = torch.zeros((T * H * W, dim), dtype=out_dtype, device=dev)
    txt_part = torch.empty((max(p["n_local"] for p in plans), Lt, dim), dtype=out_dtype, device=dev)
    # one text output per layer of a step: a sharded layer's all-reduce of its text mean runs
    # asynchronously (NCCL's stream) while the next, independent layer computes; a step ends
    # once all of its all-reduces completed (inside the timed region)
    txt_outs = [torch.empty((Lt, dim), dtype=torch.float32, device=dev) for _ in range(32)]
    pending = []
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    lib = s2b200.lib()
    sp = s2b200._stream_ptr(stream)
    vp = lambda t: s2b200._ptr(t)  # noqa: E731

    def layer(i, ev=None):
        p = plans[i % 2]
        v_in, t_in = inputs[i % 4]
        # packed [heads, n_rows, 128] operands: leading slices of the flat workspaces
        qf, kf, vf = (w.view(-1)[: heads * p["n_rows"] * 128] for w in ws)
        if ev:
            ev[0].record(stream)
        rc = lib.s2_qk_norm_rope(sp, vp(v_in), vp(t_in), s2b200.S2_F16, heads, 1e-5, vp(gam_d), vp(p["tab"]),
                                 vp(p["rows"]), p["n_rows"], mode, vp(qf), vp(kf), vp(vf))
        if rc:
            raise RuntimeError(s2b200.last_error())
        if ev:
            ev[1].record(stream)
        rc = lib.s2_window_attention(sp, mode, vp(qf), vp(kf), vp(vf), heads, p["n_rows"], vp(p["cu"]),
                                     p["n_local"], Lt, vp(p["rows"]), vp(p["work"]), p["work"].shape[0],
                                     vp(vid_out), vp(txt_part), vp(err))
        if rc:
            raise RuntimeError(s2b200.last_error())
        if ev:
            ev[2].record(stream)
        rc = lib.s2_text_window_sum(sp, mode, vp(txt_part), p["n_local"], Lt, dim, 1.0 / p["n_total"], 0,
                                    vp(txt_outs[i]))
        if rc:
            raise RuntimeError(s2b200.last_error())
        if ev:
            ev[3].record(stream)
        if args.shard and world > 1:
            pending.append(dist.all_reduce(txt_outs[i], async_op=True))

    def end_step():
        while pending:
            pending.pop().wait()  # the current stream waits for the collective

    layers_per_step = 32
    t_w = time.time()
    with nvtx_range(torch, "attention_stage"):
        for _ in range(args.warmup):
            for i in range(layers_per_step):
                layer(i)
            end_step()
    torch.cuda.synchronize()
    n_pre = preroll_steps((time.time() - t_w) * 1e3 / max(1, args.warmup), dist, dev)
    if int(err.item()) != 0:
        raise RuntimeError(f"attention kernel device error {int(err.item())}")

    n_ev = layers_per_step * args.steps
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(n_ev)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        for _ in range(n_pre):
            for i in range(layers_per_step):
                layer(i)
            end_step()
        start.record(stream)
        for s in range(args.steps):
            for i in range(layers_per_step):
                layer(i, evs[s * layers_per_step + i])
            end_step()
        end.record(stream)
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    ms = start.elapsed_time(end)
    if int(err.item()) != 0:
        raise RuntimeError(f"attention kernel device error {int(err.item())}")
    t_pro = np.array([e[0].elapsed_time(e[1]) for e in evs])
    t_att = np.array([e[1].elapsed_time(e[2]) for e in evs])
    t_txt = np.array([e[2].elapsed_time(e[3]) for e in evs])
    ms_t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())

    step_flops_local = 16 * (plans[0]["flops"] + plans[1]["flops"])
    tot = torch.tensor([step_flops_local], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(tot)
    step_flops_all = float(tot.item())
    ms_per_step = ms / args.steps
    value = step_flops_all / (ms_per_step * 1e-3) / 1e12

    # roofline of the attention kernel (per-launch mean, both layer kinds)
    att_plain = float(np.mean(t_att[0::2]))
    att_shift = float(np.mean(t_att[1::2]))
    flops_launch = (plans[0]["flops"] + plans[1]["flops"]) / 2
    att_ms = (att_plain + att_shift) / 2
    achieved = flops_launch / (att_ms * 1e-3) / 1e12
    peaks, peak_src = load_peaks()
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    traffic = profile_traffic("window_attention_cfg2.md")
    # the prologue's own rows: this rank's video rows (all L at N = 1) and the text rows
    vid_local = sum(p["n_rows"] - p["n_local"] * Lt for p in plans) / 2
    pro_bytes = synth.prologue_bytes(vid_local, Lt, heads, 2)
    pro_moved = synth.prologue_bytes_moved(vid_local, Lt, (plans[0]["n_rows"] + plans[1]["n_rows"]) / 2, heads, 2)
    pro_gbs = pro_bytes / (float(np.mean(t_pro)) * 1e-3) / 1e9
    hbm_peak = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))

    # end-to-end through the host-buffer C-ABI call (layer objects, pinned host memory)
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, torch, s2b200, synth, dev, rank, world, grid, heads, Lt, gam, fr, mode, override,
                      step_flops_all, dist)

    extra = {}
    if not args.no_cfg3:
        extra["config3"] = run_cfg3(args, torch, s2b200, synth, dev, rank, world, dist)
    if not args.no_euler:
        extra["euler_step"] = run_euler(args, torch, s2b200, synth, dev, rank, world, dist)
    if world == 1 and not args.no_vae:
        extra["vae_attention"] = run_vae(args, torch, s2b200, synth, dev)
        extra["vae_layers"] = run_vae_layers(args, torch, s2b200, synth, dev)

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
                "scaling": "strong" if args.shard and world > 1 else "weak", "vs_baseline": None,
                "dtype": "f16" if args.mode == "f16" else "f16 (bf16 out)", "data": "synthetic",
                "config": workload_config(args),
                "pct_of_peak": 100.0 * value / world / peak,
                "gpu_launches": 3 * layers_per_step * args.steps,
                "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                             "frac": achieved / peak, "traffic": traffic,
                             "peak_source": f"{peak_src} bf16 dense (burst)",
                             "kernel": "window_attention_kernel", "flops_per_launch": flops_launch,
                             "ms_per_launch": {"plain": att_plain, "shifted": att_shift}},
                "kernels": {"prologue_ms": float(np.mean(t_pro)), "attention_ms": att_ms,
                            "text_sum_ms": float(np.mean(t_txt)), "prologue_gbs": pro_gbs,
                            "prologue_hbm_frac": pro_gbs / hbm_peak,
                            "prologue_moved_gbs": pro_moved / (float(np.mean(t_pro)) * 1e-3) / 1e9},
                "clocks": clk.summary()}
        if e2e:
            line["e2e"] = e2e
        line.update(extra)
        if world == 1 and not args.no_cpu_baseline:
            cb = cpu_reference_sample(grid, Lt, heads)
            line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def run_e2e(args, torch, s2b200, synth, dev, rank, world, grid, heads, Lt, gam, fr, mode, override, step_flops_all,
            dist):
    T, H, W = grid
    L, dim = T * H * W, heads * 128
    stream = torch.cuda.current_stream()
    layers = []
    for shifted in (0, 1):
        lay = s2b200.SeedVR2DiTBlockAttention(device=dev.index, mode=mode, window_override=override)
        lay.load_param(shifted=shifted, dim=dim, heads=heads)
        lay.load_model(gam[0], gam[1], fr, gam[2], gam[3])
        if args.shard and world > 1:
            lay.set_window_subset(s2b200.shard_windows(s2b200.make_windows(T, H, W, shifted, override), Lt, world)[rank])
        layers.append(lay)
    vid_np, txt_np, _, _ = synth.layer_inputs(grid, heads=heads, text_len=Lt, seed=666 + rank)
    hv = torch.from_numpy(vid_np.astype(np.float16)).pin_memory().numpy()
    ht = torch.from_numpy(txt_np.astype(np.float16)).pin_memory().numpy()
    out_np = np.float16 if mode == s2b200.MODE_F16 else np.uint16
    io = s2b200.S2_F16 if mode == s2b200.MODE_F16 else s2b200.S2_F32
    if io == s2b200.S2_F32:
        hv = torch.from_numpy(vid_np).pin_memory().numpy()
        ht = torch.from_numpy(txt_np).pin_memory().numpy()
        out_np = np.float32
    ov = torch.empty((L, dim), dtype={np.float16: torch.float16, np.float32: torch.float32}[out_np]).pin_memory().numpy()
    ot = torch.empty((Lt, dim), dtype=torch.float32).pin_memory().numpy()
    shape = np.array(grid, np.int32)
    layers_per_step = 32
    steps = max(1, min(args.steps, args.e2e_steps))
    for i in range(2):
        layers[i % 2].forward_host(hv, ht, shape, io, ov, ot, stream=stream)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(steps):
        for i in range(layers_per_step):
            layers[i % 2].forward_host(hv, ht, shape, io, ov, ot, stream=stream)
    end.record(stream)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    ms_t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_step = float(ms_t.item()) / steps
    h2d = layers_per_step * (hv.nbytes + ht.nbytes)
    d2h = layers_per_step * (ov.nbytes + ot.nbytes)
    for lay in layers:
        lay.close()
    return {"value": step_flops_all / (ms_step * 1e-3) / 1e12, "unit": UNIT, "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h), "ms_per_step": ms_step, "steps": steps,
            "path": "s2_attention_layer_forward_host (pinned host buffers)"}


def run_euler(args, torch, s2b200, synth, dev, rank, world, dist):
    """One DiT Euler step at 720p (config 2): on this GPU (N = 1), or sharded by
    window over all ranks (N > 1: strong scaling, one step split across GPUs).
    Returns a dict (on every rank; rank 0 prints it)."""
    t0 = time.perf_counter()
    m = s2b200.SeedVR2DiT(device=dev.index)
    m.load_input(synth.dit_input_weights(2560))
    m.load_output(synth.dit_output_weights(2560))
    for i in range(32):
        m.load_block(i, synth.block_weights_device(2560, 20, 6912, s2b200.block_flags(i)["shared"], seed=100 + i,
                                                   device=dev))
    comm = None
    if world > 1:
        comm = s2b200.Comm.create(dev.index, rank, world)
        m.set_comm(comm)
    load_s = time.perf_counter() - t0
    noise, cond, text = synth.dit_latents(synth.DIT_CFG2_LATENT)
    n, c, t = (torch.from_numpy(a).to(dev) for a in (noise, cond, text))
    x0 = torch.empty_like(n)
    stream = torch.cuda.current_stream()
    with nvtx_range(torch, "euler_step_eager"):  # the first call runs eagerly (one launch per kernel)
        m.euler_step(n, c, t, 1000.0, x0, stream=stream)
    for _ in range(max(3, args.warmup) - 1):  # capture, replays
        m.euler_step(n, c, t, 1000.0, x0, stream=stream)
    torch.cuda.synchronize()
    t_w = time.time()
    m.euler_step(n, c, t, 1000.0, x0, stream=stream)
    torch.cuda.synchronize()
    n_pre = preroll_steps((time.time() - t_w) * 1e3, dist, dev)
    if m.device_error() != 0:
        raise RuntimeError("DiT device error")
    steps = max(1, args.euler_steps)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(dev.index) as clk:
        for _ in range(n_pre):
            m.euler_step(n, c, t, 1000.0, x0, stream=stream)
        ev[0].record(stream)
        for i in range(steps):
            m.euler_step(n, c, t, 1000.0, x0, stream=stream)
            ev[i + 1].record(stream)
        torch.cuda.synchronize()
    per = [ev[i].elapsed_time(ev[i + 1]) for i in range(steps)]
    ms = float(np.mean(per))
    if dist:
        ms_t = torch.tensor([ms, float(min(per))], dtype=torch.float64, device=dev)
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
        ms = float(ms_t[0].item())
        per = [float(ms_t[1].item())]
    ok = bool(torch.isfinite(x0).all().item())
    L = 6 * 45 * 80
    gemm = sum(synth.block_gemm_flops(L, 58, 2560, 6912, last=(i == 31)) for i in range(32))
    att = 16 * sum(synth.attention_flops(s2b200.make_windows(6, 45, 80, sh), 58, 20) for sh in (0, 1))
    # end to end: pinned host noise / condition / text in, x0 out, copies inside the timed region
    hn, hc, ht = (torch.from_numpy(a).pin_memory().numpy() for a in (noise, cond, text))
    hx = torch.empty(noise.shape, dtype=torch.float32).pin_memory().numpy()
    m.euler_step_host(hn, hc, ht, 1000.0, hx, stream=stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = max(1, min(steps, args.e2e_steps))
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(e2e_steps):
        m.euler_step_host(hn, hc, ht, 1000.0, hx, stream=stream)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    if dist:
        e_t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(e_t, op=dist.ReduceOp.MAX)
        e2e_ms = float(e_t.item())
    launches = m.last_launches()
    m.close()
    if comm is not None:
        comm.close()
    cpu_ref = cpu_euler_estimate() if (args.cpu_euler and rank == 0 and world == 1) else None
    return {"workload": "DiT Euler step at 720p: latent 33x6x90x160 -> 21,600 tokens, 58 text tokens x 5120, "
                        "32 blocks (dim 2560, 20 heads, SwiGLU 6912), t = 1000, one step, cfg 1",
            "ms_per_step": ms, "ms_min": float(min(per)), "steps": steps, "higher_is_better": False,
            "gemm_tflop_per_step": gemm / 1e12, "attention_tflop_per_step": att / 1e12,
            "tflops_overall": (gemm + att) / (ms * 1e-3) / 1e12, "gpu_launches_per_step": launches,
            "cuda_graph": True, "n_gpus": world,
            "sharding": "one step split by window across the GPUs (NCCL text all-reduce per block; the row "
                        "exchange at every plain/shifted boundary stored by the MLP output GEMM into the next "
                        "owner's buffer over NVLink), strong scaling" if world > 1 else "one GPU",
            "finite": ok, "weights_load_s": load_s,
            "e2e": {"ms_per_step": e2e_ms, "unit": "ms", "steps": e2e_steps,
                    "h2d_bytes_per_step": int(hn.nbytes + hc.nbytes + ht.nbytes),
                    "d2h_bytes_per_step": int(hx.nbytes), "path": "s2_dit_euler_step_host (pinned host buffers)"},
            "clocks": clk.summary(), **({"cpu_reference": cpu_ref} if cpu_ref else {})}


def run_cfg3(args, torch, s2b200, synth, dev, rank, world, dist):
    """the 1080p x 45f ragged shifted-window stress test, one
    plain and one shifted attention layer per step (prologue, attention, text
    mean through s2_attention_layer_forward), fp16 QKV in, fp16 out. At N > 1
    each layer's windows are split across the ranks by LPT on S_w^2 and the
    text partial sums are all-reduced (strong scaling); value = all ranks'
    algorithmic FLOPs / max-over-ranks device time."""
    grid = synth.GRIDS["cfg3"]
    T, H, W = grid
    heads, Lt, dim = 20, 58, 2560
    mode = s2b200.MODE_F16 if args.mode == "f16" else s2b200.MODE_BF16_REF
    vid, txt, gam, fr = synth.layer_inputs(grid, heads=heads, text_len=Lt, seed=77)
    v = torch.from_numpy(vid).to(dev, torch.float16)
    t = torch.from_numpy(txt).to(dev, torch.float16)
    del vid
    layers, flops = [], 0.0
    for shifted in (0, 1):
        wins = s2b200.make_windows(T, H, W, shifted)
        lay = s2b200.SeedVR2DiTBlockAttention(device=dev.index, mode=mode)
        lay.load_param(shifted=shifted, dim=dim, heads=heads)
        lay.load_model(gam[0], gam[1], fr, gam[2], gam[3])
        lay.set_runtime_shape(T, H, W)
        ids = np.arange(len(wins))
        if world > 1:
            ids = s2b200.shard_windows(wins, Lt, world)[rank]
            lay.set_window_subset(ids)
        flops += synth.attention_flops(wins[ids], Lt, heads)
        layers.append(lay)
    vo = torch.zeros((T * H * W, dim), dtype=s2b200.mode_dtype(mode), device=dev)
    tos = [torch.empty((Lt, dim), dtype=torch.float32, device=dev) for _ in layers]
    stream = torch.cuda.current_stream()

    def step():
        # each layer's text all-reduce overlaps the next, independent layer; the step ends
        # once both completed
        pending = []
        for lay, to in zip(layers, tos):
            lay.forward(v, t, vo, to, stream=stream)
            if dist:
                pending.append(dist.all_reduce(to, async_op=True))
        for h in pending:
            h.wait()

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    steps = max(1, args.cfg3_steps)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(dev.index) as clk:
        for _ in range(2):
            step()
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    for lay in layers:
        if lay.device_error() != 0:
            raise RuntimeError("config-3 attention device error")
    tot = torch.tensor([ms, flops], dtype=torch.float64, device=dev)
    if dist:
        ms_t = tot[:1].clone()
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
        fl = tot[1:].clone()
        dist.all_reduce(fl)
        ms, flops = float(ms_t.item()), float(fl.item())
    for lay in layers:
        lay.close()
    return {"workload": "config 3: 1080p x 45f, grid 12x67x120 = 96,480 tokens, 20 heads x 128, 58 text tokens, "
                        "reference windows 3x15x27 (100 plain / 125 shifted); one plain + one shifted layer per step",
            "value": flops / (ms * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": ms, "steps": steps,
            "tflop_per_step": flops / 1e12, "n_gpus": world,
            "scaling": "strong (windows split across ranks, NCCL text all-reduce overlapped with the next layer)"
            if world > 1 else "one GPU",
            "gpu_launches_per_step": 6, "clocks": clk.summary()}


def run_vae_layers(args, torch, s2b200, synth, dev):
    """The VAE's GroupNorm, space-time shuffle (512 -> 4096 channels, temporal
    ratio 2) and 3x3x3 Conv3D (512 -> 512, causal: two replicated leading
    frames) at the config-4 latent, 512 x 6 x 90 x 160; device ms per forward,
    achieved HBM bandwidth (GroupNorm: read x once, write y once) and tensor
    throughput (2 x MACs)."""
    C, T, H, W = synth.VAE_CFG4
    rng = np.random.default_rng(3)
    x = torch.randn((C, T, H, W), device=dev)
    stream = torch.cuda.current_stream()
    peaks, _ = load_peaks()
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    steps = max(1, args.vae_steps)

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    out = {}
    gn = s2b200.DynamicFramewiseGroupNorm(device=dev.index)
    gn.load_param(C)
    gn.load_model(rng.standard_normal(C).astype(np.float32) * 0.1, 1 + 0.1 * rng.standard_normal(C).astype(np.float32))
    y = torch.empty_like(x)
    ms = timed(lambda: gn.forward(x, y, stream=stream))
    algo = 2 * x.numel() * 4
    out["group_norm"] = {"ms": ms, "gbs": algo / (ms * 1e-3) / 1e9, "hbm_frac": algo / (ms * 1e-3) / 1e9 / hbm,
                         "algorithmic_bytes": algo, "launches": gn.last_launches()}
    gn.close()
    del y
    P = C * 8
    st = s2b200.DynamicSpaceTimeShuffle(device=dev.index)
    st.load_param(C, P)
    st.load_model(rng.standard_normal(P).astype(np.float32) * 0.02,
                  (rng.standard_normal((P, C)) / np.sqrt(C)).astype(np.float32))
    ys = torch.empty((C, 2 * T - 1, 2 * H, 2 * W), device=dev)
    ms = timed(lambda: st.forward(x, ys, stream=stream))
    fl = 2.0 * T * H * W * P * C
    algo = x.numel() * 4 + ys.numel() * 4
    out["space_time_shuffle"] = {"ms": ms, "tflops": fl / (ms * 1e-3) / 1e12, "gbs": algo / (ms * 1e-3) / 1e9,
                                 "hbm_frac": algo / (ms * 1e-3) / 1e9 / hbm, "launches": st.last_launches(),
                                 "shape": f"{C} x {T}x{H}x{W} -> {C} x {2 * T - 1}x{2 * H}x{2 * W}"}
    if st.device_error() != 0:
        raise RuntimeError("space-time shuffle device error")
    st.close()
    del ys
    cv = s2b200.Convolution3D(device=dev.index)
    cv.load_param(C, C, kernel=(3, 3, 3), pad=(0, 1, 1, 0, 1, 1))
    cv.load_model((rng.standard_normal((C, C, 3, 3, 3)) / np.sqrt(27 * C)).astype(np.float32),
                  rng.standard_normal(C).astype(np.float32) * 0.02)
    xc = torch.randn((C, T + 2, H, W), device=dev)
    yc = torch.empty((C, T, H, W), device=dev)
    ms = timed(lambda: cv.forward(xc, yc, stream=stream))
    fl = 2.0 * T * H * W * C * C * 27
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    out["conv3d"] = {"ms": ms, "tflops": fl / (ms * 1e-3) / 1e12, "frac_of_peak": fl / (ms * 1e-3) / 1e12 / peak,
                     "tflop": fl / 1e12, "launches": cv.last_launches(),
                     "shape": f"{C} -> {C}, 3x3x3, input {T + 2}x{H}x{W} (causal pad), output {T}x{H}x{W}"}
    if cv.device_error() != 0:
        raise RuntimeError("conv3d device error")
    cv.close()
    out["workload"] = "VAE layers at the config-4 latent: 512 channels x 6 frames x 90 x 160"
    return out


def run_vae(args, torch, s2b200, synth, dev):
    """VAE mid-block attention (config 4) on this GPU; returns a dict."""
    shape = synth.VAE_CFG4
    x, w = synth.vae_inputs(shape)
    lay = s2b200.DynamicFramewiseSpatialAttention(device=dev.index)
    lay.load_param(shape[0])
    lay.load_model(w)
    xd = torch.from_numpy(x).to(dev)
    y = torch.empty_like(xd)
    stream = torch.cuda.current_stream()
    t_w = time.time()
    for _ in range(max(3, args.warmup)):
        lay.forward(xd, y, stream=stream)
    torch.cuda.synchronize()
    n_pre = preroll_steps((time.time() - t_w) * 1e3 / max(3, args.warmup), None, dev)
    steps = max(1, args.vae_steps)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clk:
        for _ in range(n_pre):
            lay.forward(xd, y, stream=stream)
        e0.record(stream)
        for _ in range(steps):
            lay.forward(xd, y, stream=stream)
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    if lay.device_error() != 0:
        raise RuntimeError("VAE attention device error")
    # the attention core alone (the same kernel as in the layer), on the layer's own operands
    C, T, H, W = shape
    N = H * W
    q, k, v, o = (torch.randn((T * N, 512), device=dev).half() for _ in range(4))
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    for _ in range(2):
        s2b200.spatial_attention(q, k, v, C, T, N, o, err, stream=stream)
    e0.record(stream)
    for _ in range(steps):
        s2b200.spatial_attention(q, k, v, C, T, N, o, err, stream=stream)
    e1.record(stream)
    torch.cuda.synchronize()
    core_ms = e0.elapsed_time(e1) / steps
    af = synth.vae_attention_flops(shape)
    hx = torch.from_numpy(x).pin_memory().numpy()
    hy = torch.empty(x.shape, dtype=torch.float32).pin_memory().numpy()
    lay.forward_host(hx, y=hy)
    t0 = time.perf_counter()
    lay.forward_host(hx, y=hy)
    e2e_ms = (time.perf_counter() - t0) * 1e3
    lay.close()
    return {"workload": "VAE mid-block attention, C 512, 6 frames x 90x160 = 14,400 tokens per frame",
            "ms_per_forward": ms, "attention_core_ms": core_ms,
            "attention_tflops": af / (core_ms * 1e-3) / 1e12, "attention_tflop": af / 1e12,
            "projection_tflop": synth.vae_projection_flops(shape) / 1e12, "gpu_launches_per_forward": 5,
            "e2e_ms": e2e_ms, "clocks": clk.summary()}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--mode", choices=["f16", "bf16"], default="f16")
    ap.add_argument("--override", action="store_true", help="BASELINE.json's 6x15x20 windows")
    ap.add_argument("--shard", action="store_true",
                    help="split one clip's windows across ranks (the default when N > 1)")
    ap.add_argument("--weak", action="store_true", help="N > 1: one clip per rank instead (weak scaling)")
    ap.add_argument("--no-cfg3", action="store_true", help="skip the config-3 (1080p) stage")
    ap.add_argument("--cfg3-steps", type=int, default=5)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-euler", action="store_true", help="skip the DiT Euler-step measurement")
    ap.add_argument("--euler-steps", type=int, default=5)
    ap.add_argument("--cpu-euler", action="store_true",
                    help="also time the reference's CPU block code on the Euler-step shape (about 3 min, N = 1)")
    ap.add_argument("--no-vae", action="store_true", help="skip the VAE attention measurement")
    ap.add_argument("--vae-steps", type=int, default=5)
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not args.weak:
        args.shard = True
    if args.weak:
        args.shard = False
    if args.impl == "reference":
        run_reference_arm(args, rank)
        return
    run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
