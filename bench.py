#!/usr/bin/env python3
"""Benchmark: DiT ODE-step evals/s of the B200 engine (or of the reference CPU path).

Workload (default): one Euler flow-matching solve per utterance for one latent
patch -- 10 steps of the 18-layer DiT velocity forward with classifier-free
guidance (cond + uncond rows in one launch), CFG scale 2.0 (v4 form),
64 utterances (128 CFG rows) per GPU, L = 64 tokens per row (60 FM-history
tokens in the v4 layout with its attention mask and position ids, plus 4 noise
frames), speaker x-vectors, bf16 weights with fp32 accumulation, the whole
solve captured in one CUDA graph.  Weights are random-init N(0, 0.02) (seed 1)
in the real architecture; inputs are seeded synthetic tensors of the real
shapes.  One "eval" = one CFG-pair velocity evaluation, so a solve is
n_utt * nfe evals.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs one process per GPU under torch.distributed.run (launched here if
not already); every rank solves its own shard of utterances (weak scaling, no
collective on the data path); times are CUDA-event device times, max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(HERE, "dots.tts.cpp_b200")
sys.path.insert(0, PKG)

METRIC = "DiT ODE-step evals/sec"
UNIT = "evals/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--n-utt", type=int, default=64, help="utterances per GPU")
    ap.add_argument("--fm-len", type=int, default=60, help="FM history tokens (L = fm_len + patch)")
    ap.add_argument("--patch", type=int, default=4)
    ap.add_argument("--nfe", type=int, default=10)
    ap.add_argument("--layers", type=int, default=18)
    ap.add_argument("--dtype", choices=["both", "bf16", "fp8"], default="both",
                    help="block projection weights: bf16, e4m3 with per-channel scales, or both "
                         "(bf16 is the headline line, the e4m3 run is added under the key fp8)")
    ap.add_argument("--cfg-scale", type=float, default=2.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-roofline", action="store_true")
    ap.add_argument("--no-pe", action="store_true", help="skip the PatchEncoder stream measurement")
    ap.add_argument("--no-llm", action="store_true", help="skip the LLM decoder step measurement")
    ap.add_argument("--no-voc", action="store_true", help="skip the BigVGAN decoder measurement")
    ap.add_argument("--global-utt", type=int, default=2048,
                    help="strong-scaling line (key global_solve): this many utterances split evenly over the "
                         "ranks, each rank solving its shard in batches of at most --max-batch; 0 skips it")
    ap.add_argument("--max-batch", type=int, default=128,
                    help="utterances per solve in the global_solve line (throughput peaks at 64-128)")
    ap.add_argument("--global-steps", type=int, default=2, help="timed passes over the global workload")
    ap.add_argument("--part", choices=["all", "dit", "pe", "llm", "voc", "attn"], default="all",
                    help="run one part alone and print its JSON object (profiling drivers): dit = the DiT solve "
                         "(bf16 unless --dtype fp8), pe = PatchEncoder prefill + decode, llm = LLM steps, "
                         "voc = BigVGAN decode, attn = the attention sublayer")
    ap.add_argument("--pe-steps", type=int, default=125, help="PatchEncoder decode steps per pass")
    ap.add_argument("--sweep", action="store_true",
                    help="per-GPU sweep instead of the benchmark line: batch 16..256 at L = 64 and L = 16/64/256 "
                         "at batch 64, bf16 and e4m3, one JSON line per point")
    return ap.parse_args()


def maybe_relaunch(args):
    """--gpus N > 1 outside torchrun: relaunch this script under it."""
    if args.gpus > 1 and "WORLD_SIZE" not in os.environ:
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={args.gpus}",
               "--master-addr", "127.0.0.1", "--master-port", str(29500 + os.getpid() % 1000)] + sys.argv
        sys.exit(subprocess.call(cmd))


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples (every 200 ms) during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        loaded = [s for s in sm if mx and s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- workload
def make_inputs(args, rank):
    import synth
    seed = 1000 + rank
    w = synth.dit_weights(1, n_layers=args.layers)
    fc, fu = synth.fm_history(seed, args.n_utt, args.fm_len, w)
    z0 = synth.normal(seed, "z0", (args.n_utt, args.patch, 128), 1.0)
    spk = synth.normal(seed, "spk", (args.n_utt, 512), 1.0 / np.sqrt(512.0))
    return w, fc, fu, z0, spk


def workload_config(args, n, dtype="bf16"):
    L = args.fm_len + args.patch
    cfg = {"workload": f"DiT Euler solve, {args.layers} layers, CFG pair, v4 FM layout",
           "n_utt_per_gpu": args.n_utt, "cfg_rows_per_gpu": 2 * args.n_utt, "seq_len": L,
           "fm_len": args.fm_len, "patch": args.patch, "nfe": args.nfe, "cfg_scale": args.cfg_scale}
    if dtype == "f32":
        cfg.update({"weights": "fp32 (the reference's host arithmetic)",
                    "sample": "CFG-pair evals of this workload's first utterance at step t = 0"})
        return cfg
    cfg.update({
        "weights": ("bf16 (fp32 accumulate, fp32 residual)" if dtype == "bf16" else
                    "block projections e4m3 x e4m3 (per-channel weight scales, per-row activation scales), "
                    "fp32 accumulate; adaLN/input/output bf16; fp32 residual"),
        "global_utterances": args.n_utt * n,
        "parallelism": f"utterance shards x{n}, no collective",
        "l2": "working set > L2: %s of weights streamed per forward" % ("0.69 GB" if dtype == "bf16" else "0.36 GB"),
        "graph": "whole solve in one CUDA graph"})
    return cfg


def cpu_reference_eval(args, w, fc, fu, z0, spk, ffn_mode):
    """One CFG-pair velocity eval (cond row + uncond row, step t = 0) through the
    reference's own include/dit_manual.h built in oracle/_ref, wired like
    src/e2e_pipeline_v4.cpp:438-506.  Returns seconds."""
    sys.path.insert(0, os.path.join(HERE, "oracle"))
    import oracle as O
    orc, ref = O.Oracle(), O.Reference()
    # all host threads (torch.distributed.run sets OMP_NUM_THREADS=1 per process)
    ncpu = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    orc.set_threads(ncpu)
    ref.set_threads(ncpu)
    L = args.fm_len + args.patch
    mask = orc.fm_mask(L, args.fm_len, args.patch)
    pos = orc.fm_pos(L, args.fm_len, args.patch)
    cond = orc.compute_cond(w, 0.0, spk[0], 1.5, n_layers=args.layers)
    coord = orc.linear_rows(z0[0], w["coordinate_proj.weight"], w["coordinate_proj.bias"])
    xs = []
    for buf in (fc, fu):
        x = np.zeros((L, 1024), np.float32)
        x[:args.fm_len] = buf[0]
        x[args.fm_len:] = coord
        xs.append(x)
    t = time.perf_counter()
    for x in xs:
        ref.dit_velocity(w, args.layers, x, cond, mask, pos, ffn_mode=ffn_mode, n_out=args.patch)
    return time.perf_counter() - t, ref.num_threads()


def cpu_batched_eval(args, inputs):
    """The batched CPU throughput line: one velocity forward of every CFG row of
    the workload (2 x n_utt rows, step t = 0) through a PyTorch fp32
    restatement of the reference's arithmetic (oracle/torch_cpu.py) on all
    host threads; one untimed warm-up forward first."""
    import torch
    sys.path.insert(0, os.path.join(HERE, "oracle"))
    import oracle as O
    import torch_cpu
    w, fc, fu, z0, spk = inputs
    ncpu = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    torch.set_num_threads(ncpu)
    orc = O.Oracle()
    L = args.fm_len + args.patch
    mask = orc.fm_mask(L, args.fm_len, args.patch)
    pos = orc.fm_pos(L, args.fm_len, args.patch)
    n = args.n_utt
    x = np.zeros((2 * n, L, 1024), np.float32)
    cond = np.zeros((2 * n, 1024), np.float32)
    for u in range(n):
        c = orc.compute_cond(w, 0.0, spk[u], 1.5, n_layers=args.layers)
        coord = orc.linear_rows(z0[u], w["coordinate_proj.weight"], w["coordinate_proj.bias"])
        for r, buf in ((2 * u, fc), (2 * u + 1, fu)):
            x[r, :args.fm_len] = buf[u]
            x[r, args.fm_len:] = coord
            cond[r] = c
    m = torch_cpu.BatchedDiT(w, args.layers)
    m.velocity(x[:2], cond[:2], mask, pos, n_out=args.patch)
    t = time.perf_counter()
    m.velocity(x, cond, mask, pos, n_out=args.patch)
    secs = time.perf_counter() - t
    return {"value": n / secs, "unit": UNIT, "cores": ncpu, "kind": "port",
            "sample": "one velocity forward of all %d CFG rows (L=%d, %d layers, fp32) batched through "
                      "PyTorch/MKL on the host (oracle/torch_cpu.py), %.1f s" % (2 * n, L, args.layers, secs)}


def run_reference(args, rank, world):
    """--impl reference: the reference CPU path (as shipped) on the host cores."""
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(HERE, "oracle"))
    import oracle as O
    if not O.Reference.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libdtts_ref.so was not built"}))
        return
    w, fc, fu, z0, spk = make_inputs(args, 0)
    for _ in range(args.warmup):
        cpu_reference_eval(args, w, fc, fu, z0, spk, O.FFN_AS_WRITTEN)
    tot, cores = 0.0, 1
    for _ in range(args.steps):
        dt, cores = cpu_reference_eval(args, w, fc, fu, z0, spk, O.FFN_AS_WRITTEN)
        tot += dt
    value = args.steps / tot
    sample = ("one CFG-pair velocity eval per step (cond + uncond row, L=%d, %d layers) through the "
              "reference's manual_dit_block as shipped (include/dit_manual.h; FFN on token 0 only)"
              % (args.fm_len + args.patch, args.layers))
    print(json.dumps({
        "metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * tot / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args, 1, "f32"),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "reference", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def load_traffic():
    """Per-launch DRAM traffic of the dominant GEMM from the committed ncu summary."""
    p = os.path.join(HERE, "profiles", "gemm_traffic.json")
    try:
        with open(p) as f:
            return json.load(f)
    except (OSError, ValueError):
        return None


def library_e4m3_peak(dev, seconds=1.5):
    """Dense e4m3 x e4m3 -> bf16 GEMM throughput of the vendor library on this
    GPU (cuBLASLt through torch._scaled_mm, 8192 x 8192 x 8192, per-tensor
    scales): a burst of 10 launches after warm-up, and sustained over about
    `seconds` under the power cap, the two ways the bf16 peaks are measured.
    The e4m3 roofline's denominator; None where the library call fails."""
    import torch
    n = 8192
    try:
        g = torch.Generator(device=dev)
        g.manual_seed(0)
        a = torch.randn(n, n, device=dev, generator=g).to(torch.float8_e4m3fn)
        b = torch.randn(n, n, device=dev, generator=g).to(torch.float8_e4m3fn).t()   # column-major operand
        one = torch.ones((), device=dev, dtype=torch.float32)

        def run(k):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(k):
                torch._scaled_mm(a, b, one, one, out_dtype=torch.bfloat16)
            e1.record()
            e1.synchronize()
            return e0.elapsed_time(e1) / 1e3 / k   # seconds per GEMM

        run(5)
        burst = run(10)
        sustained = run(max(10, int(seconds / burst)))
        del a, b
        torch.cuda.empty_cache()
    except (RuntimeError, AttributeError, TypeError, ValueError):
        return None
    flop = 2.0 * n ** 3
    return {"burst": flop / burst / 1e12, "sustained": flop / sustained / 1e12,
            "source": "cuBLASLt e4m3 GEMM measured by this run (torch._scaled_mm, 8192^3, "
                      f"sustained over {seconds} s)"}


def measure(args, dtype, world, local_rank, dist, inputs):
    """Times one engine (dtype "bf16" or "fp8") on this rank: the resident-input
    solve loop (value), the same through host buffers (e2e), then the in-place
    launch timeline and each GEMM alone (roofline).  Every rank takes the same
    collective steps."""
    import torch
    import dtts
    dev = torch.device("cuda", local_rank)
    w, fc, fu, z0, spk = inputs
    eng = dtts.DiT(w, n_layers=args.layers, device=local_rank,
                   dtype=dtts.DTYPE_FP8 if dtype == "fp8" else dtts.DTYPE_BF16)
    stream = torch.cuda.Stream(device=dev)
    eng.set_stream(stream.cuda_stream)
    kw = dict(spk_scale=1.5, nfe=args.nfe, cfg_scale=args.cfg_scale, cfg_form=dtts.CFG_V4,
              layout=dtts.LAYOUT_FM_MASK, use_graph=True)

    # ---- resident inputs (value)
    d_fc, d_fu = torch.from_numpy(fc).to(dev), torch.from_numpy(fu).to(dev)
    d_z0, d_spk = torch.from_numpy(z0).to(dev), torch.from_numpy(spk).to(dev)
    d_z = torch.empty_like(d_z0)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            eng.solve(d_fc, d_fu, d_z0, d_spk, z_out=d_z, mem=dtts.MEM_DEVICE, **kw)
        eng.sync()
        launches_per_solve = eng.last_launch_count()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        clk = ClockSampler(local_rank)
        clk.start()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            eng.solve(d_fc, d_fu, d_z0, d_spk, z_out=d_z, mem=dtts.MEM_DEVICE, **kw)
        e1.record(stream)
        eng.sync()
        torch.cuda.synchronize()
        clocks = clk.stop()
        ms = e0.elapsed_time(e1)
        if dist:
            dist.barrier()

    # ---- end to end through the public API with pinned host buffers (e2e)
    e2e_ms = None
    h2d = fc.nbytes + fu.nbytes + z0.nbytes + spk.nbytes
    d2h = z0.nbytes
    if not args.no_e2e:
        p_fc, p_fu = torch.from_numpy(fc).pin_memory(), torch.from_numpy(fu).pin_memory()
        p_z0, p_spk = torch.from_numpy(z0).pin_memory(), torch.from_numpy(spk).pin_memory()
        p_z = torch.empty_like(p_z0).pin_memory()
        hfc, hfu, hz0, hspk, hz = (t.numpy() for t in (p_fc, p_fu, p_z0, p_spk, p_z))
        with torch.cuda.stream(stream):
            for _ in range(max(1, args.warmup)):
                eng.solve(hfc, hfu, hz0, hspk, z_out=hz, mem=dtts.MEM_HOST, **kw)
            if dist:
                dist.barrier()
            torch.cuda.synchronize()
            # each call copies in, solves and copies out before it returns: the
            # host clock around the loop is what the API costs a caller
            t0 = time.perf_counter()
            for _ in range(args.steps):
                eng.solve(hfc, hfu, hz0, hspk, z_out=hz, mem=dtts.MEM_HOST, **kw)
            torch.cuda.synchronize()
            e2e_ms = (time.perf_counter() - t0) * 1000.0
            if dist:
                dist.barrier()

    # ---- max over ranks
    t = torch.tensor([ms, e2e_ms if e2e_ms is not None else 0.0], device=dev, dtype=torch.float64)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms_max = float(t[0]), float(t[1])

    evals = args.n_utt * args.nfe * args.steps * world
    value = evals / (ms / 1000.0)
    e2e_value = evals / (e2e_ms_max / 1000.0) if e2e_ms is not None else None

    # ---- roofline of the dominant kernel: the four per-block tcgen05 GEMMs,
    # timed in place (events around every launch of the captured solve, on the
    # engine stream, replayed right after the timed region) and, for
    # reference, each one alone (20 back-to-back launches)
    roof, attn_us, kernels, alone, timeline_ms = None, None, {}, {}, None
    if not args.no_roofline:
        with torch.cuda.stream(stream):
            tl = eng.solve_timeline(d_fc, d_fu, d_z0, d_z, spk=d_spk, spk_scale=1.5, nfe=args.nfe,
                                    cfg_scale=args.cfg_scale, cfg_form=dtts.CFG_V4, layout=dtts.LAYOUT_FM_MASK,
                                    reps=3)
            names = {0: "gemm_qkv", 1: "gemm_o", 2: "gemm_ffn1", 3: "gemm_ffn2", 4: "attention", 5: "ln_modulate",
                     6: "gemm_adaln", 7: "gemm_input"}
            flops = {}
            for kind, name in names.items():
                us, fl, by = eng.profile(kind, iters=20)
                alone[name] = round(us, 2)
                flops[name] = fl
        timeline_ms = sum(v[0] for v in tl.values()) / 1000.0
        kernels = {k: {"us_per_launch": round(v[0] / v[1], 2), "launches_per_solve": v[1],
                       "share": round(v[0] / (timeline_ms * 1000.0), 4)} for k, v in tl.items() if v[1]}
        gem = ("gemm_qkv", "gemm_o", "gemm_ffn1", "gemm_ffn2")
        f = sum(flops[n] for n in gem)                                 # one block's four GEMMs
        tt = sum(tl[n][0] / tl[n][1] for n in gem)                     # their mean in-place durations
        achieved = f / (tt * 1e-6) / 1e12
        peaks = {}
        try:
            with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as fh:
                peaks = json.load(fh)
        except (OSError, ValueError):
            pass
        peak = peaks.get("bf16_tflops_sustained", 1400.0)
        burst = peaks.get("bf16_tflops", 1590.0)
        src = ("measured bf16_tflops_sustained (kernels timed inside the long solve)" if "bf16_tflops_sustained" in peaks
               else "fallback sustained figure")
        lib8 = None
        if dtype == "fp8":
            # the e4m3 denominator: the library's e4m3 GEMM measured here, else
            # twice the bf16 figure (B200's dense e4m3 : bf16 tensor-rate ratio)
            lib8 = library_e4m3_peak(dev)
            if lib8:
                peak, burst, src = lib8["sustained"], lib8["burst"], lib8["source"]
            else:
                peak, burst = 2 * peak, 2 * burst
                src = "2 x " + src + " (dense e4m3 = 2 x bf16 tensor rate; the library e4m3 GEMM failed)"
        tr = load_traffic() if dtype == "bf16" else None
        roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "traffic": tr.get("bytes_per_launch") if tr else None,
                "kernel": "gemm_tc_kernel (tcgen05): QKV + O + FFN1 + FFN2 of one block, FLOP-weighted",
                "peak_source": src, "frac_of_burst_peak": achieved / burst,
                "algorithmic_flops_per_launch": f,
                "traffic_source": tr.get("source") if tr else None}
        if lib8:
            roof["frac_of_2x_bf16_sustained"] = achieved / (2 * peaks.get("bf16_tflops_sustained", 1400.0))
        attn_us = kernels["attention"]["us_per_launch"]
    eng.close()
    return {"value": value, "ms_per_step": ms / args.steps,
            "e2e": None if e2e_value is None else {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                                                    "d2h_bytes_per_step": d2h},
            "roofline": roof, "attention_us_per_layer": attn_us, "kernels_in_place": kernels,
            "timeline_solve_ms": timeline_ms, "kernels_alone_us": alone, "clocks": clocks,
            "gpu_launches": launches_per_solve * args.steps}


def measure_global(args, world, rank, local_rank, dist):
    """Config 5: args.global_utt utterances (one config-3 patch solve each) split
    evenly over the ranks (shard.shard_range), every rank solving its shard in
    batches of at most args.max_batch utterances with inputs resident on its
    GPU; bf16 and, with --dtype both, e4m3.  Whole-job evals/s over the max of
    the ranks' device times (strong scaling: the total work is fixed)."""
    import torch
    import dtts
    import shard
    import synth
    dev = torch.device("cuda", local_rank)
    lo, hi = shard.shard_range(args.global_utt, world, rank)
    n_local = hi - lo
    chunks = []
    u = lo
    while u < hi:
        chunks.append(min(args.max_batch, hi - u))
        u += chunks[-1]
    # one seeded batch of inputs, reused by every chunk of the same size: the
    # work of a solve does not depend on the values
    w = synth.dit_weights(1, n_layers=args.layers)
    nb = max(chunks) if chunks else 0
    res = {}
    for dtype in (("bf16", "fp8") if args.dtype == "both" else (args.dtype,)):
        eng = dtts.DiT(w, n_layers=args.layers, device=local_rank,
                       dtype=dtts.DTYPE_FP8 if dtype == "fp8" else dtts.DTYPE_BF16)
        stream = torch.cuda.Stream(device=dev)
        eng.set_stream(stream.cuda_stream)
        kw = dict(spk_scale=1.5, nfe=args.nfe, cfg_scale=args.cfg_scale, cfg_form=dtts.CFG_V4,
                  layout=dtts.LAYOUT_FM_MASK, use_graph=True)
        d = {}
        if nb:
            fc, fu = synth.fm_history(5000, nb, args.fm_len, w)
            z0 = synth.normal(5000, "z0", (nb, args.patch, 128), 1.0)
            spk = synth.normal(5000, "spk", (nb, 512), 1.0 / np.sqrt(512.0))
            d = {k: torch.from_numpy(v).to(dev) for k, v in (("fc", fc), ("fu", fu), ("z0", z0), ("spk", spk))}
            d["z"] = torch.empty_like(d["z0"])

        def one_pass():
            for c in chunks:
                eng.solve(d["fc"][:c], d["fu"][:c], d["z0"][:c], d["spk"][:c], z_out=d["z"][:c], mem=dtts.MEM_DEVICE,
                          **kw)

        with torch.cuda.stream(stream):
            one_pass()
            eng.sync()
            if dist:
                dist.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.global_steps):
                one_pass()
            e1.record(stream)
            eng.sync()
            torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        if dist:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t[0])
        evals = args.global_utt * args.nfe * args.global_steps
        res[dtype] = {"value": evals / (ms / 1000.0), "unit": UNIT, "ms_per_pass": ms / args.global_steps,
                      "gpu_launches": eng.last_launch_count() * len(chunks) * args.global_steps}
        eng.close()
        if dist:
            dist.barrier()
    return {"global_utterances": args.global_utt, "utterances_per_rank": n_local, "batches_per_rank": chunks,
            "scaling": "strong", "passes": args.global_steps,
            "inputs": "one seeded batch of the largest solve size, reused by every batch of the shard",
            **res}


def run_sweep(args, local_rank):
    """Per-GPU sweep of config 5: batch (utterances per solve) 16..256 at L = 64
    and sequence length L = 16 / 64 / 256 at 64 utterances, bf16 and e4m3; one
    JSON line per point with the solve's evals/s and the in-place kernel times."""
    import torch
    torch.cuda.set_device(local_rank)
    points = [(b, 60) for b in (16, 32, 64, 128, 256)] + [(64, 12), (64, 252)]
    for n_utt, fm_len in points:
        a = argparse.Namespace(**vars(args))
        a.n_utt, a.fm_len, a.no_e2e = n_utt, fm_len, True
        inputs = make_inputs(a, 0)
        for dtype in (("bf16", "fp8") if args.dtype == "both" else (args.dtype,)):
            r = measure(a, dtype, 1, local_rank, None, inputs)
            k = r["kernels_in_place"]
            print(json.dumps({"sweep": "config5", "dtype": dtype, "n_utt": n_utt, "seq_len": fm_len + args.patch,
                              "value": r["value"], "unit": UNIT, "ms_per_step": r["ms_per_step"],
                              "roofline_frac": r["roofline"]["frac"] if r["roofline"] else None,
                              "us_per_launch": {n: v["us_per_launch"] for n, v in k.items()},
                              "clocks": r["clocks"]}), flush=True)


def cpu_pe_baseline(w, layers, frames):
    """One stream's prefill on the host cores: the reference's own patchenc_forward
    (src/modules/backbone/patchenc.cpp, built in oracle/_ref over the eager ggml
    stand-in, OpenMP matrix products) where that build exists, else the oracle's
    fp32 restatement (oracle/oracle.c)."""
    sys.path.insert(0, os.path.join(HERE, "oracle"))
    import oracle as O
    import synth
    try:
        fr = synth.normal(2, "pe.cpu", (frames, 128), 1.0)
        if O.Reference.available():
            ref = O.Reference()
            ncpu = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
            ref.set_threads(ncpu)
            t0 = time.perf_counter()
            ref.pe_forward(w, layers, fr)
            secs = time.perf_counter() - t0
            return {"prefill_frames_per_s": frames / secs, "cores": ref.num_threads(), "kind": "reference",
                    "sample": "one stream's %d-frame prefill, %d layers, through the reference's patchenc_forward "
                              "(src/modules/backbone/patchenc.cpp) built in oracle/_ref, its ggml operators from "
                              "the eager stand-in oracle/shim/ggml_eager.cpp, %.1f s" % (frames, layers, secs)}
        orc = O.Oracle()
        t0 = time.perf_counter()
        orc.pe_forward(w, layers, fr)
        secs = time.perf_counter() - t0
        cores = orc.num_threads()
    except Exception as e:   # the device figures stand without the CPU sample
        return {"error": str(e)[:200]}
    return {"prefill_frames_per_s": frames / secs, "cores": cores, "kind": "port",
            "sample": "one stream's %d-frame prefill, %d layers, through oracle/oracle.c (the fp32 "
                      "restatement of src/modules/backbone/patchenc.cpp), %.1f s" % (frames, layers, secs)}


def measure_pe(args, local_rank, cpu_sample=False):
    """PatchEncoder stream at the PatchEncoder workload: 32 streams, a 500-frame
    prefill (250 tokens each), then 125 one-patch decode steps against the KV
    cache; 24 layers, bf16, device-resident frames, CUDA events on the engine
    stream.  The decode steps are launched one host call at a time, as a
    streaming caller would, so launch gaps count.  cpu_sample: time one
    stream's prefill through the oracle's restatement on the host."""
    import torch
    import dtts
    import synth
    dev = torch.device("cuda", local_rank)
    B, prefill, steps = 32, 500, args.pe_steps
    w = synth.pe_weights(2, n_layers=24)
    pe = dtts.PatchEncoder(w, n_layers=24, max_batch=B, max_tokens=512, device=local_rank)
    stream = torch.cuda.Stream(device=dev)
    pe.set_stream(stream.cuda_stream)
    fr = torch.from_numpy(synth.normal(2, "pe.bench", (B, prefill + 4 * steps, 128), 1.0)).to(dev)
    pre_in = fr[:, :prefill].contiguous()
    steps_in = [fr[:, prefill + 4 * i:prefill + 4 * i + 4].contiguous() for i in range(steps)]
    out_pre = torch.empty((B, prefill // 4, 1536), device=dev)
    out_step = torch.empty((B, 1, 1536), device=dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    with torch.cuda.stream(stream):
        for rep in range(2):   # the first pass warms up
            pe.reset(B)
            ev[0].record(stream)
            pe.decode(pre_in, out=out_pre, mem=dtts.MEM_DEVICE)
            ev[1].record(stream)
            for i in range(steps):
                pe.decode(steps_in[i], out=out_step, mem=dtts.MEM_DEVICE)
            ev[2].record(stream)
            pe.sync()
    torch.cuda.synchronize()
    pre_ms, dec_ms = ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])
    pe.close()
    flop_pre = B * 24 * (prefill // 2) * 2 * (4 * 1024 * 1024 + 2 * 1024 * 4096)
    res = {"workload": f"PatchEncoder, 24 layers, 32 streams: 500-frame prefill, then {steps} decode steps",
           "prefill_ms": pre_ms, "prefill_frames_per_s": B * prefill / (pre_ms / 1000.0),
           "prefill_gemm_tflops": flop_pre / (pre_ms / 1000.0) / 1e12,
           "decode_ms_per_step": dec_ms / steps, "decode_patches_per_s": B * steps / (dec_ms / 1000.0),
           "dtype": "bf16"}
    if cpu_sample:
        res["cpu_baseline"] = cpu_pe_baseline(w, 24, prefill)
    return res


def cpu_llm_reference(w, layers, batch):
    """The reference's own llm_kv_cache_init / llm_kv_cache_step (oracle/_ref) on
    one sequence on the host: a 1-token prompt alone, then with one step; the
    step time is the difference.  None when oracle/_ref is absent."""
    sys.path.insert(0, os.path.join(HERE, "oracle"))
    import oracle as O
    import synth
    if not O.Reference.available():
        return None
    try:
        ref = O.Reference()
        p1 = synth.normal(4, "llm.cpu_prompt", (1, 1536), 1.0)
        s1 = synth.normal(4, "llm.cpu_step", (1, 1536), 1.0)
        t0 = time.perf_counter()
        ref.llm_run(w, layers, p1, s1[:0])
        t1 = time.perf_counter()
        ref.llm_run(w, layers, p1, s1)
        t2 = time.perf_counter()
    except Exception as e:   # the device figures stand without the CPU sample
        return {"error": str(e)[:200]}
    step_s = max(1e-9, (t2 - t1) - (t1 - t0))
    return {"step_ms_per_sequence": step_s * 1000.0, "steps_per_s": 1.0 / (step_s * batch), "cores": 1,
            "kind": "reference",
            "sample": "one sequence through the reference's llm_kv_cache_init / llm_kv_cache_step "
                      "(oracle/_ref, single-threaded loops), %d layers: a 1-token prompt alone, then with "
                      "one step; the step is the difference (%.1f s in all). steps_per_s is for %d "
                      "sequences, which the reference steps one after another" % (layers, t2 - t0, batch)}


def measure_llm(args, local_rank, cpu_sample=False):
    """LLM decoder step at the autoregressive loop's batch: 28 layers of
    Qwen2.5-1.5B (synthetic weights), 64 sequences prefilled with 64-token
    prompts, then 16 steps of one embedding each (device-resident inputs,
    CUDA events on the engine stream, one host call per step).  cpu_sample:
    time the reference's own llm_kv_cache_init / llm_kv_cache_step on one
    sequence on the host (oracle/_ref), if present."""
    import torch
    import dtts
    import synth
    dev = torch.device("cuda", local_rank)
    B, n_tok, steps, layers = args.n_utt, 64, 16, 28
    w = synth.llm_weights(3, n_layers=layers)
    llm = dtts.LLM(w, n_layers=layers, max_batch=B, max_seq=n_tok + steps + 1, device=local_rank)
    if not cpu_sample:
        del w
    stream = torch.cuda.Stream(device=dev)
    llm.set_stream(stream.cuda_stream)
    emb = torch.from_numpy(synth.normal(4, "llm.bench", (B, n_tok + steps, 1536), 1.0)).to(dev)
    prompt = emb[:, :n_tok].contiguous()
    step_in = [emb[:, n_tok + i].contiguous() for i in range(steps)]
    out_p = torch.empty((B, n_tok, 1536), device=dev)
    out_s = torch.empty((B, 1536), device=dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    with torch.cuda.stream(stream):
        for rep in range(2):   # the first pass warms up
            ev[0].record(stream)
            llm.prefill(prompt, out=out_p, mem=dtts.MEM_DEVICE)
            ev[1].record(stream)
            for i in range(steps):
                llm.step(step_in[i], out=out_s, mem=dtts.MEM_DEVICE)
            ev[2].record(stream)
    torch.cuda.synchronize()
    pre_ms, st_ms = ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2]) / steps
    llm.close()
    weight_bytes = layers * 2 * (1536 * 2048 + 1536 * 1536 + 2 * 8960 * 1536 + 8960 * 1536)
    res = {"workload": f"LLM decoder, {layers} layers, {B} sequences: {n_tok}-token prefill, then {steps} steps",
           "prefill_ms": pre_ms, "step_ms": st_ms, "steps_per_s": 1000.0 / st_ms,
           "step_weight_stream_gbs": weight_bytes / (st_ms / 1000.0) / 1e9, "dtype": "bf16"}
    if cpu_sample:
        res["cpu_reference"] = cpu_llm_reference(w, layers, B)
        del w
    return res


def measure_voc(args, local_rank, cpu_sample):
    """BigVGAN decoder on one utterance of 250 latent frames (20 s of 24 kHz
    audio): device-resident latents, CUDA events on the engine stream, 2
    warm-up and 5 timed decodes; e2e through host buffers (the C ABI call
    with its copies), 3 decodes.  cpu_sample: time the reference's own
    bigvgan_decode on one frame on the host (oracle/_ref), if present."""
    import time
    import torch
    import dtts
    import synth
    dev = torch.device("cuda", local_rank)
    F, reps = 250, 5
    w = synth.voc_weights(5, aa_filter=dtts.voc_aa_filter())
    v = dtts.Vocoder(w, max_frames=F, device=local_rank)
    stream = torch.cuda.Stream(device=dev)
    v.set_stream(stream.cuda_stream)
    lat_h = synth.normal(9, "voc.bench", (F, 128), 1.0)
    lat = torch.from_numpy(lat_h).to(dev)
    out = torch.empty(F * 1920, device=dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    with torch.cuda.stream(stream):
        for _ in range(2):
            v.decode(lat, out=out, mem=dtts.MEM_DEVICE)
        ev[0].record(stream)
        for _ in range(reps):
            v.decode(lat, out=out, mem=dtts.MEM_DEVICE)
        ev[1].record(stream)
    torch.cuda.synchronize()
    ms = ev[0].elapsed_time(ev[1]) / reps
    audio_s = F * 1920 / 24000.0
    pin_in = torch.from_numpy(lat_h).pin_memory()
    pin_out = torch.empty(F * 1920, dtype=torch.float32).pin_memory()
    t0 = time.perf_counter()
    for _ in range(3):
        v.decode(pin_in.numpy(), out=pin_out.numpy(), mem=dtts.MEM_HOST)
    e2e_ms = (time.perf_counter() - t0) / 3 * 1000.0
    v.close()
    res = {"workload": f"BigVGAN decoder, one utterance of {F} latent frames ({audio_s:.0f} s of 24 kHz audio)",
           "ms_per_decode": ms, "audio_s_per_s": audio_s / (ms / 1000.0),
           "e2e": {"ms_per_decode": e2e_ms, "audio_s_per_s": audio_s / (e2e_ms / 1000.0),
                   "h2d_bytes": F * 128 * 4, "d2h_bytes": F * 1920 * 4},
           "dtype": "bf16 convolutions, fp32 LSTM / activations"}
    if cpu_sample:
        sys.path.insert(0, os.path.join(HERE, "oracle"))
        import oracle as O
        if O.Reference.available():
            import ctypes
            ref = O.Reference()
            # the reference prints progress lines from C: send fd 1 to /dev/null meanwhile
            sys.stdout.flush()
            libc = ctypes.CDLL(None)
            saved, dn = os.dup(1), os.open(os.devnull, os.O_WRONLY)
            os.dup2(dn, 1)
            try:
                t0 = time.perf_counter()
                ref.voc_decode(w, lat_h[:1])
                secs = time.perf_counter() - t0
                libc.fflush(None)
            finally:
                os.dup2(saved, 1)
                os.close(saved)
                os.close(dn)
            res["cpu_reference"] = {"audio_s_per_s": (1920 / 24000.0) / secs, "cores": 1, "kind": "reference",
                                    "sample": "one latent frame through the reference's bigvgan_decode "
                                              "(oracle/_ref, single-threaded loops), %.1f s" % secs}
    return res


def measure_attn_sublayer(args, local_rank, cpu_sample):
    """Config 1: one DiT self-attention sublayer (manual_attention), X [2][64][1024],
    fp32 and bf16 engines.  Reports the attention core's device time (post-QKV,
    pre-O; CUDA events over 50 back-to-back launches) and the whole sublayer call
    through host buffers (copies included, mean of 20 calls); with cpu_sample,
    the reference's own manual_attention (oracle/_ref) on the host for the same
    two rows."""
    import time
    import dtts
    import synth
    w = synth.dit_weights(0, n_layers=1)
    p = "velocity_field_predictor.blocks.0."
    W = [w[p + n] for n in ("attn.q_proj.weight", "attn.k_proj.weight", "attn.v_proj.weight", "attn.o_proj.weight")]
    bo = np.zeros(1024, np.float32)
    qn, kn = w[p + "attn.q_norm.weight"], w[p + "attn.k_norm.weight"]
    x = synth.normal(0, "c1.x", (2, 64, 1024), 1.0)
    res = {"workload": "attention sublayer, 2 rows x L=64 x 1024, 16 heads, RMS qk-norm, RoPE, no mask"}
    for name, dt in (("fp32", dtts.DTYPE_F32), ("bf16", dtts.DTYPE_BF16)):
        a = dtts.Attention(*W, bo, qn, kn, dtype=dt, device=local_rank)
        for _ in range(3):
            a.forward(x)
        t0 = time.perf_counter()
        for _ in range(20):
            a.forward(x)
        call_us = (time.perf_counter() - t0) / 20 * 1e6
        res[name] = {"core_us": a.profile_core(50), "sublayer_call_us_host_buffers": call_us}
        a.close()
    if cpu_sample:
        sys.path.insert(0, os.path.join(HERE, "oracle"))
        import oracle as O
        if O.Reference.available():
            ref = O.Reference()
            t0 = time.perf_counter()
            for i in range(2):
                ref.manual_attention(x[i], *W, bo, qn, kn)
            res["cpu_reference_us"] = (time.perf_counter() - t0) * 1e6
            res["cpu_reference"] = ("the reference's manual_attention (include/dit_manual.h:88) built in "
                                    "oracle/_ref, both rows, %d threads" % ref.num_threads())
    return res


def run_part(args, local_rank):
    """One part of the benchmark alone (a profiling driver): its JSON object on one line."""
    import torch
    torch.cuda.set_device(local_rank)
    cpu = not args.no_cpu_baseline
    if args.part == "dit":
        dtype = "fp8" if args.dtype == "fp8" else "bf16"
        r = measure(args, dtype, 1, local_rank, None, make_inputs(args, 0))
    elif args.part == "pe":
        r = measure_pe(args, local_rank, cpu)
    elif args.part == "llm":
        r = measure_llm(args, local_rank, cpu)
    elif args.part == "voc":
        r = measure_voc(args, local_rank, cpu)
    else:
        r = measure_attn_sublayer(args, local_rank, cpu)
    print(json.dumps({"part": args.part, **r}))


def run_ours(args, rank, world, local_rank):
    import torch
    dist = None
    if world > 1:
        import torch.distributed as dist
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    torch.cuda.set_device(local_rank)
    inputs = make_inputs(args, rank)
    head_dtype = "fp8" if args.dtype == "fp8" else "bf16"
    head = measure(args, head_dtype, world, local_rank, dist, inputs)
    extra = measure(args, "fp8", world, local_rank, dist, inputs) if args.dtype == "both" else None
    glob = measure_global(args, world, rank, local_rank, dist) if args.global_utt > 0 else None
    pe = measure_pe(args, local_rank, rank == 0 and not args.no_cpu_baseline) \
        if (world == 1 and not args.no_pe) else None
    llm = measure_llm(args, local_rank, rank == 0 and not args.no_cpu_baseline) \
        if (world == 1 and not args.no_llm) else None
    voc = measure_voc(args, local_rank, rank == 0 and not args.no_cpu_baseline) \
        if (world == 1 and not args.no_voc) else None
    attn1 = measure_attn_sublayer(args, local_rank, rank == 0 and not args.no_cpu_baseline) \
        if world == 1 else None

    # ---- CPU baseline: reference code (per-token FFN) on the host, rank 0, N = 1
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(HERE, "oracle"))
        import oracle as O
        if O.Reference.available():
            w, fc, fu, z0, spk = inputs
            secs, cores = cpu_reference_eval(args, w, fc, fu, z0, spk, O.FFN_PER_TOKEN)
            cpu = {"value": 1.0 / secs, "unit": UNIT, "cores": cores, "kind": "reference",
                   "sample": "one CFG-pair eval (2 rows, L=%d, %d layers) through the reference's "
                             "include/dit_manual.h (FFN per token) built in oracle/_ref, %.1f s"
                             % (args.fm_len + args.patch, args.layers, secs)}

    # ---- batched CPU line: all 128 rows of the workload through MKL at once
    cpu_batched = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_batched = cpu_batched_eval(args, inputs)

    if rank == 0:
        line = {
            "metric": METRIC, "value": head["value"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16" if head_dtype == "bf16" else "e4m3",
            "data": "synthetic (seeded N(0,1) inputs, N(0,0.02) weights)",
            "config": workload_config(args, world, head_dtype),
        }
        for k in ("e2e", "roofline", "attention_us_per_layer", "kernels_in_place", "timeline_solve_ms",
                  "kernels_alone_us"):
            line[k] = head[k]
        line["cpu_baseline"] = cpu
        if cpu_batched:
            line["cpu_batched"] = cpu_batched
        line["clocks"] = head["clocks"]
        line["gpu_launches"] = head["gpu_launches"]
        if pe:
            line["patch_encoder"] = pe
        if llm:
            line["llm_step"] = llm
        if voc:
            line["vocoder"] = voc
        if attn1:
            line["attention_sublayer"] = attn1
        if glob:
            line["global_solve"] = glob
        if extra:
            line["fp8"] = {"dtype": "e4m3", "weights": workload_config(args, world, "fp8")["weights"],
                           **{k: extra[k] for k in ("value", "ms_per_step", "e2e", "roofline", "attention_us_per_layer",
                                                    "kernels_in_place", "clocks", "gpu_launches")}}
        print(json.dumps(line))
    if dist:
        dist.destroy_process_group()


def main():
    args = parse()
    maybe_relaunch(args)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, rank, world)
    elif args.sweep:
        run_sweep(args, local_rank)
    elif args.part != "all":
        run_part(args, local_rank)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
