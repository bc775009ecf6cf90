#!/usr/bin/env python3
"""Benchmark of the B200 encoder hot path (bark3-wgpu's Conformer encoder).

Default workload: BASELINE config 5 as written -- ONE batch of 256 seeded
utterances, lengths uniform in 10-60 s, transcribed from 16 kHz audio (mel,
conv subsampling, the 24-block 4-bit LUT encoder, greedy TDT).  Under
torchrun the batch is sharded across the ranks by longest-processing-time
over the encoder cost (b3_shard_lpt), one process per GPU, no collective on
the data path ("scaling": "strong").  --scaling weak gives every rank its own
256-utterance batch instead.  One step = the whole batch once.  Metric: RTFx =
audio seconds transcribed per second, whole job.

  value  device-resident inputs (HBM), CUDA events on the library's stream,
         max over ranks; the per-step working set (GBs of activations) is far
         larger than L2, so no flush is needed between steps.
  e2e    the same through the host-pointer C ABI call: pinned host audio
         copied in and the token buffers copied out inside every timed step.

--impl reference times the reference's CPU pipeline (the C restatement of
src/mel.rs, src/sub.rs, src/cpu/* and src/tdt.rs in oracle/, all host cores)
on utterances of the same batch.  It loads only the oracle library, never
the product's.
"""
from __future__ import annotations

import argparse
import atexit
import json
import os
import pathlib
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from __graft_entry__ import load_oracle, load_package  # noqa: E402

N_LAYERS = 24
METRIC = "RTFx (audio-s/s), batched transcription"
VOCAB = 1025        # 1024 tokens + blank
MAX_TOKENS = 1024   # token slots per utterance in the output buffer


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--utterances", type=int, default=256)
    ap.add_argument("--scaling", default="strong", choices=["strong", "weak"],
                    help="strong: one batch of --utterances sharded across the ranks (LPT; BASELINE config 5); "
                         "weak: every rank its own batch of --utterances")
    ap.add_argument("--seconds", type=float, default=0.0,
                    help="every utterance this many seconds long instead of U(10, 60) (e.g. --utterances 1 "
                         "--seconds 30: BASELINE config 2's single 30 s clip)")
    ap.add_argument("--shard", default="",
                    help="R:N -- on one GPU, time the share rank R of an N-GPU strong-scaling job would get "
                         "(diagnostic; the line says so)")
    ap.add_argument("--no-sweep", action="store_true", help="skip the K1 M-sweep recorded in the N=1 line")
    ap.add_argument("--ref-utterances", type=int, default=16,
                    help="--impl reference: utterances of the batch its steps cycle through")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="budget of the CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--seed", type=int, default=5)
    ap.add_argument("--workload", default="audio", choices=["audio", "transcribe", "encoder", "linear"],
                    help="audio: 16 kHz audio -> tokens (mel, subsampling, encoder, greedy TDT) over the "
                         "config-5 batch; transcribe: the same from subsampled features; encoder: the "
                         "encoder alone; linear: K1 GEMM shape sweep (config 1)")
    return ap.parse_args()


SWEEP_SHAPES = [(1875, 4096, 1024), (2048, 4096, 1024), (4096, 4096, 1024), (8192, 4096, 1024),
                (16384, 4096, 1024), (8192, 1024, 4096), (8192, 3072, 1024), (110894, 4096, 1024)]


def k1_sweep(pkg, syn, enc, shapes, warmup, steps, seed):
    """BASELINE config 1 (M=1875, K=1024, N=4096, f32 activations, bias) and
    the M >= 2048 shapes of the north-star GEMM target, through
    b3_linear_lut4 with device pointers (config 1's uncentred level tables).
    The K1 launch is timed alone with CUDA events on the library's stream
    (the f32 -> f16 conversion of A is a separate, separately timed kernel);
    TFLOP/s against the burst bf16 peak (a kernel timed in isolation)."""
    import ctypes

    import torch

    L = pkg.lib()
    pk, pk_kind = peaks()
    rng = np.random.default_rng(seed)
    rows = []
    for m, n, k in shapes:
        codes, lut16 = syn.make_lut4(rng, n, k)
        a = torch.randn(m, k, device="cuda")
        bias = torch.randn(n, device="cuda") * 0.01
        tc = torch.from_numpy(codes).cuda()
        tl = torch.from_numpy(lut16.view(np.int16)).cuda()
        out = torch.empty(m, n, device="cuda")
        torch.cuda.synchronize()
        for _ in range(warmup):
            enc.linear_lut4(a, tc, tl, bias, out=out)
        enc.sync()
        L.b3_profile(enc.ctx, 1)
        for _ in range(steps):
            enc.linear_lut4(a, tc, tl, bias, out=out)
        vals = {}
        for kind in (pkg_kind("gemm_lut4"), pkg_kind("convert")):
            t, f, b, nl = ctypes.c_double(), ctypes.c_double(), ctypes.c_double(), ctypes.c_int64()
            pkg.check(L.b3_profile_read(enc.ctx, kind, ctypes.byref(t), ctypes.byref(f), ctypes.byref(b),
                                        ctypes.byref(nl)))
            vals[kind] = (t.value, f.value, b.value, nl.value)
        L.b3_profile(enc.ctx, 0)
        t, f, b, nl = vals[pkg_kind("gemm_lut4")]
        tflops = f / (t / 1000.0) / 1e12
        peak = pk.get("bf16_tflops")
        ct = vals[pkg_kind("convert")]
        rows.append({"m": m, "n": n, "k": k, "us_per_launch": round(1000 * t / nl, 2),
                     "TFLOP/s": round(tflops, 1), "frac_of_burst_peak": round(tflops / peak, 4),
                     "alg_GB/s": round(b / t / 1e6, 1), "convert_us": round(1000 * ct[0] / max(1, ct[3]), 2)})
        del a, out, tc, tl
    return rows, f"bf16_tflops (burst) of {pk_kind}"


def run_linear_sweep(args):
    """--workload linear: one JSON line per K1 shape (see k1_sweep)."""
    pkg = load_package()
    import bark3_b200.synthetic as syn

    enc = pkg.Encoder(0)
    rows, peak_src = k1_sweep(pkg, syn, enc, SWEEP_SHAPES, args.warmup, args.steps, args.seed)
    for r in rows:
        print(json.dumps({"workload": "k1 LUT4 linear", **r, "peak": peak_src}), flush=True)
    enc.close()


def pkg_kind(name):
    return KINDS.index(name)


KINDS = ["gemm_lut4", "gemm_f16", "attention", "layernorm", "dwconv", "convert", "other", "decoder", "frontend"]


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def job_batch(args, world, syn):
    """(seconds, frames) of every utterance of the whole job, in batch order;
    pure Python (loads no library)."""
    import bark3_b200 as pkg

    def lengths(seed):
        if args.seconds > 0:
            return [args.seconds] * args.utterances
        return [float(x) for x in syn.batch_lengths(seed, args.utterances)]

    if args.scaling == "strong":
        secs = lengths(args.seed)
    else:
        secs = [x for r in range(world) for x in lengths(args.seed + 1000 * r)]
    return secs, [pkg.frames_for_seconds(x) for x in secs]


def batch_for_rank(args, rank, world, pkg, syn):
    """(seconds per utterance, frames per utterance) of this rank's share."""
    if args.shard:   # one GPU standing in for rank R of an N-GPU strong job
        rank, world = (int(v) for v in args.shard.split(":"))
    if args.scaling == "strong":
        secs, frames = job_batch(args, 1, syn)
        if world == 1:
            return secs, frames
        rank_of = pkg.shard_lpt(frames, world)
        mine = [i for i in range(len(frames)) if rank_of[i] == rank]
        return [secs[i] for i in mine], [frames[i] for i in mine]
    if args.seconds > 0:
        return job_batch(args, 1, syn)
    secs = [float(x) for x in syn.batch_lengths(args.seed + 1000 * rank, args.utterances)]
    return secs, [pkg.frames_for_seconds(x) for x in secs]


def job_config(args, world, syn):
    """The `config` object of the JSON line: the whole job's workload (both
    arms print the same one)."""
    secs, frames = job_batch(args, world, syn)
    decode = args.workload in ("audio", "transcribe")
    return {
        "workload": {"audio": "config 5: batched transcription, 16 kHz audio -> tokens (mel, conv subsampling, "
                              "24-block 4-bit LUT encoder, greedy TDT)",
                     "transcribe": "config-5 batch from subsampled features: 4-bit encoder + greedy TDT",
                     "encoder": "config-5 batch through the 24-block 4-bit LUT encoder"}[args.workload],
        "utterances": len(secs), "audio_s": round(sum(secs), 1), "frames": int(sum(frames)),
        "lengths_s": f"{args.seconds:g} each" if args.seconds > 0 else "U(10,60) seeded", "seed": args.seed,
        "layers": N_LAYERS,
        "d_model": 1024, "heads": 8, "ffn": 4096, "conv_kernel": 9,
        "weights": "random-init 4-bit codes + 16-entry f16 LUT per row (levels N(0,0.02) sorted, row-centred)",
        "input": ("synthetic audio: white noise U(-0.1,0.1) + 3 sines of amplitude 0.1, 16 kHz f32"
                  if args.workload == "audio" else "synthetic (T,4096) subsampled features, f32"),
        "decoder": (f"2-layer LSTM 640, joint 640, vocab {VOCAB - 1}+blank, durations 0..4, random-init"
                    if decode else None),
        "l2": "per-step working set (%.2f GB of encoder activations per GPU) > L2, no flush"
              % (sum(frames) / world * 4096 * 2 * 3 / 1e9),
        "parallelism": (f"one batch LPT-sharded over {world} GPU(s), no collective" if args.scaling == "strong"
                        else f"one batch per GPU x{world}, no collective"),
    }


class ClockSampler:
    """nvidia-smi samples (every 100 ms) of the SM clock and throttle reasons.

    Started before the warm-up steps and stopped after the end-to-end steps
    that follow the timed ones, so that nvidia-smi is already sampling when
    the timed region begins; `mark(t0, t1)` records the timed region's
    wall-clock window, and the summary keeps the samples inside it. A region
    too short to hold a sample (a few fast steps on many GPUs) falls back to
    the loaded samples around it (warm-up and end-to-end steps), and says
    so."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.window = None
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def mark(self, t0, t1):
        """The timed region ran from wall-clock t0 to t1 (time.time())."""
        self.window = (t0, t1)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.proc = None

    def summary(self):
        self.f.flush()
        text = pathlib.Path(self.f.name).read_text()
        os.unlink(self.f.name)
        return summarize_clocks(text, self.window)


def summarize_clocks(text, window):
    """Median SM clock and the throttle reasons seen, from nvidia-smi CSV rows
    (timestamp, index, clocks.sm, clocks.max.sm, power.draw, reasons.active,
    hw_slowdown, hw_thermal_slowdown, sw_thermal_slowdown, sw_power_cap)."""
    import datetime

    rows = []
    for line in text.splitlines():
        parts = [p.strip() for p in line.split(",")]
        if len(parts) < 10:
            continue
        try:
            ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
            rows.append((ts, float(parts[2]), float(parts[3]), float(parts[4]), parts[6:10]))
        except ValueError:
            continue
    if not rows:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
    span = "timed steps"
    chosen = rows
    if window is not None:
        inside = [r for r in rows if window[0] <= r[0] <= window[1]]
        if inside:
            chosen = inside
        else:
            chosen = [r for r in rows if r[3] > 300.0] or rows
            span = "loaded samples around the timed steps (warm-up, end-to-end); none fell inside them"
    loaded = [r for r in chosen if r[3] > 300.0] or chosen
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    reasons = sorted({names[i] for r in loaded for i, v in enumerate(r[4]) if v.lower() == "active"})
    return {"sm_mhz": statistics.median(r[1] for r in loaded), "sm_max_mhz": max(r[2] for r in rows),
            "reasons": reasons, "samples": len(loaded), "span": span}


def make_cpu_pipeline(oracle, syn, pkg, weights, workload):
    """The reference's CPU path restated (oracle): one utterance in, tokens
    (or the pooler) out, every stage on all host cores."""
    enc = oracle.OracleEncoder(weights, N_LAYERS)
    dec = oracle.OracleTdt(weights) if workload in ("audio", "transcribe") else None
    fb = oracle.mel_filters() if workload == "audio" else None

    def run(x):
        if workload == "audio":
            mel, nv = oracle.mel(np.concatenate([np.zeros(4000, np.float32), x]), fb)
            x = oracle.subsample(mel, nv, weights)
        pooled = enc.encode(x)
        if dec is not None:
            dec.decode(pooled)

    return run


def cpu_input(syn, rng, workload, secs, frames):
    return syn.synth_audio(rng, secs) if workload == "audio" else syn.sub_features(rng, frames)


def cpu_baseline_sample(oracle, syn, pkg, weights, secs, frames, budget_s, seed, workload):
    """The oracle (restated reference CPU pipeline, all host cores) on the
    first utterances of the batch, in turn, until the time budget is spent."""
    run = make_cpu_pipeline(oracle, syn, pkg, weights, workload)
    rng = np.random.default_rng(seed)
    done_audio, used, n = 0.0, 0.0, 0
    for s, t in zip(secs, frames):
        x = cpu_input(syn, rng, workload, s, t)
        t0 = time.perf_counter()
        run(x)
        used += time.perf_counter() - t0
        done_audio += s
        n += 1
        if used >= budget_s:
            break
    return done_audio / used, n, done_audio, used


def make_weights(args, syn):
    weights = syn.encoder_weights(seed=args.seed, n_layers=N_LAYERS, layout="lut4")
    if args.workload in ("audio", "transcribe"):
        weights.update(syn.decoder_weights(seed=args.seed, vocab=VOCAB))
    if args.workload == "audio":
        weights.update(syn.frontend_weights(seed=args.seed))
    return weights


def host_threads() -> int:
    """Every host core this process may run on (the reference's CPU path
    runs on all of them, rayon's default)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU pipeline (restated in C, all host
    cores) on the utterances of the same batch, one utterance per step,
    cycling through the first --ref-utterances of the batch.  Only rank 0
    runs; the oracle library is the only native code it loads."""
    if rank != 0:
        return
    pkg = load_package()          # the package's pure-Python helpers; its CUDA library is never loaded here
    import bark3_b200.synthetic as syn
    oracle = load_oracle()
    oracle.set_threads(host_threads())   # torchrun sets OMP_NUM_THREADS=1 for every rank
    secs, frames = job_batch(args, world, syn)
    weights = make_weights(args, syn)
    one = make_cpu_pipeline(oracle, syn, pkg, weights, args.workload)
    rng = np.random.default_rng(args.seed)
    k = max(1, min(len(frames), args.ref_utterances))
    subs = [cpu_input(syn, rng, args.workload, secs[i], frames[i]) for i in range(k)]

    for w in range(args.warmup):
        one(subs[w % len(subs)])
    audio, wall = 0.0, 0.0
    for k in range(args.steps):
        i = k % len(subs)
        t0 = time.perf_counter()
        one(subs[i])
        wall += time.perf_counter() - t0
        audio += secs[i]
    v = audio / wall
    cores = oracle.threads()
    sample = (f"{args.steps} utterances, cycling the first {len(subs)} of the batch "
              f"({sum(secs[:len(subs)]):.1f} audio-s, {min(secs[:len(subs)]):.1f}-{max(secs[:len(subs)]):.1f} s), "
              f"one per step, {args.workload} pipeline on {cores} host threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "audio-s/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * wall / args.steps, 3),
        "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": job_config(args, world, syn),
        "reference_path": {"audio": "src/mel.rs + src/sub.rs + src/cpu/* encoder + src/tdt.rs greedy TDT",
                           "transcribe": "src/cpu/* encoder + src/tdt.rs greedy TDT",
                           "encoder": "src/cpu/* encoder"}[args.workload]
                          + ", restated in C (oracle/), AVX2/F16C FMA",
        "cpu_baseline": {"value": round(v, 3), "unit": "audio-s/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(v, 3), "unit": "audio-s/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.workload == "linear":
        if rank == 0:
            run_linear_sweep(args)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))

    pkg = load_package()
    import bark3_b200.synthetic as syn

    secs, frames = batch_for_rank(args, rank, world, pkg, syn)
    M = int(sum(frames))
    cu = np.concatenate([[0], np.cumsum(frames)]).astype(np.int32)
    audio = float(sum(secs))

    decode = args.workload in ("audio", "transcribe")
    audio_in = args.workload == "audio"
    weights = make_weights(args, syn)
    enc = pkg.Encoder(local)
    enc.load(weights)
    enc.finalize(N_LAYERS)

    # inputs: pinned host copy (e2e) and device-resident copy (value)
    rng = np.random.default_rng(args.seed + 17 * rank)
    if audio_in:
        waves = [syn.synth_audio(rng, s) for s in secs]
        soff = np.concatenate([[0], np.cumsum([len(x) for x in waves])]).astype(np.int64)
        host_in = torch.empty((int(soff[-1]),), dtype=torch.float32, pin_memory=True)
        hv = host_in.numpy()
        for i, x in enumerate(waves):
            hv[soff[i]:soff[i + 1]] = x
        del waves
    else:
        host_in = torch.empty((M, 4096), dtype=torch.float32, pin_memory=True)
        hv = host_in.numpy()
        for i in range(len(frames)):
            hv[cu[i]:cu[i + 1]] = syn.sub_features(rng, frames[i])
    host_out = torch.empty((M, 640), dtype=torch.float32, pin_memory=True)
    dev_in = host_in.cuda()
    dev_out = torch.empty((M, 640), dtype=torch.float32, device="cuda")
    n_utt = len(frames)
    dev_tok = torch.zeros((n_utt, MAX_TOKENS, 3), dtype=torch.int32, device="cuda")
    dev_cnt = torch.zeros(n_utt, dtype=torch.int32, device="cuda")
    host_tok = np.zeros((n_utt, MAX_TOKENS, 3), dtype=np.uint32)
    host_cnt = np.zeros(n_utt, dtype=np.int32)
    torch.cuda.synchronize()
    stream = torch.cuda.ExternalStream(enc.stream)
    L = pkg.lib()

    def step_device():
        if audio_in:
            pkg.check(L.b3_transcribe_audio(enc.ctx, dev_in.data_ptr(), soff.ctypes.data, n_utt, dev_tok.data_ptr(),
                                            dev_cnt.data_ptr(), MAX_TOKENS, pkg.B3_DEVICE_PTRS))
        elif decode:
            pkg.check(L.b3_transcribe_batch(enc.ctx, dev_in.data_ptr(), cu.ctypes.data, n_utt, dev_tok.data_ptr(),
                                            dev_cnt.data_ptr(), MAX_TOKENS, pkg.B3_DEVICE_PTRS))
        else:
            enc.encode_batch(dev_in, cu, out=dev_out)

    def step_host(hin, hout):
        if audio_in:
            pkg.check(L.b3_transcribe_audio(enc.ctx, hin.ctypes.data, soff.ctypes.data, n_utt, host_tok.ctypes.data,
                                            host_cnt.ctypes.data, MAX_TOKENS, 0))
        elif decode:
            pkg.check(L.b3_transcribe_batch(enc.ctx, hin.ctypes.data, cu.ctypes.data, n_utt, host_tok.ctypes.data,
                                            host_cnt.ctypes.data, MAX_TOKENS, 0))
        else:
            enc.encode_batch(hin, cu, out=hout)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ── value: device-resident inputs ──
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(local).__enter__()   # already sampling when the timed steps start
    atexit.register(clk.__exit__, None, None, None)   # stopped on any exit path
    for _ in range(args.warmup):
        step_device()
    enc.sync()
    L.b3_profile(enc.ctx, 1)
    barrier()
    torch.cuda.synchronize()
    enc.sync()
    t_wall0 = time.time()
    ev0.record(stream)
    for _ in range(args.steps):
        step_device()
    ev1.record(stream)
    enc.sync()
    torch.cuda.synchronize()
    clk.mark(t_wall0, time.time())
    ms = ev0.elapsed_time(ev1)
    prof = {}
    import ctypes
    for kind, name in enumerate(KINDS):
        a, f, b, n = ctypes.c_double(), ctypes.c_double(), ctypes.c_double(), ctypes.c_int64()
        pkg.check(L.b3_profile_read(enc.ctx, kind, ctypes.byref(a), ctypes.byref(f), ctypes.byref(b), ctypes.byref(n)))
        prof[name] = {"ms": a.value, "flops": f.value, "bytes": b.value, "launches": n.value}
    L.b3_profile(enc.ctx, 0)
    launches = int(sum(p["launches"] for p in prof.values()))
    ms_max = max_over_ranks(ms)
    # whole-job audio: every rank's share (strong: the one batch; weak: N batches)
    tot = torch.tensor([audio], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(tot)
    job_audio = float(tot.item())
    value = job_audio * args.steps / (ms_max / 1000.0)
    # ── e2e: host buffers through the host-pointer ABI call ──
    barrier()
    hin, hout = host_in.numpy(), host_out.numpy()
    step_host(hin, hout)  # warm the staging buffers
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step_host(hin, hout)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e_value = job_audio * args.steps / (e2e_ms / 1000.0)
    clk.__exit__(None, None, None)
    clocks = clk.summary()

    # per-rank attribution: step time, clocks and the per-kind split of every rank
    mine = {"rank": rank, "utterances": n_utt, "frames": M, "audio_s": round(audio, 1),
            "longest_frames": int(max(frames)) if frames else 0,
            "ms_per_step": round(ms / args.steps, 3), "sm_mhz": clocks.get("sm_mhz"),
            "reasons": clocks.get("reasons"),
            "kernels_ms_per_step": {k: round(v["ms"] / args.steps, 3) for k, v in prof.items() if v["launches"]}}
    ranks = [None] * world
    if world > 1:
        dist.all_gather_object(ranks, mine)
    else:
        ranks = [mine]

    pk, pk_kind = peaks()
    g = prof["gemm_lut4"]
    achieved = g["flops"] / (g["ms"] / 1000.0) / 1e12 if g["ms"] > 0 else None
    peak = pk.get("bf16_tflops_sustained") or pk.get("bf16_tflops")
    traffic_file = ROOT / "profiles" / "k1_gemm_lut4_traffic.json"
    traffic = json.loads(traffic_file.read_text()).get("bytes_per_launch") if traffic_file.exists() else None

    sweep = None
    if rank == 0 and world == 1 and not args.no_sweep:
        rows, peak_src = k1_sweep(pkg, syn, enc, SWEEP_SHAPES[:5], 3, 10, args.seed)
        sweep = {"kernel": "k1 LUT4 linear alone (b3_linear_lut4, device pointers)", "peak": peak_src,
                 "shapes": rows}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        oracle = load_oracle()
        oracle.set_threads(host_threads())
        v, n, a_s, used = cpu_baseline_sample(oracle, syn, pkg, weights, secs, frames, args.cpu_seconds, args.seed,
                                              args.workload)
        cpu = {"value": round(v, 3), "unit": "audio-s/s", "cores": oracle.threads(), "kind": "port",
               "sample": f"first {n} utterances of the batch ({a_s:.1f} audio-s, {used:.1f} s wall), "
                         + args.workload + " pipeline, in turn"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "audio-s/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 3),
            "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
            "dtype": "f16", "data": "synthetic",
            "config": job_config(args, world, syn),
            "roofline": {"kernel": "k1_gemm (LUT4, tcgen05)", "bound": "tensor",
                         "achieved": round(achieved, 1) if achieved else None,
                         "peak": peak, "unit": "TFLOP/s",
                         "frac": round(achieved / peak, 4) if achieved else None,
                         "peak_source": f"bf16_tflops_sustained of {pk_kind}",
                         "traffic": traffic,
                         "launches": g["launches"], "gemm_ms_share": round(g["ms"] / ms, 4) if ms else None},
            "kernels": {k: {"ms_per_step": round(v["ms"] / args.steps, 3),
                            "TFLOP/s": round(v["flops"] / v["ms"] / 1e9, 1) if v["ms"] and v["flops"] else None,
                            "GB/s": round(v["bytes"] / v["ms"] / 1e6, 1) if v["ms"] else None,
                            "launches": v["launches"]} for k, v in prof.items() if v["launches"]},
            "gpu_launches": launches,
            "clocks": clocks,
            "ranks": ranks,
            "e2e": {"value": round(e2e_value, 2), "unit": "audio-s/s",
                    "h2d_bytes_per_step": int(host_in.numel() * 4),
                    "d2h_bytes_per_step": int(n_utt * (MAX_TOKENS * 12 + 4)) if decode else int(M * 640 * 4),
                    "bytes_are": "rank 0's per step"},
            "cpu_baseline": cpu,
            "k1_sweep": sweep,
        }
        if args.shard:
            line["emulated_shard"] = (f"rank {args.shard.split(':')[0]} of a {args.shard.split(':')[1]}-GPU "
                                      "strong-scaling job, timed alone on one GPU: value is that share's "
                                      "throughput, not a whole-job number")
        print(json.dumps(line), flush=True)
    enc.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
