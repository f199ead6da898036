#!/usr/bin/env python
"""Benchmark: RTF^-1 (seconds of output audio per wall-second) of the RVC
VITS synthesizer on B200: v2-48k SynthesizerTrnMs768NSFsid,
256 independent 10 s chunks (1000 frames -> 480000 samples each) sharded
evenly by chunk across the ranks, no collective on the data path.

    python bench.py [--gpus N --steps K --warmup W]           # our CUDA path
    python bench.py --impl reference ...                      # reference CPU arm

A step is one pass of the synthesizer over the rank's share of the 256 chunks
(groups of --group chunks per library call).  `value` is timed with inputs
already resident in HBM; `e2e` runs the same step through the public API
(`CudaSynthesizer.infer_batch`) from pinned host buffers, host<->device copies
included.  The reference arm times the reference's own numpy code (its
``runtime`` package, copied into the git-ignored ``oracle/_ref`` by
``make -C oracle ref``, which travels with the working tree) on a bounded
sample of the same workload, on the host cores; without that copy it times the
oracle port.  The line also carries BASELINE config 0 (one 10 s v2-40k chunk
per call) measured the same way, under ``config0``.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "rvc-vulkan_b200"))

import numpy as np  # noqa: E402

METRIC = "seconds of output audio per wall-second (RTF^-1)"
UNIT = "audio-s/s"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p["bf16_tflops_sustained"]), float(p["hbm_gbs"]), "measured"
    except Exception:  # noqa: BLE001
        return 1590.0, 1400.0, 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:  # noqa: BLE001
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 8:
                self.rows.append(parts)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:  # noqa: BLE001
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[4 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def make_inputs(n_unique, P, upp, sr_seed=0):
    from rvc_cuda import synthetic as syn
    ins = [syn.make_vits_inputs(P, 1000 + i) for i in range(n_unique)]
    noise = [syn.make_vits_noise(P, upp, 5000 + i) for i in range(n_unique)]
    return ins, noise


def _reference():
    """The reference's own numpy runtime (the git-ignored ``oracle/_ref`` copy,
    made by ``make -C oracle ref``), or None where it is absent; the CPU legs
    then time the oracle port instead."""
    from oracle import reference as oref
    if os.environ.get("RVC_BENCH_CPU", "") == "port" or not oref.available():
        return None
    oref.activate("numpy")
    return oref


def cpu_kind():
    return "reference" if _reference() is not None else "port"


def cpu_what():
    return ("the reference's own numpy code (runtime/, RVC_BACKEND=numpy)" if cpu_kind() == "reference"
            else "CPU oracle (numpy restatement of the reference's numpy backend)")


_REF_MODELS: dict = {}


def cpu_sample(sr, P, w, cfg, steps=1):
    """Time the synthesizer on the host cores on one chunk of P frames: the
    reference's ``SynthesizerTrn.infer_controlled`` (``runtime/models/vits.py:2551``)
    when its runtime is available, else the oracle port."""
    from rvc_cuda import synthetic as syn
    ref = _reference()
    upp = int(np.prod(cfg[12]))
    phone, pitch, nsff0, sid = syn.make_vits_inputs(P, 1)
    nz, ns = syn.make_vits_noise(P, upp, 2)
    if ref is not None:
        key = ("synth", sr)
        if key not in _REF_MODELS:
            _REF_MODELS[key] = ref.synthesizer(w, cfg)
        net = _REF_MODELS[key]
        fn = lambda: net.infer_controlled(phone, pitch, nsff0, sid, nz, ns)  # noqa: E731
    else:
        from oracle import vits as OV
        fn = lambda: OV.synth(w, cfg, phone, pitch, nsff0, sid, nz, ns)  # noqa: E731
    ts = []
    for _ in range(steps):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return P * upp / sr, ts


def blas_threads():
    try:
        import threadpoolctl
        return max(i.get("num_threads", 1) for i in threadpoolctl.threadpool_info())
    except Exception:  # noqa: BLE001
        return os.cpu_count() or 1


def synth_config(args, world):
    """The config-3 workload's description, shared by the device arm and the
    reference arm (the reference arm times bounded samples of it)."""
    from rvc_cuda import synthetic as syn
    sr, P = args.sr, args.frames
    upp = int(np.prod(syn.vits_config_array(sr)[12]))
    return {"workload": f"config3 v2-{sr // 1000}k synthesizer, {args.chunks} chunks x {P} frames "
                        f"({P * upp / sr:.0f} s each), sharded by chunk",
            "chunks": args.chunks, "frames": P, "sr": sr, "group": args.group, "precision": args.precision,
            "l2": "inputs larger than L2 (GBs per step)",
            "parallelism": f"chunk-sharded x{world}, no collective"}


def run_reference(args, world, rank):
    if rank != 0:
        return
    from rvc_cuda import synthetic as syn
    w = syn.make_vits_weights(args.sr, 0)
    cfg = syn.vits_config_array(args.sr)
    audio_s, _ = cpu_sample(args.sr, args.ref_frames, w, cfg, steps=args.warmup)
    _, ts = cpu_sample(args.sr, args.ref_frames, w, cfg, steps=args.steps)
    t = sum(ts)
    value = audio_s * len(ts) / t
    cores = blas_threads()
    sample = (f"1 chunk of {args.ref_frames} frames ({audio_s:.2f} s audio) per step of the config-3 "
              f"workload (one of its {args.chunks} chunks), v2-{args.sr // 1000}k, " + cpu_what())
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t / len(ts), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": synth_config(args, world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": cpu_kind(), "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def hubert_cpu_sample(T, steps=1):
    """Time HuBERT-base on the host cores on one chunk: the reference's
    ``HubertEncoder.encode`` (``runtime/models/hubert.py:564``) when available,
    else the oracle port."""
    from rvc_cuda import synthetic as syn
    x = syn.make_hubert_input(T, 1)
    ref = _reference()
    if ref is not None:
        if "hubert" not in _REF_MODELS:
            _REF_MODELS["hubert"] = ref.hubert(syn.make_hubert_weights(0))
        enc = _REF_MODELS["hubert"]
        fn = lambda: enc.encode(x, version=2)  # noqa: E731
    else:
        from oracle import hubert as OH
        sd = OH.prepare(syn.make_hubert_weights(0))
        fn = lambda: OH.encode(sd, x)  # noqa: E731
    ts = []
    for _ in range(steps):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return T / 16000.0, ts


def run_hubert(args, world, rank, local):
    """HuBERT-base over chunks of --samples 16 kHz samples."""
    import torch

    from rvc_cuda import _lib, synthetic as syn
    from rvc_cuda.hubert import CudaHubert, out_len

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    T, G = args.samples, args.group
    m = CudaHubert(syn.make_hubert_weights(0), device=local, precision=args.precision)
    ctx = m.ctx
    L = out_len(T)
    assert args.chunks % world == 0, "chunks must split evenly across ranks"
    n_local = args.chunks // world
    n_unique = min(args.unique, n_local)
    xs = [syn.make_hubert_input(T, 100 + i)[0] for i in range(n_unique)]
    h_x = torch.empty((n_local, T), dtype=torch.float32, pin_memory=True).numpy()
    h_y = torch.empty((n_local, L, 768), dtype=torch.float32, pin_memory=True).numpy()
    for j in range(n_local):
        h_x[j] = xs[(rank * n_local + j) % n_unique]
    d_x = ctx.alloc(h_x.nbytes)
    ctx.h2d(d_x, h_x)
    d_y = ctx.alloc(h_y.nbytes)
    groups = [(s, min(G, n_local - s)) for s in range(0, n_local, G)]

    def step_device():
        for s, g in groups:
            _lib.check(_lib.lib.rvc_cuda_hubert_encode_device(m.handle, g, T, _lib._p(d_x + s * T * 4), 2,
                                                              _lib._p(d_y + s * L * 768 * 4)))

    def step_e2e():
        for s, g in groups:
            h_y[s:s + g] = m.encode_equal(h_x[s:s + g])

    stream = torch.cuda.ExternalStream(ctx.stream(), device=local)

    def timed(fn, steps):
        barrier()
        ctx.sync()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        ctx.sync()
        torch.cuda.synchronize()
        barrier()
        return e0.elapsed_time(e1) / 1e3

    for _ in range(args.warmup):
        step_device()
    ctx.sync()
    n0 = _lib.launch_count()
    with ClockSampler(local) as clk:
        t = timed(step_device, args.steps)
    launches = _lib.launch_count() - n0
    # per-launch kernel times for the roofline: a separate pass of the same steps
    # (the events and labels cost host time, so they stay out of the timed region)
    ctx.profile(True)
    timed(step_device, args.steps)
    prof_n, prof_ms, prof_flops = ctx.profile_read()
    if args.profile_out and rank == 0:
        with open(args.profile_out, "w") as f:
            f.write(ctx.profile_dump())
    ctx.profile(False)
    t = max_over_ranks(t)
    audio_per_step = args.chunks * T / 16000.0
    value = audio_per_step * args.steps / t
    step_e2e()
    te = max_over_ranks(timed(step_e2e, args.steps))
    e2e = audio_per_step * args.steps / te
    if rank == 0:
        pb, ps, hbm, src = peaks()
        achieved = prof_flops / (prof_ms / 1e3) / 1e12 if prof_ms > 0 else None
        line = {
            "metric": "seconds of input audio encoded per wall-second (HuBERT-base)", "value": value,
            "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * t / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f32 (BF16x3 split on tcgen05, fp32 accumulate)" if args.precision == "bf16x3" else "f32",
            "data": f"synthetic: seeded random-init weights, {n_unique} distinct seeded chunks tiled",
            "config": {"workload": f"config1 HuBERT-base, {args.chunks} chunks x {T} samples -> [{L},768], "
                                   "sharded by chunk", "chunks": args.chunks, "samples": T, "group": G,
                       "precision": args.precision, "l2": "inputs larger than L2",
                       "parallelism": f"chunk-sharded x{world}, no collective"},
            "roofline": {"bound": "tensor", "kernel": "tc_conv_kernel (GEMMs and convs, all launches)",
                         "achieved": achieved, "peak": ps, "unit": "TFLOP/s",
                         "frac": (achieved / ps) if achieved else None, "traffic": None,
                         "peak_source": f"{src} bf16 dense sustained",
                         "note": "useful fp32 FLOPs / tensor-core kernel time; BF16x3 => frac <= 1/3",
                         "launches": prof_n, "kernel_ms_per_step": prof_ms / args.steps},
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": h_x.nbytes * world,
                    "d2h_bytes_per_step": h_y.nbytes * world},
            "gpu_launches": launches,
            "clocks": clk.summary(),
            "finite": bool(np.isfinite(h_y).all()),
        }
        if world == 1 and not args.no_cpu:
            audio_s, ts = hubert_cpu_sample(T, steps=1)
            line["cpu_baseline"] = {"value": audio_s / ts[0], "unit": UNIT, "cores": blas_threads(), "kind": cpu_kind(),
                                    "sample": f"1 chunk of {T} samples ({audio_s:.1f} s audio), " + cpu_what()}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def retrieval_cpu_sample(N, D, F, steps=1):
    """Time the retrieval stage on the host cores on F queries: top-8 L2
    search (the reference's ``runtime.retrieval.search_l2``, ``runtime/retrieval.py:35-82``,
    when available, else the oracle port) and the pipeline's (1/d)^2 blend."""
    from oracle import retrieval as OR
    from rvc_cuda import synthetic as syn
    db = syn.make_index(N, D, 0)
    q = syn.make_queries(F, D, 1)
    ref = _reference()
    if ref is not None:
        from runtime.retrieval import search_l2

        def fn():
            sc, ix = search_l2(q, db, k=8)
            w = np.square(1.0 / sc)
            w /= w.sum(axis=1, keepdims=True)
            return np.sum(db[ix] * np.expand_dims(w, axis=2), axis=1)
    else:
        fn = lambda: OR.blend(q, db, 8)  # noqa: E731
    ts = []
    for _ in range(steps):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return F / 50.0, ts


def run_retrieval(args, world, rank, local):
    """BASELINE config 4's retrieval stage: F = 50 frames/s x --audio-s queries
    against a --index-rows x 768 index, top-8 + inverse-squared-distance blend + mix."""
    import torch

    from rvc_cuda import _lib, synthetic as syn
    from rvc_cuda.retrieval import CudaIndex

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    N, D = args.index_rows, 768
    F_total = int(round(args.audio_s * 50))
    assert F_total % world == 0, "queries must split evenly across ranks"
    F = F_total // world
    db = syn.make_index(N, D, 0)
    idx = CudaIndex(db, device=local, precision=args.precision)
    ctx = idx.ctx
    h_q = torch.empty((F, D), dtype=torch.float32, pin_memory=True).numpy()
    h_f = torch.empty((F, D), dtype=torch.float32, pin_memory=True).numpy()
    h_o = torch.empty((F, D), dtype=torch.float32, pin_memory=True).numpy()
    h_q[:] = syn.make_queries(F, D, 1 + rank)
    h_f[:] = syn.make_queries(F, D, 100 + rank)
    d_q, d_f, d_o = ctx.alloc(h_q.nbytes), ctx.alloc(h_f.nbytes), ctx.alloc(h_o.nbytes)
    ctx.h2d(d_q, h_q)
    ctx.h2d(d_f, h_f)

    def step_device():
        _lib.check(_lib.lib.rvc_cuda_index_blend_device(idx.handle, _lib._p(d_q), F, D, 8, 0, 0.75, _lib._p(d_f),
                                                        _lib._p(d_o)))

    def step_e2e():
        h_o[:] = idx.blend(h_q, 8, feats=h_f, index_rate=0.75)

    stream = torch.cuda.ExternalStream(ctx.stream(), device=local)

    def timed(fn, steps):
        barrier()
        ctx.sync()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        ctx.sync()
        torch.cuda.synchronize()
        barrier()
        return e0.elapsed_time(e1) / 1e3

    for _ in range(args.warmup):
        step_device()
    ctx.sync()
    n0 = _lib.launch_count()
    with ClockSampler(local) as clk:
        t = timed(step_device, args.steps)
    launches = _lib.launch_count() - n0
    # per-launch kernel times for the roofline: a separate pass of the same steps
    # (the events and labels cost host time, so they stay out of the timed region)
    ctx.profile(True)
    timed(step_device, args.steps)
    prof_n, prof_ms, prof_flops = ctx.profile_read()
    if args.profile_out and rank == 0:
        with open(args.profile_out, "w") as f:
            f.write(ctx.profile_dump())
    ctx.profile(False)
    t = max_over_ranks(t)
    audio_per_step = F_total / 50.0
    value = audio_per_step * args.steps / t
    step_e2e()
    te = max_over_ranks(timed(step_e2e, args.steps))
    if rank == 0:
        pb, ps, hbm, src = peaks()
        achieved = prof_flops / (prof_ms / 1e3) / 1e12 if prof_ms > 0 else None
        line = {
            "metric": "seconds of audio retrieved per wall-second (top-8 L2 search + blend)", "value": value,
            "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * t / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32 (BF16x3 GEMM on tcgen05 + float64 re-rank)",
            "data": "synthetic: index and queries ~N(0,1), seeded",
            "config": {"workload": f"config4 retrieval stage: {F_total} queries ({args.audio_s:g} s of frames) "
                                   f"x {N} x {D} index, top-8, blend, index_rate 0.75",
                       "queries": F_total, "index_rows": N, "dim": D, "precision": args.precision,
                       "l2": "index (614 MB) larger than L2",
                       "parallelism": f"queries sharded x{world}, index replicated, no collective"},
            "roofline": {"bound": "tensor", "kernel": "tc_conv_kernel (q . d GEMM)", "achieved": achieved,
                         "peak": ps, "unit": "TFLOP/s", "frac": (achieved / ps) if achieved else None,
                         "traffic": None, "peak_source": f"{src} bf16 dense sustained",
                         "note": "useful 2*F*N*D FLOPs / GEMM time; BF16x3 => frac <= 1/3",
                         "launches": prof_n, "kernel_ms_per_step": prof_ms / args.steps},
            "e2e": {"value": audio_per_step * args.steps / te, "unit": UNIT,
                    "h2d_bytes_per_step": 2 * h_q.nbytes * world, "d2h_bytes_per_step": h_o.nbytes * world},
            "gpu_launches": launches,
            "clocks": clk.summary(),
            "finite": bool(np.isfinite(h_o).all()),
        }
        if world == 1 and not args.no_cpu:
            audio_s, ts = retrieval_cpu_sample(N, D, 500, steps=1)
            line["cpu_baseline"] = {"value": audio_s / ts[0], "unit": UNIT, "cores": blas_threads(), "kind": cpu_kind(),
                                    "sample": f"500 queries ({audio_s:g} s of frames) x {N} x {D}, " + cpu_what()}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def run_retrieval_reference(args, world, rank):
    if rank != 0:
        return
    retrieval_cpu_sample(args.index_rows, 768, 500, steps=max(1, min(args.warmup, 1)))
    audio_s, ts = retrieval_cpu_sample(args.index_rows, 768, 500, steps=args.steps)
    t = sum(ts)
    value = audio_s * len(ts) / t
    line = {
        "impl": "reference", "metric": "seconds of audio retrieved per wall-second (top-8 L2 search + blend)",
        "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * t / len(ts), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded)",
        "config": {"workload": "config4 retrieval stage, CPU sample", "queries": 500, "index_rows": args.index_rows},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": blas_threads(), "kind": cpu_kind(),
                         "sample": f"500 queries per step x {args.index_rows} x 768, " + cpu_what()},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def rmvpe_cpu_sample(T, steps=1):
    """Time RMVPE on the host cores on one clip: the reference's
    ``RMVPE.infer_from_audio`` (``runtime/models/rmvpe.py:927``) when available,
    else the oracle port."""
    from rvc_cuda import synthetic as syn
    sd = syn.make_rmvpe_weights(0)
    x = syn.make_rmvpe_input(T, 1)
    ref = _reference()
    if ref is not None:
        if "rmvpe" not in _REF_MODELS:
            _REF_MODELS["rmvpe"] = ref.rmvpe(sd)
        m = _REF_MODELS["rmvpe"]
        fn = lambda: m.infer_from_audio(x)  # noqa: E731
    else:
        from oracle import rmvpe as ORM
        fn = lambda: ORM.infer(sd, x)  # noqa: E731
    ts = []
    for _ in range(steps):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return T / 16000.0, ts


def run_rmvpe(args, world, rank, local):
    """RMVPE over clips of --samples 16 kHz samples."""
    import torch

    from rvc_cuda import _lib, synthetic as syn
    from rvc_cuda.rmvpe import CudaRmvpe, frames

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    T, G = args.samples, args.group
    m = CudaRmvpe(syn.make_rmvpe_weights(0), device=local)
    ctx = m.ctx
    F = frames(T)
    assert args.chunks % world == 0, "chunks must split evenly across ranks"
    n_local = args.chunks // world
    n_unique = min(args.unique, n_local)
    xs = [syn.make_rmvpe_input(T, 100 + i) for i in range(n_unique)]
    h_x = torch.empty((n_local, T), dtype=torch.float32, pin_memory=True).numpy()
    h_f = torch.empty((n_local, F), dtype=torch.float32, pin_memory=True).numpy()
    for j in range(n_local):
        h_x[j] = xs[(rank * n_local + j) % n_unique]
    d_x, d_f = ctx.alloc(h_x.nbytes), ctx.alloc(h_f.nbytes)
    ctx.h2d(d_x, h_x)
    groups = [(s, min(G, n_local - s)) for s in range(0, n_local, G)]

    def step_device():
        for s, g in groups:
            _lib.check(_lib.lib.rvc_cuda_rmvpe_infer_device(m.handle, g, T, _lib._p(d_x + s * T * 4), 0.03,
                                                            _lib._p(d_f + s * F * 4), None))

    def step_e2e():
        for s, g in groups:
            h_f[s:s + g] = m.infer_batch(h_x[s:s + g])

    stream = torch.cuda.ExternalStream(ctx.stream(), device=local)

    def timed(fn, steps):
        barrier()
        ctx.sync()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        ctx.sync()
        torch.cuda.synchronize()
        barrier()
        return e0.elapsed_time(e1) / 1e3

    for _ in range(args.warmup):
        step_device()
    ctx.sync()
    n0 = _lib.launch_count()
    with ClockSampler(local) as clk:
        t = timed(step_device, args.steps)
    launches = _lib.launch_count() - n0
    if args.profile_out:  # per-layer times: a separate pass, outside the timed region
        ctx.profile(True)
        timed(step_device, args.steps)
        if rank == 0:
            with open(args.profile_out, "w") as f:
                f.write(ctx.profile_dump())
        ctx.profile(False)
    t = max_over_ranks(t)
    audio_per_step = args.chunks * T / 16000.0
    value = audio_per_step * args.steps / t
    step_e2e()
    te = max_over_ranks(timed(step_e2e, args.steps))
    if rank == 0:
        pb, ps, hbm, src = peaks()
        # fp32 SIMT network: roofline against the fp32 CUDA-core peak (148 SMs x 128 FMA/clk x 2 x max clock)
        fp32_peak = 148 * 128 * 2 * 1.965e9 / 1e12
        gflop_chunk = rmvpe_gflop(T)
        achieved = gflop_chunk * args.chunks * args.steps / t / 1e3
        line = {
            "metric": "seconds of input audio pitch-tracked per wall-second (RMVPE)", "value": value,
            "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * t / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32 (float64 STFT)",
            "data": f"synthetic: seeded random-init weights, {n_unique} distinct seeded clips tiled",
            "config": {"workload": f"config2 RMVPE, {args.chunks} clips x {T} samples -> {F} frames, sharded by clip",
                       "chunks": args.chunks, "samples": T, "group": G, "l2": "inputs larger than L2",
                       "parallelism": f"clip-sharded x{world}, no collective"},
            "roofline": {"bound": "fp32 SIMT", "kernel": "whole step (U-Net convs dominate)", "achieved": achieved,
                         "peak": fp32_peak, "unit": "TFLOP/s", "frac": achieved / fp32_peak, "traffic": None,
                         "peak_source": "nominal fp32 FMA peak at max clock (no measured fp32 figure)",
                         "note": f"{gflop_chunk:.1f} GFLOP of convs/GEMMs per clip over the step time"},
            "e2e": {"value": audio_per_step * args.steps / te, "unit": UNIT,
                    "h2d_bytes_per_step": h_x.nbytes * world, "d2h_bytes_per_step": h_f.nbytes * world},
            "gpu_launches": launches,
            "clocks": clk.summary(),
            "finite": bool(np.isfinite(h_f).all()),
        }
        if world == 1 and not args.no_cpu:
            audio_s, ts = rmvpe_cpu_sample(T, steps=1)
            line["cpu_baseline"] = {"value": audio_s / ts[0], "unit": UNIT, "cores": blas_threads(), "kind": cpu_kind(),
                                    "sample": f"1 clip of {T} samples ({audio_s:.1f} s audio), " + cpu_what()}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def rmvpe_gflop(T):
    """Algorithmic GFLOP of one RMVPE clip: every conv / convT (useful taps) / GEMM."""
    from rvc_cuda import synthetic as syn
    F = 1 + T // 160
    Fp = 32 * ((F - 1) // 32 + 1)
    fl = 0.0
    for l, (ci, co) in enumerate(syn.RMVPE_ENC):
        px = (Fp >> l) * (128 >> l)
        for j in range(4):
            cin = ci if j == 0 else co
            fl += 2 * px * 9 * (cin * co + co * co) + (2 * px * cin * co if cin != co else 0)
    px = (Fp >> 5) * 4
    for i, (ci, co) in enumerate(syn.RMVPE_INTER):
        for j in range(4):
            cin = ci if j == 0 else co
            fl += 2 * px * 9 * (cin * co + co * co) + (2 * px * cin * co if cin != co else 0)
    for i, (ci, co) in enumerate(syn.RMVPE_DEC):
        l = 4 - i
        px = (Fp >> l) * (128 >> l)
        fl += 2 * px * ci * co * 2.25
        for j in range(4):
            cin = 2 * co if j == 0 else co
            fl += 2 * px * 9 * (cin * co + co * co) + (2 * px * cin * co if cin != co else 0)
    fl += 2 * Fp * 128 * 9 * 16 * 3 + 2 * Fp * 384 * 1536 + 2 * 2 * Fp * 768 * 256 + 2 * Fp * 512 * 360
    return fl / 1e9


def run_rmvpe_reference(args, world, rank):
    if rank != 0:
        return
    T = args.samples
    rmvpe_cpu_sample(T, steps=1)
    audio_s, ts = rmvpe_cpu_sample(T, steps=args.steps)
    t = sum(ts)
    value = audio_s * len(ts) / t
    line = {
        "impl": "reference", "metric": "seconds of input audio pitch-tracked per wall-second (RMVPE)",
        "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * t / len(ts), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded)",
        "config": {"workload": "config2 RMVPE, CPU sample", "samples": T},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": blas_threads(), "kind": cpu_kind(),
                         "sample": f"1 clip of {T} samples per step, " + cpu_what()},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_hubert_reference(args, world, rank):
    if rank != 0:
        return
    T = args.samples
    hubert_cpu_sample(T, steps=args.warmup)
    audio_s, ts = hubert_cpu_sample(T, steps=args.steps)
    t = sum(ts)
    value = audio_s * len(ts) / t
    line = {
        "impl": "reference", "metric": "seconds of input audio encoded per wall-second (HuBERT-base)",
        "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * t / len(ts), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded)",
        "config": {"workload": "config1 HuBERT-base, CPU sample", "samples": T},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": blas_threads(), "kind": cpu_kind(),
                         "sample": f"1 chunk of {T} samples per step, " + cpu_what()},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def pipeline_cpu_estimate(chunk_samples, frames_total, audio_s):
    """CPU time of the config-4 pipeline, composed from bounded samples of each
    stage on the host cores: the reference's models where its runtime is
    available, else the oracle port (HuBERT, RMVPE, v2-40k synthesizer, top-8
    retrieval against the 200000 x 768 index), timed on short inputs and scaled
    by the workload's samples / frames, plus the reference's
    own scipy ``filtfilt`` and the oracle's split / change_rms on the full
    signal.  Returns (seconds per workload, sample description)."""
    from scipy import signal

    from oracle import dsp as OD
    from rvc_cuda import synthetic as syn
    w = syn.make_vits_weights(40000, 0)
    cfg = syn.vits_config_array(40000)
    out_s, ts = cpu_sample(40000, 100, w, cfg, steps=1)
    synth_s = ts[0] / 100 * frames_total
    hs, ts = hubert_cpu_sample(48000, steps=1)
    hub_s = ts[0] / 48000 * chunk_samples
    rs_, ts = rmvpe_cpu_sample(48000, steps=1)
    rmv_s = ts[0] / 48000 * chunk_samples
    qs, tq = retrieval_cpu_sample(200000, 768, 100, steps=1)
    ret_s = tq[0] / 100 * (frames_total // 2)
    a = syn.make_speech_audio(audio_s, seed=0)
    bh, ah = signal.butter(N=5, Wn=48, btype="high", fs=16000)
    t0 = time.perf_counter()
    hp = signal.filtfilt(bh, ah, a)
    OD.split_points(hp, 160, 6 * 16000, 38 * 16000)
    OD.change_rms(hp, np.zeros(int(audio_s * 40000), np.float32) + 0.1, 16000, 40000, 0.25)
    dsp_s = time.perf_counter() - t0
    total = synth_s + hub_s + rmv_s + ret_s + dsp_s
    desc = (f"stage samples scaled to the workload: synth 100 frames -> {frames_total} frames ({synth_s:.1f} s), "
            f"HuBERT 3 s -> {chunk_samples / 16000:.0f} s ({hub_s:.1f} s), RMVPE 3 s -> {chunk_samples / 16000:.0f} s "
            f"({rmv_s:.1f} s), retrieval 100 -> {frames_total // 2} queries ({ret_s:.1f} s), filtfilt/split/"
            f"change_rms on the full signal ({dsp_s:.2f} s)")
    return total, desc


def pipeline_workload(audio_s):
    """Chunk samples (with the pipeline's 1 s pads) and synthesizer frames of a
    conversion of ``audio_s`` seconds under the default config (x_pad 1,
    x_query 6, x_center 38, x_max 41): chunks cut near every 38 s."""
    n = int(audio_s * 16000)
    cuts = list(range(38 * 16000, n, 38 * 16000)) if n + 160 > 41 * 16000 else []
    bounds = [0] + cuts + [n]
    samples = sum(bounds[i + 1] - bounds[i] + 2 * 16000 for i in range(len(bounds) - 1))
    return samples, samples // 160


def run_pipeline(args, world, rank, local):
    """end-to-end conversion of --audio-s seconds of 16 kHz
    speech-like audio through ``rvc_cuda.pipeline.Pipeline`` (high-pass,
    silence split, RMVPE f0, HuBERT, top-8 retrieval against a 200000 x 768
    index at index_rate 0.75, x2 interpolation, protect 0.33, v2-40k
    synthesizer, change_rms 0.25, int16), one clip per rank."""
    import types

    import torch

    from rvc_cuda import _lib, synthetic as syn
    from rvc_cuda.hubert import CudaHubert
    from rvc_cuda.pipeline import Pipeline
    from rvc_cuda.retrieval import CudaIndex
    from rvc_cuda.rmvpe import CudaRmvpe
    from rvc_cuda.synth import CudaSynthesizer

    torch.cuda.set_device(local)
    os.environ.setdefault("RVC_FIXED_SEED", "1234")
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    hub = CudaHubert(syn.make_hubert_weights(0), device=local)
    net = CudaSynthesizer(syn.make_vits_weights(40000, 0), syn.vits_config_array(40000), device=local,
                          precision=args.precision)
    index = CudaIndex(syn.make_index(args.index_rows, 768, 0), device=local)
    cfg = types.SimpleNamespace(x_pad=1, x_query=6, x_center=38, x_max=41, device=f"cuda:{local}")
    pipe = Pipeline(40000, cfg)
    pipe.model_rmvpe = CudaRmvpe(syn.make_rmvpe_weights(0), device=local, own_stream=True)
    audio = syn.make_speech_audio(args.audio_s, seed=rank)
    ctx = hub.ctx
    stage = [0.0, 0.0, 0.0]
    out = {}

    def step():
        sr, wav = pipe.pipeline(hub, net, 0, audio, stage, 0, "rmvpe", index, 0.75, True, 40000, 0, 0.25, 2, 0.33,
                                slice_length=args.slice_length)
        out["wav"] = wav

    stream = torch.cuda.ExternalStream(ctx.stream(), device=local)

    def timed(fn, steps):
        barrier()
        ctx.sync()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        t_wall = time.perf_counter()
        for _ in range(steps):
            fn()
        e1.record(stream)
        ctx.sync()
        torch.cuda.synchronize()
        t_wall = time.perf_counter() - t_wall
        barrier()
        return e0.elapsed_time(e1) / 1e3, t_wall

    for _ in range(args.warmup):
        step()
    stage[:] = [0.0, 0.0, 0.0]
    n0 = _lib.launch_count()
    with ClockSampler(local) as clk:
        t, t_wall = timed(step, args.steps)
    launches = _lib.launch_count() - n0
    stage_timed = list(stage)
    # per-launch tensor-core conv times for the roofline: a separate pass (the
    # events cost host time, which this host-driven pipeline would pay in full)
    ctx.profile(True)
    timed(step, args.steps)
    prof_n, prof_ms, prof_flops = ctx.profile_read()
    ctx.profile(False)
    t = max_over_ranks(t)
    value = world * args.audio_s * args.steps / t
    wav = out["wav"]
    if rank == 0:
        pb, ps, hbm, src = peaks()
        achieved = prof_flops / (prof_ms / 1e3) / 1e12 if prof_ms > 0 else None
        line = {
            "metric": METRIC + ", end-to-end conversion", "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 (BF16x3 tensor-core GEMMs; float64 filtfilt / split)",
            "data": "synthetic: seeded random-init weights, seeded speech-like audio (3 harmonics on a random-walk "
                    "f0 80-300 Hz, pink noise -20 dB, 0.5 s silences every 8 s), one clip per rank",
            "config": {"workload": f"config4 end-to-end pipeline, {args.audio_s:g} s at 16 kHz -> v2-40k, "
                                   f"rmvpe f0, index {args.index_rows}x768 rate 0.75, rms_mix 0.25, protect 0.33",
                       "audio_s": args.audio_s, "index_rows": args.index_rows, "slice_length": args.slice_length,
                       "split": "default config (x_pad 1, x_query 6, x_center 38, x_max 41)",
                       "l2": "working set larger than L2 (index 614 MB, GBs of activations per step)",
                       "parallelism": f"one clip per rank x{world}, no collective"},
            "roofline": {"bound": "tensor", "kernel": "tc_conv_kernel (implicit-GEMM conv/linear, all launches)",
                         "achieved": achieved, "peak": ps, "unit": "TFLOP/s",
                         "frac": (achieved / ps) if achieved else None, "traffic": None,
                         "peak_source": f"{src} bf16 dense sustained", "launches": prof_n,
                         "kernel_ms_per_step": prof_ms / args.steps},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": audio.nbytes * world,
                    "d2h_bytes_per_step": wav.nbytes * world,
                    "note": "the pipeline takes host audio and returns host int16 by contract: value is this "
                            "end-to-end measurement (stage round trips included)"},
            "stage_s_per_step": {"retrieval_interp": stage_timed[0] / args.steps,
                                 "f0": stage_timed[1] / args.steps, "synth": stage_timed[2] / args.steps},
            "host_wall_s_per_step": t_wall / args.steps,
            "gpu_launches": launches,
            "clocks": clk.summary(),
            "out_samples": int(wav.size),
        }
        if world == 1 and not args.no_cpu:
            samples, frames = pipeline_workload(args.audio_s)
            cpu_s, desc = pipeline_cpu_estimate(samples, frames, args.audio_s)
            line["cpu_baseline"] = {"value": args.audio_s / cpu_s, "unit": UNIT, "cores": blas_threads(),
                                    "kind": cpu_kind(), "sample": desc}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def run_pipeline_reference(args, world, rank):
    if rank != 0:
        return
    samples, frames = pipeline_workload(args.audio_s)
    ts, desc = [], ""
    for _ in range(args.steps):
        cpu_s, desc = pipeline_cpu_estimate(samples, frames, args.audio_s)
        ts.append(cpu_s)
    t = sum(ts)
    value = args.audio_s * len(ts) / t
    line = {
        "impl": "reference", "metric": METRIC + ", end-to-end conversion", "value": value, "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t / len(ts),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": {"workload": f"config4 end-to-end pipeline, {args.audio_s:g} s, CPU stage samples",
                   "audio_s": args.audio_s, "index_rows": 200000},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": blas_threads(), "kind": cpu_kind(), "sample": desc},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config0_figure(args, local, timed, max_over_ranks, world):
    """BASELINE config 0, the north star's v2-40k target: one 10 s chunk
    (--frames frames) of the v2-40k synthesizer per library call (B = 1) on
    every rank, timed like the headline (device-resident inputs; then through
    ``CudaSynthesizer.infer_batch`` from pinned host buffers)."""
    import torch

    from rvc_cuda import _lib, synthetic as syn
    from rvc_cuda.synth import CudaSynthesizer
    P = args.frames
    m = CudaSynthesizer(syn.make_vits_weights(40000, 0), syn.vits_config_array(40000), device=local,
                        precision=args.precision)
    ctx, upp = m.ctx, m.upp
    phone, pitch, nsff0, sid = syn.make_vits_inputs(P, 7)
    nz, ns = syn.make_vits_noise(P, upp, 8)

    def pinned(a):
        t = torch.empty(a.shape, dtype={np.float32: torch.float32, np.int64: torch.int64}[a.dtype.type],
                        pin_memory=True).numpy()
        t[...] = a
        return t

    host = [pinned(np.ascontiguousarray(a)) for a in (phone, pitch.astype(np.int64), nsff0.astype(np.float32),
                                                      np.asarray(sid, np.int64).reshape(1), nz,
                                                      ns.reshape(1, -1))]
    h_wave = pinned(np.zeros((1, P * upp), np.float32))
    dev = []
    for a in host:
        p = ctx.alloc(a.nbytes)
        ctx.h2d(p, a)
        dev.append(p)
    d_wave = ctx.alloc(h_wave.nbytes)

    def step_device():
        _lib.check(_lib.lib.rvc_cuda_synth_infer_device(m.handle, 1, P, *[_lib._p(p) for p in dev],
                                                        _lib._p(d_wave)))

    def step_e2e():
        h_wave[:] = m.infer_batch(*host)

    for _ in range(args.warmup):
        step_device()
    t = max_over_ranks(timed(step_device, args.steps))
    step_e2e()
    te = max_over_ranks(timed(step_e2e, args.steps))
    audio = world * P * upp / 40000.0 * args.steps
    for p in dev + [d_wave]:
        ctx.free(p)
    m.close()
    return {"workload": f"config0 v2-40k synthesizer, one {P}-frame chunk ({P * upp / 40000:.0f} s) per call, "
                        f"B=1, on each of {world} GPU(s)",
            "value": audio / t, "unit": UNIT, "ms_per_chunk": 1e3 * t / args.steps,
            "e2e": {"value": audio / te, "unit": UNIT, "h2d_bytes_per_step": sum(a.nbytes for a in host) * world,
                    "d2h_bytes_per_step": h_wave.nbytes * world},
            "steps": args.steps, "warmup": args.warmup}


# DRAM bytes of the tensor-core conv launches for one v2-48k chunk of 1000 frames, from an ncu
# capture of the GeneratorNSF convs of an 8-chunk call (75.6 GB) plus enc_p / flow / conv_pre
# (76 MB per chunk, 4-chunk capture); traffic grows with rows.
SYNTH_DRAM_BYTES_48K_PER_1000_FRAMES = 9.53e9


def synth_traffic(sr, P, chunks):
    if sr != 48000:
        return None
    return SYNTH_DRAM_BYTES_48K_PER_1000_FRAMES * chunks * P / 1000.0


def run_ours(args, world, rank, local):
    import torch

    from rvc_cuda import _lib, synthetic as syn
    from rvc_cuda.synth import CudaSynthesizer

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    sr, P, G = args.sr, args.frames, args.group
    w = syn.make_vits_weights(sr, 0)
    cfg = syn.vits_config_array(sr)
    m = CudaSynthesizer(w, cfg, device=local, precision=args.precision)
    ctx = m.ctx
    upp, H, D = m.upp, m.hidden, m.arch["phone_dim"]
    assert args.chunks % world == 0, "chunks must split evenly across ranks"
    n_local = args.chunks // world
    from rvc_cuda.multi import shard
    ids = shard(args.chunks, world, rank)  # contiguous chunk range of this rank
    n_unique = min(args.unique, n_local)
    ins, noise = make_inputs(n_unique, P, upp)

    def pinned(shape, dtype):
        tdt = {np.float32: torch.float32, np.int64: torch.int64}[dtype]
        return torch.empty(shape, dtype=tdt, pin_memory=True).numpy()

    h_phone = pinned((n_local, P, D), np.float32)
    h_pitch = pinned((n_local, P), np.int64)
    h_f0 = pinned((n_local, P), np.float32)
    h_sid = pinned((n_local,), np.int64)
    h_nz = pinned((n_local, H, P), np.float32)
    h_ns = pinned((n_local, P * upp), np.float32)
    h_wave = pinned((n_local, P * upp), np.float32)
    for j, c in enumerate(ids):
        u = c % n_unique
        h_phone[j], h_pitch[j], h_f0[j], h_sid[j] = ins[u][0][0], ins[u][1][0], ins[u][2][0], ins[u][3][0]
        h_nz[j], h_ns[j] = noise[u][0][0], noise[u][1].reshape(-1)
    host = [h_phone, h_pitch, h_f0, h_sid, h_nz, h_ns]
    dev = []
    for a in host:
        p = ctx.alloc(a.nbytes)
        ctx.h2d(p, a)
        dev.append(p)
    d_wave = ctx.alloc(h_wave.nbytes)
    groups = [(s, min(G, n_local - s)) for s in range(0, n_local, G)]

    def step_device():
        for s, g in groups:
            ptrs = [dev[i] + s * (host[i].nbytes // n_local) for i in range(6)]
            _lib.check(_lib.lib.rvc_cuda_synth_infer_device(m.handle, g, P, *[_lib._p(p) for p in ptrs],
                                                            _lib._p(d_wave + s * (h_wave.nbytes // n_local))))

    def step_e2e():
        # the public call a user makes for many chunks: groups of G synthesized
        # with each group's host<->device copies overlapping the next group
        h_wave[:] = m.infer_batch(h_phone, h_pitch, h_f0, h_sid, h_nz, h_ns, group=G)

    stream = torch.cuda.ExternalStream(ctx.stream(), device=local)

    def timed(fn, steps):
        barrier()
        ctx.sync()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        ctx.sync()
        torch.cuda.synchronize()
        barrier()
        return e0.elapsed_time(e1) / 1e3

    for _ in range(args.warmup):
        step_device()
    ctx.sync()
    n0 = _lib.launch_count()
    with ClockSampler(local) as clk:
        t = timed(step_device, args.steps)
    launches = _lib.launch_count() - n0
    # per-launch kernel times for the roofline: a separate pass of the same steps
    # (the events and labels cost host time, so they stay out of the timed region)
    ctx.profile(True)
    timed(step_device, args.steps)
    prof_n, prof_ms, prof_flops = ctx.profile_read()
    if args.profile_out and rank == 0:
        with open(args.profile_out, "w") as f:
            f.write(ctx.profile_dump())
    ctx.profile(False)
    t = max_over_ranks(t)
    audio_per_step = args.chunks * P * upp / sr
    value = audio_per_step * args.steps / t
    # end-to-end through the public API (host buffers, copies included)
    step_e2e()
    te = max_over_ranks(timed(step_e2e, args.steps))
    e2e = audio_per_step * args.steps / te
    h2d = sum(a.nbytes for a in host) * world
    d2h = h_wave.nbytes * world
    ok = bool(np.isfinite(h_wave).all())
    cfg0 = None if args.no_config0 else config0_figure(args, local, timed, max_over_ranks, world)

    if rank == 0:
        pb, ps, hbm, src = peaks()
        achieved = prof_flops / (prof_ms / 1e3) / 1e12 if prof_ms > 0 else None
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * t / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": "f32 (BF16x3 split on tcgen05, fp32 accumulate)" if args.precision == "bf16x3" else "f32",
            "data": f"synthetic: seeded random-init weights, {n_unique} distinct seeded chunks tiled",
            "config": synth_config(args, world),
            "roofline": {"bound": "tensor",
                         "kernel": "tc_conv_kernel + tcn_conv_kernel (implicit-GEMM convs, all launches)",
                         "achieved": achieved, "peak": ps, "unit": "TFLOP/s",
                         "frac": (achieved / ps) if achieved else None,
                         "traffic": synth_traffic(sr, P, n_local),
                         "traffic_note": "DRAM bytes of this rank's conv launches per step: ncu captures of "
                                         "8- and 4-chunk v2-48k calls (dram__bytes_read.sum + dram__bytes_write.sum over the "
                                         "conv launches) scaled by chunks x frames; a lower bound, as the smaller "
                                         "call keeps its early-stage tensors in L2",
                         "peak_source": f"{src} bf16 dense sustained",
                         "note": "achieved = useful fp32 GEMM FLOPs / kernel time; BF16x3 runs 3 bf16 MMAs per "
                                 "useful MAC, so frac <= 1/3 by construction",
                         "launches": prof_n, "kernel_ms_per_step": prof_ms / args.steps},
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches,
            "clocks": clk.summary(),
            "finite": ok,
        }
        if cfg0 is not None:
            line["config0"] = cfg0
        if world == 1 and not args.no_cpu:
            cpu_sample(sr, args.ref_frames, w, cfg, steps=1)  # untimed: first-call costs (allocation, JIT)
            audio_s, ts = cpu_sample(sr, args.ref_frames, w, cfg, steps=1)
            line["cpu_baseline"] = {
                "value": audio_s / ts[0], "unit": UNIT, "cores": blas_threads(), "kind": cpu_kind(),
                "sample": f"1 chunk of {args.ref_frames} frames ({audio_s:.2f} s audio) after one untimed call, "
                          + cpu_what()}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def _lib_ctx():
    from rvc_cuda import _lib
    return _lib.get_context()


def run_layer(args):
    """Single-GPU layer cases for timing and ncu captures (one process, no JSON
    line): ``--layer conv`` runs ``rvc_cuda.ops.conv1d`` on [1,C,T] ("same"
    padding, dilation --dil), ``synth`` ``CudaSynthesizer.infer_batch`` on
    --batch seeded chunks of --frames frames, ``hubert`` ``CudaHubert.encode_equal``
    on --batch chunks of --samples samples; each --reps times, printing the wall
    time of the last."""
    from rvc_cuda import synthetic as syn
    rs = np.random.RandomState(0)
    if args.layer == "conv":
        from rvc_cuda import ops
        C, K, T, d = args.C, args.K, args.T, args.dil
        x = rs.standard_normal((1, C, T)).astype(np.float32)
        w = (rs.standard_normal((C, C, K)) / np.sqrt(C * K)).astype(np.float32)
        b = rs.standard_normal(C).astype(np.float32)
        for _ in range(args.reps):
            t0 = time.perf_counter()
            y = ops.conv1d(x, w, b, 1, (K - 1) * d // 2, d)
            dt = time.perf_counter() - t0
        ctx = _lib_ctx()
        ctx.profile(True)  # one more call with CUDA events around the conv kernel
        ops.conv1d(x, w, b, 1, (K - 1) * d // 2, d)
        n, ms, fl = ctx.profile_read()
        ctx.profile(False)
        print(f"conv C={C} K={K} dil={d} T={T}: {dt * 1e3:.2f} ms (host API, incl. copies); kernel "
              f"{ms * 1e3:.1f} us over {n} launch(es), {fl / (ms / 1e3) / 1e12 if ms else 0:.1f} TFLOP/s useful; "
              f"mean|y|={np.abs(y).mean():.4f}")
    elif args.layer == "synth":
        from rvc_cuda.synth import CudaSynthesizer
        m = CudaSynthesizer(syn.make_vits_weights(args.sr, 0), syn.vits_config_array(args.sr))
        B, P = args.batch, args.frames
        ins = [syn.make_vits_inputs(P, i) for i in range(B)]
        noise = [syn.make_vits_noise(P, m.upp, 50 + i) for i in range(B)]
        a = (np.concatenate([i[0] for i in ins]), np.concatenate([i[1] for i in ins]),
             np.concatenate([i[2] for i in ins]), np.concatenate([i[3] for i in ins]),
             np.concatenate([n[0] for n in noise]), np.stack([n[1].reshape(-1) for n in noise]))
        for _ in range(args.reps):
            t0 = time.perf_counter()
            out = m.infer_batch(*a)
            dt = time.perf_counter() - t0
        print(f"synth sr={args.sr} B={B} P={P}: {dt * 1e3:.2f} ms, {B * P * m.upp / args.sr / dt:.1f}x realtime, "
              f"std={out.std():.4f}")
    else:
        from rvc_cuda.hubert import CudaHubert
        m = CudaHubert(syn.make_hubert_weights(0))
        x = np.concatenate([syn.make_hubert_input(args.samples, i) for i in range(args.batch)], axis=0)
        for _ in range(args.reps):
            t0 = time.perf_counter()
            y = m.encode_equal(x)
            dt = time.perf_counter() - t0
        print(f"hubert B={args.batch} T={args.samples}: {dt * 1e3:.2f} ms, "
              f"{args.batch * args.samples / 16000 / dt:.1f}x realtime, std={y.std():.4f}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--chunks", type=int, default=256)
    ap.add_argument("--frames", type=int, default=1000)
    ap.add_argument("--sr", type=int, default=48000)
    ap.add_argument("--group", type=int, default=32)
    ap.add_argument("--unique", type=int, default=16)
    ap.add_argument("--precision", default="bf16x3", choices=["bf16x3", "simt"])
    ap.add_argument("--ref-frames", type=int, default=1000,
                    help="frames of the CPU sample chunk (default: the config's own 1000-frame chunk; about 14 s "
                         "per chunk for the reference's numpy code on 16 host threads)")
    ap.add_argument("--no-config0", action="store_true", help="skip the v2-40k config-0 figure")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--profile-out", default="", help="write the per-layer conv profile (CSV) here")
    ap.add_argument("--layer", default="conv", choices=["conv", "synth", "hubert"], help="--workload layer: the case")
    ap.add_argument("--C", type=int, default=32, help="layer conv: channels")
    ap.add_argument("--K", type=int, default=3, help="layer conv: kernel size")
    ap.add_argument("--T", type=int, default=1920000, help="layer conv: time steps")
    ap.add_argument("--dil", type=int, default=1, help="layer conv: dilation")
    ap.add_argument("--batch", type=int, default=2, help="layer synth / hubert: chunks per call")
    ap.add_argument("--reps", type=int, default=2, help="layer: repetitions")
    ap.add_argument("--workload", default="synth",
                    choices=["synth", "hubert", "retrieval", "rmvpe", "pipeline", "layer"],
                    help="synth: config 3 (headline); hubert: config 1 (HuBERT-base encoder); "
                         "retrieval: config 4's top-8 search + blend; rmvpe: config 2; "
                         "pipeline: config 4 end to end; layer: one layer case for timing / ncu (--layer)")
    ap.add_argument("--slice-length", type=float, default=0.0, help="pipeline: slice_length (0 = config default)")
    ap.add_argument("--samples", type=int, default=160000, help="hubert / rmvpe: samples per chunk")
    ap.add_argument("--audio-s", type=float, default=60.0, help="retrieval: seconds of frames (50 per s)")
    ap.add_argument("--index-rows", type=int, default=200000, help="retrieval: index rows")
    args = ap.parse_args()
    world, rank, local = dist_setup()
    if args.workload == "layer":
        run_layer(args)
    elif args.workload == "pipeline":
        if args.impl == "reference":
            run_pipeline_reference(args, world, rank)
        else:
            run_pipeline(args, world, rank, local)
    elif args.workload == "rmvpe":
        if args.impl == "reference":
            run_rmvpe_reference(args, world, rank)
        else:
            run_rmvpe(args, world, rank, local)
    elif args.workload == "retrieval":
        if args.impl == "reference":
            run_retrieval_reference(args, world, rank)
        else:
            run_retrieval(args, world, rank, local)
    elif args.workload == "hubert":
        if args.impl == "reference":
            run_hubert_reference(args, world, rank)
        else:
            run_hubert(args, world, rank, local)
    elif args.impl == "reference":
        run_reference(args, world, rank)
    else:
        run_ours(args, world, rank, local)


if __name__ == "__main__":
    main()
