"""Per-layer microbenchmarks of librvc_cuda (single GPU), for timing and ncu.

    python -m rvc_cuda.microbench conv --C 32 --K 3 --T 1920000 [--dil 1] [--reps 2]
    python -m rvc_cuda.microbench synth --sr 48000 --B 2 --P 1000 [--reps 2]
    python -m rvc_cuda.microbench hubert --B 4 --T 160000 [--reps 2]

`conv` runs rvc_cuda.ops.conv1d ([1,C,T] -> [1,C,T], "same" padding) `reps`
times; `synth` runs CudaSynthesizer.infer_batch on B seeded chunks; `hubert`
runs CudaHubert.encode_equal on B seeded chunks of T samples.  Each prints the
wall time of the last repetition.
"""

from __future__ import annotations

import argparse
import time

import numpy as np


def _conv(args):
    from rvc_cuda import ops

    rs = np.random.RandomState(0)
    C, K, T, d = args.C, args.K, args.T, args.dil
    x = rs.standard_normal((1, C, T)).astype(np.float32)
    w = (rs.standard_normal((C, C, K)) / np.sqrt(C * K)).astype(np.float32)
    b = rs.standard_normal(C).astype(np.float32)
    for _ in range(args.reps):
        t0 = time.perf_counter()
        y = ops.conv1d(x, w, b, 1, (K - 1) * d // 2, d)
        dt = time.perf_counter() - t0
    print(f"conv C={C} K={K} dil={d} T={T}: {dt * 1e3:.2f} ms (host API, incl. copies) mean|y|={np.abs(y).mean():.4f}")


def _synth(args):
    from rvc_cuda import synthetic as syn
    from rvc_cuda.synth import CudaSynthesizer

    w = syn.make_vits_weights(args.sr, 0)
    m = CudaSynthesizer(w, syn.vits_config_array(args.sr))
    B, P = args.B, args.P
    ins = [syn.make_vits_inputs(P, i) for i in range(B)]
    nz = np.concatenate([syn.make_vits_noise(P, m.upp, 50 + i)[0] for i in range(B)])
    ns = np.stack([syn.make_vits_noise(P, m.upp, 50 + i)[1].reshape(-1) for i in range(B)])
    phone = np.concatenate([i[0] for i in ins])
    pitch = np.concatenate([i[1] for i in ins])
    f0 = np.concatenate([i[2] for i in ins])
    sid = np.concatenate([i[3] for i in ins])
    for _ in range(args.reps):
        t0 = time.perf_counter()
        out = m.infer_batch(phone, pitch, f0, sid, nz, ns)
        dt = time.perf_counter() - t0
    print(f"synth sr={args.sr} B={B} P={P}: {dt * 1e3:.2f} ms, {B * P * m.upp / args.sr / dt:.1f}x realtime, "
          f"std={out.std():.4f}")


def _hubert(args):
    from rvc_cuda import synthetic as syn
    from rvc_cuda.hubert import CudaHubert

    m = CudaHubert(syn.make_hubert_weights(0))
    x = np.concatenate([syn.make_hubert_input(args.T, i) for i in range(args.B)], axis=0)
    for _ in range(args.reps):
        t0 = time.perf_counter()
        y = m.encode_equal(x)
        dt = time.perf_counter() - t0
    print(f"hubert B={args.B} T={args.T}: {dt * 1e3:.2f} ms, {args.B * args.T / 16000 / dt:.1f}x realtime, "
          f"std={y.std():.4f}")


def main():
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    c = sub.add_parser("conv")
    c.add_argument("--C", type=int, default=32)
    c.add_argument("--K", type=int, default=3)
    c.add_argument("--T", type=int, default=1920000)
    c.add_argument("--dil", type=int, default=1)
    c.add_argument("--reps", type=int, default=2)
    s = sub.add_parser("synth")
    s.add_argument("--sr", type=int, default=48000)
    s.add_argument("--B", type=int, default=2)
    s.add_argument("--P", type=int, default=1000)
    s.add_argument("--reps", type=int, default=2)
    h = sub.add_parser("hubert")
    h.add_argument("--B", type=int, default=4)
    h.add_argument("--T", type=int, default=160000)
    h.add_argument("--reps", type=int, default=2)
    args = ap.parse_args()
    {"conv": _conv, "synth": _synth, "hubert": _hubert}[args.cmd](args)


if __name__ == "__main__":
    main()
