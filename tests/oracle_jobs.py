"""Oracle runs executed in worker processes (spawned, so they never inherit a
CUDA context), used by the GPU tests to overlap the CPU oracle's work with
their own device work.  Test infrastructure: imports only numpy, the oracle
and the synthetic-data generators (no GPU)."""

from __future__ import annotations

import os

import numpy as np


def _limit_threads(n):
    try:
        import threadpoolctl  # noqa: PLC0415

        return threadpoolctl.threadpool_limits(n)
    except Exception:  # noqa: BLE001
        return None


def synth_chunk(sr: int, P: int, wseed: int, iseed: int, nseed: int, tap_names, threads: int):
    """``oracle.vits.synth`` on one seeded chunk: (waveform, {tap: array})."""
    from oracle import vits as OV  # noqa: PLC0415
    from rvc_cuda import synthetic as syn  # noqa: PLC0415

    _lim = _limit_threads(threads)  # noqa: F841  (kept alive for the call)
    w = syn.make_vits_weights(sr, wseed)
    cfg = syn.vits_config_array(sr)
    phone, pitch, nsff0, sid = syn.make_vits_inputs(P, iseed)
    upp = int(np.prod(cfg[12]))
    nz, ns = syn.make_vits_noise(P, upp, nseed)
    taps: dict = {}
    wav = OV.synth(w, cfg, phone, pitch, nsff0, sid, nz, ns, taps)
    keep = {k: taps[k] for k in tap_names if k in taps}
    return np.asarray(wav, np.float32).reshape(-1), keep


def pool(workers: int):
    """A process pool whose workers start with ``spawn``."""
    import concurrent.futures as cf  # noqa: PLC0415
    import multiprocessing as mp  # noqa: PLC0415

    return cf.ProcessPoolExecutor(max_workers=workers, mp_context=mp.get_context("spawn"))


def threads_per_worker(workers: int) -> int:
    return max(1, (os.cpu_count() or 1) // max(1, workers))
