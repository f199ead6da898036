"""Chunk-parallel synthesis over several GPUs of one node.

The pipeline's chunks are independent once the global f0 pass is done
(``runtime/pipeline.py:821-829``; ``decode_batch`` treats them independently,
``runtime/models/vits.py:1847-1878``), so the work splits by chunk with no
collective on the data path:

* ``SynthPool``: one ``CudaSynthesizer`` per device in one process (devices from
  ``RVC_CUDA_DEVICES``, e.g. ``0,1,2,3`` or ``all``), each driven by its own
  host thread (the library's calls release the GIL).  It has the synthesizer's
  duck-typed interface (``infer`` / ``infer_controlled`` / ``prep_dec`` /
  ``decode_batch`` / ``make_noise``), so ``rvc_cuda.pipeline.Pipeline`` and the
  reference's ``Pipeline.pipeline`` take it in place of one model; chunks are
  spread over the devices by length and the waveforms come back in chunk order.
* ``shard`` / ``gather_ordered``: the same split for one process per GPU
  (``torchrun``): each rank takes its chunks, and rank 0 reassembles the
  results in chunk order through ``torch.distributed.gather_object`` (host
  objects; no device collective).
"""

from __future__ import annotations

import os
import threading
from concurrent.futures import ThreadPoolExecutor
from typing import Callable, List, Optional, Sequence

import numpy as np

__all__ = ["devices_from_env", "balance", "shard", "gather_ordered", "SynthPool"]


def devices_from_env(default: Optional[Sequence[int]] = None) -> List[int]:
    """Devices named by ``RVC_CUDA_DEVICES`` (``"0,2"``, ``"all"``); else
    ``default``, else ``[$RVC_CUDA_DEVICE or 0]``."""
    spec = os.environ.get("RVC_CUDA_DEVICES", "").strip()
    if spec:
        if spec.lower() == "all":
            from . import _lib  # noqa: PLC0415

            return list(range(_lib.device_count()))
        devs = [int(t) for t in spec.replace(" ", "").split(",") if t != ""]
        if not devs or len(set(devs)) != len(devs) or min(devs) < 0:
            raise ValueError(f"RVC_CUDA_DEVICES must list distinct device ids, got {spec!r}")
        return devs
    if default is not None:
        return list(default)
    return [int(os.environ.get("RVC_CUDA_DEVICE", "0"))]


def balance(costs: Sequence[float], n_workers: int) -> List[List[int]]:
    """Indices of ``costs`` split over ``n_workers`` bins: longest first onto
    the least-loaded bin (ties to the lower bin), each bin in ascending index
    order.  Deterministic, so every rank computes the same split."""
    if n_workers < 1:
        raise ValueError("n_workers must be >= 1")
    bins: List[List[int]] = [[] for _ in range(n_workers)]
    load = [0.0] * n_workers
    for i in sorted(range(len(costs)), key=lambda j: (-float(costs[j]), j)):
        b = min(range(n_workers), key=lambda k: (load[k], k))
        bins[b].append(i)
        load[b] += float(costs[i])
    return [sorted(b) for b in bins]


def shard(n_items: int, world: int, rank: int, costs: Optional[Sequence[float]] = None) -> List[int]:
    """Item indices rank ``rank`` of ``world`` processes: contiguous equal
    ranges (the first ``n % world`` ranks one more) for uniform items, or the
    ``balance`` split when per-item ``costs`` are given."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if costs is not None:
        if len(costs) != n_items:
            raise ValueError("costs must have one entry per item")
        return balance(costs, world)[rank]
    base, extra = divmod(n_items, world)
    start = rank * base + min(rank, extra)
    return list(range(start, start + base + (1 if rank < extra else 0)))


def gather_ordered(local_results: Sequence, local_ids: Sequence[int], n_items: int, group=None, dst: int = 0):
    """Rank ``dst`` receives every rank's ``(ids, results)`` (host objects,
    ``torch.distributed.gather_object``) and returns the results in item order;
    other ranks return None.  Raises if an item is missing or duplicated."""
    import torch.distributed as dist  # noqa: PLC0415

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    payload = (list(map(int, local_ids)), list(local_results))
    got = [None] * world if rank == dst else None
    dist.gather_object(payload, got, dst=dst, group=group)
    if rank != dst:
        return None
    out: list = [None] * n_items
    seen = np.zeros(n_items, np.int64)
    for ids, res in got:
        if len(ids) != len(res):
            raise RuntimeError("gather_ordered: a rank sent ids and results of different lengths")
        for i, r in zip(ids, res):
            if not 0 <= i < n_items:
                raise RuntimeError(f"gather_ordered: item {i} out of range")
            seen[i] += 1
            out[i] = r
    if (seen != 1).any():
        raise RuntimeError(f"gather_ordered: items missing {np.flatnonzero(seen == 0).tolist()} "
                           f"or repeated {np.flatnonzero(seen > 1).tolist()}")
    return out


class SynthPool:
    """One ``CudaSynthesizer`` per device, used as one synthesizer."""

    def __init__(self, weights: dict, config=None, sr: Optional[int] = None, devices: Optional[Sequence[int]] = None,
                 precision: str = "bf16x3", factory: Optional[Callable] = None):
        """``factory(device)`` builds a device model (default: a
        ``CudaSynthesizer`` on that device from ``weights``)."""
        self.devices = devices_from_env() if devices is None else list(devices)
        if not self.devices:
            raise ValueError("SynthPool needs at least one device")
        if factory is None:
            from .synth import CudaSynthesizer  # noqa: PLC0415

            def factory(dev):
                return CudaSynthesizer(weights, config, sr=sr, device=dev, precision=precision)
        with ThreadPoolExecutor(len(self.devices)) as ex:  # upload the weights to every device at once
            self.models = list(ex.map(factory, self.devices))
        m0 = self.models[0]
        self.upp, self.sr, self.hidden, self.arch = m0.upp, m0.sr, m0.hidden, getattr(m0, "arch", None)
        self._ex = ThreadPoolExecutor(len(self.devices), thread_name_prefix="rvc-synth-dev")
        self._rr = 0
        self._lock = threading.Lock()

    @classmethod
    def from_reference(cls, net, devices=None, precision: str = "bf16x3"):
        """From a loaded reference ``SynthesizerTrn`` (its weights and config)."""
        from .synth import CudaSynthesizer  # noqa: PLC0415

        devs = devices_from_env() if devices is None else list(devices)
        return cls(None, devices=devs, precision=precision,
                   factory=lambda d: CudaSynthesizer.from_reference(net, device=d, precision=precision))

    def close(self):
        self._ex.shutdown(wait=True)
        for m in self.models:
            m.close()

    # one chunk: the next device in turn
    def _next(self):
        with self._lock:
            m = self.models[self._rr % len(self.models)]
            self._rr += 1
        return m

    def make_noise(self, P: int, seed=None, out=None):
        return self.models[0].make_noise(P, seed, out)

    def infer_controlled(self, *a, **k):
        return self._next().infer_controlled(*a, **k)

    def infer(self, *a, **k):
        return self._next().infer(*a, **k)

    def infer_partial(self, *a, **k):
        return self._next().infer_partial(*a, **k)

    def prep_dec(self, *a, **k):
        return self.models[0].prep_dec(*a, **k)

    def decode_batch(self, preps) -> list:
        """Waveforms of ``preps`` in order; the chunks are spread over the
        devices by frame count (``balance``) and decoded concurrently, each
        device batching its equal-length chunks."""
        preps = list(preps)
        if not preps:
            return []
        costs = [p["phone"].shape[1] if p["head"] is None else p["length"] + 2 * 16 for p in preps]
        bins = balance(costs, len(self.models))
        futs = [(idx, self._ex.submit(m.decode_batch, [preps[i] for i in idx]))
                for m, idx in zip(self.models, bins) if idx]
        out: list = [None] * len(preps)
        for idx, f in futs:
            for i, w in zip(idx, f.result()):
                out[i] = w
        return out

    def infer_chunks(self, chunks) -> list:
        """``chunks``: (phone, pitch, nsff0, sid, nz, ns) tuples; waveforms
        ``[1,1,P*upp]`` in order."""
        preps = [self.models[0].prep_dec(ph, p, f, s, noise=(nz, ns)) for ph, p, f, s, nz, ns in chunks]
        return self.decode_batch(preps)
