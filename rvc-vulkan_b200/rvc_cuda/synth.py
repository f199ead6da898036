"""Model-level fast path for the VITS synthesizer (SynthesizerTrnMs768NSFsid).

Per-op dispatch moves activations host<->device at every op and does not
cover the attention matmuls, gates, SineGen or leaky_relu of the model
(``runtime/models/vits.py:1000-1014``, ``:1131-1132``, ``:1468-1501``), so the
throughput path is a whole-model call: weights are uploaded once under their
checkpoint keys (weight norm folded on the device, like the resident-weight
registration at ``runtime/models/vits.py:2279-2330``) and one library call runs
enc_p + flow + GeneratorNSF for a batch of equal-length chunks.

``CudaSynthesizer`` keeps the numpy-in / numpy-out contract of
``SynthesizerTrn.infer`` / ``infer_controlled`` (``runtime/models/vits.py:2352``,
``:2551``); ``patch_reference`` installs it on the reference class so
``runtime/pipeline.py`` and ``runtime/vc.py`` run unchanged.
"""

from __future__ import annotations

import ctypes as C
import os
from typing import Optional

import numpy as np

from . import _lib
from ._lib import check, fptr, iptr, lib

__all__ = ["CudaSynthesizer", "synth_config_from_weights", "patch_reference"]

PRECISIONS = {"bf16x3": 0, "simt": 1}


def synth_config_from_weights(w: dict, cfg=None, sr: Optional[int] = None) -> dict:
    """Architecture of a synthesizer checkpoint, derived like ``VitsConfig``
    (``runtime/models/vits.py:166-249``): encoder sizes from weight shapes,
    upsampling from the checkpoint config array."""
    hidden, phone_dim = (int(s) for s in w["enc_p.emb_phone.weight"].shape)
    n_layers = 0
    while f"enc_p.encoder.attn_layers.{n_layers}.conv_q.weight" in w:
        n_layers += 1
    erk = w["enc_p.encoder.attn_layers.0.emb_rel_k"]
    kc = int(erk.shape[2])
    n_ups = 0
    while f"dec.ups.{n_ups}.weight_v" in w:
        n_ups += 1
    if cfg is not None and len(cfg) > 14:
        rates = [int(r) for r in cfg[12]]
        kernels = [int(k) for k in cfg[14]] if cfg[14] not in (None, "") else \
            [int(w[f"dec.ups.{i}.weight_v"].shape[2]) for i in range(n_ups)]
        sr_ = int(sr) if sr else (int(cfg[17]) if len(cfg) > 17 else 48000)
    else:
        raise ValueError("CudaSynthesizer needs the checkpoint config array (rates/kernels/sr)")
    return {
        "sr": sr_, "hidden": hidden, "filter": int(w["enc_p.encoder.ffn_layers.0.conv_1.weight"].shape[0]),
        "heads": hidden // kc, "layers": n_layers, "kc": kc, "window": (int(erk.shape[1]) - 1) // 2,
        "gin": int(w["emb_g.weight"].shape[1]), "up0": int(w["dec.conv_pre.weight"].shape[0]),
        "n_ups": n_ups, "rates": rates, "kernels": kernels, "phone_dim": phone_dim,
        "n_spk": int(w["emb_g.weight"].shape[0]),
    }


class _Ready:
    """``collect()`` wrapper for ``_defer=True`` callers (``runtime/pipeline.py:1065-1072``)."""

    def __init__(self, arr):
        self._arr = arr

    def collect(self):
        return self._arr

    def abort(self):
        self._arr = None


class CudaSynthesizer:
    """Device-resident synthesizer on one GPU (one library context)."""

    def __init__(self, weights: dict, config=None, sr: Optional[int] = None, device: Optional[int] = None,
                 precision: str = "bf16x3"):
        self.arch = synth_config_from_weights(weights, config, sr)
        a = self.arch
        self.upp = int(np.prod(a["rates"]))
        self.sr = a["sr"]
        self.hidden = a["hidden"]
        self.ctx = _lib.get_context(device)
        p = os.environ.get("RVC_CUDA_PRECISION", precision)
        if p not in PRECISIONS:
            raise ValueError(f"precision must be one of {sorted(PRECISIONS)}")
        self.precision = p
        ints = [a["sr"], a["hidden"], a["filter"], a["heads"], a["layers"], a["kc"], a["window"], a["gin"],
                a["up0"], a["n_ups"], *a["rates"], *a["kernels"], a["phone_dim"], a["n_spk"], PRECISIONS[p]]
        arr = (C.c_int32 * len(ints))(*ints)
        h = C.c_int64(0)
        check(lib.rvc_cuda_synth_create(self.ctx.handle, arr, len(ints), C.byref(h)))
        self.handle = int(h.value)
        for k, v in weights.items():
            t = np.ascontiguousarray(np.asarray(v, dtype=np.float32))
            shape = (C.c_int64 * max(1, t.ndim))(*t.shape)
            check(lib.rvc_cuda_synth_set_weight(self.handle, k.encode(), fptr(t), shape, t.ndim))
        check(lib.rvc_cuda_synth_finalize(self.handle))

    @classmethod
    def from_reference(cls, net, device: Optional[int] = None, precision: str = "bf16x3"):
        """Build from a loaded reference ``SynthesizerTrn`` (its weight dict and config)."""
        c = net.cfg
        cfg = [c.spec_channels, c.segment_size, c.hidden, c.hidden, c.filter, c.n_heads, c.n_layers, 3, 0, "1",
               [3, 7, 11], [[1, 3, 5]] * 3, list(c.upsample_rates), c.upsample_initial,
               list(c.upsample_kernels), c.n_spk, c.gin_channels, c.sr]
        return cls(net._w, cfg, device=device, precision=precision)

    def close(self):
        if getattr(self, "handle", 0):
            lib.rvc_cuda_synth_destroy(self.handle)
            self.handle = 0

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass

    # ---------------------------------------------------------------- noise
    def make_noise(self, P: int, seed=None, out=None):
        """``nz [1,h,P]`` then ``ns [1,P*upp,1]`` in the order of
        ``SynthesizerTrn._make_noise`` (``runtime/models/vits.py:2337-2350``),
        honouring ``RVC_FIXED_SEED``.  ``out``: two float32 arrays of
        ``h*P`` and ``P*upp`` elements (e.g. page-locked views) the draws are
        cast into; they are returned reshaped."""
        fixed = os.environ.get("RVC_FIXED_SEED", "").strip()
        if seed is None and fixed:
            seed = int(fixed)
        rng = np.random.RandomState(seed) if seed is not None else np.random.RandomState()
        if out is None:
            nz = rng.standard_normal((1, self.hidden, P)).astype(np.float32)
            ns = rng.standard_normal((1, P * self.upp, 1)).astype(np.float32)
            return nz, ns
        nz = out[0].reshape(1, self.hidden, P)
        ns = out[1].reshape(1, P * self.upp, 1)
        np.copyto(nz, rng.standard_normal((1, self.hidden, P)), casting="same_kind")
        np.copyto(ns, rng.standard_normal((1, P * self.upp, 1)), casting="same_kind")
        return nz, ns

    # ---------------------------------------------------------------- infer
    def infer_batch(self, phone, pitch, nsff0, sid, nz, ns, group: Optional[int] = None) -> np.ndarray:
        """B equal-length chunks: ``phone [B,P,D]``, ``pitch [B,P]``, ``nsff0 [B,P]``,
        ``sid [B]``, ``nz [B,h,P]``, ``ns [B,P*upp]`` -> ``[B, P*upp]``.
        ``group``: synthesize in groups of that many chunks with the copies of
        one group overlapping the synthesis of the next (each group's result is
        that of ``infer_batch`` on those chunks)."""
        phone = np.ascontiguousarray(phone, dtype=np.float32)
        B, P, D = phone.shape
        pitch = np.ascontiguousarray(np.asarray(pitch).reshape(B, P), dtype=np.int64)
        nsff0 = np.ascontiguousarray(np.asarray(nsff0).reshape(B, P), dtype=np.float32)
        sid = np.ascontiguousarray(np.asarray(sid).reshape(B), dtype=np.int64)
        nz = np.ascontiguousarray(np.asarray(nz, dtype=np.float32).reshape(B, self.hidden, P))
        ns = np.ascontiguousarray(np.asarray(ns, dtype=np.float32).reshape(B, P * self.upp))
        out = np.empty((B, P * self.upp), np.float32)
        if group is not None and 0 < int(group) < B:
            check(lib.rvc_cuda_synth_infer_grouped(self.handle, B, int(group), P, fptr(phone), iptr(pitch),
                                                   fptr(nsff0), iptr(sid), fptr(nz), fptr(ns), fptr(out)))
            return out
        check(lib.rvc_cuda_synth_infer(self.handle, B, P, fptr(phone), iptr(pitch), fptr(nsff0), iptr(sid),
                                       fptr(nz), fptr(ns), fptr(out)))
        return out

    def infer_device(self, B: int, P: int, d_phone: int, d_pitch: int, d_nsff0: int, d_sid: int, d_nz: int,
                     d_ns: int, d_wave: int):
        """Device pointers (from this model's context): phone [B,P,D] f32, pitch [B,P] i64,
        nsff0 [B,P] f32, sid [B] i64, nz [B,h,P] f32, ns [B,P*upp] f32 -> wave [B,P*upp] f32;
        asynchronous on the context's stream."""
        check(lib.rvc_cuda_synth_infer_device(self.handle, int(B), int(P), *[C.c_void_p(v) for v in (
            d_phone, d_pitch, d_nsff0, d_sid, d_nz, d_ns, d_wave)]))

    def infer_controlled(self, phone, pitch, nsff0, sid, nz, ns, phone_gpu=None, _defer: bool = False):
        """Same contract as ``SynthesizerTrn.infer_controlled``: ``[1,1,upp*P]``."""
        phone = np.asarray(phone, dtype=np.float32)
        if phone.ndim != 3 or phone.shape[0] != 1:
            raise ValueError(f"phone must be [1,P,D], got {phone.shape}")
        P = phone.shape[1]
        wav = self.infer_batch(phone, np.asarray(pitch).reshape(1, P), np.asarray(nsff0).reshape(1, P),
                               np.asarray(sid).reshape(1), nz, ns).reshape(1, 1, -1)
        return _Ready(wav) if _defer else wav

    def infer(self, phone, pitch, nsff0, sid, seed=None, skip_head=None, return_length=None, phone_gpu=None,
              _defer: bool = False):
        """``SynthesizerTrn.infer`` (full synthesis; ``runtime/models/vits.py:2352``)."""
        P = np.asarray(phone).shape[1]
        nz, ns = self.make_noise(P, seed)
        if skip_head is not None and return_length is not None:
            return self.infer_partial(phone, pitch, nsff0, sid, nz, ns, int(skip_head), int(return_length))
        return self.infer_controlled(phone, pitch, nsff0, sid, nz, ns, _defer=_defer)

    def infer_partial(self, phone, pitch, nsff0, sid, nz, ns, skip_head: int, return_length: int) -> np.ndarray:
        """Partial synthesis (``SynthesizerTrn._infer_partial``, ``runtime/models/vits.py:2539-2548``):
        ``[1,1,upp*return_length]``, the samples of frames ``[skip_head, skip_head+return_length)``."""
        phone = np.ascontiguousarray(np.asarray(phone, dtype=np.float32))
        if phone.ndim != 3 or phone.shape[0] != 1:
            raise ValueError(f"phone must be [1,P,D], got {phone.shape}")
        P = phone.shape[1]
        if skip_head < 0 or skip_head >= P or return_length <= 0 or skip_head + return_length > P:
            raise ValueError(f"skip_head/return_length out of range: P={P}, head={skip_head}, length={return_length}")
        pitch = np.ascontiguousarray(np.asarray(pitch).reshape(P), dtype=np.int64)
        nsff0 = np.ascontiguousarray(np.asarray(nsff0).reshape(P), dtype=np.float32)
        sid = np.ascontiguousarray(np.asarray(sid).reshape(1), dtype=np.int64)
        nz = np.ascontiguousarray(np.asarray(nz, dtype=np.float32).reshape(self.hidden, P))
        ns = np.ascontiguousarray(np.asarray(ns, dtype=np.float32).reshape(P * self.upp))
        out = np.empty(return_length * self.upp, np.float32)
        check(lib.rvc_cuda_synth_infer_partial(self.handle, P, skip_head, return_length, fptr(phone), iptr(pitch),
                                               fptr(nsff0), iptr(sid), fptr(nz), fptr(ns), fptr(out)))
        return out.reshape(1, 1, -1)

    # ---------------------------------------------------------------- batched decode
    def prep_dec(self, phone, pitch, nsff0, sid, seed=None, skip_head=None, return_length=None, phone_gpu=None,
                 noise=None):
        """``SynthesizerTrn.prep_dec`` (``runtime/models/vits.py:2478-2500``): draws the
        chunk's noise in the reference's order (or takes ``noise = (nz, ns)``
        drawn beforehand by ``make_noise``) and keeps the inputs for
        ``decode_batch`` (the whole model runs there, batched on the device)."""
        phone = np.asarray(phone, dtype=np.float32)
        P = phone.shape[1]
        if skip_head is not None and return_length is not None:
            head, length = int(skip_head), int(return_length)
            if head < 0 or head >= P or length <= 0 or head + length > P:
                raise ValueError(f"skip_head/return_length out of range: P={P}, head={head}, length={length}")
        else:
            head = length = None
        nz, ns = self.make_noise(P, seed) if noise is None else noise
        return {"phone": phone, "pitch": np.asarray(pitch), "nsff0": np.asarray(nsff0, dtype=np.float32),
                "sid": np.asarray(sid), "nz": nz, "ns": ns, "head": head, "length": length}

    def decode_batch(self, preps) -> list:
        """``SynthesizerTrn.decode_batch`` (``runtime/models/vits.py:2502-2536``): one
        waveform per prep (``[1,1,upp*P]``, or the target segment for partial
        preps); full-length chunks of equal length share one batched call."""
        out: list = [None] * len(preps)
        groups: dict = {}
        for i, p in enumerate(preps):
            if p["head"] is not None:
                out[i] = self.infer_partial(p["phone"], p["pitch"], p["nsff0"], p["sid"], p["nz"], p["ns"],
                                            p["head"], p["length"])
            else:
                groups.setdefault(p["phone"].shape[1], []).append(i)
        for P, idx in groups.items():
            ps = [preps[i] for i in idx]
            waves = self.infer_batch(np.concatenate([p["phone"] for p in ps], axis=0),
                                     np.stack([p["pitch"].reshape(P) for p in ps]),
                                     np.stack([p["nsff0"].reshape(P) for p in ps]),
                                     np.concatenate([p["sid"].reshape(1) for p in ps]),
                                     np.concatenate([p["nz"].reshape(1, self.hidden, P) for p in ps]),
                                     np.stack([p["ns"].reshape(-1) for p in ps]))
            for j, i in enumerate(idx):
                out[i] = waves[j:j + 1].reshape(1, 1, -1)
        return out

    # ---------------------------------------------------------------- debug
    def keep_taps(self, on: bool = True, chunk: Optional[int] = None):
        """Record per-layer intermediates of the next calls: of every chunk
        (chunk-major), or with ``chunk`` of that chunk of a batched call only."""
        mode = 0 if not on else (1 if chunk is None else 2 + int(chunk))
        check(lib.rvc_cuda_synth_keep_taps(self.handle, mode))

    def tap(self, name: str, shape) -> np.ndarray:
        out = np.empty(int(np.prod(shape)), np.float32)
        check(lib.rvc_cuda_synth_tap(self.handle, name.encode(), fptr(out), out.size))
        return out.reshape(shape)


def patch_reference(vits_module=None, device: Optional[int] = None, precision: str = "bf16x3"):
    """Route ``SynthesizerTrn.infer_controlled`` (and thus ``infer`` for full
    synthesis), ``_infer_partial`` (``infer`` with skip_head/return_length) and
    the pipeline's batched ``prep_dec`` / ``decode_batch`` of the reference
    through ``CudaSynthesizer``.

    The class methods are replaced, not the loader, because ``runtime/vc.py``
    imports the loaders by name.  A device model is built once per
    ``SynthesizerTrn`` instance and cached on it; ``vc.get_vc`` builds a new
    instance on model switch, which drops the old cache with it.  When
    ``RVC_CUDA_DEVICES`` names several GPUs (and no ``device`` is given) the
    device model is a ``rvc_cuda.multi.SynthPool`` over them: the pipeline's
    batched decode then spreads its chunks over the devices.
    """
    if vits_module is None:
        from runtime.models import vits as vits_module  # noqa: PLC0415
    cls = vits_module.SynthesizerTrn
    if getattr(cls, "_rvc_cuda_patched", False):
        return cls

    def _model(self):
        m = self.__dict__.get("_rvc_cuda_model")
        if m is None:
            from .multi import SynthPool, devices_from_env  # noqa: PLC0415

            devs = devices_from_env() if device is None else [device]
            if len(devs) > 1:
                m = SynthPool.from_reference(self, devices=devs, precision=precision)
            else:
                m = CudaSynthesizer.from_reference(self, device=devs[0], precision=precision)
            self.__dict__["_rvc_cuda_model"] = m
        return m

    def infer_controlled(self, phone, pitch, nsff0, sid, nz, ns, phone_gpu=None, _defer=False):
        return _model(self).infer_controlled(phone, pitch, nsff0, sid, nz, ns, _defer=_defer)

    def _infer_partial(self, phone, pitch, nsff0, sid, nz, ns, head, length, phone_gpu=None):
        return _model(self).infer_partial(phone, pitch, nsff0, sid, nz, ns, int(head), int(length))

    def prep_dec(self, phone, pitch, nsff0, sid, seed=None, skip_head=None, return_length=None, phone_gpu=None):
        return _model(self).prep_dec(phone, pitch, nsff0, sid, seed, skip_head, return_length)

    def decode_batch(self, preps):
        return _model(self).decode_batch(preps)

    cls._rvc_cuda_orig_infer_controlled = cls.infer_controlled
    cls.infer_controlled = infer_controlled
    if hasattr(cls, "prep_dec") and hasattr(cls, "decode_batch"):  # the pipeline's batched decode path
        cls._rvc_cuda_orig_prep_dec = cls.prep_dec
        cls._rvc_cuda_orig_decode_batch = cls.decode_batch
        cls.prep_dec = prep_dec
        cls.decode_batch = decode_batch
    if hasattr(cls, "_infer_partial"):  # SynthesizerTrn.infer's skip_head path (vits.py:2416-2420)
        cls._rvc_cuda_orig_infer_partial = cls._infer_partial
        cls._infer_partial = _infer_partial
    cls._rvc_cuda_patched = True
    return cls
