"""Deterministic stand-ins for the models, to pin the pipeline's own steps.

The reference's ``Pipeline.pipeline`` (``runtime/pipeline.py:697``) calls
``model.encode``, ``net_g.infer`` and ``self.model_rmvpe.infer_from_audio``
(``:444-450``).  These cheap, seeded functions of their inputs replace the
networks so that a golden run of the reference's pipeline and a run of this
library's pipeline differ only in the pipeline's own signal processing and
chunking (high-pass, split, f0 post-processing, x2 interpolation, protect,
``change_rms``, int16).  The networks themselves are pinned by their own
fixtures.
"""

from __future__ import annotations

import numpy as np


class FakeHubert:
    """``encode(x [1,T], version) -> [1, L, D]`` with HuBERT's frame count
    ``L = (T - 400) // 320 + 1``: tanh of a seeded projection of four
    per-frame statistics of the audio."""

    def __init__(self, D=768, seed=0):
        self.P = np.random.RandomState(90_000 + seed).standard_normal((4, D)) * 2.0

    def encode(self, x, version=2):
        x = np.asarray(x, np.float64).reshape(-1)
        L = max(0, (x.size - 400) // 320 + 1)
        fr = np.lib.stride_tricks.sliding_window_view(x, 400)[::320][:L]
        st = np.stack([fr.mean(1) * 10, np.abs(fr).mean(1) * 4, fr.std(1) * 4, fr.max(1)], axis=1)
        return np.tanh(st @ self.P).astype(np.float32)[None]


class FakeSynth:
    """``infer(feats [1,P,D], pitch, pitchf [1,P], sid) -> [1,1,upp P]``: a sine
    at ``pitchf`` with a per-frame amplitude from the features, ``gain`` sets
    the peak (above 1 exercises the int16 peak normalisation)."""

    def __init__(self, upp=400, sr=40000, gain=1.3):
        self.upp, self.sr, self.gain = upp, sr, gain

    def infer(self, feats, pitch, pitchf, sid, phone_gpu=None, **_):
        feats = np.asarray(feats, np.float32)
        P = feats.shape[1]
        amp = np.tanh(feats[0].mean(axis=1).astype(np.float64) * 4.0) * 0.5 + 0.5
        f0 = np.asarray(pitchf, np.float64).reshape(-1)[:P]
        f0 = np.where(f0 > 0, f0, 0.0)
        ph = 2.0 * np.pi * np.cumsum(np.repeat(f0, self.upp)) / self.sr
        w = self.gain * np.repeat(amp, self.upp) * np.sin(ph)
        return w.astype(np.float32)[None, None]


class FakeRmvpe:
    """``infer_from_audio(x, thred) -> f0 [T // 160 + 1]`` Hz: 110-330 Hz from
    the frame's mean absolute level, 0 (unvoiced) below a level threshold."""

    def infer_from_audio(self, x, thred=0.03):
        x = np.asarray(x, np.float64).reshape(-1)
        n = x.size // 160 + 1
        xp = np.pad(x, (512, 512))
        lvl = np.array([np.abs(xp[i * 160:i * 160 + 1024]).mean() for i in range(n)])
        f0 = 110.0 + 220.0 * np.clip(lvl * 8.0, 0.0, 1.0)
        f0[lvl < 0.02] = 0.0
        return f0.astype(np.float32)


def config(x_pad=1, x_query=6, x_center=38, x_max=41):
    """The reference's ``Config`` attributes the pipeline reads (defaults:
    ``runtime/native_config.py:120``)."""
    import types
    return types.SimpleNamespace(x_pad=x_pad, x_query=x_query, x_center=x_center, x_max=x_max, device="cpu")
