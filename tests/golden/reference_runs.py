"""Runs of the reference's own code, unchanged, on seeded synthetic weights.

    python tests/golden/reference_runs.py --backend numpy --out refruns.npz
    python tests/golden/reference_runs.py --backend cuda  --out refruns_cuda.npz

The reference's runtime comes from ``oracle.reference`` (a checkout named by
``RVC_REFERENCE`` or the ``oracle/_ref`` copy).  With ``--backend numpy`` this
is the reference as shipped: ``make_golden.py`` stores its outputs as fixtures.
With ``--backend cuda`` the same code runs after ``rvc_cuda.register()``
(``RVC_BACKEND=cuda``: ``runtime.nn``'s float32 ops reach ``rvc_cuda.ops``
through ``runtime/backend.py:189-197``) and ``rvc_cuda.patch_reference()`` (the
model classes' methods, the pipeline's signal processing and the
``vc_single`` pool release); the GPU tests compare its outputs with the
fixtures.  The backend is a per-process choice of the reference
(``runtime/backend.py:154-158``), so each backend runs in its own process.

Cases:

* ``ops``: ``runtime.nn.conv1d`` / ``conv_transpose1d`` / ``layer_norm`` /
  ``linear`` / ``softmax`` on float32 inputs against the reference's numpy
  kernels (``runtime/nn.py:90``, ``:294``, ``:394``, ``:458``) called directly;
  records the backend the reference selected.
* ``synth``: ``SynthesizerTrn.infer_controlled`` and ``infer`` (seeded),
  ``runtime/models/vits.py:2352``, ``:2551``.
* ``pipeline``: ``Pipeline.pipeline`` (``runtime/pipeline.py:697``) with the
  reference's HubertEncoder, RMVPE and SynthesizerTrn and a FeatureIndex.
* ``vc``: ``VC.get_vc`` + ``VC.vc_single`` (``runtime/vc.py:332``, ``:440``) on a
  WAV file, through to the int16 output (pm f0).
* ``config4``: ``Pipeline.pipeline`` on BASELINE config 4's 60 s clip (numpy
  only: the fixture for the device pipeline's 60 s test).
"""

from __future__ import annotations

import argparse
import os
import sys
import tempfile
import wave

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
for _p in (ROOT, os.path.join(ROOT, "rvc-vulkan_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

from rvc_cuda import synthetic as syn  # noqa: E402

SEED = 1234               # RVC_FIXED_SEED: the synthesizer noise of every chunk
CLIP_S, CLIP_SEED = 2.5, 21
# 8 index rows: k = 8 takes them all (runtime/retrieval.py:35-82 with N <= k),
# so the blend weights are continuous in the features and no top-k decision
# is left to a float near-tie; top-k selection at scale has its own tests.
INDEX_N, INDEX_SEED = 8, 5
# f0_up_key 5: every coarse-pitch decision of this clip is >= 0.027 bins from
# a rounding point (the random-init RMVPE gives a few distinct f0 values)
PIPE_KW = dict(f0_up_key=5, f0_method="rmvpe", index_rate=0.75, if_f0=1, tgt_sr=40000, resample_sr=0,
               rms_mix_rate=0.25, version="v2", protect=0.33)


def _case_ops(out):
    from runtime import backend, nn  # noqa: PLC0415

    out["ops_backend"] = np.array(backend.get_backend())
    rs = np.random.RandomState(77)
    errs = []
    for (B, Ci, Co, T, K, s, pad, d) in [(1, 192, 384, 50, 5, 1, 2, 1), (2, 64, 64, 301, 11, 1, (25, 25), 5),
                                         (1, 32, 48, 77, 3, 2, (1, 0), 1)]:
        x = rs.standard_normal((B, Ci, T)).astype(np.float32)
        w = (rs.standard_normal((Co, Ci, K)) * 0.05).astype(np.float32)
        b = rs.standard_normal(Co).astype(np.float32)
        got = nn.conv1d(x, w, b, stride=s, padding=pad, dilation=d)
        ref = nn._conv1d_numpy(x, w, None, s, pad, d) + b[None, :, None]
        errs.append(float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30)))
    for (Ci, Co, T, K, s, p) in [(256, 128, 40, 16, 8, 4), (64, 32, 33, 4, 2, 1)]:
        x = rs.standard_normal((1, Ci, T)).astype(np.float32)
        w = (rs.standard_normal((Ci, Co, K)) * 0.05).astype(np.float32)
        b = rs.standard_normal(Co).astype(np.float32)
        got = nn.conv_transpose1d(x, w, b, stride=s, padding=p)
        ref = nn._conv_transpose1d_numpy(x, w, b, s, p, 0, 1)
        errs.append(float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30)))
    x = (rs.standard_normal((3, 70, 192)) * 3 + 1).astype(np.float32)
    g = rs.uniform(0.5, 1.5, 192).astype(np.float32)
    bb = rs.standard_normal(192).astype(np.float32)
    got = nn.layer_norm(x, g, bb, eps=1e-5)
    mu = x.astype(np.float64).mean(-1, keepdims=True)
    var = ((x.astype(np.float64) - mu) ** 2).mean(-1, keepdims=True)
    ref = ((x - mu) / np.sqrt(var + 1e-5)) * g + bb
    errs.append(float(np.abs(got - ref).max()))
    a = rs.standard_normal((2, 37, 768)).astype(np.float32)
    w = (rs.standard_normal((192, 768)) * 0.03).astype(np.float32)
    lb = rs.standard_normal(192).astype(np.float32)
    got = nn.linear(a, w, lb)
    ref = (a.astype(np.float64) @ w.T.astype(np.float64) + lb)
    errs.append(float(np.abs(got - ref).max() / np.abs(ref).max()))
    s = (rs.standard_normal((4, 9, 333)) * 5).astype(np.float32)
    got = nn.softmax(s, axis=-1)
    e = np.exp(s.astype(np.float64) - s.max(-1, keepdims=True))
    errs.append(float(np.abs(got - e / e.sum(-1, keepdims=True)).max()))
    out["ops_err"] = np.array(errs, np.float64)


def _case_synth(out):
    from oracle import reference as oref  # noqa: PLC0415

    w = syn.make_vits_weights(40000, 0)
    net = oref.synthesizer(w, syn.vits_config_array(40000))
    phone, pitch, nsff0, sid = syn.make_vits_inputs(32, 1)
    nz, ns = syn.make_vits_noise(32, net.cfg.upp, 11)
    out["synth_controlled"] = np.asarray(net.infer_controlled(phone, pitch, nsff0, sid, nz, ns), np.float32).reshape(-1)
    out["synth_seeded"] = np.asarray(net.infer(phone, pitch, nsff0, sid, seed=7), np.float32).reshape(-1)


def _models():
    from oracle import reference as oref  # noqa: PLC0415

    hub = oref.hubert(syn.make_hubert_weights(0))
    net = oref.synthesizer(syn.make_vits_weights(40000, 0), syn.vits_config_array(40000))
    return hub, net


def _index():
    from runtime.retrieval import FeatureIndex  # noqa: PLC0415

    idx = FeatureIndex(768)
    idx.add(syn.make_index(INDEX_N, 768, INDEX_SEED))
    return idx


# The pipeline makes two discrete decisions on float data: the top-8 set of
# each retrieval query (runtime/pipeline.py:547) and the coarse pitch bin,
# rint of a mel-scaled f0 (:477-482).  Float paths that agree to ~1e-5 can
# still land on opposite sides of a decision whose margin is that small, and
# a changed neighbour or pitch bin reaches every frame of the chunk through
# the text encoder's attention.  The runs record each decision's smallest
# margin, computed in float64 from their own inputs, and the test inputs are
# chosen so that every margin is far above the float paths' differences.
MIN_RET_GAP = 0.1        # squared-distance gap between the 8th and 9th neighbour
MIN_COARSE_MARGIN = 1e-3  # distance of the scaled mel f0 from a rounding point, in bins


def _record_margins():
    """Wraps ``runtime.pipeline.search_l2`` and ``Pipeline.get_f0``; returns a
    function that removes the wrappers and gives (retrieval gap, coarse margin)."""
    from runtime import pipeline as rp  # noqa: PLC0415

    st = {"gap": np.inf, "coarse": np.inf}
    orig_search, orig_f0 = rp.search_l2, rp.Pipeline.get_f0

    def search_l2(q, vecs, k=8):
        r = orig_search(q, vecs, k=k)
        q64, v64 = np.asarray(q, np.float64), np.asarray(vecs, np.float64)
        if v64.shape[0] > k:
            d = (q64 * q64).sum(1)[:, None] + (v64 * v64).sum(1)[None, :] - 2.0 * (q64 @ v64.T)
            part = np.sort(np.partition(d, k, axis=1)[:, :k + 1], axis=1)
            st["gap"] = min(st["gap"], float((part[:, k] - part[:, k - 1]).min()))
        return r

    def get_f0(self, x, p_len, f0_up_key, f0_method, *a, **kw):
        coarse, f0bak = orig_f0(self, x, p_len, f0_up_key, f0_method, *a, **kw)
        mel = 1127.0 * np.log(1.0 + np.asarray(f0bak, np.float64) / 700.0)
        lo, hi = 1127.0 * np.log(1.0 + 50.0 / 700.0), 1127.0 * np.log(1.0 + 1100.0 / 700.0)
        m = (mel[mel > 0] - lo) * 254.0 / (hi - lo) + 1.0
        m = m[(m > 1.0) & (m < 255.0)]
        if m.size:
            st["coarse"] = min(st["coarse"], float(np.abs(m - np.floor(m) - 0.5).min()))
        return coarse, f0bak

    rp.search_l2, rp.Pipeline.get_f0 = search_l2, get_f0

    def done():
        rp.search_l2, rp.Pipeline.get_f0 = orig_search, orig_f0
        return st["gap"], st["coarse"]

    return done


def _case_pipeline(out):
    from oracle import reference as oref  # noqa: PLC0415
    from runtime.native_config import Config  # noqa: PLC0415
    from runtime.pipeline import Pipeline  # noqa: PLC0415

    hub, net = _models()
    audio = syn.make_speech_audio(CLIP_S, seed=CLIP_SEED, silence_every=1.2)
    pipe = Pipeline(40000, Config())
    pipe.model_rmvpe = oref.rmvpe(syn.make_rmvpe_weights(0))
    done = _record_margins()
    try:
        sr, y = pipe.pipeline(hub, net, 0, audio, [0.0, 0.0, 0.0], PIPE_KW["f0_up_key"], PIPE_KW["f0_method"],
                              _index(), PIPE_KW["index_rate"], PIPE_KW["if_f0"], PIPE_KW["tgt_sr"],
                              PIPE_KW["resample_sr"], PIPE_KW["rms_mix_rate"], PIPE_KW["version"], PIPE_KW["protect"])
    finally:
        out["pipeline_margins"] = np.array(done(), np.float64)
    out["pipeline_sr"] = np.array(sr)
    out["pipeline_int16"] = np.asarray(y)


def _write_wav(path, x, sr=16000):
    y = np.clip(np.round(np.asarray(x, np.float64) * 32767.0), -32768, 32767).astype("<i2")
    with wave.open(path, "wb") as f:
        f.setnchannels(1)
        f.setsampwidth(2)
        f.setframerate(sr)
        f.writeframes(y.tobytes())


def _pool_release_stand_in():
    """numpy runs only: ``vc_single`` ends with
    ``vulkan_ops.get_context().clear_pool()`` (``runtime/vc.py:532-534``), which
    raises without the Vulkan engine library (``runtime/vulkan_ops.py:3935-3945``)
    after the conversion is done.  A numpy process has no device pool to
    release, so that one call gets a stand-in whose ``clear_pool`` does
    nothing; under ``--backend cuda`` ``rvc_cuda.patch_reference()`` installs
    the library's own (which releases its cached device blocks)."""
    from runtime import vulkan_ops  # noqa: PLC0415

    orig = vulkan_ops.get_context

    class _NoPool:
        def clear_pool(self):
            return None

    def get_context():
        try:
            return orig()
        except Exception:  # noqa: BLE001 - no engine library: nothing to release
            return _NoPool()

    vulkan_ops.get_context = get_context


def _case_vc(out):
    from pathlib import Path  # noqa: PLC0415

    from runtime import vc as rvc  # noqa: PLC0415
    from runtime.models import hubert as rh, rmvpe as rr, vits as rv  # noqa: PLC0415
    from runtime.native_config import Config  # noqa: PLC0415

    w, cfg = syn.make_vits_weights(40000, 0), syn.vits_config_array(40000)
    hsd, rsd = syn.make_hubert_weights(0), syn.make_rmvpe_weights(0)
    with tempfile.TemporaryDirectory() as d:
        # files the facade looks for; their contents come from the replaced loaders
        os.makedirs(os.path.join(d, "hubert_base"))
        os.makedirs(os.path.join(d, "rmvpe"))
        for p in ("hubert_base/pytorch_model.bin", "rmvpe/rmvpe.pt", "model.pth"):
            open(os.path.join(d, p), "wb").close()
        rvc.ASSETS = Path(d)
        rvc.load_pth = lambda path: {"weight": w, "config": cfg, "version": "v2", "f0": 1}
        rv._load_ckpt = lambda path: {"weight": w, "config": cfg}
        rh.load_pth = lambda path: hsd
        rr.load_pth = lambda path: rsd
        idx_path = os.path.join(d, "model_added.npz")
        _index().save(idx_path)
        wav_path = os.path.join(d, "in.wav")
        _write_wav(wav_path, syn.make_speech_audio(CLIP_S, seed=CLIP_SEED + 1, silence_every=1.2))
        if os.environ.get("RVC_BACKEND") == "numpy":
            _pool_release_stand_in()
        v = rvc.VC(Config())
        info = v.get_vc(os.path.join(d, "model.pth"))
        if not info["success"]:
            raise RuntimeError(info.get("traceback") or info["error"])
        done = _record_margins()
        try:
            msg, (sr, y) = v.vc_single(0, wav_path, 0, "pm", idx_path, 0.75, 0, 0.25, 0.33)
        finally:
            out["vc_margins"] = np.array(done(), np.float64)
    out["vc_sr"] = np.array(sr)
    out["vc_int16"] = np.asarray(y)


# BASELINE config 4 at its full 60 s: the speech-like clip, RMVPE f0, HuBERT,
# retrieval at index_rate 0.75, protect 0.33, v2-40k synthesizer, rms mix
# 0.25, default split (two chunks near 38 s).  The index has 8 rows (no top-k
# near-ties, see INDEX_N) and f0_up_key 9 keeps every coarse-pitch decision of
# this clip >= 0.04 bins from a rounding point.
C4_SECONDS, C4_SEED, C4_KEY, C4_STRIDE = 60.0, 0, 9, 11


def config4_kwargs():
    return dict(f0_up_key=C4_KEY, f0_method="rmvpe", index_rate=0.75, if_f0=1, tgt_sr=40000, resample_sr=0,
                rms_mix_rate=0.25, version="v2", protect=0.33)


def _case_config4(out):
    from oracle import reference as oref  # noqa: PLC0415
    from runtime.native_config import Config  # noqa: PLC0415
    from runtime.pipeline import Pipeline  # noqa: PLC0415

    hub, net = _models()
    audio = syn.make_speech_audio(C4_SECONDS, seed=C4_SEED)
    pipe = Pipeline(40000, Config())
    pipe.model_rmvpe = oref.rmvpe(syn.make_rmvpe_weights(0))
    kw = config4_kwargs()
    done = _record_margins()
    try:
        sr, y = pipe.pipeline(hub, net, 0, audio, [0.0, 0.0, 0.0], kw["f0_up_key"], kw["f0_method"], _index(),
                              kw["index_rate"], kw["if_f0"], kw["tgt_sr"], kw["resample_sr"], kw["rms_mix_rate"],
                              kw["version"], kw["protect"])
    finally:
        out["config4_margins"] = np.array(done(), np.float64)
    y = np.asarray(y)
    out["config4_len"] = np.array(y.size)
    out["config4_int16_every"] = y[::C4_STRIDE].copy()


CASES = {"ops": _case_ops, "synth": _case_synth, "pipeline": _case_pipeline, "vc": _case_vc,
         "config4": _case_config4}
FIXTURE_CASES = "ops,synth,pipeline,vc"


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--backend", choices=["numpy", "cuda"], required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--cases", default=FIXTURE_CASES)
    args = ap.parse_args(argv)
    os.environ["RVC_BACKEND"] = args.backend
    os.environ["RVC_FIXED_SEED"] = str(SEED)
    from oracle import reference as oref  # noqa: PLC0415

    oref.activate(args.backend)
    if args.backend == "cuda":
        import rvc_cuda  # noqa: PLC0415

        rvc_cuda.register()
        rvc_cuda.patch_reference()
    out: dict = {}
    for name in args.cases.split(","):
        CASES[name](out)
    np.savez_compressed(args.out, **out)
    print("reference_runs:", args.backend, sorted(out))


if __name__ == "__main__":
    main()
