"""Pipeline signal processing on the CPU: the oracle against the reference's
own outputs (``tests/golden/dsp.npz``), and the device pipeline's host
orchestration (chunking, f0 assembly, alignment) run with the oracle's DSP in
place of the device calls, against whole reference pipeline runs with the
stand-in models of ``tests/golden/pipeline_fakes.py``.

The oracle restates the same numpy / scipy operations in the same order, so
everything here is compared bit-exactly.
"""

import types

import numpy as np
import pytest

from oracle import dsp as OD
from rvc_cuda import synthetic as syn
from tests.conftest import load_golden
from tests.golden import pipeline_fakes as pf
from tests.golden.make_golden import PIPE_CASES, digest

signal = pytest.importorskip("scipy.signal")
BH, AH = signal.butter(N=5, Wn=48, btype="high", fs=16000)


@pytest.fixture(scope="module")
def gold():
    return load_golden("dsp")


def test_filtfilt_oracle_matches_reference(gold, golden_meta):
    m = golden_meta["dsp"]["cases"]["hp_speech"]
    audio = syn.make_speech_audio(m["seconds"], seed=m["seed"])
    assert digest([audio]) == m["inputs_sha256"], "synthetic audio stream drifted"
    np.testing.assert_array_equal(OD.filtfilt(BH, AH, audio), gold["hp_speech"])
    np.testing.assert_array_equal(OD.filtfilt(BH, AH, gold["hp_edge_x"]), gold["hp_edge"])
    np.testing.assert_array_equal(OD.filtfilt(BH, AH, gold["hp_f64_x"]), gold["hp_f64"])
    with pytest.raises(ValueError):
        OD.filtfilt(BH, AH, gold["hp_edge_x"][:18])


def test_change_rms_oracle_matches_reference(gold, golden_meta):
    m = golden_meta["dsp"]["cases"]["rms"]
    d1 = syn.make_speech_audio(m["seconds"], seed=m["seed"])
    np.testing.assert_array_equal(OD.change_rms(d1, gold["rms_d2"], 16000, 40000, 0.25), gold["rms_out"])
    np.testing.assert_array_equal(OD.change_rms(d1, gold["rms_small_d2"], 16000, 48000, 0.6),
                                  gold["rms_small_out"])
    assert OD.change_rms(d1, np.zeros(0, np.float32), 16000, 40000, 0.25).size == 0


def test_prepare_oracle_matches_reference(gold):
    feats, pitch, pitchf = gold["prep_feats"], gold["prep_pitch"], gold["prep_pitchf"]
    f = OD.interpolate_linear(feats.transpose(0, 2, 1), 2).transpose(0, 2, 1)
    f0 = f.copy()
    n = f.shape[1]
    p, pfa = OD.align_frames(pitch, n), OD.align_frames(pitchf, n)
    np.testing.assert_array_equal(p, gold["prep_out_pitch"])
    np.testing.assert_array_equal(pfa, gold["prep_out_pitchf"])
    # with no retrieval feats0 == the interpolated features and the blend is exact arithmetic on them
    out = OD.protect_blend(f, f0, pfa, 0.33)
    np.testing.assert_array_equal(out, gold["prep_out"])


def _oracle_dsp():
    return types.SimpleNamespace(
        highpass=lambda a: OD.filtfilt(BH, AH, a),
        split_points=lambda a, tq, step, window=160: OD.split_points(a, window, tq, step),
        interpolate_linear=OD.interpolate_linear,
        protect_blend=OD.protect_blend,
        change_rms=OD.change_rms,
        to_int16=OD.to_int16,
        f0_autocorrelation=OD.f0_autocorrelation,
        resample=OD.resample,
    )


@pytest.mark.parametrize("name,kw", PIPE_CASES, ids=[c[0] for c in PIPE_CASES])
def test_pipeline_orchestration_matches_reference(name, kw, gold, golden_meta, monkeypatch):
    """The device pipeline's host logic with the oracle's DSP: split points and
    int16 output equal to the reference pipeline's, bit for bit."""
    from rvc_cuda import pipeline as P
    monkeypatch.setattr(P, "dsp", _oracle_dsp())
    m = golden_meta["dsp"]["cases"][name]
    a = syn.make_speech_audio(kw["seconds"], seed=kw["seed"], silence_every=kw["silence_every"])
    assert digest([a]) == m["inputs_sha256"]
    pipe = P.Pipeline(40000, pf.config(x_query=kw["x_query"]))
    pipe.model_rmvpe = pf.FakeRmvpe()
    starts = []
    orig = pipe.get_f0

    def get_f0(x, *args):
        starts.append(x.__array_interface__["data"][0])
        return orig(x, *args)

    pipe.get_f0 = get_f0
    sr, out = pipe.pipeline(pf.FakeHubert(D=768), pf.FakeSynth(gain=kw["gain"]), 0, a, [0.0, 0.0, 0.0],
                            kw["f0_up_key"], kw.get("f0", "rmvpe"), None, 0, True, 40000, kw.get("resample_sr", 0),
                            kw["rms"], 2, kw["protect"], slice_length=kw["slice_length"])
    assert sr == 40000 and out.dtype == np.int16 and out.size == m["out_len"]
    split = [(p - starts[0]) // 8 - pipe.t_pad for p in starts[1:]]
    np.testing.assert_array_equal(split, gold[name + "_split"])
    if name + "_int16" in gold:
        np.testing.assert_array_equal(out, gold[name + "_int16"])
    else:
        np.testing.assert_array_equal(out[::101], gold[name + "_int16_every101"])


def test_pipeline_concurrent_f0_segments_match_reference(gold, golden_meta, monkeypatch):
    """With an f0 model offering ``infer_many`` (the device RMVPE's concurrent
    segments) the pipeline's segment slicing and f0 post-processing still give
    the reference's split points and int16 output, bit for bit."""
    from rvc_cuda import pipeline as P
    name, kw = next(c for c in PIPE_CASES if c[0] == "pipe_split")
    monkeypatch.setattr(P, "dsp", _oracle_dsp())
    m = golden_meta["dsp"]["cases"][name]
    a = syn.make_speech_audio(kw["seconds"], seed=kw["seed"], silence_every=kw["silence_every"])

    class ManyRmvpe(pf.FakeRmvpe):
        calls = []

        def infer_many(self, xs, thred=0.03):
            self.calls.append(len(xs))
            return [self.infer_from_audio(x, thred) for x in xs]

    pipe = P.Pipeline(40000, pf.config(x_query=kw["x_query"]))
    pipe.model_rmvpe = ManyRmvpe()
    sr, out = pipe.pipeline(pf.FakeHubert(D=768), pf.FakeSynth(gain=kw["gain"]), 0, a, [0.0, 0.0, 0.0],
                            kw["f0_up_key"], "rmvpe", None, 0, True, 40000, 0, kw["rms"], 2, kw["protect"],
                            slice_length=kw["slice_length"])
    assert ManyRmvpe.calls and ManyRmvpe.calls[0] > 1
    assert out.size == m["out_len"]
    if name + "_int16" in gold:
        np.testing.assert_array_equal(out, gold[name + "_int16"])
    else:
        np.testing.assert_array_equal(out[::101], gold[name + "_int16_every101"])


def _pm_audio(golden_meta):
    m = golden_meta["dsp"]["cases"]["pm"]
    a = syn.make_speech_audio(m["seconds"], seed=m["seed"], silence_every=0.6, silence_len=0.2)
    a[3000:3400] += (0.3 * np.random.RandomState(91_005).standard_normal(400)).astype(np.float32)
    assert digest([a]) == m["inputs_sha256"]
    return a, m


def test_pm_f0_oracle_matches_reference(gold, golden_meta, monkeypatch):
    a, m = _pm_audio(golden_meta)
    np.testing.assert_array_equal(OD.f0_autocorrelation(a.astype(np.float64), 16000), gold["pm_f0"])
    # the device pipeline's get_f0("pm") host logic (padding, post-processing) with the oracle's f0
    from rvc_cuda import pipeline as P
    monkeypatch.setattr(P, "dsp", types.SimpleNamespace(f0_autocorrelation=OD.f0_autocorrelation))
    coarse, f0bak = P.Pipeline(40000, pf.config()).get_f0(a.astype(np.float64), m["p_len"], 4, "pm")
    np.testing.assert_array_equal(coarse, gold["pm_coarse"])
    np.testing.assert_array_equal(f0bak, gold["pm_f0bak"])


@pytest.mark.parametrize("method", ["fft", "linear", "sinc"])
def test_resample_oracle_matches_reference(method, gold):
    for sr, tag in ((48000, "48k"), (16000, "16k")):
        np.testing.assert_array_equal(OD.resample(gold["rs_x"], 40000, sr, method), gold[f"rs_{method}_{tag}"])


def test_pipeline_rejects_what_is_not_on_the_device_path():
    from rvc_cuda import pipeline as P
    pipe = P.Pipeline(40000, pf.config())
    with pytest.raises(RuntimeError):  # no model_fcpe assigned
        pipe.get_f0(np.zeros(1000), 6, 0, "fcpe")
    with pytest.raises(ValueError):
        pipe.get_f0(np.zeros(1000), 6, 0, "crepe")
    with pytest.raises(NotImplementedError):
        pipe.pipeline(None, None, 0, np.zeros(16000, np.float32), [0, 0, 0], 0, "rmvpe", None, 0, False, 40000,
                      0, 1, 2, 0.33)
