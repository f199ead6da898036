"""Pipeline signal processing on the device (C ABI) against the reference's
outputs (``tests/golden/dsp.npz``) and the oracle, and the device pipeline
end to end.

Bars: the x2 interpolation, protect blend, int16 conversion and split points
are bit-exact (the same float32 / float64 operations in the same order).
``filtfilt`` runs the float64 DF2T recursion in blocks, each entered
after a warm-up from a zero state; for this filter float64 DF2T carries
~1e-7 relative rounding noise of its own (its zero-input responses grow to
~2e7 before they decay), which differs between any two evaluation orders, so
the bar is |error| <= 1e-6 x the signal's peak (bit-exact over the first
blocks, which start from the true initial state).  ``change_rms`` sums the RMS
frames in float64 rather than numpy's float32 pairwise order and uses the
device ``powf``: rel 1e-5.  Whole pipelines with the stand-in models: the
same split points, int16 within 2 LSB; with the device models against the
oracle models: the waveform tolerance of the models (1e-3 of full scale,
33 LSB).
"""

import numpy as np
import pytest

from oracle import dsp as OD
from rvc_cuda import synthetic as syn
from tests.conftest import load_golden
from tests.golden import pipeline_fakes as pf
from tests.golden.make_golden import PIPE_CASES

pytestmark = pytest.mark.gpu

from rvc_cuda import dsp  # noqa: E402
signal = pytest.importorskip("scipy.signal")
BH, AH = signal.butter(N=5, Wn=48, btype="high", fs=16000)


@pytest.fixture(scope="module")
def gold():
    return load_golden("dsp")


def _close_hp(y, ref):
    assert y.dtype == np.float64 and y.shape == ref.shape
    assert np.abs(y - ref).max() <= 1e-6 * max(1.0, np.abs(ref).max())


def test_filtfilt_matches_reference(gold, golden_meta):
    m = golden_meta["dsp"]["cases"]["hp_speech"]
    audio = syn.make_speech_audio(m["seconds"], seed=m["seed"])
    _close_hp(dsp.highpass(audio), gold["hp_speech"])
    _close_hp(dsp.filtfilt(BH, AH, gold["hp_edge_x"]), gold["hp_edge"])
    _close_hp(dsp.filtfilt(BH, AH, gold["hp_f64_x"]), gold["hp_f64"])
    with pytest.raises(Exception):
        dsp.filtfilt(BH, AH, gold["hp_edge_x"][:18])


def test_filtfilt_long_against_oracle():
    audio = syn.make_speech_audio(60.0, seed=0)
    _close_hp(dsp.highpass(audio), OD.filtfilt(BH, AH, audio))
    x = np.random.RandomState(5).standard_normal(100_003)  # float64, ragged block count
    b, a = signal.butter(N=3, Wn=0.2)
    _close_hp(dsp.filtfilt(b, a, x), OD.filtfilt(b, a, x))


@pytest.mark.parametrize("name,kw", PIPE_CASES, ids=[c[0] for c in PIPE_CASES])
def test_split_points_match_reference(name, kw, gold):
    a = syn.make_speech_audio(kw["seconds"], seed=kw["seed"], silence_every=kw["silence_every"])
    t_max = int(kw["slice_length"] * 16000) if kw["slice_length"] > 0 else 41 * 16000
    if a.size + 160 <= t_max:
        assert gold[name + "_split"].size == 0
        return
    step = min(38 * 16000, t_max)
    tq = kw["x_query"] * 16000
    # on the reference's filtered signal (the oracle is bit-exact to scipy) ...
    assert dsp.split_points(OD.filtfilt(BH, AH, a), tq, step) == list(gold[name + "_split"])
    # ... and on the device's own
    assert dsp.split_points(dsp.highpass(a), tq, step) == list(gold[name + "_split"])


def test_split_points_against_oracle_edges():
    rs = np.random.RandomState(7)
    x = np.abs(rs.standard_normal(5000))
    x[1000:1400] = 0.0  # an exact-zero plateau: the first index of the minimum wins
    for tq, step in ((300, 700), (50, 1000), (5000, 2500), (0, 900)):
        assert dsp.split_points(x, tq, step) == OD.split_points(x, 160, tq, step)


def test_interp_protect_match_reference(gold):
    feats, pitchf = gold["prep_feats"], gold["prep_out_pitchf"]
    f = dsp.interpolate_linear(feats, 2, axis=1)
    np.testing.assert_array_equal(f, OD.interpolate_linear(feats.transpose(0, 2, 1), 2).transpose(0, 2, 1))
    np.testing.assert_array_equal(dsp.protect_blend(f, f, pitchf, 0.33), gold["prep_out"])
    rs = np.random.RandomState(3)
    x = rs.standard_normal((2, 37, 5)).astype(np.float32)
    for scale, axis in ((2, 1), (3, -1), (1.5, 0)):
        np.testing.assert_array_equal(dsp.interpolate_linear(x, scale, axis), OD.interpolate_linear(x, scale, axis))
    f1, f0 = rs.standard_normal((2, 1, 50, 768)).astype(np.float32)
    pf_ = rs.uniform(-1, 3, (1, 50)).astype(np.float32)
    np.testing.assert_array_equal(dsp.protect_blend(f1, f0, pf_, 0.2), OD.protect_blend(f1, f0, pf_, 0.2))


def test_change_rms_matches_reference(gold, golden_meta):
    m = golden_meta["dsp"]["cases"]["rms"]
    d1 = syn.make_speech_audio(m["seconds"], seed=m["seed"])
    np.testing.assert_allclose(dsp.change_rms(d1, gold["rms_d2"], 16000, 40000, 0.25), gold["rms_out"],
                               rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(dsp.change_rms(d1, gold["rms_small_d2"], 16000, 48000, 0.6), gold["rms_small_out"],
                               rtol=1e-5, atol=1e-7)
    assert dsp.change_rms(d1, np.zeros(0, np.float32), 16000, 40000, 0.25).size == 0
    long1 = syn.make_speech_audio(60.0, seed=1)
    long2 = np.repeat(long1, 5)[: 60 * 40000] * 1.7
    np.testing.assert_allclose(dsp.change_rms(long1, long2, 16000, 40000, 0.25),
                               OD.change_rms(long1, long2, 16000, 40000, 0.25), rtol=1e-5, atol=1e-7)


def test_pm_f0_matches_reference(gold, golden_meta):
    m = golden_meta["dsp"]["cases"]["pm"]
    a = syn.make_speech_audio(m["seconds"], seed=m["seed"], silence_every=0.6, silence_len=0.2)
    a[3000:3400] += (0.3 * np.random.RandomState(91_005).standard_normal(400)).astype(np.float32)
    np.testing.assert_array_equal(dsp.f0_autocorrelation(a.astype(np.float64), 16000), gold["pm_f0"])
    from rvc_cuda.pipeline import Pipeline
    coarse, f0bak = Pipeline(40000, pf.config()).get_f0(a.astype(np.float64), m["p_len"], 4, "pm")
    np.testing.assert_array_equal(coarse, gold["pm_coarse"])
    np.testing.assert_array_equal(f0bak, gold["pm_f0bak"])
    # other rates, hops and ranges against the oracle; a silent input is all unvoiced
    x = syn.make_speech_audio(2.0, seed=8).astype(np.float64)
    for kw in ({"sr": 16000, "time_step": 0.005}, {"sr": 22050, "f0_min": 80.0, "f0_max": 600.0},
               {"sr": 16000, "voicing_threshold": 0.3}):
        sr = kw.pop("sr")
        np.testing.assert_array_equal(dsp.f0_autocorrelation(x, sr, **kw), OD.f0_autocorrelation(x, sr, **kw))
    assert not dsp.f0_autocorrelation(np.zeros(4000), 16000).any()


@pytest.mark.parametrize("method", ["fft", "linear", "sinc"])
def test_resample_matches_reference(method, gold):
    """fft: cuFFT double transforms and the device Kaiser-sinc spectral
    interpolation against numpy's pocketfft path: within 1e-6 of full scale;
    sinc: device sin / power-series I0 in the taps: 1e-6; linear: exact."""
    for sr, tag in ((48000, "48k"), (16000, "16k")):
        y = dsp.resample(gold["rs_x"], 40000, sr, method)
        ref = gold[f"rs_{method}_{tag}"]
        assert y.dtype == np.float32 and y.shape == ref.shape
        if method == "linear":
            np.testing.assert_array_equal(y, ref)
        else:
            assert np.abs(y - ref).max() <= 1e-6
    # a long odd-length signal (a cuFFT size with a large prime factor) against the oracle
    x = syn.make_speech_audio(7.3, seed=4)[:116_803]
    np.testing.assert_allclose(dsp.resample(x, 16000, 44100, method), OD.resample(x, 16000, 44100, method),
                               atol=1e-6 if method != "linear" else 0, rtol=0)


def test_to_int16_matches_oracle():
    rs = np.random.RandomState(11)
    for peak in (0.5, 0.99, 1.0, 1.7, 40.0):
        x = rs.uniform(-1, 1, 123_457).astype(np.float32)
        x *= np.float32(peak) / np.abs(x).max()
        np.testing.assert_array_equal(dsp.to_int16(x), OD.to_int16(x))
    np.testing.assert_array_equal(dsp.to_int16(np.zeros(1000, np.float32)), np.zeros(1000, np.int16))


@pytest.mark.parametrize("name,kw", PIPE_CASES, ids=[c[0] for c in PIPE_CASES])
def test_device_pipeline_with_stand_ins_matches_reference(name, kw, gold, golden_meta):
    from rvc_cuda.pipeline import Pipeline
    m = golden_meta["dsp"]["cases"][name]
    a = syn.make_speech_audio(kw["seconds"], seed=kw["seed"], silence_every=kw["silence_every"])
    pipe = Pipeline(40000, pf.config(x_query=kw["x_query"]))
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
    assert sr == 40000 and out.size == m["out_len"]
    np.testing.assert_array_equal([(p - starts[0]) // 8 - pipe.t_pad for p in starts[1:]], gold[name + "_split"])
    ref = gold[name + "_int16"] if name + "_int16" in gold else None
    got = out if ref is not None else out[::101]
    ref = ref if ref is not None else gold[name + "_int16_every101"]
    assert np.abs(got.astype(np.int32) - ref.astype(np.int32)).max() <= 2


class _OracleHubert:
    def __init__(self, sd):
        from oracle import hubert as OH
        self.OH, self.p = OH, OH.prepare(sd)

    def encode(self, x, version=2):
        return self.OH.encode(self.p, np.asarray(x, np.float32), version=version)


class _OracleSynth:
    def __init__(self, w, sr):
        from oracle import vits as OV
        self.OV, self.w, self.cfg = OV, w, syn.vits_config_array(sr)
        self.upp = int(np.prod(syn.VITS_V2_40K[1] if sr == 40000 else syn.VITS_V2_48K[1]))

    def infer(self, phone, pitch, nsff0, sid, phone_gpu=None, seed=1234):
        P = phone.shape[1]
        nz, ns = syn.make_vits_noise(P, self.upp, seed)
        return self.OV.synth(self.w, self.cfg, phone, np.asarray(pitch, np.int64), nsff0, sid, nz, ns)


class _OracleRmvpe:
    def __init__(self, sd):
        from oracle import rmvpe as ORm
        self.ORm, self.sd = ORm, sd

    def infer_from_audio(self, x, thred=0.03):
        return self.ORm.infer(self.sd, np.asarray(x, np.float32), thred)


def test_device_pipeline_end_to_end_against_oracle(monkeypatch):
    """Device HuBERT + RMVPE + synthesizer + retrieval + DSP through
    ``rvc_cuda.pipeline.Pipeline`` against the same host logic driving the
    oracle models and the oracle DSP (1.6 s, split in two chunks, retrieval
    0.75, rms mix 0.25, protect 0.33)."""
    import types
    from rvc_cuda import pipeline as P
    from rvc_cuda.hubert import CudaHubert
    from rvc_cuda.rmvpe import CudaRmvpe
    from rvc_cuda.synth import CudaSynthesizer
    monkeypatch.setenv("RVC_FIXED_SEED", "1234")
    a = syn.make_speech_audio(1.6, seed=9, silence_every=0.8)
    hsd, rsd, vw = syn.make_hubert_weights(0), syn.make_rmvpe_weights(0), syn.make_vits_weights(40000, 0)
    db = syn.make_index(3000, 768, 1)
    kw = dict(f0_up_key=1, f0_method="rmvpe", index_rate=0.75, if_f0=True, tgt_sr=40000, resample_sr=0,
              rms_mix_rate=0.25, version=2, protect=0.33, slice_length=1.0)
    cfg = pf.config(x_query=1)

    pipe = P.Pipeline(40000, cfg)
    pipe.model_rmvpe = CudaRmvpe(rsd)
    _, out = pipe.pipeline(CudaHubert(hsd), CudaSynthesizer(vw, syn.vits_config_array(40000)), 0, a, [0.0, 0.0, 0.0],
                           file_index=db, **kw)

    shim = types.SimpleNamespace(
        highpass=lambda x: OD.filtfilt(BH, AH, x),
        split_points=lambda x, tq, step, window=160: OD.split_points(x, window, tq, step),
        interpolate_linear=OD.interpolate_linear, protect_blend=OD.protect_blend,
        change_rms=OD.change_rms, to_int16=OD.to_int16)

    class _OracleIndex:
        nlist = 0  # brute force (no IVF structure)

        def blend(self, q, k=8, mode="pipeline", feats=None, index_rate=1.0):
            from oracle import retrieval as OR
            sc, ix = OR.search_l2(q, db, k)
            w = np.square(1.0 / sc)
            w /= np.maximum(w.sum(axis=1, keepdims=True), 1e-12)
            b = np.sum(db[ix] * w[:, :, None], axis=1)
            return b * index_rate + feats * (1 - index_rate)

    monkeypatch.setattr(P, "dsp", shim)
    monkeypatch.setattr(P.Pipeline, "_resolve_index", staticmethod(lambda f, r: _OracleIndex()))
    opipe = P.Pipeline(40000, cfg)
    opipe.model_rmvpe = _OracleRmvpe(rsd)
    _, ref = opipe.pipeline(_OracleHubert(hsd), _OracleSynth(vw, 40000), 0, a, [0.0, 0.0, 0.0],
                            file_index=db, **kw)
    assert out.shape == ref.shape and out.dtype == np.int16
    assert np.abs(out.astype(np.int32) - ref.astype(np.int32)).max() <= 33


class _Proxy:
    """Forwards every attribute; not an instance of the library's model classes,
    so the pipeline takes its host-buffer path."""

    def __init__(self, m):
        self._m = m

    def __getattr__(self, k):
        return getattr(self._m, k)


@pytest.mark.parametrize("ivf", [False, True])
def test_device_resident_chain_equals_host_buffer_path(monkeypatch, ivf):
    """The HBM-resident chunk chain runs the same kernels as the host-buffer
    path: identical int16 output (2 chunks, retrieval brute force / IVF,
    protect, change_rms)."""
    from rvc_cuda import pipeline as P
    from rvc_cuda.hubert import CudaHubert
    from rvc_cuda.retrieval import CudaIndex
    from rvc_cuda.rmvpe import CudaRmvpe
    from rvc_cuda.synth import CudaSynthesizer
    monkeypatch.setenv("RVC_FIXED_SEED", "77")
    a = syn.make_speech_audio(2.2, seed=12, silence_every=1.0)
    hub = CudaHubert(syn.make_hubert_weights(0))
    net = CudaSynthesizer(syn.make_vits_weights(40000, 0), syn.vits_config_array(40000))
    db = syn.make_index(4000, 768, 3)
    index = CudaIndex(db)
    if ivf:
        rs = np.random.RandomState(1)
        cent = db[rs.choice(4000, 16, replace=False)]
        d = ((db[:, None, :] - cent[None]) ** 2).sum(-1)
        index.set_ivf(cent, d.argmin(1))
    pipe = P.Pipeline(40000, pf.config(x_query=1))
    pipe.model_rmvpe = CudaRmvpe(syn.make_rmvpe_weights(0), own_stream=True)  # f0 concurrently on its own stream
    kw = dict(f0_up_key=0, f0_method="rmvpe", index_rate=0.75, if_f0=True, tgt_sr=40000, resample_sr=0,
              rms_mix_rate=0.25, version=2, protect=0.33, slice_length=1.0)
    assert pipe._device_chain(hub, net, index) is hub.ctx
    _, dev = pipe.pipeline(hub, net, 0, a, [0.0, 0.0, 0.0], file_index=index, **kw)
    assert pipe._device_chain(_Proxy(hub), net, index) is None
    _, host = pipe.pipeline(_Proxy(hub), _Proxy(net), 0, a, [0.0, 0.0, 0.0], file_index=index, **kw)
    assert dev.shape == host.shape and dev.size > 40000
    np.testing.assert_array_equal(dev, host)
