"""FCPE parity: the device model (C ABI) against the reference's numpy FCPE
(golden fixtures) and the oracle.

Bars: per-layer relative L2 <= 1e-3 (north star; measured ~1e-6 with BF16x3),
the latent argmax bit-exact, f0 within 1e-4 relative (0 where unvoiced), the
log-mel within 1e-6 (float64 direct DFT against numpy's FFT).
"""

import numpy as np
import pytest

from oracle import fcpe as OF
from rvc_cuda import synthetic as syn
from tests.conftest import load_golden, rel_l2

pytestmark = pytest.mark.gpu

from rvc_cuda import fcpe as fc  # noqa: E402

GOLD = ["fcpe_t24000", "fcpe_t3001", "fcpe_t400"]
_models = {}


def _model(precision="bf16x3"):
    if precision not in _models:
        _models[precision] = fc.CudaFcpe(syn.make_fcpe_weights(0), precision=precision)
    return _models[precision]


@pytest.mark.parametrize("name", GOLD)
def test_fcpe_matches_reference_golden(name, golden_meta):
    m = golden_meta[name]
    x = syn.make_rmvpe_input(m["T"], m["input_seed"])
    g = load_golden(name)
    model = _model()
    model.keep_taps(True)
    f0, am = model.infer_batch(x[None], return_argmax=True)
    F = fc.frames(m["T"])
    assert f0.shape == (1, F) and F == g["f0"].shape[0]
    mel = model.tap("mel", (F, 128))
    assert np.abs(mel - g["mel"]).max() < 1e-4 and rel_l2(mel, g["mel"]) < 1e-6
    lat = model.tap("latent", (F, 360))
    assert rel_l2(lat, g["latent"]) < 1e-3
    np.testing.assert_array_equal(am[0], g["argmax"])
    np.testing.assert_array_equal(f0[0] == 0, g["f0"] == 0)
    np.testing.assert_allclose(f0[0], g["f0"], rtol=1e-4)
    model.keep_taps(False)


@pytest.mark.parametrize("name", ["fcpe_t24000", "fcpe_t3001"])
def test_fcpe_argmax_decoder_matches_reference_golden(name, golden_meta):
    """``decoder_mode="argmax"`` (``runtime/models/fcpe.py:318-322``): the
    latent-weighted mean of the cents over all 360 bins, summed in numpy's
    pairwise order; f0 within float32 rounding of the latent (rel 1e-4)."""
    m = golden_meta[name]
    x = syn.make_rmvpe_input(m["T"], m["input_seed"])
    g = load_golden(name)
    f0 = _model().infer(x, decoder_mode="argmax")
    assert f0.shape == g["f0_argmax"].shape
    np.testing.assert_array_equal(f0 == 0, g["f0_argmax"] == 0)
    np.testing.assert_allclose(f0, g["f0_argmax"], rtol=1e-4, atol=1e-3)
    with pytest.raises(ValueError):
        _model().infer(x, decoder_mode="median")


def test_fcpe_layers_against_oracle_and_simt():
    sd = syn.make_fcpe_weights(0)
    x = syn.make_rmvpe_input(16000, 9)
    taps = {}
    ref = OF.infer(sd, x, taps=taps)
    F = fc.frames(16000)
    for prec, tol in (("bf16x3", 1e-4), ("simt", 1e-5)):
        model = _model(prec)
        model.keep_taps(True)
        f0 = model.infer(x)
        for name in ["stack"] + [f"layer{i}" for i in range(6)]:
            assert rel_l2(model.tap(name, (F, 512)), taps[name]) < tol, (prec, name)
        assert rel_l2(model.tap("latent", (F, 360)), taps["latent"]) < tol
        np.testing.assert_allclose(f0, ref, rtol=1e-4)
        model.keep_taps(False)


def test_fcpe_batch_equals_single_and_pipeline_get_f0(golden_meta):
    model = _model()
    xs = np.stack([syn.make_rmvpe_input(9600, s) for s in (1, 2, 3)])
    fb = model.infer_batch(xs)
    for i in range(3):
        np.testing.assert_array_equal(fb[i], model.infer(xs[i]))
    # the device pipeline's get_f0("fcpe") against the reference's on the same model
    from rvc_cuda.pipeline import Pipeline
    from tests.golden import pipeline_fakes as pf
    m = golden_meta["fcpe_t24000"]
    x = syn.make_rmvpe_input(m["T"], m["input_seed"])
    g = load_golden("fcpe_t24000")
    pipe = Pipeline(40000, pf.config())
    pipe.model_fcpe = model
    coarse, f0bak = pipe.get_f0(x.astype(np.float64), m["T"] // 160 + 1, 3, "fcpe")
    assert np.abs(coarse.astype(int) - g["pipe_coarse"].astype(int)).max() <= 1
    np.testing.assert_allclose(f0bak, g["pipe_f0bak"], rtol=1e-4)
    with pytest.raises(NotImplementedError):
        model.infer(x, sr=22050)
