"""RMVPE parity: CudaRmvpe (GPU, whole model through the C ABI) against the
reference's golden outputs and the oracle.

Bars: salience argmax bit-exact, float paths within
relative L2 1e-3 (measured far tighter: the device path is fp32 with a
float64 STFT).  An argmax may only differ where the oracle's own top-2
salience margin is below 1e-5 (fp32 summation-order ties).
"""

import numpy as np
import pytest

from oracle import rmvpe as ORM
from rvc_cuda import synthetic as syn
from tests.conftest import load_golden, rel_l2

pytestmark = pytest.mark.gpu

from rvc_cuda import rmvpe as rm  # noqa: E402

_models = {}


def model(seed=0):
    if seed not in _models:
        sd = syn.make_rmvpe_weights(seed)
        _models[seed] = (sd, rm.CudaRmvpe(sd))
    return _models[seed]


def _argmax_ok(am, sal, tie=1e-5):
    ref = np.argmax(sal, axis=1)
    bad = np.nonzero(am != ref)[0]
    for t in bad:
        srt = np.sort(sal[t])
        assert srt[-1] - srt[-2] < tie, f"frame {t}: argmax {am[t]} vs {ref[t]}, margin {srt[-1] - srt[-2]}"
    return len(bad)


@pytest.mark.parametrize("name", ["rmvpe_t16000", "rmvpe_t6401"])
def test_rmvpe_matches_reference_golden(name, golden_meta):
    g = golden_meta[name]
    _, m = model(g["weight_seed"])
    x = syn.make_rmvpe_input(g["T"], g["input_seed"])
    gold = load_golden(name)
    m.keep_taps(True)
    f0, am = m.infer_batch(x[None], return_argmax=True)
    F = gold["f0"].shape[0]
    Fp = 32 * ((F - 1) // 32 + 1)
    assert f0.shape == (1, F)
    mel = m.tap("mel", (Fp, 128))[:F].T
    np.testing.assert_allclose(mel, gold["mel"], rtol=1e-5, atol=1e-5)
    sal = m.tap("salience", (Fp, 360))[:F]
    assert rel_l2(sal, gold["salience"]) <= 1e-4
    np.testing.assert_array_equal(am[0], gold["argmax"])
    np.testing.assert_allclose(f0[0], gold["f0"], rtol=1e-5, atol=1e-3)


def test_rmvpe_per_layer_against_oracle():
    sd, m = model(0)
    x = syn.make_rmvpe_input(16000, 5)
    taps = {}
    ref_f0 = ORM.infer(sd, x, taps=taps)
    m.keep_taps(True)
    f0, am = m.infer_batch(x[None], return_argmax=True)
    F = ref_f0.shape[0]
    Fp = 32 * ((F - 1) // 32 + 1)
    for l in range(5):
        r = taps[f"enc{l}"][0].transpose(1, 2, 0)  # [H,W,C]
        H, W, Cc = r.shape
        got = m.tap(f"enc{l}", (H, W, 2 * Cc))[:, :, Cc:]
        assert rel_l2(got, r) <= 1e-4, (l, rel_l2(got, r))
    r = taps["inter"][0].transpose(1, 2, 0)
    assert rel_l2(m.tap("inter", r.shape), r) <= 1e-4
    for i in range(5):
        r = taps[f"dec{i}"][0].transpose(1, 2, 0)
        assert rel_l2(m.tap(f"dec{i}", r.shape), r) <= 1e-4, (i, rel_l2(m.tap(f"dec{i}", r.shape), r))
    assert rel_l2(m.tap("cnn", (Fp, 384)), taps["cnn"]) <= 1e-4
    assert rel_l2(m.tap("gru", (Fp, 512)), taps["gru"]) <= 1e-4
    sal = m.tap("salience", (Fp, 360))[:F]
    assert rel_l2(sal, taps["salience"]) <= 1e-4
    _argmax_ok(am[0], taps["salience"])
    np.testing.assert_allclose(f0[0], ref_f0, rtol=1e-4, atol=1e-2)


def test_rmvpe_full_size_config2():
    """10 s of 16 kHz audio -> 1001 frames, argmax vs the oracle."""
    sd, m = model(0)
    x = syn.make_rmvpe_input(160000, 0)
    taps = {}
    ref_f0 = ORM.infer(sd, x, taps=taps)
    f0, am = m.infer_batch(x[None], return_argmax=True)
    assert f0.shape == (1, 1001) and np.isfinite(f0).all()
    assert _argmax_ok(am[0], taps["salience"]) == 0
    np.testing.assert_allclose(f0[0], ref_f0, rtol=1e-4, atol=1e-2)


def test_rmvpe_batch_equals_single_and_bad_input():
    """A batch and its clips one by one: the same argmax; f0 within fp32
    rounding (the deep convs split their channel sums by the batch's tile
    count, so the summation order may differ)."""
    _, m = model(0)
    xs = np.stack([syn.make_rmvpe_input(9000, s) for s in (1, 2, 3)])
    fb, ab = m.infer_batch(xs, return_argmax=True)
    for i in range(3):
        f1, a1 = m.infer_batch(xs[i][None], return_argmax=True)
        np.testing.assert_array_equal(ab[i], a1[0])
        np.testing.assert_allclose(fb[i], f1[0], rtol=1e-5, atol=1e-4)
        np.testing.assert_array_equal(f1[0], m.infer_from_audio(xs[i]))
    with pytest.raises(ValueError):
        m.infer_from_audio(np.zeros(512, np.float32))
    with pytest.raises(ValueError):
        m.infer_from_audio(np.zeros((2, 1000), np.float32))
    assert rm.frames(160000) == 1001 and rm.frames(513) == 4
