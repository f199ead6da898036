"""HuBERT parity: CudaHubert (GPU, whole encoder through the C ABI) against the
oracle and the reference's golden vectors.

Bar (float paths): relative L2 <= 1e-3 per layer and on
the output features, on identical seeded weights and inputs.
"""

import numpy as np
import pytest

from oracle import hubert as OH
from rvc_cuda import synthetic as syn
from tests.conftest import load_golden, rel_l2

pytestmark = pytest.mark.gpu

from rvc_cuda import hubert as hub  # noqa: E402

TOL = 1e-3
_models = {}


def model(seed=0, precision="bf16x3"):
    key = (seed, precision)
    if key not in _models:
        sd = syn.make_hubert_weights(seed)
        _models[key] = (OH.prepare(sd), hub.CudaHubert(sd, precision=precision))
    return _models[key]


@pytest.mark.parametrize("name", ["hubert_t8000", "hubert_t3201"])
def test_hubert_matches_golden(name, golden_meta):
    g = golden_meta[name]
    _, m = model(g["weight_seed"])
    x = syn.make_hubert_input(g["T"], g["input_seed"])
    gold = load_golden(name)
    m.keep_taps(True)
    out = m.encode(x, version=2)
    assert out.shape == (1,) + gold["out"].shape
    assert rel_l2(out[0], gold["out"]) <= TOL
    L = gold["conv"].shape[0]
    assert rel_l2(m.tap("conv6", (L, 512)), gold["conv"]) <= TOL
    out1 = m.encode(x, version=1)
    assert out1.shape == (1,) + gold["out_v1"].shape
    assert rel_l2(out1[0], gold["out_v1"]) <= TOL


def test_hubert_per_layer():
    sd, m = model(0)
    x = syn.make_hubert_input(16000, 7)
    taps = {}
    ref = OH.encode(sd, x, taps)
    m.keep_taps(True)
    out = m.encode(x)
    L = ref.shape[1]
    for i in range(7):
        r = taps[f"conv{i}"]
        got = m.tap(f"conv{i}", r.shape)
        assert rel_l2(got, r) <= TOL, (f"conv{i}", rel_l2(got, r))
    for name in ["proj", "pos"] + [f"layer{i}" for i in range(12)]:
        got = m.tap(name, (L, 768))
        assert rel_l2(got, taps[name]) <= TOL, (name, rel_l2(got, taps[name]))
    assert rel_l2(out[0], ref[0]) <= TOL


def test_hubert_simt_path_is_fp32_exact_to_oracle():
    sd, m = model(0, "simt")
    x = syn.make_hubert_input(8000, 3)
    ref = OH.encode(sd, x)
    out = m.encode(x)
    assert rel_l2(out[0], ref[0]) <= 2e-5


def test_hubert_batch_equals_single():
    _, m = model(0)
    xs = np.concatenate([syn.make_hubert_input(12000, s) for s in (11, 12, 13)], axis=0)
    yb = m.encode_equal(xs)
    for i in range(3):
        yi = m.encode(xs[i:i + 1])
        assert np.abs(yb[i] - yi[0]).max() <= 1e-6


def test_hubert_encode_batch_ragged_lengths():
    _, m = model(0)
    xs = [syn.make_hubert_input(T, s) for T, s in ((8000, 1), (3201, 2), (8000, 4), (5555, 5))]
    ys = m.encode_batch(xs)
    assert len(ys) == 4
    for x, y in zip(xs, ys):
        y1 = m.encode(x)
        assert y.shape == y1.shape == (1, hub.out_len(x.shape[1]), 768)
        assert np.abs(y - y1).max() <= 1e-6


def test_hubert_full_size_config1():
    """160000 samples -> [1,499,768] against the oracle."""
    sd, m = model(0)
    x = syn.make_hubert_input(160000, 0)
    out = m.encode(x)
    assert out.shape == (1, 499, 768)
    assert np.isfinite(out).all()
    ref = OH.encode(sd, x)
    assert rel_l2(out[0], ref[0]) <= TOL
    # post-LN rows (gamma 1, beta 0): zero mean, unit variance
    assert np.abs(out[0].mean(axis=1)).max() < 1e-4
    assert np.abs(out[0].var(axis=1) - 1.0).max() < 1e-2


def test_hubert_minimum_length_and_bad_inputs():
    _, m = model(0)
    T = 400  # the shortest input giving one frame
    assert hub.out_len(T) == 1 and hub.out_len(T - 1) == 0
    sd, _ = model(0)
    x = syn.make_hubert_input(T, 9)
    out = m.encode(x)
    assert out.shape == (1, 1, 768)
    assert rel_l2(out[0], OH.encode(sd, x)[0]) <= TOL
    with pytest.raises(ValueError):
        m.encode(syn.make_hubert_input(T - 1, 9))
    with pytest.raises(ValueError):
        m.encode(x, version=3)
    with pytest.raises(ValueError):
        m.encode(np.zeros((2, 1000), np.float32))
