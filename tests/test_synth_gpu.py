"""Synthesizer parity: CudaSynthesizer (GPU, whole model through the C ABI)
against the oracle and the reference's golden vectors.

Bars: waveform max-abs error <= 1e-3 and per-layer
relative L2 <= 1e-3, on identical seeded weights, inputs and noise.
"""

import numpy as np
import pytest

from oracle import vits as OV
from rvc_cuda import synthetic as syn
from tests.conftest import load_golden, rel_l2

pytestmark = pytest.mark.gpu

from rvc_cuda import synth  # noqa: E402

WAVE_TOL = 1e-3
LAYER_TOL = 1e-3
_models = {}


def model(sr, seed, precision="bf16x3"):
    key = (sr, seed, precision)
    if key not in _models:
        w = syn.make_vits_weights(sr, seed)
        _models[key] = (w, synth.CudaSynthesizer(w, syn.vits_config_array(sr), precision=precision))
    return _models[key]


def run_case(sr, P, wseed, iseed, nseed, precision="bf16x3"):
    w, m = model(sr, wseed, precision)
    phone, pitch, nsff0, sid = syn.make_vits_inputs(P, iseed)
    nz, ns = syn.make_vits_noise(P, m.upp, nseed)
    m.keep_taps(True)
    wav = m.infer_controlled(phone, pitch, nsff0, sid, nz, ns)
    taps = {}
    ref = OV.synth(w, syn.vits_config_array(sr), phone, pitch, nsff0, sid, nz, ns, taps)
    return m, wav, ref, taps



@pytest.mark.parametrize("name", ["vits40k_p32", "vits48k_p24", "vits40k_p7"])
def test_synth_matches_golden(name, golden_meta):
    g = golden_meta[name]
    w, m = model(g["sr"], g["weight_seed"])
    phone, pitch, nsff0, sid = syn.make_vits_inputs(g["P"], g["input_seed"])
    nz, ns = syn.make_vits_noise(g["P"], g["upp"], g["noise_seed"])
    wav = m.infer_controlled(phone, pitch, nsff0, sid, nz, ns)
    gold = load_golden(name)
    assert wav.shape == (1, 1, g["P"] * g["upp"])
    err = np.abs(wav.reshape(-1) - gold["wave"]).max()
    assert err <= WAVE_TOL, err


@pytest.mark.parametrize("sr,P", [(40000, 64), (48000, 40)])
def test_synth_per_layer(sr, P):
    m, wav, ref, taps = run_case(sr, P, 0, 5, 55)
    H = m.hidden
    checks = {"enc.embed": (P, H), "enc.l0": (P, H), "enc.l5": (P, H), "enc.zp": (P, H), "flow.z": (P, H),
              "dec.har": (P * m.upp,), "dec.pre": (P, 512)}
    L = P
    for i, r in enumerate(m.arch["rates"]):
        L *= r
        checks[f"dec.s{i}.ups"] = (L, 512 >> (i + 1))
        checks[f"dec.s{i}.out"] = (L, 512 >> (i + 1))
    worst = {}
    for k, shp in checks.items():
        got = m.tap(k, shp)
        worst[k] = rel_l2(got, taps[k])
    bad = {k: v for k, v in worst.items() if not v <= LAYER_TOL}
    assert not bad, (bad, worst)
    assert np.abs(wav - ref).max() <= WAVE_TOL


def test_synth_simt_precision_agrees():
    _, wav, ref, _ = run_case(40000, 20, 0, 6, 66, precision="simt")
    assert np.abs(wav - ref).max() <= WAVE_TOL


def test_synth_batch_equals_single():
    w, m = model(40000, 0)
    P, B = 24, 3
    ins = [syn.make_vits_inputs(P, 100 + i) for i in range(B)]
    noise = [syn.make_vits_noise(P, m.upp, 200 + i) for i in range(B)]
    batch = m.infer_batch(np.concatenate([i[0] for i in ins]), np.concatenate([i[1] for i in ins]),
                          np.concatenate([i[2] for i in ins]), np.concatenate([i[3] for i in ins]),
                          np.concatenate([n[0] for n in noise]), np.stack([n[1].reshape(-1) for n in noise]))
    for i in range(B):
        one = m.infer_controlled(*ins[i], *noise[i]).reshape(-1)
        np.testing.assert_allclose(batch[i], one, rtol=0, atol=1e-6)


def test_grouped_infer_equals_per_group_calls():
    """``infer_batch(..., group=G)`` (copies of one group overlapping the next
    group's synthesis on separate streams) gives exactly the per-group
    ``infer_batch`` results, the short last group included, twice in a row
    (the double buffers are reused)."""
    w, m = model(48000, 0)
    P, B, G = 40, 5, 2
    ins = [syn.make_vits_inputs(P, 300 + i) for i in range(B)]
    noise = [syn.make_vits_noise(P, m.upp, 400 + i) for i in range(B)]
    args = (np.concatenate([i[0] for i in ins]), np.concatenate([i[1] for i in ins]),
            np.concatenate([i[2] for i in ins]), np.concatenate([i[3] for i in ins]),
            np.concatenate([n[0] for n in noise]), np.stack([n[1].reshape(-1) for n in noise]))
    ref = np.concatenate([m.infer_batch(*[a[s:s + G] for a in args]) for s in range(0, B, G)])
    for _ in range(2):
        got = m.infer_batch(*args, group=G)
        np.testing.assert_array_equal(got, ref)
    assert np.array_equal(m.infer_batch(*args, group=B), m.infer_batch(*args))


def test_synth_long_chunk_properties():
    """Full 10 s chunk (P=1000): output shape, finite, bounded, deterministic."""
    w, m = model(40000, 0)
    phone, pitch, nsff0, sid = syn.make_vits_inputs(1000, 9)
    nz, ns = syn.make_vits_noise(1000, m.upp, 99)
    a = m.infer_controlled(phone, pitch, nsff0, sid, nz, ns)
    b = m.infer_controlled(phone, pitch, nsff0, sid, nz, ns)
    assert a.shape == (1, 1, 400000)
    assert np.isfinite(a).all() and np.abs(a).max() <= 1.0
    np.testing.assert_array_equal(a, b)
    assert 0.05 < a.std() < 0.8


def test_enc_p_long_sequence_key_split():
    """The text encoder on one 10 s chunk (P = 1000: 8 query tiles x 2 heads,
    so the tensor-core attention splits the keys and merges the ranges)
    against the oracle's text encoder, layer by layer."""
    w, m = model(40000, 0)
    P = 1000
    phone, pitch, nsff0, sid = syn.make_vits_inputs(P, 9)
    nz, ns = syn.make_vits_noise(P, m.upp, 99)
    m.keep_taps(True)
    m.infer_controlled(phone, pitch, nsff0, sid, nz, ns)
    taps = {}
    OV.text_encoder(w, OV.VitsShape(w, syn.vits_config_array(40000)), phone, pitch, taps)
    for k in ("enc.embed", "enc.l0", "enc.l3", "enc.l5"):
        err = rel_l2(m.tap(k, (P, m.hidden)), taps[k])
        assert err <= LAYER_TOL, (k, err)


def test_seeded_infer_matches_infer_controlled():
    w, m = model(40000, 0)
    phone, pitch, nsff0, sid = syn.make_vits_inputs(16, 3)
    a = m.infer(phone, pitch, nsff0, sid, seed=1234)
    nz, ns = syn.make_vits_noise(16, m.upp, 1234)
    b = m.infer_controlled(phone, pitch, nsff0, sid, nz, ns)
    np.testing.assert_array_equal(a, b)


def test_bad_inputs_raise():
    w, m = model(40000, 0)
    phone, pitch, nsff0, sid = syn.make_vits_inputs(8, 3)
    nz, ns = syn.make_vits_noise(8, m.upp, 1)
    with pytest.raises(ValueError):
        m.infer_controlled(phone, pitch + 300, nsff0, sid, nz, ns)
    with pytest.raises(ValueError):
        m.infer_controlled(phone, pitch, nsff0, np.array([5]), nz, ns)


@pytest.mark.parametrize("name", ["vits40k_p96_part", "vits48k_p40_part"])
def test_partial_synthesis_matches_golden(name, golden_meta):
    """infer with skip_head / return_length (SynthesizerTrn._infer_partial)."""
    g = golden_meta[name]
    w, m = model(g["sr"], g["weight_seed"])
    phone, pitch, nsff0, sid = syn.make_vits_inputs(g["P"], g["input_seed"])
    nz, ns = syn.make_vits_noise(g["P"], g["upp"], g["noise_seed"])
    wav = m.infer_partial(phone, pitch, nsff0, sid, nz, ns, g["head"], g["length"])
    gold = load_golden(name)
    assert wav.shape == (1, 1, g["length"] * g["upp"])
    assert np.abs(wav.reshape(-1) - gold["wave"]).max() <= WAVE_TOL


def test_partial_equals_slice_of_full_interior():
    """Away from the segment edges, partial synthesis equals the full synthesis'
    samples (the reference's stated property, runtime/models/vits.py:2381-2388)."""
    w, m = model(40000, 0)
    P, head, length = 120, 60, 24
    phone, pitch, nsff0, sid = syn.make_vits_inputs(P, 21)
    nz, ns = syn.make_vits_noise(P, m.upp, 22)
    full = m.infer_controlled(phone, pitch, nsff0, sid, nz, ns).reshape(-1)
    part = m.infer_partial(phone, pitch, nsff0, sid, nz, ns, head, length).reshape(-1)
    seg = full[head * m.upp:(head + length) * m.upp]
    assert np.abs(part - seg).max() <= WAVE_TOL
    with pytest.raises(ValueError):
        m.infer_partial(phone, pitch, nsff0, sid, nz, ns, P - 4, 8)


def test_prep_dec_decode_batch_ragged_and_partial():
    """The pipeline's batched decode (prep_dec + decode_batch): equal-length
    chunks share a call, other lengths and partial preps run on their own; each
    result equals the single-chunk path with the same noise up to fp32
    rounding (the kernel plans follow the batch: column-tile widths and
    attention key splits differ between a batch of two and one chunk)."""
    w, m = model(40000, 0)
    ins = [syn.make_vits_inputs(P, 30 + i) for i, P in enumerate((48, 48, 33))]
    preps = [m.prep_dec(*x, seed=100 + i) for i, x in enumerate(ins)]
    preps.append(m.prep_dec(*ins[2], seed=200, skip_head=10, return_length=12))
    waves = m.decode_batch(preps)
    assert [wv.shape[-1] for wv in waves] == [48 * m.upp, 48 * m.upp, 33 * m.upp, 12 * m.upp]
    for x, p, wv in zip(ins, preps[:3], waves[:3]):
        ref = m.infer_controlled(x[0], x[1], x[2], x[3], p["nz"], p["ns"])
        assert np.abs(wv - ref).max() <= 1e-4
    pp = preps[3]
    ref = m.infer_partial(*ins[2], pp["nz"], pp["ns"], 10, 12)
    assert np.abs(waves[3] - ref).max() <= 1e-4


def test_synth_pool_matches_one_device():
    """``rvc_cuda.multi.SynthPool`` (the multi-GPU entry of the pipeline and of
    ``patch_reference`` under ``RVC_CUDA_DEVICES``): chunks spread over the
    devices (two GPUs when present, else two models on GPU 0) come back in
    order, equal to one device's ``decode_batch`` up to fp32 rounding (the
    batch sizes per call differ, and with them the kernel plans)."""
    from rvc_cuda import _lib
    from rvc_cuda.multi import SynthPool

    w, m = model(40000, 0)
    devs = [0, 1] if _lib.device_count() >= 2 else [0, 0]
    pool = SynthPool(w, syn.vits_config_array(40000), devices=devs)
    ins = [syn.make_vits_inputs(P, 60 + i) for i, P in enumerate((48, 20, 48, 33, 48))]
    preps = [m.prep_dec(*x, seed=300 + i) for i, x in enumerate(ins)]
    got = pool.decode_batch(preps)
    ref = m.decode_batch(preps)
    assert [g.shape for g in got] == [r.shape for r in ref]
    for g, r in zip(got, ref):
        assert np.abs(g - r).max() <= 1e-4
    pool.close()
