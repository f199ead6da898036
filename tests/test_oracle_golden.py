"""Pin the oracle: it must reproduce the reference's own outputs.

The golden vectors were produced by running the reference's numpy CPU path
(``tests/golden/make_golden.py``).  Oracle and reference are both float32
numpy; they differ only in BLAS summation order, so the bar here is far
tighter than the CUDA parity bar.
"""

import numpy as np
import pytest

from tests.conftest import load_golden, rel_l2
from oracle import hubert as OH
from oracle import ops as O
from oracle import retrieval as OR
from oracle import vits as OV
from rvc_cuda import synthetic as syn
from tests.golden.make_golden import digest, weights_digest

VITS = ["vits40k_p32", "vits48k_p24", "vits40k_p7"]
HUB = ["hubert_t8000", "hubert_t3201"]


@pytest.mark.parametrize("name", VITS)
def test_vits_oracle_matches_reference(name, golden_meta):
    m = golden_meta[name]
    w = syn.make_vits_weights(m["sr"], m["weight_seed"])
    assert weights_digest(w) == m["weights_sha256"], "synthetic weight stream drifted"
    phone, pitch, nsff0, sid = syn.make_vits_inputs(m["P"], m["input_seed"])
    nz, ns = syn.make_vits_noise(m["P"], m["upp"], m["noise_seed"])
    assert digest([phone, pitch, nsff0, sid, nz, ns]) == m["inputs_sha256"]
    g = load_golden(name)
    taps = {}
    wav = OV.synth(w, syn.vits_config_array(m["sr"]), phone, pitch, nsff0, sid, nz, ns, taps)
    assert rel_l2(taps["enc.l5"], g["enc_h"]) < 1e-5
    assert rel_l2(taps["enc.m"], g["enc_m"]) < 1e-5
    assert rel_l2(taps["enc.logs"], g["enc_logs"]) < 1e-5
    assert rel_l2(taps["flow.z"], g["flow_z"]) < 1e-5
    assert wav.size == g["wave"].size
    assert np.abs(wav.reshape(-1) - g["wave"]).max() < 1e-5


@pytest.mark.parametrize("name", HUB)
def test_hubert_oracle_matches_reference(name, golden_meta):
    m = golden_meta[name]
    sd = syn.make_hubert_weights(m["weight_seed"])
    assert weights_digest(sd) == m["weights_sha256"]
    x = syn.make_hubert_input(m["T"], m["input_seed"])
    g = load_golden(name)
    taps = {}
    out = OH.encode(OH.prepare(sd), x, taps)
    assert rel_l2(taps["conv6"], g["conv"]) < 1e-5
    assert out.shape[1:] == g["out"].shape
    assert rel_l2(out[0], g["out"]) < 1e-5
    out1 = OH.encode(OH.prepare(sd), x, version=1)
    assert out1.shape[1:] == g["out_v1"].shape
    assert rel_l2(out1[0], g["out_v1"]) < 1e-5


def test_ops_oracle_matches_reference(golden_meta):
    g = load_golden("ops")
    for c in golden_meta["ops"]["cases"]:
        i = c["i"]
        if c["op"] == "conv1d":
            pad = tuple(c["padding"]) if isinstance(c["padding"], list) else c["padding"]
            y = O.conv1d(g[f"conv1d_{i}_x"], g[f"conv1d_{i}_w"], g[f"conv1d_{i}_b"],
                         c["stride"], pad, c["dilation"])
            np.testing.assert_allclose(y, g[f"conv1d_{i}_y"], rtol=1e-5, atol=1e-5)
        else:
            y = O.conv_transpose1d(g[f"convt_{i}_x"], g[f"convt_{i}_w"], g[f"convt_{i}_b"],
                                   c["stride"], c["padding"])
            np.testing.assert_allclose(y, g[f"convt_{i}_y"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(O.layer_norm(g["ln_x"], g["ln_g"], g["ln_b"]), g["ln_y"],
                               rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(O.softmax(g["sm_x"]), g["sm_y"], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(O.gelu_erf(g["gelu_x"]), g["gelu_y"], rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(O.leaky_relu(g["leaky_x"], 0.1), g["leaky_y"])


RET = ["ret_f200_n20000", "ret_f64_n3000_d256", "ret_f37_n5", "ret_f9_n1000_d60"]


@pytest.mark.parametrize("name", RET)
def test_retrieval_oracle_matches_reference(name, golden_meta):
    m = golden_meta[name]
    db = syn.make_index(m["N"], m["D"], m["index_seed"])
    q = syn.make_queries(m["F"], m["D"], m["query_seed"])
    assert digest([db, q]) == m["inputs_sha256"]
    g = load_golden(name)
    sc, ix = OR.search_l2(q, db, k=m["k"])
    np.testing.assert_array_equal(ix, g["inds"])
    np.testing.assert_allclose(sc, g["scores"], rtol=1e-6, atol=1e-4)
    n = g["blend"].shape[0]
    np.testing.assert_allclose(OR.blend(q[:n], db, k=m["k"]), g["blend"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("name", ["rmvpe_t16000", "rmvpe_t6401"])
def test_rmvpe_oracle_matches_reference(name, golden_meta):
    from oracle import rmvpe as ORM
    m = golden_meta[name]
    sd = syn.make_rmvpe_weights(m["weight_seed"])
    assert weights_digest(sd) == m["weights_sha256"]
    x = syn.make_rmvpe_input(m["T"], m["input_seed"])
    assert digest([x]) == m["inputs_sha256"]
    g = load_golden(name)
    mel = ORM.log_mel(x)
    np.testing.assert_allclose(mel, g["mel"], rtol=1e-5, atol=1e-5)
    sal = ORM.salience(sd, g["mel"])
    assert rel_l2(sal, g["salience"]) < 1e-5
    np.testing.assert_array_equal(np.argmax(sal, axis=1), g["argmax"])
    np.testing.assert_allclose(ORM.decode(sal), g["f0"], rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("name", ["vits40k_p96_part", "vits48k_p40_part"])
def test_partial_synthesis_oracle_matches_reference(name, golden_meta):
    m = golden_meta[name]
    w = syn.make_vits_weights(m["sr"], m["weight_seed"])
    assert weights_digest(w) == m["weights_sha256"]
    phone, pitch, nsff0, sid = syn.make_vits_inputs(m["P"], m["input_seed"])
    nz, ns = syn.make_vits_noise(m["P"], m["upp"], m["noise_seed"])
    assert digest([phone, pitch, nsff0, sid, nz, ns]) == m["inputs_sha256"]
    wav = OV.synth_partial(w, syn.vits_config_array(m["sr"]), phone, pitch, nsff0, sid, nz, ns, m["head"],
                           m["length"])
    g = load_golden(name)
    assert wav.size == g["wave"].size == m["length"] * m["upp"]
    assert np.abs(wav.reshape(-1) - g["wave"]).max() < 1e-5


IVF = ["ivf_n8000_d256", "ivf_n40_d16_edge"]


@pytest.mark.parametrize("name", IVF)
def test_ivf_oracle_matches_reference(name, golden_meta):
    """The restated IVF strict search and blend against the reference's own
    ``_ivf_strict_search`` / ``_vc_prepare`` on the same index structure."""
    from oracle import dsp as OD
    m = golden_meta[name]
    vecs = syn.make_index(m["N"], m["D"], 100 + m["seed"])
    q = syn.make_queries(m["F"], m["D"], 200 + m["seed"])
    if m["edge"]:
        g0 = load_golden(name)
        c = g0["centroids"]
        q[:5] = c[-1] + 0.01 * q[:5]
    g = load_golden(name)
    buckets = OR.ivf_buckets(g["assignments"], g["centroids"].shape[0])
    for npb in (1, 3):
        sc, ix = OR.ivf_strict_search(g["centroids"], vecs, buckets, q, k=8, nprobe=npb)
        np.testing.assert_array_equal(ix, g[f"inds_p{npb}"])
        np.testing.assert_array_equal(sc, g[f"scores_p{npb}"])
    # the pipeline's IVF blend, mix, x2 interpolation and protect (nprobe 1)
    feats = (q[None] * 0.5).astype(np.float32)
    sc, ix = OR.ivf_strict_search(g["centroids"], vecs, buckets, feats[0], k=8, nprobe=1)
    mixed = (OR.ivf_blend(vecs, sc, ix)[None] * 0.75 + feats * (1 - 0.75)).astype(np.float32)
    f = OD.interpolate_linear(mixed, 2, axis=1)
    f0 = OD.interpolate_linear(feats, 2, axis=1)
    pitchf = np.full((1, 2 * m["F"]), 150.0, np.float32)
    pitchf[0, ::3] = 0.0
    np.testing.assert_array_equal(OD.protect_blend(f, f0, pitchf, 0.33), g["prep_feats"])


FCPE = ["fcpe_t24000", "fcpe_t3001", "fcpe_t400"]


@pytest.mark.parametrize("name", FCPE)
def test_fcpe_oracle_matches_reference(name, golden_meta):
    from oracle import fcpe as OF
    m = golden_meta[name]
    sd = syn.make_fcpe_weights(m["weight_seed"])
    assert weights_digest(sd) == m["weights_sha256"]
    x = syn.make_rmvpe_input(m["T"], m["input_seed"])
    g = load_golden(name)
    mel = OF.log_mel(x)
    np.testing.assert_array_equal(mel, g["mel"])
    lat = OF.latent(sd, mel)
    assert rel_l2(lat, g["latent"]) < 1e-5
    np.testing.assert_array_equal(lat.argmax(axis=1), g["argmax"])
    np.testing.assert_allclose(OF.decode(lat, sd["cent_table"]), g["f0"], rtol=1e-5)
