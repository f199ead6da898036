"""The reference's own code, unchanged, on the CUDA backend.

A child process (``tests/golden/reference_runs.py --backend cuda``) imports
the reference's runtime from ``oracle/_ref``, calls ``rvc_cuda.register()``
with ``RVC_BACKEND=cuda`` and ``rvc_cuda.patch_reference()``, then runs:

* ``runtime.nn.conv1d`` / ``conv_transpose1d`` / ``layer_norm`` / ``linear`` /
  ``softmax`` (dispatched to ``rvc_cuda.ops`` by ``runtime/backend.py:189-197``)
  against the reference's numpy kernels called directly;
* ``SynthesizerTrn.infer_controlled`` and seeded ``infer``
  (``runtime/models/vits.py:2352``, ``:2551``);
* ``Pipeline.pipeline`` (``runtime/pipeline.py:697``) with the reference's
  HubertEncoder, RMVPE and SynthesizerTrn objects and a FeatureIndex;
* ``VC.get_vc`` + ``VC.vc_single`` (``runtime/vc.py:332``, ``:440``) on a WAV
  file, through to the int16 output (its closing ``clear_pool`` reaches
  rvc_cuda's pool release instead of raising).

The outputs are compared with the same runs on the reference's numpy backend
(``tests/golden/refruns.npz``, made by ``tests/golden/make_golden.py``):
waveform max-abs <= 1e-3, int16 within 33 LSB (1e-3 of full scale).  The
pipeline's discrete decisions (top-k neighbours, coarse pitch bins) are kept
away from float near-ties by the inputs, and both runs check their margins
(``reference_runs.MIN_RET_GAP``, ``MIN_COARSE_MARGIN``): a neighbour or pitch
bin that flips on a tie reaches every frame of a chunk through the text
encoder's attention.
"""

import os
import subprocess
import sys
import tempfile

import numpy as np
import pytest

from oracle import reference as oref
from rvc_cuda import _lib  # noqa: F401  (a missing library fails the module)
from tests.conftest import ROOT, load_golden

pytestmark = pytest.mark.gpu

WAVE_TOL = 1e-3
INT16_TOL = 33


@pytest.fixture(scope="module")
def cuda_runs():
    if not oref.available():
        pytest.fail("the reference runtime copy is missing: run `make -C oracle ref REF=<checkout>` "
                    "(__graft_entry__.build() does it where the checkout is present)")
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "runs.npz")
        env = dict(os.environ)
        env.pop("RVC_BACKEND", None)
        r = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "golden", "reference_runs.py"),
                            "--backend", "cuda", "--out", out], env=env, capture_output=True, text=True,
                           timeout=900)
        assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
        yield dict(np.load(out))


@pytest.fixture(scope="module")
def numpy_runs():
    return load_golden("refruns")


def test_register_routes_nn_ops_to_cuda(cuda_runs):
    assert str(cuda_runs["ops_backend"]) == "cuda"
    # conv / convT / linear: relative to the output's peak (BF16x3 ~1e-5);
    # layer_norm / softmax: absolute
    assert (cuda_runs["ops_err"] <= 2e-4).all(), cuda_runs["ops_err"]


def test_real_synthesizer_infer_through_patch(cuda_runs, numpy_runs):
    for k in ("synth_controlled", "synth_seeded"):
        err = float(np.abs(cuda_runs[k] - numpy_runs[k]).max())
        assert cuda_runs[k].shape == numpy_runs[k].shape and err <= WAVE_TOL, (k, err)


def _margins_ok(runs, case):
    from tests.golden import reference_runs as rr
    gap, coarse = runs[case + "_margins"]
    # the device run's own decisions are as far from a tie as the fixture's
    assert gap >= rr.MIN_RET_GAP and coarse >= rr.MIN_COARSE_MARGIN, (case, gap, coarse)


def test_real_pipeline_pipeline_through_patch(cuda_runs, numpy_runs):
    _margins_ok(cuda_runs, "pipeline")
    a, b = cuda_runs["pipeline_int16"], numpy_runs["pipeline_int16"]
    assert int(cuda_runs["pipeline_sr"]) == int(numpy_runs["pipeline_sr"]) == 40000
    assert a.dtype == np.int16 and a.shape == b.shape
    assert np.abs(a.astype(np.int32) - b.astype(np.int32)).max() <= INT16_TOL


def test_real_vc_single_runs_to_int16(cuda_runs, numpy_runs):
    _margins_ok(cuda_runs, "vc")
    a, b = cuda_runs["vc_int16"], numpy_runs["vc_int16"]
    assert int(cuda_runs["vc_sr"]) == 40000
    assert a.dtype == np.int16 and a.shape == b.shape and a.size > 40000
    assert np.abs(a.astype(np.int32) - b.astype(np.int32)).max() <= INT16_TOL
