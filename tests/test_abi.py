"""C-ABI checks that need no GPU: the library loads, exports every function
that include/rvc_cuda.h declares, and reports errors through the
status + last-error convention instead of crashing."""

import ctypes as C
import os
import re

import numpy as np
import pytest

from tests.conftest import ROOT

HEADER = os.path.join(ROOT, "include", "rvc_cuda.h")


def declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^int32_t\s+(rvc_cuda_\w+)\(", src, flags=re.M)))


def test_header_declares_entry_points():
    names = declared()
    assert "rvc_cuda_synth_infer" in names and "rvc_cuda_conv1d" in names
    assert len(names) >= 30


def test_library_exports_every_declared_symbol():
    from rvc_cuda import _lib
    missing = [n for n in declared() if not hasattr(_lib.lib, n)]
    assert not missing, missing
    assert set(declared()) == set(_lib.EXPORTED)


def test_version_and_device_count():
    from rvc_cuda import _lib
    assert _lib.lib.rvc_cuda_version() >= 100
    assert _lib.device_count() >= 0


def test_bad_device_is_an_error_not_a_crash():
    from rvc_cuda import _lib
    h = C.c_int64(0)
    rc = _lib.lib.rvc_cuda_create(9999, C.byref(h))
    assert rc == _lib.RVC_E_ARG
    assert "9999" in _lib.last_error()
    with pytest.raises(ValueError):
        _lib.check(rc)


def test_invalid_handles_report_state_errors():
    from rvc_cuda import _lib
    assert _lib.lib.rvc_cuda_sync(123456, 10) == -4
    assert "invalid context handle" in _lib.last_error()
    assert _lib.lib.rvc_cuda_synth_finalize(987654) == -4
    out = np.zeros(4, np.float32)
    assert _lib.lib.rvc_cuda_synth_tap(987654, b"x", _lib.fptr(out), 4) == -4


def test_last_error_truncates_safely():
    from rvc_cuda import _lib
    _lib.lib.rvc_cuda_sync(123456, 10)
    buf = C.create_string_buffer(8)
    n = _lib.lib.rvc_cuda_last_error(buf, 8)
    assert n > 8 and len(buf.value) == 7


def test_hubert_out_len_matches_conv_stack_arithmetic():
    from rvc_cuda import hubert

    def ref_len(T):
        for i, k in enumerate((10, 3, 3, 3, 3, 2, 2)):
            if T < k:
                return 0
            T = (T - k) // (5 if i == 0 else 2) + 1
        return T

    for T in (0, 1, 399, 400, 401, 3201, 8000, 16000, 160000, 160001, 480000):
        assert hubert.out_len(T) == ref_len(T), T
    assert hubert.out_len(160000) == 499


def test_hubert_patch_reference_replaces_class_methods():
    from rvc_cuda import hubert

    class FakeEncoder:
        def encode(self, x, version=2):
            return "numpy"

        def encode_batch(self, xs, version=2):
            return ["numpy"]

    class FakeModule:
        HubertEncoder = FakeEncoder

    cls = hubert.patch_reference(FakeModule)
    assert cls is FakeEncoder and cls._rvc_cuda_patched
    assert FakeEncoder.encode is not FakeEncoder._rvc_cuda_orig_encode
    assert FakeEncoder.encode_batch is not FakeEncoder._rvc_cuda_orig_encode_batch
    assert hubert.patch_reference(FakeModule) is FakeEncoder  # idempotent


def test_retrieval_patch_reference_replaces_module_functions():
    import types

    from rvc_cuda import retrieval

    ret_mod = types.SimpleNamespace(search_l2=lambda *a, **k: "numpy", weighted_blend=lambda *a, **k: "numpy")
    pipe_mod = types.SimpleNamespace(search_l2=ret_mod.search_l2, _ivf_strict_search=lambda *a, **k: "numpy")
    retrieval.patch_reference(ret_mod, pipe_mod)
    assert ret_mod.search_l2 is retrieval.search_l2 and pipe_mod.search_l2 is retrieval.search_l2
    assert pipe_mod._ivf_strict_search is retrieval.ivf_strict_search
    with pytest.raises(NotImplementedError):  # inner-product indexes are refused before any device work
        retrieval.ivf_strict_search(types.SimpleNamespace(metric="IP"), np.zeros((1, 4), np.float32))
    assert ret_mod.weighted_blend is retrieval.weighted_blend
    assert ret_mod._rvc_cuda_orig_search_l2() == "numpy"


def test_dsp_patch_reference_replaces_pipeline_functions():
    import types

    from rvc_cuda import dsp

    sig = types.SimpleNamespace(filtfilt=lambda b, a, x: "scipy", butter=lambda *a, **k: "butter")
    pipe_mod = types.SimpleNamespace(signal=sig, change_rms=lambda *a: "numpy", interpolate_linear=lambda *a: "numpy")
    dsp.patch_reference(pipe_mod)
    assert pipe_mod.change_rms is dsp.change_rms and pipe_mod.interpolate_linear is dsp.interpolate_linear
    assert pipe_mod.signal is not sig and pipe_mod.signal.butter is sig.butter
    assert pipe_mod._rvc_cuda_orig_signal.filtfilt(0, 0, 0) == "scipy"
    with pytest.raises(ValueError):  # other padding modes are not on the device path
        pipe_mod.signal.filtfilt([1.0], [1.0], [0.0] * 10, padtype="even")
    assert dsp.patch_reference(pipe_mod) is pipe_mod  # idempotent


def test_fcpe_patch_reference_replaces_infer():
    import types

    from rvc_cuda import fcpe

    class FakeFcpe:
        def infer(self, x, sr=16000, decoder_mode="local_argmax", threshold=0.006):
            return "numpy"

    mod = types.SimpleNamespace(FCPE=FakeFcpe)
    cls = fcpe.patch_reference(mod)
    assert cls is FakeFcpe and FakeFcpe.infer is not FakeFcpe._rvc_cuda_orig_infer
    assert fcpe.patch_reference(mod) is FakeFcpe  # idempotent
    assert fcpe.frames(16000) == 101 and fcpe.frames(159) == 1


def test_rmvpe_frames_and_patch_reference():
    from rvc_cuda import rmvpe

    assert rmvpe.frames(160000) == 1001 and rmvpe.frames(16000) == 101

    class FakeRmvpe:
        def infer_from_audio(self, x, thred=0.03):
            return "numpy"

    class FakeModule:
        RMVPE = FakeRmvpe

    cls = rmvpe.patch_reference(FakeModule)
    assert cls is FakeRmvpe and FakeRmvpe.infer_from_audio is not FakeRmvpe._rvc_cuda_orig_infer_from_audio


def test_synth_patch_reference_replaces_full_and_partial_paths():
    from rvc_cuda import synth

    class FakeSynth:
        def infer_controlled(self, *a, **k):
            return "numpy"

        def _infer_partial(self, *a, **k):
            return "numpy"

        def prep_dec(self, *a, **k):
            return "numpy"

        def decode_batch(self, *a, **k):
            return "numpy"

    class FakeModule:
        SynthesizerTrn = FakeSynth

    cls = synth.patch_reference(FakeModule)
    assert cls is FakeSynth
    assert FakeSynth.infer_controlled is not FakeSynth._rvc_cuda_orig_infer_controlled
    assert FakeSynth._infer_partial is not FakeSynth._rvc_cuda_orig_infer_partial
    assert FakeSynth.decode_batch is not FakeSynth._rvc_cuda_orig_decode_batch
    assert FakeSynth.prep_dec is not FakeSynth._rvc_cuda_orig_prep_dec


def test_vc_pool_release_shim_on_the_reference_module():
    """``VC.vc_single`` ends with ``vulkan_ops.get_context().clear_pool()``
    (``runtime/vc.py:532-534``), which raises without the Vulkan engine.  After
    ``patch_vc_pool_release()`` the reference's own ``get_context`` (from the
    ``oracle/_ref`` copy, in a child process) yields rvc_cuda's pool release,
    and installing twice keeps one wrapper.  No GPU is touched: with no open
    context the release has nothing to do."""
    import subprocess
    import sys

    from oracle import reference as oref

    if not oref.available():
        pytest.skip("reference runtime copy not built (make -C oracle ref)")
    code = (
        "import sys; sys.path[:0] = [%r, %r]\n"
        "from oracle import reference as r; r.activate('numpy')\n"
        "from runtime import vulkan_ops as v\n"
        "try:\n    v.get_context(); raised = False\nexcept RuntimeError:\n    raised = True\n"
        "import rvc_cuda; rvc_cuda.patch_vc_pool_release(); rvc_cuda.patch_vc_pool_release()\n"
        "c = v.get_context(); c.clear_pool()\n"
        "print(raised, type(c).__name__, v.get_context.__wrapped__.__module__)\n"
    ) % (ROOT, os.path.join(ROOT, "rvc-vulkan_b200"))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300,
                       env=dict(os.environ, RVC_BACKEND="numpy"))
    assert r.returncode == 0, r.stderr[-3000:]
    assert r.stdout.split()[-3:] == ["True", "_DevicePool", "runtime.vulkan_ops"], r.stdout
