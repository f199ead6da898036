"""rvc_cuda: B200-native (sm_100a) backend for the RVC inference hot path.

Drop-in for jiangchengnay/rvc-vulkan's numpy runtime:

* ``register()`` adds the ``cuda`` operator backend to ``runtime.backend``
  (``runtime/backend.py:57-70``); ``RVC_BACKEND=cuda`` then routes the
  ``runtime.nn`` float32 ops through ``rvc_cuda.ops``.
* ``patch_reference()`` installs the whole-model fast paths
  (``rvc_cuda.synth.patch_reference`` for ``SynthesizerTrn``,
  ``rvc_cuda.hubert.patch_reference`` for ``HubertEncoder``,
  ``rvc_cuda.retrieval.patch_reference`` for the brute-force ``search_l2``,
  ``rvc_cuda.rmvpe.patch_reference`` for ``RMVPE.infer_from_audio``,
  ``rvc_cuda.fcpe.patch_reference`` for ``FCPE.infer``,
  ``rvc_cuda.dsp.patch_reference`` for the pipeline's ``filtfilt``,
  ``change_rms`` and ``interpolate_linear``).

Importing this package does not touch the GPU; the shared library is loaded
on first use of ``rvc_cuda.ops`` / ``rvc_cuda.synth`` and raises if missing.
"""

from __future__ import annotations

__all__ = ["register", "patch_reference", "probe"]


def probe() -> bool:
    """True when librvc_cuda loads and a B200 (sm_100) is visible."""
    try:
        from . import _lib  # noqa: PLC0415

        if _lib.device_count() < 1:
            return False
        _lib.get_context()
        return True
    except Exception:  # noqa: BLE001 - a failed probe means "not available"
        return False


def register(name: str = "cuda") -> None:
    """Register the operator module with ``runtime.backend`` (before the first
    ``get_backend()`` call, which caches the choice: ``runtime/backend.py:154-158``)."""
    from runtime import backend  # noqa: PLC0415

    if name not in backend._BACKENDS:
        backend.register_backend(name, "rvc_cuda.ops", label="cuda (B200 sm_100a)", probe=probe)


def patch_reference(device=None, precision: str = "bf16x3") -> None:
    """Install the model-level CUDA paths on the reference's model classes and
    the device signal processing in ``runtime.pipeline``."""
    from . import dsp, fcpe, hubert, retrieval, rmvpe, synth  # noqa: PLC0415

    synth.patch_reference(device=device, precision=precision)
    hubert.patch_reference(device=device, precision=precision)
    retrieval.patch_reference()
    rmvpe.patch_reference(device=device)
    fcpe.patch_reference(device=device, precision=precision)
    dsp.patch_reference()
