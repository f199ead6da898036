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
  ``change_rms`` and ``interpolate_linear``) and makes ``VC.vc_single``'s
  closing pool release work without the Vulkan engine library
  (``patch_vc_pool_release``).

Importing this package does not touch the GPU; the shared library is loaded
on first use of ``rvc_cuda.ops`` / ``rvc_cuda.synth`` and raises if missing.
"""

from __future__ import annotations

__all__ = ["register", "patch_reference", "patch_vc_pool_release", "probe"]


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
    patch_vc_pool_release()


class _DevicePool:
    """What ``VC.vc_single`` gets from ``vulkan_ops.get_context()`` when the
    Vulkan engine is absent: its one call, ``clear_pool()``, returns the cached
    free device blocks of every rvc_cuda context to the driver, as
    ``VulkanContext.clear_pool`` does for the engine's output pool
    (``runtime/vulkan_ops.py:618-633``)."""

    def clear_pool(self) -> None:
        from . import _lib  # noqa: PLC0415

        _lib.release_pools()


def patch_vc_pool_release() -> None:
    """``VC.vc_single`` ends every conversion, in a ``finally``, with
    ``vulkan_ops.get_context().clear_pool()`` (``runtime/vc.py:532-534``);
    ``get_context`` raises when ``rvc_core.dll`` is missing
    (``runtime/vulkan_ops.py:3935-3945``), which would turn every finished
    conversion into an exception.  ``get_context`` is wrapped: the Vulkan
    context when the engine loads, otherwise ``_DevicePool``.  Pure Python;
    ``runtime/vc.py`` itself is unchanged."""
    from runtime import vulkan_ops  # noqa: PLC0415

    orig = vulkan_ops.get_context
    if getattr(orig, "_rvc_cuda_pool", False):
        return
    pool = _DevicePool()

    def get_context():
        try:
            return orig()
        except Exception:  # noqa: BLE001 - no Vulkan engine: the device pool is rvc_cuda's
            return pool

    get_context._rvc_cuda_pool = True
    get_context.__wrapped__ = orig
    vulkan_ops.get_context = get_context
