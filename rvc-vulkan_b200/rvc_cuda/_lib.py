"""ctypes binding of librvc_cuda.so (declarations in include/rvc_cuda.h).

Mirrors the reference's ctypes layer for its Vulkan engine
(``runtime/_vulkan.py``): the shared library is found next to this package
(or at ``$RVC_CUDA_LIB``), every call returns an int32 status and a non-zero
status becomes an exception carrying the library's last error message
(``runtime/_vulkan.py:320-324``).  There is no CPU fallback: if the library
cannot be loaded, importing this module raises.
"""

from __future__ import annotations

import ctypes as C
import os
import threading
import weakref

import numpy as np

__all__ = ["lib", "check", "Context", "get_context", "device_count", "RvcCudaError", "PinnedBuffer"]

RVC_E_ARG = -1
RVC_E_TIMEOUT = -3
RVC_E_OOM = -5


class RvcCudaError(RuntimeError):
    """Error raised by a librvc_cuda call (status < 0)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"librvc_cuda error {code}: {msg}")
        self.code = code


def _find_lib() -> str:
    env = os.environ.get("RVC_CUDA_LIB")
    if env:
        return env
    return os.path.join(os.path.dirname(os.path.abspath(__file__)), "librvc_cuda.so")


_path = _find_lib()
if not os.path.isfile(_path):
    raise ImportError(
        f"librvc_cuda.so not found at {_path}: build it first (make -C rvc-vulkan_b200, "
        "or __graft_entry__.build()); the cuda backend has no CPU fallback")
lib = C.CDLL(_path)

_i32, _i64, _f32, _f64 = C.c_int32, C.c_int64, C.c_float, C.c_double
_p = C.c_void_p
_fp = C.POINTER(C.c_float)
_ip64 = C.POINTER(C.c_int64)

_SIGS = {
    "rvc_cuda_version": ([], _i32),
    "rvc_cuda_last_error": ([C.c_char_p, _i64], _i32),
    "rvc_cuda_launch_count": ([C.POINTER(_i64)], _i32),
    "rvc_cuda_device_count": ([C.POINTER(_i32)], _i32),
    "rvc_cuda_create": ([_i32, C.POINTER(_i64)], _i32),
    "rvc_cuda_destroy": ([_i64], _i32),
    "rvc_cuda_sync": ([_i64, _i32], _i32),
    "rvc_cuda_stream": ([_i64, C.POINTER(_p)], _i32),
    "rvc_cuda_set_mem_cap": ([_i64, _i64], _i32),
    "rvc_cuda_release_pool": ([_i64], _i32),
    "rvc_cuda_alloc": ([_i64, _i64, C.POINTER(_p)], _i32),
    "rvc_cuda_free": ([_i64, _p], _i32),
    "rvc_cuda_h2d": ([_i64, _p, _p, _i64], _i32),
    "rvc_cuda_d2h": ([_i64, _p, _p, _i64], _i32),
    "rvc_cuda_profile": ([_i64, _i32], _i32),
    "rvc_cuda_profile_dump": ([_i64, C.c_char_p, _i64], _i32),
    "rvc_cuda_profile_read": ([_i64, C.POINTER(_i64), C.POINTER(_f64), C.POINTER(_f64)], _i32),
    "rvc_cuda_conv1d": ([_i64, _fp, _i32, _i32, _i32, _fp, _i32, _i32, _fp, _i32, _i32, _i32, _i32, _fp, _i32], _i32),
    "rvc_cuda_conv_transpose1d": ([_i64, _fp, _i32, _i32, _i32, _fp, _i32, _i32, _fp, _i32, _i32, _i32, _i32, _fp,
                                   _i32], _i32),
    "rvc_cuda_matmul": ([_i64, _fp, _fp, _i32, _i32, _i32, _fp], _i32),
    "rvc_cuda_layer_norm": ([_i64, _fp, _i64, _i32, _fp, _fp, _f32, _fp], _i32),
    "rvc_cuda_conv2d": ([_i64, _fp, _i32, _i32, _i32, _i32, _fp, _i32, _i32, _i32, _fp, _i32, _i32, _i32, _i32,
                         _fp], _i32),
    "rvc_cuda_rmsnorm": ([_i64, _fp, _i64, _i32, _fp, _f32, _fp], _i32),
    "rvc_cuda_softmax": ([_i64, _fp, _i64, _i32, _fp], _i32),
    "rvc_cuda_elementwise": ([_i64, _i32, _fp, _fp, _i64, _f32, _fp], _i32),
    "rvc_cuda_embedding": ([_i64, _ip64, _i64, _fp, _i32, _i32, _fp], _i32),
    "rvc_cuda_gating": ([_i64, _fp, _fp, _i32, _i32, _i32, _fp], _i32),
    "rvc_cuda_rel_attention": ([_i64, _fp, _fp, _fp, _fp, _fp, _i32, _i32, _i32, _i32, _i32, _fp], _i32),
    "rvc_cuda_rel_attention_noalloc": ([_i64, _p, _p, _p, _p, _p, _i32, _i32, _i32, _i32, _i32, _p], _i32),
    "rvc_cuda_im2col1d": ([_i64, _fp, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _fp], _i32),
    "rvc_cuda_synth_create": ([_i64, C.POINTER(_i32), _i32, C.POINTER(_i64)], _i32),
    "rvc_cuda_synth_destroy": ([_i64], _i32),
    "rvc_cuda_synth_set_weight": ([_i64, C.c_char_p, _fp, _ip64, _i32], _i32),
    "rvc_cuda_synth_finalize": ([_i64], _i32),
    "rvc_cuda_synth_infer": ([_i64, _i32, _i32, _fp, _ip64, _fp, _ip64, _fp, _fp, _fp], _i32),
    "rvc_cuda_synth_infer_grouped": ([_i64, _i32, _i32, _i32, _fp, _ip64, _fp, _ip64, _fp, _fp, _fp], _i32),
    "rvc_cuda_synth_infer_device": ([_i64, _i32, _i32, _p, _p, _p, _p, _p, _p, _p], _i32),
    "rvc_cuda_synth_infer_partial": ([_i64, _i32, _i32, _i32, _fp, _ip64, _fp, _ip64, _fp, _fp, _fp], _i32),
    "rvc_cuda_synth_tap": ([_i64, C.c_char_p, _fp, _i64], _i32),
    "rvc_cuda_synth_keep_taps": ([_i64, _i32], _i32),
    "rvc_cuda_hubert_create": ([_i64, _i32, C.POINTER(_i64)], _i32),
    "rvc_cuda_hubert_destroy": ([_i64], _i32),
    "rvc_cuda_hubert_set_weight": ([_i64, C.c_char_p, _fp, _ip64, _i32], _i32),
    "rvc_cuda_hubert_finalize": ([_i64], _i32),
    "rvc_cuda_hubert_out_len": ([_i64, C.POINTER(_i64)], _i32),
    "rvc_cuda_hubert_encode": ([_i64, _i32, _i64, _fp, _i32, _fp], _i32),
    "rvc_cuda_hubert_encode_device": ([_i64, _i32, _i64, _p, _i32, _p], _i32),
    "rvc_cuda_hubert_tap": ([_i64, C.c_char_p, _fp, _i64], _i32),
    "rvc_cuda_hubert_keep_taps": ([_i64, _i32], _i32),
    "rvc_cuda_fcpe_create": ([_i64, _i32, C.POINTER(_i64)], _i32),
    "rvc_cuda_fcpe_destroy": ([_i64], _i32),
    "rvc_cuda_fcpe_set_weight": ([_i64, C.c_char_p, _fp, _ip64, _i32], _i32),
    "rvc_cuda_fcpe_finalize": ([_i64], _i32),
    "rvc_cuda_fcpe_infer": ([_i64, _i32, _i64, _fp, _f32, _fp, C.POINTER(_i32)], _i32),
    "rvc_cuda_fcpe_infer_mode": ([_i64, _i32, _i64, _fp, _f32, _i32, _fp, C.POINTER(_i32)], _i32),
    "rvc_cuda_fcpe_infer_device": ([_i64, _i32, _i64, _p, _f32, _p, _p], _i32),
    "rvc_cuda_fcpe_tap": ([_i64, C.c_char_p, _fp, _i64], _i32),
    "rvc_cuda_fcpe_keep_taps": ([_i64, _i32], _i32),
    "rvc_cuda_rmvpe_create": ([_i64, C.POINTER(_i64)], _i32),
    "rvc_cuda_rmvpe_destroy": ([_i64], _i32),
    "rvc_cuda_rmvpe_set_weight": ([_i64, C.c_char_p, _fp, _ip64, _i32], _i32),
    "rvc_cuda_rmvpe_finalize": ([_i64], _i32),
    "rvc_cuda_rmvpe_frames": ([_i64, C.POINTER(_i64)], _i32),
    "rvc_cuda_rmvpe_infer": ([_i64, _i32, _i64, _fp, _f32, _fp, C.POINTER(_i32)], _i32),
    "rvc_cuda_rmvpe_infer_device": ([_i64, _i32, _i64, _p, _f32, _p, _p], _i32),
    "rvc_cuda_rmvpe_tap": ([_i64, C.c_char_p, _fp, _i64], _i32),
    "rvc_cuda_rmvpe_keep_taps": ([_i64, _i32], _i32),
    "rvc_cuda_filtfilt": ([_i64, _p, _i32, _p, _i32, _p, _i32, _i64, _p], _i32),
    "rvc_cuda_split_points": ([_i64, _p, _i64, _i32, _i64, _i64, _p, _i64, C.POINTER(_i64)], _i32),
    "rvc_cuda_interp_linear": ([_i64, _fp, _i64, _i32, _f64, _fp, _i64], _i32),
    "rvc_cuda_protect": ([_i64, _fp, _fp, _fp, _i64, _i32, _f32, _fp], _i32),
    "rvc_cuda_change_rms": ([_i64, _fp, _i64, _i32, _fp, _i64, _i32, _f64, _fp], _i32),
    "rvc_cuda_to_int16": ([_i64, _fp, _i64, _p], _i32),
    "rvc_cuda_interp_linear_device": ([_i64, _p, _i64, _i32, _f64, _p, _i64], _i32),
    "rvc_cuda_protect_device": ([_i64, _p, _p, _p, _i64, _i32, _f32, _p], _i32),
    "rvc_cuda_change_rms_device": ([_i64, _p, _i64, _i32, _p, _i64, _i32, _f64, _p], _i32),
    "rvc_cuda_to_int16_device": ([_i64, _p, _i64, _p], _i32),
    "rvc_cuda_index_ivf_blend_device": ([_i64, _p, _i64, _i32, _i32, _i32, _f64, _p, _p], _i32),
    "rvc_cuda_d2d": ([_i64, _p, _p, _i64], _i32),
    "rvc_cuda_h2d_async": ([_i64, _p, _p, _i64], _i32),
    "rvc_cuda_host_alloc": ([_i64, C.POINTER(_p)], _i32),
    "rvc_cuda_host_free": ([_p], _i32),
    "rvc_cuda_resample": ([_i64, _p, _i32, _i64, _i32, _i32, _i32, _fp, _i64], _i32),
    "rvc_cuda_f0_autocorr": ([_i64, _p, _i64, _i32, _i32, _i32, _i32, _i32, _p, _f64, _fp, _i64], _i32),
    "rvc_cuda_index_create": ([_i64, _fp, _i64, _i32, _i32, C.POINTER(_i64)], _i32),
    "rvc_cuda_index_destroy": ([_i64], _i32),
    "rvc_cuda_index_search": ([_i64, _fp, _i64, _i32, _i32, _fp, _ip64], _i32),
    "rvc_cuda_index_search_device": ([_i64, _p, _i64, _i32, _i32, _p, _p], _i32),
    "rvc_cuda_index_blend": ([_i64, _fp, _i64, _i32, _i32, _i32, _f64, _fp, _fp], _i32),
    "rvc_cuda_index_blend_device": ([_i64, _p, _i64, _i32, _i32, _i32, _f64, _p, _p], _i32),
    "rvc_cuda_index_set_ivf": ([_i64, _fp, _i32, _ip64], _i32),
    "rvc_cuda_index_ivf_search": ([_i64, _fp, _i64, _i32, _i32, _i32, _fp, _ip64], _i32),
    "rvc_cuda_index_ivf_blend": ([_i64, _fp, _i64, _i32, _i32, _i32, _f64, _fp, _fp], _i32),
}
for _name, (_args, _ret) in _SIGS.items():
    _fn = getattr(lib, _name)
    _fn.argtypes = _args
    _fn.restype = _ret
EXPORTED = tuple(_SIGS)


def last_error() -> str:
    buf = C.create_string_buffer(4096)
    lib.rvc_cuda_last_error(buf, len(buf))
    return buf.value.decode("utf-8", "replace")


def check(rc: int) -> None:
    """Raise for a negative status: ValueError for bad arguments (the
    reference's callers catch ValueError to pick another path,
    ``runtime/nn.py:286-289``), RvcCudaError otherwise."""
    if rc == 0:
        return
    msg = last_error()
    if rc == RVC_E_ARG:
        raise ValueError(msg)
    raise RvcCudaError(rc, msg)


def fptr(a: np.ndarray):
    return a.ctypes.data_as(_fp) if a is not None else None


def iptr(a: np.ndarray):
    return a.ctypes.data_as(_ip64)


def launch_count() -> int:
    n = _i64(0)
    check(lib.rvc_cuda_launch_count(C.byref(n)))
    return int(n.value)


def device_count() -> int:
    n = _i32(0)
    check(lib.rvc_cuda_device_count(C.byref(n)))
    return int(n.value)


class Context:
    """One CUDA context (stream + workspace) on one device."""

    def __init__(self, device: int = 0):
        h = _i64(0)
        check(lib.rvc_cuda_create(int(device), C.byref(h)))
        self.handle = int(h.value)
        self.device = int(device)
        _live.add(self)

    def close(self):
        if getattr(self, "handle", 0):
            lib.rvc_cuda_destroy(self.handle)
            self.handle = 0

    def sync(self, timeout_ms: int = 0):
        check(lib.rvc_cuda_sync(self.handle, int(timeout_ms)))

    def stream(self) -> int:
        s = _p()
        check(lib.rvc_cuda_stream(self.handle, C.byref(s)))
        return int(s.value or 0)

    def set_mem_cap(self, nbytes: int):
        check(lib.rvc_cuda_set_mem_cap(self.handle, int(nbytes)))

    def release_pool(self):
        """Return this context's cached free device blocks to the driver."""
        check(lib.rvc_cuda_release_pool(self.handle))

    def alloc(self, nbytes: int) -> int:
        p = _p()
        check(lib.rvc_cuda_alloc(self.handle, int(nbytes), C.byref(p)))
        return int(p.value)

    def free(self, dptr: int):
        check(lib.rvc_cuda_free(self.handle, _p(dptr)))

    def h2d(self, dptr: int, arr: np.ndarray):
        arr = np.ascontiguousarray(arr)
        check(lib.rvc_cuda_h2d(self.handle, _p(dptr), arr.ctypes.data_as(_p), arr.nbytes))

    def d2h(self, arr: np.ndarray, dptr: int):
        check(lib.rvc_cuda_d2h(self.handle, arr.ctypes.data_as(_p), _p(dptr), arr.nbytes))

    def h2d_async(self, dptr: int, arr: np.ndarray):
        """Host-to-device copy enqueued without waiting for the stream.  ``arr``
        (page-locked, from ``PinnedBuffer``, for a copy that overlaps) must stay
        unchanged and alive until the next ``sync`` / ``d2h`` of this context."""
        if not (arr.flags.c_contiguous):
            raise ValueError("h2d_async needs a contiguous source")
        check(lib.rvc_cuda_h2d_async(self.handle, _p(dptr), arr.ctypes.data_as(_p), arr.nbytes))

    def d2d(self, dst: int, src: int, nbytes: int):
        """Device-to-device copy, asynchronous on this context's stream."""
        check(lib.rvc_cuda_d2d(self.handle, _p(dst), _p(src), int(nbytes)))

    def profile(self, enable: bool):
        check(lib.rvc_cuda_profile(self.handle, 1 if enable else 0))

    def profile_read(self):
        n, ms, fl = _i64(0), _f64(0), _f64(0)
        check(lib.rvc_cuda_profile_read(self.handle, C.byref(n), C.byref(ms), C.byref(fl)))
        return int(n.value), float(ms.value), float(fl.value)

    def profile_dump(self) -> str:
        buf = C.create_string_buffer(1 << 20)
        n = lib.rvc_cuda_profile_dump(self.handle, buf, len(buf))
        if n < 0:
            check(n)
        return buf.value.decode()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


_ctx_lock = threading.Lock()
_contexts: dict = {}
_live: "weakref.WeakSet[Context]" = weakref.WeakSet()


def release_pools() -> None:
    """Return the cached free device blocks of every open context of this
    process (models' own contexts included) to the driver."""
    for c in list(_live):
        if getattr(c, "handle", 0):
            c.release_pool()


def get_context(device: int | None = None) -> Context:
    """Process-wide context per device (``$RVC_CUDA_DEVICE`` or 0 by default)."""
    if device is None:
        device = int(os.environ.get("RVC_CUDA_DEVICE", "0"))
    with _ctx_lock:
        c = _contexts.get(device)
        if c is None:
            c = Context(device)
            _contexts[device] = c
        return c


class PinnedBuffer:
    """Page-locked host memory (``rvc_cuda_host_alloc``) with numpy views."""

    def __init__(self, nbytes: int):
        p = _p()
        check(lib.rvc_cuda_host_alloc(int(max(16, nbytes)), C.byref(p)))
        self.ptr = int(p.value)
        self.nbytes = int(max(16, nbytes))

    def view(self, dtype, count: int, offset: int = 0) -> np.ndarray:
        """``count`` elements of ``dtype`` starting ``offset`` bytes in."""
        dt = np.dtype(dtype)
        if offset < 0 or offset + count * dt.itemsize > self.nbytes:
            raise ValueError("pinned view out of range")
        buf = (C.c_char * (count * dt.itemsize)).from_address(self.ptr + offset)
        return np.frombuffer(buf, dtype=dt, count=count)

    def close(self):
        if getattr(self, "ptr", 0):
            lib.rvc_cuda_host_free(_p(self.ptr))
            self.ptr = 0

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass
