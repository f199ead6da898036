"""The reference's own Python runtime, loaded from ``oracle/_ref``.

TEST INFRASTRUCTURE ONLY.  ``make -C oracle ref REF=<checkout>`` copies the
reference's ``runtime/`` package and ``torch_compat.py`` into ``oracle/_ref``
(git-ignored); this module puts that copy on ``sys.path`` and builds the
reference's models on the seeded synthetic checkpoints of
``rvc_cuda.synthetic`` by replacing their file loaders, as the reference's
models read checkpoints from disk:

* ``runtime.models.vits._load_ckpt`` (``runtime/models/vits.py:157-160``),
* ``runtime.models.hubert.load_pth`` (imported at ``runtime/models/hubert.py:115``),
* ``runtime.models.rmvpe.load_pth`` (imported at ``runtime/models/rmvpe.py:50``).

The operator backend is chosen from ``RVC_BACKEND`` at the reference's first
``get_backend()`` call and kept for the process (``runtime/backend.py:154-158``),
so a process that needs both the numpy and the cuda backend runs one of them
in a child process.  Only ``tests/``, ``bench.py``'s reference arm and
``tests/golden/make_golden.py`` use this module.
"""

from __future__ import annotations

import os
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")


def root() -> str | None:
    """Directory holding the reference's ``runtime`` package, or None: an
    explicit ``RVC_REFERENCE`` checkout first, then the ``oracle/_ref`` copy."""
    for d in (os.environ.get("RVC_REFERENCE", ""), REF_DIR):
        if d and os.path.isfile(os.path.join(d, "runtime", "models", "vits.py")):
            return d
    return None


def available() -> bool:
    return root() is not None


def activate(backend: str = "numpy") -> str:
    """Put the reference on ``sys.path`` (first) and select its operator
    backend for this process; returns the directory used."""
    d = root()
    if d is None:
        raise RuntimeError("the reference runtime is not available: run `make -C oracle ref REF=<checkout>`")
    os.environ.setdefault("RVC_BACKEND", backend)
    if d not in sys.path:
        sys.path.insert(0, d)
    return d


def synthesizer(w: dict, cfg: list):
    """``runtime.models.vits.SynthesizerTrn`` on a synthetic checkpoint."""
    from runtime.models import vits  # noqa: PLC0415

    vits._load_ckpt = lambda path: {"weight": w, "config": cfg}
    return vits.SynthesizerTrn("synthetic.pth")


def hubert(sd: dict):
    """``runtime.models.hubert.HubertEncoder`` on a synthetic state dict (the
    constructor checks that ``pytorch_model.bin`` exists, so an empty one is
    made in a temporary directory)."""
    from runtime.models import hubert as rh  # noqa: PLC0415

    rh.load_pth = lambda path: sd
    with tempfile.TemporaryDirectory() as d:
        open(os.path.join(d, "pytorch_model.bin"), "wb").close()
        return rh.HubertEncoder(d)


def rmvpe(sd: dict):
    """``runtime.models.rmvpe.RMVPE`` on a synthetic state dict."""
    from runtime.models import rmvpe as rr  # noqa: PLC0415

    rr.load_pth = lambda path: sd
    return rr.RMVPE(os.path.join(tempfile.gettempdir(), "rmvpe.pt"))
