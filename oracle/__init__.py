"""CPU oracle for the RVC inference hot path (test infrastructure only).

A numpy restatement of jiangchengnay/rvc-vulkan's numpy-backend inference for
the VITS synthesizer (``oracle.vits``), the HuBERT encoder (``oracle.hubert``)
and the per-op math (``oracle.ops``).  Pinned against outputs of the
reference itself by the fixtures under ``tests/golden/``.  ``oracle.reference``
loads the reference's own runtime from ``oracle/_ref`` (a git-ignored copy made
by ``make -C oracle ref``).  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline and reference arms may import this package.
"""
