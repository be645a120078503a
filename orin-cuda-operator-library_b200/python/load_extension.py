"""Loader with the reference's Python entry point, ``load_operatorlib``.

The reference's tests do ``from load_extension import load_operatorlib`` and
call ``load_operatorlib(verbose=...)`` before using ``torch.ops.operatorlib``
(reference python/load_extension.py:17).  Here the binding is prebuilt in
the tree (``operatorlib/_operatorlib_torch.so``, sm_100a), so loading means
registering that library with torch; nothing is compiled at import time.
Put this directory on ``sys.path`` (or PYTHONPATH) and the reference's
scripts run unchanged.
"""
from __future__ import annotations

import sys
from pathlib import Path

_PKG_PARENT = Path(__file__).resolve().parents[1]
if str(_PKG_PARENT) not in sys.path:
    sys.path.insert(0, str(_PKG_PARENT))


def load_operatorlib(verbose: bool = False) -> None:
    """Registers torch.ops.operatorlib.{reduce_sum, softmax, transpose,
    rmsnorm, gemm, attention}; raises if the CUDA library is not built."""
    import operatorlib

    operatorlib.load_operatorlib(verbose=verbose)


if __name__ == "__main__":
    load_operatorlib(verbose=True)
