"""Drop-in module name of the reference's pgf_rmsnorm.py: re-exports icml_b200.pgf_rmsnorm.

Put this directory first on PYTHONPATH and the reference's training
scripts import the CUDA implementation under their own module names.
"""
import os as _os
import sys as _sys

_root = _os.path.dirname(_os.path.dirname(_os.path.dirname(_os.path.abspath(__file__))))
if _root not in _sys.path:
    _sys.path.append(_root)

from icml_b200.pgf_rmsnorm import *  # noqa: E402,F401,F403
from icml_b200 import pgf_rmsnorm as _impl  # noqa: E402

__all__ = list(getattr(_impl, "__all__", []))
