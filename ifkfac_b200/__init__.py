"""ifkfac_b200 — B200 (sm_100a) implementation of IFKFAC's curvature hot path.

The streaming TSQR, damping fold, four triangular solves and the fp32 update
epilogue run in libifk.so (C ABI: include/ifk.h); this package keeps the
reference's Python front end (IFKFAC, RawActivationHooks, the functional
triangular API) on top of it.  The shared library is loaded on first use and
there is no CPU fallback.
"""
from ._lib import IFKError, lib  # noqa: F401

__version__ = "0.1.0"


def __getattr__(name):
    # Lazy imports keep `import ifkfac_b200` cheap and free of CUDA work.
    if name in ("IFKFAC",):
        from .ifkfac import IFKFAC
        return IFKFAC
    if name in ("RawActivationHooks", "IFKFACRankError"):
        from . import activation_hooks as ah
        return getattr(ah, name)
    raise AttributeError(name)
