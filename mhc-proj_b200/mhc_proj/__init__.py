"""mhc_proj -- batched n=4 Birkhoff projection for manifold-constrained
hyper-connections, with hand-written CUDA kernels for B200 (sm_100a).

Drop-in for the reference package of the same name (mhc_proj/__init__.py of
Aoblex/mHC-proj): ``mhc_proj.MHCProjectionN4``, ``mhc_proj.MHCSinkhornN4`` and
the low-level ``mhc_proj.torch.*`` functions.  ``mhc_proj.MHCProjectionN4HRes``
and ``mhc_proj.MHCSinkhornN4HRes`` add the projection and the Sinkhorn-Knopp
pair fused with the mHC layer's H_res producer.  The
native extension is required; there is no CPU fallback.
"""
# torch first so that libc10 and the CUDA runtime resolve for the extension.
import torch as _torch  # noqa: F401

try:
    from ._internal import *  # noqa: F401,F403  (exports the `torch` submodule)
    from . import _internal
except ImportError as e:  # pragma: no cover - exercised only on a broken install
    raise ImportError(
        "mhc_proj: the native extension is not built or failed to load "
        "(run `python mhc-proj_b200/build.py`): " + str(e)) from e

from .module import MHCProjectionN4, MHCProjectionN4HRes, MHCSinkhornN4, MHCSinkhornN4HRes  # noqa: E402

__version__ = "0.1.0"
__all__ = ["MHCProjectionN4", "MHCProjectionN4HRes", "MHCSinkhornN4", "MHCSinkhornN4HRes", "torch"]
