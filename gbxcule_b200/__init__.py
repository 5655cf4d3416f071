"""gbxcule_b200: B200-native (sm_100a) vectorized Game Boy core.

Drop-in for the vectorized backend of bkase/gbxcule: ``GbxVecCudaBackend``
(alias ``WarpVecCudaBackend``) and ``ResetCache`` keep the reference's
constructor keywords, methods and error behaviour; every device operation runs
in libgbx (``csrc/``, C ABI in ``include/gbx.h``).
"""

__version__ = "0.1.0"


def __getattr__(name):
    if name in ("GbxVecCudaBackend", "WarpVecCudaBackend"):
        from . import backend

        return getattr(backend, name)
    if name == "ResetCache":
        from .reset_cache import ResetCache

        return ResetCache
    raise AttributeError(name)
