"""huncho_b200: a B200-native (sm_100a) Kev scoring forward behind huncho's Backend trait.

The compute path is libhuncho_kev.so (CUDA kernels + the C ABI of
include/huncho_kev.h); this package holds the host-side mirror of the
reference's Backend trait (backend.py), its calibration and answer semantics
(calibration.py, engine.py), cross-request collation (collate.py), replica
pools and sharding (replicas.py), the synthetic workload generator (synth.py)
and the in-tree build (build.py).
"""
from .errors import (BackendError, CalibrationError, HunchoError, PackageError, RequestError, UnavailableError,
                     UnsupportedError, WorkerFailedError)

__all__ = ["BackendError", "CalibrationError", "HunchoError", "PackageError", "RequestError", "UnavailableError",
           "UnsupportedError", "WorkerFailedError", "KevBackend", "ForwardInput", "ForwardOutput"]


def __getattr__(name):
    # The backend loads the native library; import it on first use so that
    # the calibration / synthetic-workload helpers work without a build.
    if name in ("KevBackend", "ForwardInput", "ForwardOutput", "BatchLimits", "Capabilities"):
        from . import backend
        return getattr(backend, name)
    raise AttributeError(name)
