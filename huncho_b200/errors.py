"""Error kinds of huncho-core's `Error` enum that the Kev backend raises
(crates/huncho-core/src/error.rs:10-45)."""


class HunchoError(Exception):
    kind = "internal"


class BackendError(HunchoError):
    """Error::Backend: invalid request for the backend, or failed inference."""
    kind = "backend"


class UnsupportedError(HunchoError):
    """Error::Unsupported."""
    kind = "unsupported"


class PackageError(HunchoError):
    """Error::Package: unreadable or inconsistent model package."""
    kind = "package"


class CalibrationError(HunchoError):
    """Error::Calibration."""
    kind = "calibration"


class RequestError(HunchoError):
    """Error::Request: the request itself is invalid (error.rs:16-17)."""
    kind = "request"


class UnavailableError(HunchoError):
    """JobResult::Unavailable (huncho-api coalesce.rs:13-17): the batch queue
    is full or closed, so the request was not admitted."""
    kind = "unavailable"


class WorkerFailedError(HunchoError):
    """JobResult::WorkerFailed: the collation worker failed outside the
    backend (the group's callers all receive it)."""
    kind = "worker_failed"
