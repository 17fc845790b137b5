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
