"""Exception hierarchy shared by the public API and the dispatch runtime.

Mirrors the reference's ``radeon_kernels.errors`` (src/radeon_kernels/errors.py:1-11):
every expected user-facing failure derives from :class:`RadeonKernelsError`, and
configuration problems carry the offending path.
"""


class RadeonKernelsError(Exception):
    """Base class for expected, user-facing failures."""


class ConfigError(RadeonKernelsError):
    """A manifest, pack or key file is malformed; ``path`` names the offending item."""

    def __init__(self, path: str, message: str) -> None:
        self.path = path
        self.message = message
        super().__init__(f"{path}: {message}")


class NativeLibraryError(RadeonKernelsError):
    """The compiled sm_100a kernel library is missing or cannot run on this machine."""
