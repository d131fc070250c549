"""Environment constraints of dispatch entries and kernel packs.

Matching follows the reference's ``EnvironmentConstraint``
(src/radeon_kernels/runtime/compatibility.py:26-127): architecture, warp size, toolkit
ABI, Python ABI and PyTorch build must be equal; the constraint's ``features`` must be a
subset of the fingerprint's.  Overlap and subset relations drive the manifest
validator's priority rules.  The architecture pattern also accepts ``sm_*`` names.
"""

from __future__ import annotations

import re
from dataclasses import dataclass
from typing import Any, Mapping

from radeon_kernels.errors import ConfigError
from radeon_kernels.runtime.fingerprint import (
    ARCHITECTURE_PATTERN,
    EnvironmentFingerprint,
    FingerprintError,
    normalize_rocm_abi,
)

_REQUIRED = ("architecture", "wavefront_size", "rocm_abi", "python_abi", "pytorch_version")
_ALLOWED = frozenset(_REQUIRED) | {"features"}
_ARCHITECTURE_RE = re.compile(ARCHITECTURE_PATTERN)
_PYTHON_ABI_RE = re.compile(r"^cp\d+$")


def _is_feature(item: Any) -> bool:
    return isinstance(item, str) and bool(item) and item.replace("_", "").isalnum()


@dataclass(frozen=True)
class EnvironmentConstraint:
    architecture: str
    wavefront_size: int
    rocm_abi: str
    python_abi: str
    pytorch_version: str
    features: frozenset[str] = frozenset()

    @classmethod
    def from_mapping(cls, value: Mapping[str, Any], path: str) -> EnvironmentConstraint:
        if not isinstance(value, Mapping):
            raise ConfigError(path, "expected a mapping")
        unknown = set(value) - _ALLOWED
        if unknown:
            raise ConfigError(path, f"unknown fields: {sorted(unknown)}")
        missing = set(_REQUIRED) - set(value)
        if missing:
            raise ConfigError(path, f"missing fields: {sorted(missing)}")

        architecture = value["architecture"]
        if not isinstance(architecture, str) or _ARCHITECTURE_RE.fullmatch(architecture) is None:
            raise ConfigError(f"{path}.architecture", "expected a gfx* or sm_* architecture")
        warp = value["wavefront_size"]
        if isinstance(warp, bool) or warp not in (32, 64):
            raise ConfigError(f"{path}.wavefront_size", "expected 32 or 64")
        features = value.get("features", [])
        if isinstance(features, (str, bytes)) or not isinstance(features, list):
            raise ConfigError(f"{path}.features", "expected a list")
        if not all(_is_feature(item) for item in features):
            raise ConfigError(f"{path}.features", "contains an invalid feature")
        python_abi = value["python_abi"]
        if not isinstance(python_abi, str) or _PYTHON_ABI_RE.fullmatch(python_abi) is None:
            raise ConfigError(f"{path}.python_abi", "expected a cpXY ABI tag")
        torch_version = value["pytorch_version"]
        if not isinstance(torch_version, str) or not torch_version:
            raise ConfigError(f"{path}.pytorch_version", "expected an exact build version")
        try:
            abi = normalize_rocm_abi(value["rocm_abi"])
        except FingerprintError as error:
            raise ConfigError(f"{path}.rocm_abi", "expected MAJOR.MINOR") from error
        return cls(architecture, warp, abi, python_abi, torch_version, frozenset(features))

    def _same_target(self, other: EnvironmentConstraint | EnvironmentFingerprint) -> bool:
        return (
            self.architecture == other.architecture
            and self.wavefront_size == other.wavefront_size
            and self.rocm_abi == other.rocm_abi
            and self.python_abi == other.python_abi
            and self.pytorch_version == other.pytorch_version
        )

    def matches(self, fingerprint: EnvironmentFingerprint) -> bool:
        return self._same_target(fingerprint) and self.features <= set(fingerprint.features)

    def overlaps(self, other: EnvironmentConstraint) -> bool:
        return self._same_target(other)

    def is_subset_of(self, other: EnvironmentConstraint) -> bool:
        return self._same_target(other) and self.features >= other.features

    def is_strict_subset_of(self, other: EnvironmentConstraint) -> bool:
        return self.is_subset_of(other) and self.features != other.features

    def to_dict(self) -> dict[str, Any]:
        return {
            "architecture": self.architecture,
            "wavefront_size": self.wavefront_size,
            "rocm_abi": self.rocm_abi,
            "python_abi": self.python_abi,
            "pytorch_version": self.pytorch_version,
            "features": sorted(self.features),
        }
