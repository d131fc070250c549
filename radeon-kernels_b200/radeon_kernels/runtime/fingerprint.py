"""Environment fingerprint: the exact-match key of dispatch entries and kernel packs.

Same six fields as the reference's ``EnvironmentFingerprint``
(src/radeon_kernels/runtime/fingerprint.py:38-129) so manifests stay drop-in, with the
NVIDIA meanings filled in:

* ``architecture``   -- ``sm_100a`` on B200 (``sm_<major><minor>`` plus the ``a`` suffix
  for architectures whose kernels are built arch-specific); AMD ``gfx*`` names still parse;
* ``wavefront_size`` -- the warp size, 32;
* ``rocm_abi``       -- the field name is kept by the manifest schema; on CUDA builds of
  PyTorch it holds the CUDA runtime ABI ``MAJOR.MINOR`` (``torch.version.cuda``);
* ``python_abi``, ``pytorch_version`` -- unchanged;
* ``features``       -- hardware features the kernels rely on (``tcgen05``, ``tma``).

Detection is done once per device by the operator runtimes.
"""

from __future__ import annotations

import re
import sys
from dataclasses import dataclass
from typing import Any, Iterable, Mapping

from radeon_kernels.errors import RadeonKernelsError

ARCHITECTURE_PATTERN = r"^(gfx[0-9a-f]+|sm_[0-9]{2,3}[af]?)$"
_ARCHITECTURE_RE = re.compile(ARCHITECTURE_PATTERN)
_ABI_RE = re.compile(r"^(\d+)\.(\d+)")
_PYTHON_ABI_RE = re.compile(r"^cp\d{2,3}$")
_FEATURE_RE = re.compile(r"^[A-Za-z0-9_]+$")
_FIELDS = ("architecture", "wavefront_size", "rocm_abi", "python_abi", "pytorch_version", "features")

# Compute capabilities whose kernels are compiled for the arch-specific ("a") target.
_ARCH_SPECIFIC_MAJORS = {9, 10}
_FEATURES_BY_MAJOR = {9: ("tma", "wgmma"), 10: ("tcgen05", "tma")}


class FingerprintError(RadeonKernelsError):
    """The local GPU environment cannot be identified safely."""


def normalize_rocm_abi(value: str) -> str:
    """Reduce a toolkit version string (``12.8``, ``7.2.4``, ``12.8.93``) to ``MAJOR.MINOR``."""

    if not isinstance(value, str):
        raise FingerprintError(f"invalid toolkit version: {value!r}")
    found = _ABI_RE.match(value.strip())
    if found is None:
        raise FingerprintError(f"invalid toolkit version: {value!r}")
    return f"{int(found.group(1))}.{int(found.group(2))}"


def _clean_features(values: Iterable[Any]) -> tuple[str, ...]:
    result = set()
    for item in values:
        if not isinstance(item, str) or _FEATURE_RE.fullmatch(item) is None:
            raise FingerprintError(f"invalid architecture feature: {item!r}")
        result.add(item)
    return tuple(sorted(result))


def cuda_architecture_name(major: int, minor: int) -> str:
    suffix = "a" if major in _ARCH_SPECIFIC_MAJORS else ""
    return f"sm_{major}{minor}{suffix}"


@dataclass(frozen=True)
class EnvironmentFingerprint:
    architecture: str
    wavefront_size: int
    rocm_abi: str
    python_abi: str
    pytorch_version: str
    features: tuple[str, ...] = ()

    def __post_init__(self) -> None:
        if not isinstance(self.architecture, str) or _ARCHITECTURE_RE.fullmatch(self.architecture) is None:
            raise FingerprintError(f"invalid GPU architecture: {self.architecture!r}")
        if isinstance(self.wavefront_size, bool) or self.wavefront_size not in (32, 64):
            raise FingerprintError("wavefront size must be 32 or 64")
        object.__setattr__(self, "rocm_abi", normalize_rocm_abi(self.rocm_abi))
        if not isinstance(self.python_abi, str) or _PYTHON_ABI_RE.fullmatch(self.python_abi) is None:
            raise FingerprintError("Python ABI must use the cpXY form")
        if not isinstance(self.pytorch_version, str) or not self.pytorch_version:
            raise FingerprintError("PyTorch version must not be empty")
        object.__setattr__(self, "features", _clean_features(self.features))

    @classmethod
    def from_mapping(cls, value: Mapping[str, Any]) -> EnvironmentFingerprint:
        extra = set(value) - set(_FIELDS)
        if extra:
            raise FingerprintError(f"unknown fingerprint fields: {sorted(extra)}")
        features = value.get("features", ())
        if isinstance(features, (str, bytes)):
            raise FingerprintError("fingerprint has missing or invalid fields")
        try:
            return cls(
                architecture=value["architecture"],
                wavefront_size=value["wavefront_size"],
                rocm_abi=value["rocm_abi"],
                python_abi=value["python_abi"],
                pytorch_version=value["pytorch_version"],
                features=tuple(features),
            )
        except (KeyError, TypeError) as error:
            raise FingerprintError("fingerprint has missing or invalid fields") from error

    @classmethod
    def detect(
        cls,
        *,
        torch_module: Any | None = None,
        device_index: int = 0,
        features: Iterable[str] | None = None,
        python_abi: str | None = None,
    ) -> EnvironmentFingerprint:
        """Fingerprint one visible GPU.  Raises :class:`FingerprintError` without one."""

        if torch_module is None:
            try:
                import torch as torch_module
            except ImportError as error:
                raise FingerprintError("PyTorch is required to detect the GPU environment") from error
        if not torch_module.cuda.is_available():
            raise FingerprintError("no visible CUDA GPU")

        hip = getattr(torch_module.version, "hip", None)
        cuda = getattr(torch_module.version, "cuda", None)
        props = torch_module.cuda.get_device_properties(device_index)
        if isinstance(hip, str) and hip:
            architecture = getattr(props, "gcnArchName", "").split(":", 1)[0]
            toolkit = hip
            detected: tuple[str, ...] = ()
        elif isinstance(cuda, str) and cuda:
            major, minor = int(props.major), int(props.minor)
            architecture = cuda_architecture_name(major, minor)
            toolkit = cuda
            detected = _FEATURES_BY_MAJOR.get(major, ())
        else:
            raise FingerprintError("the installed PyTorch build reports neither a CUDA nor a ROCm version")
        warp = getattr(props, "warp_size", 32)
        if not isinstance(warp, int):
            raise FingerprintError("PyTorch did not report the GPU warp size")
        return cls(
            architecture=architecture,
            wavefront_size=warp,
            rocm_abi=toolkit,
            python_abi=python_abi or f"cp{sys.version_info.major}{sys.version_info.minor}",
            pytorch_version=str(torch_module.__version__),
            features=tuple(detected if features is None else features),
        )

    def to_dict(self) -> dict[str, Any]:
        return {
            "architecture": self.architecture,
            "wavefront_size": self.wavefront_size,
            "rocm_abi": self.rocm_abi,
            "python_abi": self.python_abi,
            "pytorch_version": self.pytorch_version,
            "features": list(self.features),
        }
