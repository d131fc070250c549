"""SHA-256 verified loading of precompiled kernel-pack artifacts.

Same contract as the reference's ``PrecompiledArtifactLoader``
(src/radeon_kernels/runtime/loader.py:64-121): an artifact path must stay inside the pack
root, its SHA-256 must equal the manifest's digest, and ``python_extension`` artifacts are
imported by the module name their single ``PyInit_*`` symbol declares.

One deliberate difference: the reference re-hashes the shared object twice on every call
(loader.py:88-89 and :117), which costs milliseconds per call on a multi-megabyte pack.
Here a digest is computed once per file *version* -- keyed by (device, inode, size,
mtime_ns) -- and recomputed whenever the file changes, so a swapped or tampered file is
still rejected before it runs, while repeated calls cost one ``stat``.
"""

from __future__ import annotations

import hashlib
import importlib.util
import re
import threading
from dataclasses import dataclass
from pathlib import Path
from types import ModuleType
from typing import Any, Callable

from radeon_kernels.errors import RadeonKernelsError
from radeon_kernels.runtime.registry import ArtifactSpec

_PYINIT = re.compile(rb"(?<![^\x00])PyInit_([A-Za-z_][A-Za-z0-9_]*)\x00")


class ArtifactError(RadeonKernelsError):
    """Base class for precompiled kernel-pack failures."""


class ArtifactIntegrityError(ArtifactError):
    """An artifact path escapes its pack or its digest does not match."""


class ArtifactLoadError(ArtifactError):
    """A verified artifact cannot be imported or lacks its entrypoint."""


def sha256_of(path: Path) -> str:
    digest = hashlib.sha256()
    with open(path, "rb") as handle:
        while chunk := handle.read(1 << 20):
            digest.update(chunk)
    return digest.hexdigest()


def extension_module_name(path: Path) -> str:
    """Module name from the single exported ``PyInit_<name>`` symbol (else the file stem)."""

    try:
        names = {found.group(1).decode("ascii") for found in _PYINIT.finditer(path.read_bytes())}
    except OSError as error:
        raise ArtifactLoadError(f"cannot inspect Python extension {path.name}: {error}") from error
    if len(names) > 1:
        raise ArtifactLoadError(f"Python extension {path.name} exports multiple PyInit symbols: {sorted(names)}")
    return names.pop() if names else path.name.split(".", 1)[0]


@dataclass(frozen=True)
class LoadedEntrypoint:
    artifact: Path
    provider: str
    entrypoint: str
    callable: Callable[..., Any]


class PrecompiledArtifactLoader:
    def __init__(self, pack_root: Path) -> None:
        try:
            self._root = Path(pack_root).resolve(strict=True)
        except OSError as error:
            raise ArtifactIntegrityError(f"kernel pack root is unavailable: {pack_root}") from error
        if not self._root.is_dir():
            raise ArtifactIntegrityError(f"kernel pack root is not a directory: {pack_root}")
        self._modules: dict[Path, ModuleType] = {}
        self._verified: dict[Path, tuple[tuple[int, int, int, int], str]] = {}
        self._lock = threading.Lock()

    @property
    def root(self) -> Path:
        return self._root

    def resolve_and_verify(self, artifact: ArtifactSpec) -> Path:
        path = (self._root / artifact.artifact).resolve()
        if not path.is_relative_to(self._root):
            raise ArtifactIntegrityError("artifact escapes the kernel pack root")
        try:
            info = path.stat()
        except OSError as error:
            raise ArtifactIntegrityError(f"artifact is missing: {artifact.artifact}") from error
        if not path.is_file():
            raise ArtifactIntegrityError(f"artifact is missing: {artifact.artifact}")
        version = (info.st_dev, info.st_ino, info.st_size, info.st_mtime_ns)
        with self._lock:
            cached = self._verified.get(path)
        if cached is not None and cached[0] == version:
            actual = cached[1]
        else:
            actual = sha256_of(path)
            with self._lock:
                self._verified[path] = (version, actual)
        if actual != artifact.sha256:
            raise ArtifactIntegrityError(
                f"artifact SHA-256 mismatch for {artifact.artifact}: expected {artifact.sha256}, got {actual}"
            )
        return path

    def load_module(self, artifact: ArtifactSpec) -> ModuleType:
        path = self.resolve_and_verify(artifact)
        if artifact.format != "python_extension":
            raise ArtifactLoadError(f"artifact format {artifact.format!r} requires a provider-specific launcher")
        with self._lock:
            module = self._modules.get(path)
        if module is not None:
            return module
        spec = importlib.util.spec_from_file_location(extension_module_name(path), path)
        if spec is None or spec.loader is None:
            raise ArtifactLoadError(f"cannot create an import specification for {path.name}")
        module = importlib.util.module_from_spec(spec)
        try:
            spec.loader.exec_module(module)
        except Exception as error:  # an import failure of any kind disqualifies the winner
            raise ArtifactLoadError(f"failed to load {path.name}: {error}") from error
        with self._lock:
            self._modules.setdefault(path, module)
            return self._modules[path]

    def load_entrypoint(self, artifact: ArtifactSpec) -> LoadedEntrypoint:
        module = self.load_module(artifact)
        function = getattr(module, artifact.entrypoint, None)
        if not callable(function):
            raise ArtifactLoadError(f"artifact {artifact.artifact} does not export callable {artifact.entrypoint!r}")
        return LoadedEntrypoint(
            artifact=self.resolve_and_verify(artifact),
            provider=artifact.provider,
            entrypoint=artifact.entrypoint,
            callable=function,
        )
