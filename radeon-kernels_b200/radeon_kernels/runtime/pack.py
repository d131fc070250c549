"""Kernel pack directory model: ``manifest.json`` + artifacts under ``lib/``.

Manifest format of the reference (src/radeon_kernels/runtime/pack.py:40-157), unchanged:
``{schema_version: "1.0", pack_id, pack_version: X.Y.Z, environment, artifacts: [...]}``
where each artifact names the operator/semantic version it serves, the provider, relative
path, entrypoint, SHA-256, format and evidence id.  One artifact per operator version,
artifact paths unique.
"""

from __future__ import annotations

import json
import re
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Mapping

from radeon_kernels.errors import ConfigError
from radeon_kernels.runtime.compatibility import EnvironmentConstraint
from radeon_kernels.runtime.fingerprint import EnvironmentFingerprint
from radeon_kernels.runtime.loader import PrecompiledArtifactLoader
from radeon_kernels.runtime.registry import ArtifactSpec, identifier

_VERSION_RE = re.compile(r"^\d+\.\d+$")
_PACK_VERSION_RE = re.compile(r"^\d+\.\d+\.\d+$")
_ARTIFACT_FIELDS = frozenset(
    {"operator", "semantic_version", "provider", "artifact", "entrypoint", "sha256", "format", "evidence_id"}
)
_PACK_FIELDS = frozenset({"schema_version", "pack_id", "pack_version", "environment", "artifacts"})


def _version(value: Any, path: str, pattern: re.Pattern[str]) -> str:
    if not isinstance(value, str) or pattern.fullmatch(value) is None:
        raise ConfigError(path, "invalid version")
    return value


def _fields(value: Mapping[str, Any], path: str, expected: frozenset[str]) -> None:
    if set(value) - expected:
        raise ConfigError(path, f"unknown fields: {sorted(set(value) - expected)}")
    if expected - set(value):
        raise ConfigError(path, f"missing fields: {sorted(expected - set(value))}")


@dataclass(frozen=True)
class KernelPackArtifact:
    operator: str
    semantic_version: str
    artifact: ArtifactSpec
    evidence_id: str

    @classmethod
    def from_mapping(cls, value: Any, path: str) -> KernelPackArtifact:
        if not isinstance(value, Mapping):
            raise ConfigError(path, "expected a mapping")
        _fields(value, path, _ARTIFACT_FIELDS)
        spec = ArtifactSpec.from_mapping(
            {key: value[key] for key in ("provider", "artifact", "entrypoint", "sha256", "format")}, path
        )
        return cls(
            operator=identifier(value["operator"], f"{path}.operator"),
            semantic_version=_version(value["semantic_version"], f"{path}.semantic_version", _VERSION_RE),
            artifact=spec,
            evidence_id=identifier(value["evidence_id"], f"{path}.evidence_id"),
        )

    def to_dict(self) -> dict[str, Any]:
        return {
            "operator": self.operator,
            "semantic_version": self.semantic_version,
            **self.artifact.to_dict(),
            "evidence_id": self.evidence_id,
        }


@dataclass(frozen=True)
class KernelPack:
    root: Path
    schema_version: str
    pack_id: str
    pack_version: str
    environment: EnvironmentConstraint
    artifacts: tuple[KernelPackArtifact, ...]

    @classmethod
    def from_directory(cls, root: Path, *, verify_artifacts: bool = True) -> KernelPack:
        try:
            base = Path(root).resolve(strict=True)
        except OSError as error:
            raise ConfigError(str(root), "kernel pack directory does not exist") from error
        manifest = base / "manifest.json"
        where = str(manifest)
        try:
            value = json.loads(manifest.read_text(encoding="utf-8"))
        except OSError as error:
            raise ConfigError(where, str(error)) from error
        except json.JSONDecodeError as error:
            raise ConfigError(where, f"invalid JSON: {error.msg}") from error
        if not isinstance(value, Mapping):
            raise ConfigError(where, "expected a mapping")
        _fields(value, where, _PACK_FIELDS)
        schema = _version(value["schema_version"], f"{where}.schema_version", _VERSION_RE)
        if schema != "1.0":
            raise ConfigError(f"{where}.schema_version", f"unsupported version {schema!r}")
        if not isinstance(value["artifacts"], list) or not value["artifacts"]:
            raise ConfigError(f"{where}.artifacts", "expected a non-empty list")
        pack = cls(
            root=base,
            schema_version=schema,
            pack_id=identifier(value["pack_id"], f"{where}.pack_id"),
            pack_version=_version(value["pack_version"], f"{where}.pack_version", _PACK_VERSION_RE),
            environment=EnvironmentConstraint.from_mapping(value["environment"], f"{where}.environment"),
            artifacts=tuple(
                KernelPackArtifact.from_mapping(item, f"{where}.artifacts[{index}]")
                for index, item in enumerate(value["artifacts"])
            ),
        )
        keys = [(item.operator, item.semantic_version) for item in pack.artifacts]
        if len(set(keys)) != len(keys):
            raise ConfigError(f"{where}.artifacts", "operator semantic versions must be unique")
        paths = [item.artifact.artifact for item in pack.artifacts]
        if len(set(paths)) != len(paths):
            raise ConfigError(f"{where}.artifacts", "artifact paths must be unique")
        if verify_artifacts:
            loader = PrecompiledArtifactLoader(pack.root)
            for item in pack.artifacts:
                loader.resolve_and_verify(item.artifact)
        return pack

    def matches(self, fingerprint: EnvironmentFingerprint) -> bool:
        return self.environment.matches(fingerprint)

    def get(self, operator: str, semantic_version: str) -> KernelPackArtifact:
        for item in self.artifacts:
            if item.operator == operator and item.semantic_version == semantic_version:
                return item
        raise ConfigError(self.pack_id, f"pack has no artifact for {operator!r} semantic version {semantic_version!r}")
