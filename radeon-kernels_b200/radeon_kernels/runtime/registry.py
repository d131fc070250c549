"""Static dispatch manifests: strict parsing, region-overlap validation, lookup.

The manifest format is the reference's ``dispatch/*.json`` schema 1.0, unchanged, so a
manifest written for the reference parses here and vice versa
(src/radeon_kernels/runtime/registry.py:59-401):

* workload values are constraints: a scalar is an exact, *type-exact* match (``True`` is
  not ``1``), ``[lo, hi]`` an inclusive positive integer range, ``{"one_of": [...]}`` a set;
* entries whose environment and workload regions overlap must differ in priority, and the
  higher-priority one must be a strict subset of the lower one -- a manifest therefore
  never has two equally good answers for one call;
* unknown or missing fields are errors, never ignored.

On B200 the ``artifact.format`` values stay ``python_extension`` (a pybind module whose
named entrypoint is called with the launch parameters).
"""

from __future__ import annotations

import json
import re
from dataclasses import dataclass
from pathlib import Path, PurePosixPath
from types import MappingProxyType
from typing import Any, Iterable, Mapping

from radeon_kernels.errors import ConfigError
from radeon_kernels.runtime.compatibility import EnvironmentConstraint
from radeon_kernels.runtime.fingerprint import EnvironmentFingerprint

IDENTIFIER_RE = re.compile(r"^[a-z][a-z0-9_.-]*$")
_VERSION_RE = re.compile(r"^\d+\.\d+$")
_SHA256_RE = re.compile(r"^[0-9a-f]{64}$")
_SCHEMA_VERSION = "1.0"
_ARTIFACT_FORMATS = ("python_extension", "hsaco")


def _require_mapping(value: Any, path: str) -> Mapping[str, Any]:
    if not isinstance(value, Mapping) or not all(isinstance(key, str) for key in value):
        raise ConfigError(path, "expected a mapping" if not isinstance(value, Mapping) else "keys must be strings")
    return value


def _check_fields(value: Mapping[str, Any], path: str, *, allowed: Iterable[str], required: Iterable[str]) -> None:
    allowed, required = set(allowed), set(required)
    if set(value) - allowed:
        raise ConfigError(path, f"unknown fields: {sorted(set(value) - allowed)}")
    if required - set(value):
        raise ConfigError(path, f"missing fields: {sorted(required - set(value))}")


def identifier(value: Any, path: str) -> str:
    if not isinstance(value, str) or IDENTIFIER_RE.fullmatch(value) is None:
        raise ConfigError(path, "expected a lowercase identifier")
    return value


def _version(value: Any, path: str) -> str:
    if not isinstance(value, str) or _VERSION_RE.fullmatch(value) is None:
        raise ConfigError(path, "expected MAJOR.MINOR")
    return value


def _scalar(value: Any, path: str) -> str | int | float | bool:
    if isinstance(value, (str, int, float, bool)):
        return value
    raise ConfigError(path, "expected a string, number or boolean")


def _same(value: Any, expected: Any) -> bool:
    return type(value) is type(expected) and value == expected


def _is_int(value: Any) -> bool:
    return isinstance(value, int) and not isinstance(value, bool)


@dataclass(frozen=True)
class _Span:
    """Closed interval of positive integers."""

    low: int
    high: int


def _tagged(items: Iterable[Any]) -> frozenset[tuple[type, Any]]:
    # Values are compared type-exactly: True is not 1, 1 is not 1.0.
    return frozenset((type(item), item) for item in items)


def _domain(constraint: ValueConstraint) -> _Span | frozenset[tuple[type, Any]]:
    if constraint.kind == "range":
        return _Span(*constraint.value)
    return _tagged(constraint.values())


def _ints_of(members: frozenset[tuple[type, Any]]) -> list[int]:
    return [value for kind, value in members if kind is int]


def _intersects(a: _Span | frozenset, b: _Span | frozenset) -> bool:
    if isinstance(a, _Span) and isinstance(b, _Span):
        return max(a.low, b.low) <= min(a.high, b.high)
    if isinstance(a, _Span) or isinstance(b, _Span):
        span, members = (a, b) if isinstance(a, _Span) else (b, a)
        return any(span.low <= value <= span.high for value in _ints_of(members))
    return bool(a & b)


def _within(a: _Span | frozenset, b: _Span | frozenset) -> bool:
    """Every value admitted by ``a`` is admitted by ``b`` (a span inside a finite set only as a
    single point: the manifest language never enumerates a whole span)."""

    if isinstance(a, frozenset):
        if isinstance(b, frozenset):
            return a <= b
        return all(kind is int and b.low <= value <= b.high for kind, value in a)
    if isinstance(b, _Span):
        return b.low <= a.low and a.high <= b.high
    return a.low == a.high and (int, a.low) in b


@dataclass(frozen=True)
class ValueConstraint:
    """Admissible values of one workload field.

    Manifest forms (schema 1.0): a bare scalar (``kind == "eq"``), ``[low, high]`` -- an
    inclusive range of positive integers (``"range"``) -- or ``{"one_of": [...]}`` (``"one_of"``).
    Matching, overlap and containment are computed on a common domain: a span of integers or
    a finite set of type-tagged scalars.
    """

    kind: str
    value: Any

    @classmethod
    def from_raw(cls, raw: Any, path: str) -> ValueConstraint:
        if isinstance(raw, Mapping):
            _check_fields(_require_mapping(raw, path), path, allowed={"one_of"}, required={"one_of"})
            listed = raw["one_of"]
            if not isinstance(listed, list) or not listed:
                raise ConfigError(f"{path}.one_of", "expected a non-empty list")
            members = tuple(_scalar(item, f"{path}.one_of") for item in listed)
            if len(_tagged(members)) != len(members):
                raise ConfigError(f"{path}.one_of", "contains duplicate values")
            return cls("one_of", members)
        if isinstance(raw, list):
            ends = raw if len(raw) == 2 and all(_is_int(end) for end in raw) else None
            if ends is None or not 0 < ends[0] <= ends[1]:
                raise ConfigError(path, "integer ranges must be [minimum, maximum]")
            return cls("range", (ends[0], ends[1]))
        return cls("eq", _scalar(raw, path))

    def values(self) -> tuple[Any, ...]:
        """Representative values: all of them for eq/one_of, the ends of a range."""

        if self.kind == "range":
            return tuple(sorted(set(self.value)))
        return self.value if self.kind == "one_of" else (self.value,)

    def matches(self, candidate: Any) -> bool:
        domain = _domain(self)
        if isinstance(domain, _Span):
            return _is_int(candidate) and domain.low <= candidate <= domain.high
        return (type(candidate), candidate) in domain

    def overlaps(self, other: ValueConstraint) -> bool:
        return _intersects(_domain(self), _domain(other))

    def is_subset_of(self, other: ValueConstraint) -> bool:
        return _within(_domain(self), _domain(other))

    def to_raw(self) -> Any:
        return {"range": list, "one_of": lambda v: {"one_of": list(v)}}.get(self.kind, lambda v: v)(self.value)


@dataclass(frozen=True)
class WorkloadConstraint:
    values: Mapping[str, ValueConstraint]

    @classmethod
    def from_mapping(cls, raw: Mapping[str, Any], path: str) -> WorkloadConstraint:
        raw = _require_mapping(raw, path)
        if not raw:
            raise ConfigError(path, "must contain at least one constraint")
        parsed = {}
        for key, item in raw.items():
            if IDENTIFIER_RE.fullmatch(key) is None:
                raise ConfigError(path, f"invalid workload field: {key!r}")
            parsed[key] = ValueConstraint.from_raw(item, f"{path}.{key}")
        return cls(parsed)

    def matches(self, signature: Mapping[str, Any]) -> bool:
        return all(key in signature and rule.matches(signature[key]) for key, rule in self.values.items())

    def overlaps(self, other: WorkloadConstraint) -> bool:
        # A field constrained on one side only does not separate the regions.
        return all(self.values[key].overlaps(other.values[key]) for key in self.values.keys() & other.values.keys())

    def is_subset_of(self, other: WorkloadConstraint) -> bool:
        return all(key in self.values and self.values[key].is_subset_of(rule) for key, rule in other.values.items())

    def is_strict_subset_of(self, other: WorkloadConstraint) -> bool:
        if not self.is_subset_of(other):
            return False
        if set(self.values) > set(other.values):
            return True
        return any(not rule.is_subset_of(self.values[key]) for key, rule in other.values.items())

    def to_dict(self) -> dict[str, Any]:
        return {key: rule.to_raw() for key, rule in self.values.items()}


@dataclass(frozen=True)
class ArtifactSpec:
    provider: str
    artifact: str
    entrypoint: str
    sha256: str
    format: str = "python_extension"

    @classmethod
    def from_mapping(cls, raw: Mapping[str, Any], path: str) -> ArtifactSpec:
        raw = _require_mapping(raw, path)
        _check_fields(
            raw,
            path,
            allowed={"provider", "artifact", "entrypoint", "sha256", "format"},
            required={"provider", "artifact", "entrypoint", "sha256"},
        )
        artifact = raw["artifact"]
        if not isinstance(artifact, str) or not artifact:
            raise ConfigError(f"{path}.artifact", "expected a relative path")
        posix = PurePosixPath(artifact)
        if posix.is_absolute() or ".." in posix.parts or posix.as_posix() != artifact:
            raise ConfigError(f"{path}.artifact", "must be a normalized relative path")
        entrypoint = raw["entrypoint"]
        if not isinstance(entrypoint, str) or not entrypoint.isidentifier():
            raise ConfigError(f"{path}.entrypoint", "expected a Python/C identifier")
        digest = raw["sha256"]
        if not isinstance(digest, str) or _SHA256_RE.fullmatch(digest) is None:
            raise ConfigError(f"{path}.sha256", "expected a lowercase SHA-256")
        kind = raw.get("format", "python_extension")
        if kind not in _ARTIFACT_FORMATS:
            raise ConfigError(f"{path}.format", "expected python_extension or hsaco")
        return cls(identifier(raw["provider"], f"{path}.provider"), artifact, entrypoint, digest, kind)

    def to_dict(self) -> dict[str, Any]:
        return {
            "provider": self.provider,
            "artifact": self.artifact,
            "entrypoint": self.entrypoint,
            "sha256": self.sha256,
            "format": self.format,
        }


_ENTRY_FIELDS = ("id", "priority", "environment", "workload", "winner", "launch", "fallbacks", "evidence_id")


def _identifier_list(raw: Any, path: str) -> tuple[str, ...]:
    if not isinstance(raw, list):
        raise ConfigError(path, "expected a list")
    items = tuple(identifier(item, path) for item in raw)
    if len(set(items)) != len(items):
        raise ConfigError(path, "contains duplicates")
    return items


@dataclass(frozen=True)
class DispatchEntry:
    id: str
    priority: int
    environment: EnvironmentConstraint
    workload: WorkloadConstraint
    winner: ArtifactSpec
    launch: Mapping[str, str | int | float | bool]
    fallbacks: tuple[str, ...]
    evidence_id: str

    @classmethod
    def from_mapping(cls, raw: Mapping[str, Any], path: str) -> DispatchEntry:
        raw = _require_mapping(raw, path)
        _check_fields(raw, path, allowed=_ENTRY_FIELDS, required=_ENTRY_FIELDS)
        priority = raw["priority"]
        if not _is_int(priority) or priority < 0:
            raise ConfigError(f"{path}.priority", "expected a non-negative integer")
        launch_raw = _require_mapping(raw["launch"], f"{path}.launch")
        launch = {}
        for key, item in launch_raw.items():
            if IDENTIFIER_RE.fullmatch(key) is None:
                raise ConfigError(f"{path}.launch", f"invalid parameter: {key!r}")
            launch[key] = _scalar(item, f"{path}.launch.{key}")
        return cls(
            id=identifier(raw["id"], f"{path}.id"),
            priority=priority,
            environment=EnvironmentConstraint.from_mapping(raw["environment"], f"{path}.environment"),
            workload=WorkloadConstraint.from_mapping(raw["workload"], f"{path}.workload"),
            winner=ArtifactSpec.from_mapping(raw["winner"], f"{path}.winner"),
            launch=MappingProxyType(launch),
            fallbacks=_identifier_list(raw["fallbacks"], f"{path}.fallbacks"),
            evidence_id=identifier(raw["evidence_id"], f"{path}.evidence_id"),
        )

    def matches(self, fingerprint: EnvironmentFingerprint, signature: Mapping[str, Any]) -> bool:
        return self.environment.matches(fingerprint) and self.workload.matches(signature)

    def to_dict(self) -> dict[str, Any]:
        return {
            "id": self.id,
            "priority": self.priority,
            "environment": self.environment.to_dict(),
            "workload": self.workload.to_dict(),
            "winner": self.winner.to_dict(),
            "launch": dict(self.launch),
            "fallbacks": list(self.fallbacks),
            "evidence_id": self.evidence_id,
        }


_MANIFEST_FIELDS = ("schema_version", "operator", "semantic_version", "default_fallbacks", "entries")


@dataclass(frozen=True)
class DispatchManifest:
    schema_version: str
    operator: str
    semantic_version: str
    default_fallbacks: tuple[str, ...]
    entries: tuple[DispatchEntry, ...]

    @classmethod
    def from_mapping(cls, raw: Mapping[str, Any], path: str = "dispatch") -> DispatchManifest:
        raw = _require_mapping(raw, path)
        _check_fields(raw, path, allowed=_MANIFEST_FIELDS, required=_MANIFEST_FIELDS)
        if not isinstance(raw["entries"], list):
            raise ConfigError(f"{path}.entries", "expected a list")
        if not isinstance(raw["default_fallbacks"], list) or not raw["default_fallbacks"]:
            raise ConfigError(f"{path}.default_fallbacks", "expected a non-empty list")
        schema = _version(raw["schema_version"], f"{path}.schema_version")
        if schema != _SCHEMA_VERSION:
            raise ConfigError(f"{path}.schema_version", f"unsupported dispatch schema version {schema!r}")
        manifest = cls(
            schema_version=schema,
            operator=identifier(raw["operator"], f"{path}.operator"),
            semantic_version=_version(raw["semantic_version"], f"{path}.semantic_version"),
            default_fallbacks=_identifier_list(raw["default_fallbacks"], f"{path}.default_fallbacks"),
            entries=tuple(
                DispatchEntry.from_mapping(item, f"{path}.entries[{index}]")
                for index, item in enumerate(raw["entries"])
            ),
        )
        manifest._check_regions(path)
        return manifest

    def _check_regions(self, path: str) -> None:
        ids = [entry.id for entry in self.entries]
        if len(set(ids)) != len(ids):
            raise ConfigError(f"{path}.entries", "entry ids must be unique")
        for index, first in enumerate(self.entries):
            for second in self.entries[index + 1 :]:
                if not (first.environment.overlaps(second.environment) and first.workload.overlaps(second.workload)):
                    continue
                if first.priority == second.priority:
                    raise ConfigError(f"{path}.entries", f"ambiguous overlapping entries {first.id!r} and {second.id!r}")
                high, low = (first, second) if first.priority > second.priority else (second, first)
                nested = high.environment.is_subset_of(low.environment) and high.workload.is_subset_of(low.workload)
                narrower = high.environment.is_strict_subset_of(low.environment) or high.workload.is_strict_subset_of(
                    low.workload
                )
                if not (nested and narrower):
                    raise ConfigError(
                        f"{path}.entries", f"higher-priority entry {high.id!r} must be a strict subset of {low.id!r}"
                    )

    @classmethod
    def from_file(cls, path: Path) -> DispatchManifest:
        try:
            payload = json.loads(Path(path).read_text(encoding="utf-8"))
        except OSError as error:
            raise ConfigError(str(path), str(error)) from error
        except json.JSONDecodeError as error:
            raise ConfigError(str(path), f"invalid JSON: {error.msg}") from error
        return cls.from_mapping(payload, str(path))

    def to_dict(self) -> dict[str, Any]:
        return {
            "schema_version": self.schema_version,
            "operator": self.operator,
            "semantic_version": self.semantic_version,
            "default_fallbacks": list(self.default_fallbacks),
            "entries": [entry.to_dict() for entry in self.entries],
        }


class DispatchRegistry:
    """All manifests known to a runtime, keyed by (operator, semantic version)."""

    def __init__(self, manifests: Iterable[DispatchManifest] = ()) -> None:
        self._by_key: dict[tuple[str, str], DispatchManifest] = {}
        for manifest in manifests:
            self.add(manifest)

    def add(self, manifest: DispatchManifest) -> None:
        key = (manifest.operator, manifest.semantic_version)
        if key in self._by_key:
            raise ConfigError("dispatch", f"duplicate manifest for {key[0]} {key[1]}")
        self._by_key[key] = manifest

    def get(self, operator: str, semantic_version: str) -> DispatchManifest:
        try:
            return self._by_key[(operator, semantic_version)]
        except KeyError as error:
            raise ConfigError(
                "dispatch", f"no manifest for operator {operator!r} semantic version {semantic_version!r}"
            ) from error

    def keys(self) -> tuple[tuple[str, str], ...]:
        return tuple(sorted(self._by_key))

    @classmethod
    def from_directory(cls, directory: Path) -> DispatchRegistry:
        directory = Path(directory)
        if not directory.is_dir():
            raise ConfigError(str(directory), "dispatch directory does not exist")
        files = sorted(directory.rglob("*.json"))
        if not files:
            raise ConfigError(str(directory), "contains no dispatch manifests")
        return cls(DispatchManifest.from_file(path) for path in files)
