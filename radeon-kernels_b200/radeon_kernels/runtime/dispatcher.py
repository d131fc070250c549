"""Static dispatch: (operator, version, signature, fingerprint) -> decision.

Semantics of the reference's ``Dispatcher.select`` (src/radeon_kernels/runtime/dispatcher.py:
57-100): an entry is a candidate when its environment and workload both match; the
highest-priority candidate wins (the manifest validator makes it unique); with no candidate
the manifest's ``default_fallbacks`` apply.  The decision -- as the dictionary that
``explain_last_dispatch`` renders -- is recorded before any kernel runs.  Manifests hold a
handful of entries, so selection is one pass over them.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Mapping

from radeon_kernels.runtime.explain import record_dispatch
from radeon_kernels.runtime.fingerprint import EnvironmentFingerprint
from radeon_kernels.runtime.registry import ArtifactSpec, DispatchEntry, DispatchRegistry

NO_MATCH_REASON = "no compatible environment and workload region matched"


@dataclass(frozen=True)
class DispatchRequest:
    operator: str
    semantic_version: str
    signature: Mapping[str, Any]


@dataclass(frozen=True)
class DispatchDecision:
    operator: str
    semantic_version: str
    fingerprint: EnvironmentFingerprint
    entry_id: str | None
    winner: ArtifactSpec | None
    launch: Mapping[str, str | int | float | bool]
    fallbacks: tuple[str, ...]
    evidence_id: str | None
    reason: str

    @property
    def matched(self) -> bool:
        return self.winner is not None

    @classmethod
    def for_entry(cls, request: DispatchRequest, fingerprint: EnvironmentFingerprint, entry: DispatchEntry) -> DispatchDecision:
        return cls(request.operator, request.semantic_version, fingerprint, entry.id, entry.winner, entry.launch,
                   entry.fallbacks, entry.evidence_id, f"matched dispatch entry {entry.id!r} at priority {entry.priority}")

    @classmethod
    def unmatched(cls, request: DispatchRequest, fingerprint: EnvironmentFingerprint, fallbacks: tuple[str, ...]) -> DispatchDecision:
        return cls(request.operator, request.semantic_version, fingerprint, None, None, {}, fallbacks, None, NO_MATCH_REASON)

    def to_dict(self) -> dict[str, Any]:
        """The record ``get_last_dispatch()`` returns (keys callers parse)."""

        env = self.fingerprint
        chosen = self.winner
        return {
            "operator": self.operator,
            "semantic_version": self.semantic_version,
            **{key: getattr(env, key) for key in ("architecture", "rocm_abi", "python_abi", "pytorch_version")},
            "entry_id": self.entry_id,
            "selected": None if chosen is None else f"{chosen.provider}/{chosen.entrypoint}",
            "artifact": None if chosen is None else chosen.artifact,
            "launch": dict(self.launch),
            "fallbacks": list(self.fallbacks),
            "evidence_id": self.evidence_id,
            "reason": self.reason,
        }


class Dispatcher:
    def __init__(self, registry: DispatchRegistry) -> None:
        self.registry = registry

    def select(self, request: DispatchRequest, fingerprint: EnvironmentFingerprint) -> DispatchDecision:
        manifest = self.registry.get(request.operator, request.semantic_version)
        candidates = [entry for entry in manifest.entries if entry.matches(fingerprint, request.signature)]
        if candidates:
            decision = DispatchDecision.for_entry(request, fingerprint, max(candidates, key=lambda entry: entry.priority))
        else:
            decision = DispatchDecision.unmatched(request, fingerprint, manifest.default_fallbacks)
        record_dispatch(decision.to_dict())
        return decision
