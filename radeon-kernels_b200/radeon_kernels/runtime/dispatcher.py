"""Exact-match static dispatch: (operator, version, signature, fingerprint) -> decision.

Behaviour of the reference's ``Dispatcher.select`` (src/radeon_kernels/runtime/dispatcher.py:57-100):
every entry whose environment and workload match is a candidate, the highest priority wins
(the manifest validator guarantees it is unique), and a miss yields the manifest's
``default_fallbacks``.  The decision is recorded for ``explain_last_dispatch`` before any
kernel runs.  Selection is a linear scan: manifests hold a handful of entries.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Mapping

from radeon_kernels.runtime.explain import record_dispatch
from radeon_kernels.runtime.fingerprint import EnvironmentFingerprint
from radeon_kernels.runtime.registry import ArtifactSpec, DispatchRegistry


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

    def to_dict(self) -> dict[str, Any]:
        winner = self.winner
        return {
            "operator": self.operator,
            "semantic_version": self.semantic_version,
            "architecture": self.fingerprint.architecture,
            "rocm_abi": self.fingerprint.rocm_abi,
            "python_abi": self.fingerprint.python_abi,
            "pytorch_version": self.fingerprint.pytorch_version,
            "entry_id": self.entry_id,
            "selected": f"{winner.provider}/{winner.entrypoint}" if winner else None,
            "artifact": winner.artifact if winner else None,
            "launch": dict(self.launch),
            "fallbacks": list(self.fallbacks),
            "evidence_id": self.evidence_id,
            "reason": self.reason,
        }


class Dispatcher:
    def __init__(self, registry: DispatchRegistry) -> None:
        self._registry = registry

    def select(self, request: DispatchRequest, fingerprint: EnvironmentFingerprint) -> DispatchDecision:
        manifest = self._registry.get(request.operator, request.semantic_version)
        best = None
        for entry in manifest.entries:
            if entry.matches(fingerprint, request.signature) and (best is None or entry.priority > best.priority):
                best = entry
        if best is not None:
            decision = DispatchDecision(
                operator=request.operator,
                semantic_version=request.semantic_version,
                fingerprint=fingerprint,
                entry_id=best.id,
                winner=best.winner,
                launch=best.launch,
                fallbacks=best.fallbacks,
                evidence_id=best.evidence_id,
                reason=f"matched dispatch entry {best.id!r} at priority {best.priority}",
            )
        else:
            decision = DispatchDecision(
                operator=request.operator,
                semantic_version=request.semantic_version,
                fingerprint=fingerprint,
                entry_id=None,
                winner=None,
                launch={},
                fallbacks=manifest.default_fallbacks,
                evidence_id=None,
                reason="no compatible environment and workload region matched",
            )
        record_dispatch(decision.to_dict())
        return decision
