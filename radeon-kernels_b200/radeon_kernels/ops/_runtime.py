"""Shared static-dispatch executor: decision -> pack winner -> declared fallback.

Control flow of the reference's ``OperatorRuntime.execute``
(src/radeon_kernels/ops/_runtime.py:82-171), with the fallback chain retargeted: the
manifests of this build declare the built-in ``cuda`` provider (this library's generic
kernels) instead of ``torch``.  A manifest that only declares ``torch`` is honoured by
refusing it -- there is no torch/CPU execution path -- and the call raises
:class:`OperatorDispatchError` with the reason recorded.

Every outcome is recorded for ``explain_last_dispatch``: the winner with the pack that
served it, or the fallback with the winner's failure reason, or "none".
"""

from __future__ import annotations

from pathlib import Path
from threading import Lock
from typing import Any, Callable, Iterable, Mapping

from radeon_kernels.errors import RadeonKernelsError
from radeon_kernels.providers import native
from radeon_kernels.runtime.dispatcher import DispatchDecision, DispatchRequest, Dispatcher
from radeon_kernels.runtime.explain import record_dispatch, record_dispatch_shared
from radeon_kernels.runtime.fingerprint import EnvironmentFingerprint
from radeon_kernels.runtime.loader import ArtifactError, PrecompiledArtifactLoader
from radeon_kernels.runtime.packs import (
    BUILTIN_PACK_ROOT,
    KernelPackRegistry,
    PackResolutionError,
    default_pack_roots,
)
from radeon_kernels.runtime.registry import DispatchRegistry
from radeon_kernels.runtime.resources import builtin_dispatch_registry

FALLBACK_PROVIDER = "cuda"
WINNER_FAILURES = (PackResolutionError, ArtifactError, native.NativeProviderError, RuntimeError, TypeError, ValueError)


class OperatorDispatchError(RadeonKernelsError):
    """Neither a published winner nor a supported fallback can run."""


def record_execution(
    decision: DispatchDecision, *, selected: str, artifact: str | None, evidence_id: str | None, reason: str
) -> None:
    record = decision.to_dict()
    record.update({"selected": selected, "artifact": artifact, "evidence_id": evidence_id, "reason": reason})
    record_dispatch(record)


class DispatchingRuntime:
    """Dispatcher + pack registry + cached loaders and fingerprints (one per process)."""

    def __init__(
        self,
        *,
        registry: DispatchRegistry | None = None,
        pack_roots: Iterable[Path] | None = None,
        pack_registry: KernelPackRegistry | None = None,
        require_pack_signatures: bool = True,
        builtin_pack_roots: Iterable[Path] | None = None,
        loader_factory: Callable[[Path], PrecompiledArtifactLoader] = PrecompiledArtifactLoader,
        fingerprint_detector: Callable[..., EnvironmentFingerprint] = EnvironmentFingerprint.detect,
        cuda_provider: Any = None,
    ) -> None:
        from radeon_kernels.providers import cuda_builtin

        self.cuda_provider = cuda_provider if cuda_provider is not None else cuda_builtin
        self._dispatcher = Dispatcher(registry or builtin_dispatch_registry())
        if pack_registry is None:
            roots = tuple(pack_roots) if pack_roots is not None else default_pack_roots()
            builtin = (BUILTIN_PACK_ROOT,) if builtin_pack_roots is None and pack_roots is None else tuple(builtin_pack_roots or ())
            pack_registry = KernelPackRegistry.discover(
                roots, require_signatures=require_pack_signatures, builtin_roots=builtin
            )
        self._pack_registry = pack_registry
        self._loader_factory = loader_factory
        self._detect = fingerprint_detector
        self._loaders: dict[Path, PrecompiledArtifactLoader] = {}
        self._fingerprints: dict[int, EnvironmentFingerprint] = {}
        self._lock = Lock()
        # (operator, device, signature items) -> (entrypoint, launch, shared record).
        # Filled after a winner ran successfully; the reference re-selects, re-resolves
        # and re-hashes on every call (ops/_runtime.py:87-121), which costs far more
        # than a decode GEMV's kernel time.  Manifests and packs are immutable for the
        # lifetime of a runtime, so the decision cannot change; reset_*runtime() drops it.
        self._fast: dict[tuple, tuple[Any, Any, dict[str, Any]]] = {}
        self._fast_positional: dict[tuple, tuple[Any, Any, dict[str, Any]]] = {}

    @property
    def pack_registry(self) -> KernelPackRegistry:
        return self._pack_registry

    def fingerprint(self, torch_module: Any, device_index: int) -> EnvironmentFingerprint:
        found = self._fingerprints.get(device_index)
        if found is None:
            found = self._detect(torch_module=torch_module, device_index=device_index)
            self._fingerprints[device_index] = found
        return found

    def loader(self, root: Path) -> PrecompiledArtifactLoader:
        with self._lock:
            if root not in self._loaders:
                self._loaders[root] = self._loader_factory(root)
            return self._loaders[root]

    @staticmethod
    def fast_key(operator: str, device_index: int, signature: Mapping[str, Any]) -> tuple:
        return (operator, device_index, tuple(sorted(signature.items())))

    def fast_call(self, key: tuple, arguments: tuple[Any, ...]) -> Any | None:
        """Run a cached winner for ``key`` (operator-specific positional key), or None."""

        cached = self._fast_positional.get(key)
        if cached is None:
            return None
        entry, launch, record = cached
        result = entry(*arguments, **launch)
        if result is None:
            raise native.NativeProviderError("native entrypoint returned no output")
        record_dispatch_shared(record)
        return result

    def fast_alias(self, key: tuple, signature_key: tuple) -> None:
        """Let positional ``key`` reuse the cached winner stored under ``signature_key``."""

        cached = self._fast.get(signature_key)
        if cached is not None:
            self._fast_positional[key] = cached

    def fast_lookup(self, key: tuple) -> tuple[Any, Any, dict[str, Any]] | None:
        return self._fast.get(key)

    def fast_store(self, key: tuple, entry: Any, launch: Any, decision: DispatchDecision, reason: str) -> None:
        record = decision.to_dict()
        record.update(
            {
                "selected": f"{decision.winner.provider}/{decision.winner.entrypoint}",
                "artifact": decision.winner.artifact,
                "evidence_id": decision.evidence_id,
                "reason": reason,
            }
        )
        self._fast[key] = (entry, launch, record)

    def decide(self, operator: str, version: str, signature: Mapping[str, Any], fingerprint: EnvironmentFingerprint):
        return self._dispatcher.select(DispatchRequest(operator, version, signature), fingerprint)

    def resolve(self, decision: DispatchDecision, fingerprint: EnvironmentFingerprint):
        return self._pack_registry.resolve(
            fingerprint=fingerprint,
            operator=decision.operator,
            semantic_version=decision.semantic_version,
            artifact=decision.winner,
            evidence_id=decision.evidence_id,
        )

    def run_fallback(
        self,
        decision: DispatchDecision,
        winner_failure: str | None,
        fallback: Callable[[], Any],
        fallback_selected: str,
        error_type: type[RadeonKernelsError],
        failure_message: str,
    ) -> Any:
        reason = decision.reason if winner_failure is None else f"{decision.reason}; winner unavailable: {winner_failure}"
        if FALLBACK_PROVIDER in decision.fallbacks:
            try:
                result = fallback()
            except Exception as error:
                record_execution(
                    decision, selected="none", artifact=None, evidence_id=None, reason=f"cuda fallback failed: {error}"
                )
                raise
            record_execution(
                decision,
                selected=fallback_selected,
                artifact=None,
                evidence_id=None,
                reason=f"{reason}; executed declared cuda fallback",
            )
            return result
        skipped = [name for name in decision.fallbacks if name != FALLBACK_PROVIDER]
        note = f"; declared fallbacks {skipped} are not available on this build" if skipped else ""
        record_execution(
            decision,
            selected="none",
            artifact=None,
            evidence_id=None,
            reason=f"{reason}{note}; no supported fallback is available",
        )
        raise error_type(failure_message)


class OperatorRuntime(DispatchingRuntime):
    """Static-dispatch executor for operators whose winner returns a new tensor (gemv)."""

    def execute(
        self,
        *,
        operator: str,
        semantic_version: str,
        signature: Mapping[str, Any],
        device_index: int,
        torch_module: Any,
        native_arguments: tuple[Any, ...],
        fallback: Callable[[], Any],
        fallback_selected: str,
    ) -> Any:
        key = self.fast_key(operator, device_index, signature)
        cached = self.fast_lookup(key)
        if cached is not None:
            entry, launch, record = cached
            result = entry(*native_arguments, **launch)
            if result is None:
                raise native.NativeProviderError("native entrypoint returned no output")
            record_dispatch_shared(record)
            return result
        fingerprint = self.fingerprint(torch_module, device_index)
        decision = self.decide(operator, semantic_version, signature, fingerprint)
        failure: str | None = None
        if decision.matched:
            try:
                resolved = self.resolve(decision, fingerprint)
                loader = self.loader(resolved.pack.root)
                result = native.execute(loader, resolved.load_spec, decision.launch, *native_arguments)
                reason = f"{decision.reason}; loaded pack {resolved.pack.pack_id} {resolved.pack.pack_version}"
                record_execution(
                    decision,
                    selected=f"{decision.winner.provider}/{decision.winner.entrypoint}",
                    artifact=decision.winner.artifact,
                    evidence_id=decision.evidence_id,
                    reason=reason,
                )
                entry = getattr(loader, "load_entrypoint")(resolved.load_spec).callable
                self.fast_store(key, entry, dict(decision.launch), decision, reason)
                return result
            except WINNER_FAILURES as error:
                failure = str(error)
        return self.run_fallback(
            decision,
            failure,
            fallback,
            fallback_selected,
            OperatorDispatchError,
            f"no approved implementation is available for {operator} {semantic_version}",
        )


_DEFAULT: OperatorRuntime | None = None
_DEFAULT_LOCK = Lock()


def default_operator_runtime() -> OperatorRuntime:
    global _DEFAULT
    if _DEFAULT is None:
        with _DEFAULT_LOCK:
            if _DEFAULT is None:
                _DEFAULT = OperatorRuntime()
    return _DEFAULT


def reset_operator_runtime() -> None:
    global _DEFAULT
    with _DEFAULT_LOCK:
        _DEFAULT = None


__all__ = [
    "DispatchingRuntime",
    "OperatorDispatchError",
    "OperatorRuntime",
    "default_operator_runtime",
    "reset_operator_runtime",
]
