"""Per-context record of the last dispatch decision and its 7-line explanation.

Format-compatible with the reference (src/radeon_kernels/runtime/explain.py:8-46): the
record lives in a ``ContextVar`` (so it is per thread and per asyncio task), is stored and
returned as deep copies, and ``explain_last_dispatch`` prints exactly the lines
``operator, architecture, selected, artifact, evidence, fallbacks, reason``.
"""

from __future__ import annotations

from contextvars import ContextVar
from copy import deepcopy
from typing import Any, Mapping

_LAST: ContextVar[dict[str, Any] | None] = ContextVar("radeon_kernels_last_dispatch", default=None)

_NO_DISPATCH = "No Radeon kernel dispatch has been performed in this context."


def record_dispatch(value: Mapping[str, Any]) -> None:
    _LAST.set(deepcopy(dict(value)))


def record_dispatch_shared(value: dict[str, Any]) -> None:
    """Record a dispatch dict that the caller promises never to mutate (no copy).

    Used by the operator runtimes' decision cache: a cached record is created once per
    (operator, signature, device) and shared; readers only ever get deep copies.
    """

    _LAST.set(value)


def get_last_dispatch() -> dict[str, Any] | None:
    value = _LAST.get()
    return None if value is None else deepcopy(value)


def clear_last_dispatch() -> None:
    _LAST.set(None)


def explain_last_dispatch() -> str:
    value = _LAST.get()
    if value is None:
        return _NO_DISPATCH
    fallbacks = value.get("fallbacks") or []
    lines = (
        ("operator", value["operator"]),
        ("architecture", value["architecture"]),
        ("selected", value.get("selected") or "none"),
        ("artifact", value.get("artifact") or "none"),
        ("evidence", value.get("evidence_id") or "none"),
        ("fallbacks", " -> ".join(fallbacks) if fallbacks else "none"),
        ("reason", value["reason"]),
    )
    return "\n".join(f"{name}: {text}" for name, text in lines)
