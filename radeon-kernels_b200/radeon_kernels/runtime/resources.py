"""Package data: the built-in dispatch manifests and operator contracts.

Equivalent of the reference's ``builtin_dispatch_registry``
(src/radeon_kernels/runtime/resources.py:34-43): every ``dispatch/*.json`` shipped with
the package is parsed strictly (including the region-overlap validator) into one registry.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any, Mapping

from radeon_kernels.errors import ConfigError
from radeon_kernels.runtime.registry import DispatchManifest, DispatchRegistry

PACKAGE_ROOT = Path(__file__).resolve().parents[1]
DISPATCH_DIR = PACKAGE_ROOT / "dispatch"
CONTRACTS_DIR = PACKAGE_ROOT / "contracts"


def builtin_dispatch_registry() -> DispatchRegistry:
    manifests = []
    for path in sorted(DISPATCH_DIR.glob("*.json")):
        try:
            payload = json.loads(path.read_text(encoding="utf-8"))
        except json.JSONDecodeError as error:
            raise ConfigError("built-in dispatch", f"invalid JSON: {error.msg}") from error
        manifests.append(DispatchManifest.from_mapping(payload, str(path)))
    if not manifests:
        raise ConfigError("built-in dispatch", "contains no manifests")
    return DispatchRegistry(manifests)


def builtin_contract(operator: str, semantic_version: str) -> Mapping[str, Any]:
    path = CONTRACTS_DIR / f"{operator}-{semantic_version}.json"
    try:
        value = json.loads(path.read_text(encoding="utf-8"))
    except (OSError, json.JSONDecodeError) as error:
        raise ConfigError(str(path), f"cannot read contract: {error}") from error
    if value.get("operator") != operator or value.get("semantic_version") != semantic_version:
        raise ConfigError(str(path), "contract identity does not match request")
    return value
