"""Publication of the built-in sm_100a kernel pack (build-time helper).

The build compiles the pack's ``python_extension`` artifact; this module then writes the
pack's ``manifest.json`` (artifact digests, environment of the build) and refreshes the
``sha256`` of every dispatch entry whose winner is that artifact, so dispatch and pack stay
consistent.  It plays the role of the reference's developer-side publish step
(developer/promotion/publish_approved.py), minus the approval workflow and signing: the
built-in pack is trusted by location (see ``radeon_kernels.runtime.packs``).

Files are rewritten only when their content changes.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path
from typing import Any

from radeon_kernels.runtime.loader import sha256_of
from radeon_kernels.runtime.resources import DISPATCH_DIR

PACK_ID = "rk-sm100a"
PACK_VERSION = "0.1.0"
ARTIFACT = "lib/rk_sm100a.so"
# (operator, semantic version) -> (entrypoint, evidence id)
ENTRYPOINTS = {
    ("gemm", "1.0"): ("gemm_out", "rk-sm100a-gemm"),
    ("gemv", "1.0"): ("gemv", "rk-sm100a-gemv"),
    ("swiglu", "1.0"): ("silu_mul", "rk-sm100a-swiglu"),
    ("rms_norm", "1.0"): ("rms_norm", "rk-sm100a-rms_norm"),
    ("add_rms_norm", "1.0"): ("add_rms_norm", "rk-sm100a-add_rms_norm"),
    ("gemm_swiglu", "1.0"): ("gemm_swiglu", "rk-sm100a-gemm_swiglu"),
    ("paged_attention_decode", "1.0"): ("paged_attention_decode", "rk-sm100a-paged_attention_decode"),
    ("sdpa", "1.0"): ("sdpa", "rk-sm100a-sdpa"),
}


def build_environment() -> dict[str, Any]:
    """Environment constraint of packs built here (the PyTorch/CUDA the binding links)."""

    import torch

    from radeon_kernels.runtime.fingerprint import normalize_rocm_abi

    return {
        "architecture": "sm_100a",
        "wavefront_size": 32,
        "rocm_abi": normalize_rocm_abi(str(torch.version.cuda)),
        "python_abi": f"cp{sys.version_info.major}{sys.version_info.minor}",
        "pytorch_version": str(torch.__version__),
        "features": ["tcgen05", "tma"],
    }


def _write_if_changed(path: Path, payload: Any) -> bool:
    text = json.dumps(payload, indent=2) + "\n"
    if path.exists() and path.read_text(encoding="utf-8") == text:
        return False
    path.write_text(text, encoding="utf-8")
    return True


def publish_builtin_pack(
    pack_dir: Path, artifact_path: Path, *, refresh_dispatch: bool = True, rewrite: bool = True
) -> str:
    """Write ``pack_dir/manifest.json`` for ``artifact_path``; returns its SHA-256."""

    digest = sha256_of(artifact_path)
    manifest = {
        "schema_version": "1.0",
        "pack_id": PACK_ID,
        "pack_version": PACK_VERSION,
        "environment": build_environment(),
        "artifacts": [
            {
                "operator": operator,
                "semantic_version": version,
                "provider": "native",
                "artifact": ARTIFACT,
                "entrypoint": entrypoint,
                "sha256": digest,
                "format": "python_extension",
                "evidence_id": evidence,
            }
            for (operator, version), (entrypoint, evidence) in ENTRYPOINTS.items()
        ],
    }
    # KernelPack requires unique artifact paths per pack entry; one shared object serves
    # several operators, so each operator gets its own hard link under lib/.
    for item in manifest["artifacts"]:
        item["artifact"] = f"lib/{item['operator']}/rk_sm100a.so"
        link = pack_dir / item["artifact"]
        link.parent.mkdir(parents=True, exist_ok=True)
        if rewrite or not link.exists() or sha256_of(link) != digest:
            if link.exists():
                link.unlink()
            try:
                link.hardlink_to(artifact_path)
            except OSError:
                link.write_bytes(artifact_path.read_bytes())
    _write_if_changed(pack_dir / "manifest.json", manifest)
    if refresh_dispatch:
        refresh_dispatch_digests(manifest)
    return digest


def refresh_dispatch_digests(manifest: dict[str, Any], dispatch_dir: Path = DISPATCH_DIR) -> list[Path]:
    """Point every dispatch winner that names a pack artifact at its current digest."""

    by_path = {item["artifact"]: item["sha256"] for item in manifest["artifacts"]}
    changed = []
    for path in sorted(dispatch_dir.glob("*.json")):
        payload = json.loads(path.read_text(encoding="utf-8"))
        dirty = False
        for entry in payload.get("entries", []):
            winner = entry.get("winner", {})
            digest = by_path.get(winner.get("artifact"))
            if digest is not None and winner.get("sha256") != digest:
                winner["sha256"] = digest
                dirty = True
        if dirty and _write_if_changed(path, payload):
            changed.append(path)
    return changed
