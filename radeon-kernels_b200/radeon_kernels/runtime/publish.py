"""Publication of the built-in sm_100a kernel pack (build-time helper).

The build compiles the pack's ``python_extension`` artifact; this module then

* writes the pack's ``manifest.json`` (artifact digests, environment of the build) and
  refreshes the ``sha256`` of every dispatch entry whose winner is that artifact, so
  dispatch and pack stay consistent (the build links reproducibly, so the digests change
  only when the sources or the toolchain do);
* signs the manifest (``manifest.sig.json``, Ed25519) when a release private key is
  available -- the public half is in ``radeon_kernels/keys/trusted-keys.json``, the private
  half never enters the source tree -- and removes a signature the manifest no longer
  matches;
* on request (``make_release`` / ``write_index``) packs the signed pack into a release
  archive plus a signed pack-index record in the reference's release format, which
  ``radeon_kernels.runtime.installer`` (and the reference's installer) install and verify.

It plays the role of the reference's developer-side publish step
(developer/promotion/publish_approved.py) without the approval workflow.  Files are
rewritten only when their content changes.
"""

from __future__ import annotations

import gzip
import io
import json
import sys
import tarfile
from pathlib import Path
from typing import Any

from radeon_kernels.runtime.loader import sha256_of
from radeon_kernels.runtime.resources import DISPATCH_DIR
from radeon_kernels.runtime.signing import sign, verify_detached_file

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


def load_private_key(path: Path) -> tuple[Any, str]:
    """(Ed25519 private key, key id) from a PEM file named ``<key_id>.pem``."""

    from cryptography.hazmat.primitives import serialization

    key = serialization.load_pem_private_key(Path(path).read_bytes(), password=None)
    return key, Path(path).stem


def sign_manifest(pack_dir: Path, private_key: Any | None, key_id: str | None, keyring: Any | None = None) -> bool:
    """Writes ``manifest.sig.json`` for the current manifest (returns True), or -- without a
    key -- removes a signature that no longer verifies against ``keyring`` (returns False)."""

    manifest = Path(pack_dir) / "manifest.json"
    target = Path(pack_dir) / "manifest.sig.json"
    if private_key is not None and key_id is not None:
        envelope = sign(private_key, key_id, "manifest.json", manifest.read_bytes())
        _write_if_changed(target, envelope.to_dict())
        return True
    if target.exists() and keyring is not None:
        try:
            verify_detached_file(manifest, target, keyring, signed_file="manifest.json")
        except Exception:  # noqa: BLE001 -- any failure: the signature is stale
            target.unlink()
    return False


def _tar_member(tar: tarfile.TarFile, name: str, data: bytes | None, mode: int) -> None:
    info = tarfile.TarInfo(name)
    info.mtime, info.uid, info.gid, info.uname, info.gname = 0, 0, 0, "", ""
    if data is None:
        info.type, info.mode = tarfile.DIRTYPE, 0o755
        tar.addfile(info)
    else:
        info.size, info.mode = len(data), mode
        tar.addfile(info, io.BytesIO(data))


def make_release(pack_dir: Path, out_dir: Path, *, approval_id: str, compresslevel: int = 6) -> dict[str, Any]:
    """Packs a signed pack directory into ``<pack_id>-<version>.tar.gz`` under ``out_dir``
    (byte-reproducible: sorted members, zero times and owners) and returns its index record."""

    pack_dir = Path(pack_dir)
    manifest_bytes = (pack_dir / "manifest.json").read_bytes()
    manifest = json.loads(manifest_bytes)
    signature = json.loads((pack_dir / "manifest.sig.json").read_text(encoding="utf-8"))
    pack_id, version = manifest["pack_id"], manifest["pack_version"]
    files = {"manifest.json": manifest_bytes, "manifest.sig.json": (pack_dir / "manifest.sig.json").read_bytes()}
    for item in manifest["artifacts"]:
        files[item["artifact"]] = (pack_dir / item["artifact"]).read_bytes()
    dirs = sorted({str(Path(name).parent) for name in files if str(Path(name).parent) != "."})
    raw = io.BytesIO()
    with tarfile.open(fileobj=raw, mode="w", format=tarfile.PAX_FORMAT) as tar:
        _tar_member(tar, pack_id, None, 0)
        for directory in dirs:
            _tar_member(tar, f"{pack_id}/{directory}", None, 0)
        for name in sorted(files):
            _tar_member(tar, f"{pack_id}/{name}", files[name], 0o755 if name.endswith(".so") else 0o644)
    out_dir = Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    release = out_dir / f"{pack_id}-{version}.tar.gz"
    with release.open("wb") as handle, gzip.GzipFile(filename="", mode="wb", fileobj=handle, mtime=0,
                                                     compresslevel=compresslevel) as zipped:
        zipped.write(raw.getvalue())
    return {
        "pack_id": pack_id,
        "pack_version": version,
        "environment": manifest["environment"],
        "manifest_sha256": sha256_of(pack_dir / "manifest.json"),
        "manifest_signature": signature,
        "release_file": release.name,
        "release_sha256": sha256_of(release),
        "release_size": release.stat().st_size,
        "artifacts": manifest["artifacts"],
        "approval_id": approval_id,
    }


def write_index(records: list[dict[str, Any]], path: Path, private_key: Any, key_id: str) -> Path:
    """Writes a pack index ``path`` and its detached signature ``<stem>.sig.json``."""

    path = Path(path)
    index = {"schema_version": "1.0", "packs": records}
    _write_if_changed(path, index)
    envelope = sign(private_key, key_id, path.name, path.read_bytes())
    _write_if_changed(path.with_name(path.name[: -len(".json")] + ".sig.json"), envelope.to_dict())
    return path


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
