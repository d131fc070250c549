"""Installing and verifying released kernel packs.

Release format shared with the reference, so a release published for one installs with the
other (reference: src/radeon_kernels/runtime/installer.py; ``verify_installed_pack`` at
:251-285):

* a **release archive** ``<pack_id>-<pack_version>.tar.gz`` holds exactly
  ``<pack_id>/manifest.json``, ``<pack_id>/manifest.sig.json`` (a detached Ed25519 signature
  of the manifest, ``radeon_kernels.runtime.signing``) and every artifact the manifest lists
  under ``<pack_id>/``;
* a **pack index** ``{"schema_version": "1.0", "packs": [record, ...]}`` (published signed,
  ``pack-index/<operator>-<version>.json`` + ``.sig.json``) describes each release: pack id
  and version, environment constraint, manifest digest and signature, archive name, digest
  and size, the artifact list and the approval id.

Installation checks, in order: the index record for this machine's fingerprint, the
archive's size and SHA-256 against the record, every archive member's path (relative, no
``..``, inside ``<pack_id>/``, regular files only, exactly the expected set), then after
extraction into a staging directory the manifest signature against the trusted keyring, the
artifacts' digests, and the installed manifest, signature, identity, environment and
artifact list against the record.  Only then is the staging directory moved into place.
"""

from __future__ import annotations

import hmac
import json
import os
import shutil
import tarfile
import tempfile
from dataclasses import dataclass
from pathlib import Path, PurePosixPath
from typing import Any, Mapping

from radeon_kernels.errors import ConfigError, RadeonKernelsError
from radeon_kernels.runtime.compatibility import EnvironmentConstraint
from radeon_kernels.runtime.fingerprint import EnvironmentFingerprint
from radeon_kernels.runtime.pack import KernelPack, KernelPackArtifact
from radeon_kernels.runtime.signing import (
    DetachedSignature,
    TrustedKeyring,
    builtin_trusted_keyring,
    sha256_file,
    verify_detached_file,
)

MAX_MEMBERS = 256
_RECORD_FIELDS = frozenset(
    {"pack_id", "pack_version", "environment", "manifest_sha256", "manifest_signature", "release_file",
     "release_sha256", "release_size", "artifacts", "approval_id"}
)


class PackInstallError(RadeonKernelsError):
    """A release or an installed pack failed a check; nothing was installed."""


def _text(value: Any, where: str) -> str:
    if not isinstance(value, str) or not value:
        raise ConfigError(where, "expected non-empty text")
    return value


def _sha(value: Any, where: str) -> str:
    text = _text(value, where)
    if len(text) != 64 or text.strip("0123456789abcdef"):
        raise ConfigError(where, "expected a lowercase SHA-256")
    return text


@dataclass(frozen=True)
class IndexedPack:
    """One release as a pack index describes it."""

    pack_id: str
    pack_version: str
    environment: EnvironmentConstraint
    manifest_sha256: str
    manifest_signature: DetachedSignature
    release_file: str
    release_sha256: str
    release_size: int
    artifacts: tuple[KernelPackArtifact, ...]
    approval_id: str

    @classmethod
    def from_mapping(cls, value: Any, path: str) -> IndexedPack:
        if not isinstance(value, Mapping):
            raise ConfigError(path, "expected a mapping")
        extra, absent = set(value) - _RECORD_FIELDS, _RECORD_FIELDS - set(value)
        if extra or absent:
            raise ConfigError(path, f"unknown={sorted(extra)}, missing={sorted(absent)}")
        size = value["release_size"]
        if isinstance(size, bool) or not isinstance(size, int) or size < 1:
            raise ConfigError(f"{path}.release_size", "expected a positive integer")
        name = _text(value["release_file"], f"{path}.release_file")
        if PurePosixPath(name).name != name or not name.endswith(".tar.gz"):
            raise ConfigError(f"{path}.release_file", "expected a .tar.gz filename")
        items = value["artifacts"]
        if not isinstance(items, list) or not items:
            raise ConfigError(f"{path}.artifacts", "expected a non-empty list")
        manifest_sha256 = _sha(value["manifest_sha256"], f"{path}.manifest_sha256")
        signature = DetachedSignature.from_mapping(value["manifest_signature"], f"{path}.manifest_signature")
        if (signature.signed_file, signature.signed_sha256) != ("manifest.json", manifest_sha256):
            raise ConfigError(f"{path}.manifest_signature", "must sign the indexed manifest SHA-256")
        return cls(
            pack_id=_text(value["pack_id"], f"{path}.pack_id"),
            pack_version=_text(value["pack_version"], f"{path}.pack_version"),
            environment=EnvironmentConstraint.from_mapping(value["environment"], f"{path}.environment"),
            manifest_sha256=manifest_sha256,
            manifest_signature=signature,
            release_file=name,
            release_sha256=_sha(value["release_sha256"], f"{path}.release_sha256"),
            release_size=size,
            artifacts=tuple(KernelPackArtifact.from_mapping(item, f"{path}.artifacts[{i}]") for i, item in enumerate(items)),
            approval_id=_text(value["approval_id"], f"{path}.approval_id"),
        )

    def expected_members(self) -> set[str]:
        root = self.pack_id
        return {f"{root}/manifest.json", f"{root}/manifest.sig.json",
                *(f"{root}/{item.artifact.artifact}" for item in self.artifacts)}


def index_records(index: Mapping[str, Any], *, path: str = "pack-index") -> tuple[IndexedPack, ...]:
    if index.get("schema_version") != "1.0":
        raise ConfigError(f"{path}.schema_version", "unsupported version")
    packs = index.get("packs")
    if not isinstance(packs, list):
        raise ConfigError(f"{path}.packs", "expected a list")
    return tuple(IndexedPack.from_mapping(item, f"{path}.packs[{i}]") for i, item in enumerate(packs))


def compatible_records(index: Mapping[str, Any], fingerprint: EnvironmentFingerprint) -> tuple[IndexedPack, ...]:
    return tuple(record for record in index_records(index) if record.environment.matches(fingerprint))


def select_record(index: Mapping[str, Any], fingerprint: EnvironmentFingerprint, release_file: str | None = None) -> IndexedPack:
    """The one indexed release for this machine (optionally the named one)."""

    candidates = [r for r in compatible_records(index, fingerprint) if release_file in (None, r.release_file)]
    if len(candidates) == 1:
        return candidates[0]
    if not candidates:
        named = f" and release {release_file!r}" if release_file else ""
        raise PackInstallError(
            f"no indexed pack matches {fingerprint.architecture}, toolkit ABI {fingerprint.rocm_abi}{named}"
        )
    raise PackInstallError("multiple compatible packs found; select one of: " + ", ".join(r.release_file for r in candidates))


def _check_archive(archive: Path, record: IndexedPack) -> None:
    try:
        size = archive.stat().st_size
    except OSError as error:
        raise PackInstallError(f"cannot read release archive {archive}: {error}") from error
    if size != record.release_size:
        raise PackInstallError(f"release size mismatch: expected {record.release_size}, got {size}")
    digest = sha256_file(archive)
    if not hmac.compare_digest(digest, record.release_sha256):
        raise PackInstallError(f"release SHA-256 mismatch: expected {record.release_sha256}, got {digest}")


def _member_path(member: tarfile.TarInfo, pack_id: str) -> PurePosixPath:
    name = member.name.rstrip("/")
    posix = PurePosixPath(name)
    if not name or posix.is_absolute() or ".." in posix.parts or posix.as_posix() != name:
        raise PackInstallError(f"release contains unsafe path {member.name!r}")
    if posix.parts[0] != pack_id:
        raise PackInstallError("release root does not match the indexed pack id")
    return posix


def _extract(archive: Path, staging: Path, record: IndexedPack) -> Path:
    try:
        tar = tarfile.open(archive, "r:gz")
    except (OSError, tarfile.TarError) as error:
        raise PackInstallError(f"cannot open release archive {archive}: {error}") from error
    with tar:
        members = tar.getmembers()
        if len(members) > MAX_MEMBERS:
            raise PackInstallError("release contains too many archive members")
        files: dict[str, tarfile.TarInfo] = {}
        seen: set[str] = set()
        for member in members:
            path = _member_path(member, record.pack_id).as_posix()
            if path in seen:
                raise PackInstallError(f"release contains duplicate path {path!r}")
            seen.add(path)
            if member.isfile():
                files[path] = member
            elif not member.isdir():
                raise PackInstallError(f"release contains unsupported member {path!r}")
        expected = record.expected_members()
        if set(files) != expected:
            raise PackInstallError(
                f"release payload differs from index: missing={sorted(expected - set(files))}, "
                f"unexpected={sorted(set(files) - expected)}"
            )
        for path, member in sorted(files.items()):
            target = staging.joinpath(*PurePosixPath(path).parts)
            target.parent.mkdir(parents=True, exist_ok=True)
            source = tar.extractfile(member)
            if source is None:
                raise PackInstallError(f"cannot read release member {path!r}")
            with source, target.open("xb") as sink:
                shutil.copyfileobj(source, sink, length=1 << 20)
            os.chmod(target, 0o755 if target.suffix in {".so", ".hsaco", ".cubin"} else 0o644)
    return staging / record.pack_id


def _identity(item: KernelPackArtifact) -> tuple[Any, ...]:
    spec = item.artifact
    return (item.operator, item.semantic_version, spec.provider, spec.artifact, spec.entrypoint, spec.sha256,
            spec.format, item.evidence_id)


def verify_installed_pack(
    pack_root: Path, *, trusted_keys: TrustedKeyring | None = None, record: IndexedPack | None = None
) -> KernelPack:
    """Signed manifest + artifact digests of an installed pack, and (with ``record``) its
    agreement with the signed index record."""

    keyring = trusted_keys or builtin_trusted_keyring()
    root = Path(pack_root)
    verify_detached_file(root / "manifest.json", root / "manifest.sig.json", keyring, signed_file="manifest.json")
    pack = KernelPack.from_directory(root, verify_artifacts=True)
    if record is None:
        return pack
    checks = (
        (hmac.compare_digest(sha256_file(pack.root / "manifest.json"), record.manifest_sha256),
         "installed manifest does not match the signed pack index"),
        (DetachedSignature.from_file(pack.root / "manifest.sig.json") == record.manifest_signature,
         "manifest signature does not match the signed pack index"),
        ((pack.pack_id, pack.pack_version) == (record.pack_id, record.pack_version),
         "installed pack identity does not match the signed pack index"),
        (pack.environment == record.environment, "installed pack environment does not match the signed pack index"),
        ([_identity(a) for a in pack.artifacts] == [_identity(a) for a in record.artifacts],
         "installed artifacts do not match the signed pack index"),
    )
    for ok, message in checks:
        if not ok:
            raise PackInstallError(message)
    return pack


def install_release(
    archive: Path,
    index: Mapping[str, Any],
    fingerprint: EnvironmentFingerprint,
    destination_root: Path,
    *,
    trusted_keys: TrustedKeyring | None = None,
    release_file: str | None = None,
) -> KernelPack:
    """Verifies ``archive`` against ``index`` and installs it as ``destination_root/<pack_id>``.

    An existing installation of the same pack id is replaced only after the new one verified.
    """

    record = select_record(index, fingerprint, release_file)
    archive = Path(archive)
    _check_archive(archive, record)
    destination_root = Path(destination_root)
    destination_root.mkdir(parents=True, exist_ok=True)
    final = destination_root / record.pack_id
    with tempfile.TemporaryDirectory(prefix=".rk-install-", dir=destination_root) as scratch:
        staged = _extract(archive, Path(scratch), record)
        verify_installed_pack(staged, trusted_keys=trusted_keys, record=record)
        if final.exists():
            shutil.rmtree(final)
        staged.rename(final)
    return verify_installed_pack(final, trusted_keys=trusted_keys, record=record)


def load_index(path: Path, *, trusted_keys: TrustedKeyring | None = None) -> dict[str, Any]:
    """Reads a pack index after verifying its detached signature (``<index>.sig.json``)."""

    path = Path(path)
    verify_detached_file(path, path.with_name(path.name[: -len(".json")] + ".sig.json"),
                         trusted_keys or builtin_trusted_keyring(), signed_file=path.name)
    return json.loads(path.read_text(encoding="utf-8"))


__all__ = [
    "IndexedPack",
    "PackInstallError",
    "compatible_records",
    "index_records",
    "install_release",
    "load_index",
    "select_record",
    "verify_installed_pack",
]
