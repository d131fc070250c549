"""Ed25519 detached signatures over release files (kernel-pack manifests).

Wire-compatible with the reference (src/radeon_kernels/runtime/signing.py:22-279): a
signature document ``{schema_version, algorithm: "ed25519", key_id, signed_file,
signed_sha256, signature}`` signs the byte string
``b"radeon-kernels-ed25519-v1\\0" + signed_file + b"\\0" + sha256_hex``, and a keyring
``{schema_version, keys: [{key_id, algorithm, public_key, status, created_at[, reason]}]}``
lists the trusted public keys (only ``active`` keys verify).  Packs signed for the
reference therefore verify here with the same keyring, and packs this build signs verify
in the reference.
"""

from __future__ import annotations

import base64
import binascii
import hashlib
import hmac
import json
import re
from dataclasses import dataclass
from pathlib import Path, PurePosixPath
from typing import Any, Mapping, Sequence

from radeon_kernels.errors import ConfigError, RadeonKernelsError

_ID_RE = re.compile(r"^[a-z][a-z0-9_.-]*$")
_SHA_RE = re.compile(r"^[0-9a-f]{64}$")
DOMAIN = b"radeon-kernels-ed25519-v1\x00"
_SIGNATURE_FIELDS = frozenset({"schema_version", "algorithm", "key_id", "signed_file", "signed_sha256", "signature"})
_KEY_FIELDS = frozenset({"key_id", "algorithm", "public_key", "status", "created_at", "reason"})


class SignatureVerificationError(RadeonKernelsError):
    """A signature is missing, malformed, made with an untrusted key or does not verify."""


def _b64(value: Any, path: str, size: int) -> bytes:
    if not isinstance(value, str):
        raise ConfigError(path, "expected base64 text")
    try:
        raw = base64.b64decode(value, validate=True)
    except (ValueError, binascii.Error) as error:
        raise ConfigError(path, "invalid base64 text") from error
    if len(raw) != size:
        raise ConfigError(path, f"expected {size} decoded bytes")
    return raw


def _key_id(value: Any, path: str) -> str:
    if not isinstance(value, str) or _ID_RE.fullmatch(value) is None:
        raise ConfigError(path, "expected a lowercase identifier")
    return value


def _relative(value: Any, path: str) -> str:
    if not isinstance(value, str) or not value:
        raise ConfigError(path, "expected a relative file path")
    posix = PurePosixPath(value)
    if posix.is_absolute() or ".." in posix.parts or posix.as_posix() != value:
        raise ConfigError(path, "expected a normalized relative file path")
    return value


def signature_payload(signed_file: str, signed_sha256: str) -> bytes:
    name = _relative(signed_file, "signature.signed_file")
    if not isinstance(signed_sha256, str) or _SHA_RE.fullmatch(signed_sha256) is None:
        raise ConfigError("signature.signed_sha256", "expected a lowercase SHA-256")
    return DOMAIN + name.encode("utf-8") + b"\x00" + signed_sha256.encode("ascii")


@dataclass(frozen=True)
class TrustedKey:
    key_id: str
    public_key: bytes
    status: str
    created_at: str
    reason: str | None = None


class TrustedKeyring:
    def __init__(self, keys: Sequence[TrustedKey]) -> None:
        if not keys:
            raise ConfigError("trusted-keys.keys", "expected at least one key")
        self._keys = {key.key_id: key for key in keys}
        if len(self._keys) != len(keys):
            raise ConfigError("trusted-keys.keys", "key ids must be unique")

    @classmethod
    def from_mapping(cls, value: Any, path: str = "trusted-keys") -> TrustedKeyring:
        if not isinstance(value, Mapping):
            raise ConfigError(path, "expected a mapping")
        if set(value) != {"schema_version", "keys"}:
            raise ConfigError(path, "expected exactly ['keys', 'schema_version']")
        if value["schema_version"] != "1.0":
            raise ConfigError(f"{path}.schema_version", "unsupported version")
        if not isinstance(value["keys"], list):
            raise ConfigError(f"{path}.keys", "expected a list")
        keys = []
        for index, item in enumerate(value["keys"]):
            where = f"{path}.keys[{index}]"
            if not isinstance(item, Mapping):
                raise ConfigError(where, "expected a mapping")
            unknown, missing = set(item) - _KEY_FIELDS, (_KEY_FIELDS - {"reason"}) - set(item)
            if unknown or missing:
                raise ConfigError(where, f"unknown={sorted(unknown)}, missing={sorted(missing)}")
            if item["algorithm"] != "ed25519":
                raise ConfigError(f"{where}.algorithm", "expected ed25519")
            if item["status"] not in ("active", "revoked"):
                raise ConfigError(f"{where}.status", "expected active or revoked")
            if not isinstance(item["created_at"], str) or not item["created_at"]:
                raise ConfigError(f"{where}.created_at", "expected a timestamp")
            reason = item.get("reason")
            if reason is not None and (not isinstance(reason, str) or not reason):
                raise ConfigError(f"{where}.reason", "expected non-empty text")
            keys.append(
                TrustedKey(
                    key_id=_key_id(item["key_id"], f"{where}.key_id"),
                    public_key=_b64(item["public_key"], f"{where}.public_key", 32),
                    status=item["status"],
                    created_at=item["created_at"],
                    reason=reason,
                )
            )
        return cls(keys)

    @classmethod
    def from_file(cls, path: Path) -> TrustedKeyring:
        try:
            value = json.loads(Path(path).read_text(encoding="utf-8"))
        except (OSError, json.JSONDecodeError) as error:
            raise ConfigError(str(path), f"cannot read trusted keys: {error}") from error
        return cls.from_mapping(value, str(path))

    def active_public_key(self, key_id: str) -> Any:
        from cryptography.hazmat.primitives.asymmetric.ed25519 import Ed25519PublicKey

        key = self._keys.get(key_id)
        if key is None:
            raise SignatureVerificationError(f"signature uses unknown key {key_id!r}")
        if key.status != "active":
            raise SignatureVerificationError(f"signature key {key_id!r} is not active")
        return Ed25519PublicKey.from_public_bytes(key.public_key)


@dataclass(frozen=True)
class DetachedSignature:
    key_id: str
    signed_file: str
    signed_sha256: str
    signature: bytes

    @classmethod
    def from_mapping(cls, value: Any, path: str = "signature") -> DetachedSignature:
        if not isinstance(value, Mapping):
            raise ConfigError(path, "expected a mapping")
        if set(value) != _SIGNATURE_FIELDS:
            raise ConfigError(path, f"expected exactly {sorted(_SIGNATURE_FIELDS)}")
        if value["schema_version"] != "1.0" or value["algorithm"] != "ed25519":
            raise ConfigError(path, "unsupported signature version or algorithm")
        digest = value["signed_sha256"]
        if not isinstance(digest, str) or _SHA_RE.fullmatch(digest) is None:
            raise ConfigError(f"{path}.signed_sha256", "expected a lowercase SHA-256")
        return cls(
            key_id=_key_id(value["key_id"], f"{path}.key_id"),
            signed_file=_relative(value["signed_file"], f"{path}.signed_file"),
            signed_sha256=digest,
            signature=_b64(value["signature"], f"{path}.signature", 64),
        )

    @classmethod
    def from_file(cls, path: Path) -> DetachedSignature:
        try:
            value = json.loads(Path(path).read_text(encoding="utf-8"))
        except (OSError, json.JSONDecodeError) as error:
            raise SignatureVerificationError(f"cannot read detached signature {path}: {error}") from error
        try:
            return cls.from_mapping(value, str(path))
        except ConfigError as error:
            raise SignatureVerificationError(str(error)) from error


def signature_document(*, private_key: Any, key_id: str, signed_file: str, signed_sha256: str) -> dict[str, str]:
    """Sign ``signed_file`` (by its digest) with an Ed25519 private key."""

    signature = private_key.sign(signature_payload(signed_file, signed_sha256))
    return {
        "schema_version": "1.0",
        "algorithm": "ed25519",
        "key_id": _key_id(key_id, "signature.key_id"),
        "signed_file": signed_file,
        "signed_sha256": signed_sha256,
        "signature": base64.b64encode(signature).decode("ascii"),
    }


def verify_detached_content(
    content: bytes,
    signature: DetachedSignature | Mapping[str, Any],
    keyring: TrustedKeyring,
    *,
    signed_file: str,
) -> DetachedSignature:
    from cryptography.exceptions import InvalidSignature

    envelope = signature if isinstance(signature, DetachedSignature) else DetachedSignature.from_mapping(signature)
    expected = _relative(signed_file, "signed_file")
    if envelope.signed_file != expected:
        raise SignatureVerificationError(f"signature names {envelope.signed_file!r}, expected {expected!r}")
    actual = hashlib.sha256(content).hexdigest()
    if not hmac.compare_digest(actual, envelope.signed_sha256):
        raise SignatureVerificationError(
            f"signed file SHA-256 mismatch: expected {envelope.signed_sha256}, got {actual}"
        )
    key = keyring.active_public_key(envelope.key_id)
    try:
        key.verify(envelope.signature, signature_payload(envelope.signed_file, envelope.signed_sha256))
    except InvalidSignature as error:
        raise SignatureVerificationError("invalid Ed25519 signature") from error
    return envelope


def verify_detached_file(
    file_path: Path, signature_path: Path, keyring: TrustedKeyring, *, signed_file: str | None = None
) -> DetachedSignature:
    try:
        content = Path(file_path).read_bytes()
    except OSError as error:
        raise SignatureVerificationError(f"cannot read signed file {file_path}: {error}") from error
    return verify_detached_content(
        content, DetachedSignature.from_file(signature_path), keyring, signed_file=signed_file or Path(file_path).name
    )


def builtin_trusted_keyring() -> TrustedKeyring:
    """Release keys shipped with the package (``radeon_kernels/keys/trusted-keys.json``)."""

    return TrustedKeyring.from_file(Path(__file__).resolve().parents[1] / "keys" / "trusted-keys.json")
