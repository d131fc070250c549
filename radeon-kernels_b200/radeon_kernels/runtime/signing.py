"""Ed25519 detached signatures over release files (pack manifests, pack indexes).

Format (shared with the reference so packs and keyrings move between the two,
src/radeon_kernels/runtime/signing.py:22-279):

* a signature document is a JSON object with exactly ``schema_version`` ("1.0"),
  ``algorithm`` ("ed25519"), ``key_id``, ``signed_file`` (a normalized relative path),
  ``signed_sha256`` (lowercase hex) and ``signature`` (base64 of 64 bytes);
* the signed message is ``b"radeon-kernels-ed25519-v1\\0" + signed_file + b"\\0" +
  signed_sha256`` -- the file is bound by name and digest, not by its bytes;
* a keyring is ``{"schema_version": "1.0", "keys": [...]}`` whose entries carry ``key_id``,
  ``algorithm`` ("ed25519"), ``public_key`` (base64 of 32 bytes), ``status`` ("active" or
  "revoked"), ``created_at`` and an optional ``reason``; only active keys verify.

The implementation here is organised around one small schema checker (``_check``) used
by both documents, an immutable :class:`DetachedSignature` that knows its own message
(:meth:`DetachedSignature.message`), and a :class:`TrustedKeyring` that maps key ids to
verifier objects.
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

MESSAGE_PREFIX = b"radeon-kernels-ed25519-v1\x00"
DOMAIN = MESSAGE_PREFIX  # name kept for callers of the first release of this module
_HEX64 = re.compile(r"[0-9a-f]{64}")
_IDENT = re.compile(r"[a-z][a-z0-9_.-]*")


class SignatureVerificationError(RadeonKernelsError):
    """A signature is missing, malformed, made with an untrusted key or does not verify."""


# ----------------------------------------------------------------------------- checks
def _check(value: Any, where: str, required: frozenset[str], optional: frozenset[str] = frozenset()) -> Mapping[str, Any]:
    """``value`` must be a mapping with all of ``required`` and nothing beyond ``optional``."""

    if not isinstance(value, Mapping):
        raise ConfigError(where, "expected a mapping")
    keys = set(value)
    missing, unknown = required - keys, keys - required - optional
    if missing or unknown:
        raise ConfigError(where, f"unknown={sorted(unknown)}, missing={sorted(missing)}")
    return value


def _text(value: Any, where: str, pattern: re.Pattern[str] | None = None, what: str = "non-empty text") -> str:
    if not isinstance(value, str) or not value or (pattern is not None and pattern.fullmatch(value) is None):
        raise ConfigError(where, f"expected {what}")
    return value


def _decoded(value: Any, where: str, size: int) -> bytes:
    try:
        raw = base64.b64decode(_text(value, where, what="base64 text"), validate=True)
    except (ValueError, binascii.Error) as error:
        raise ConfigError(where, "invalid base64 text") from error
    if len(raw) != size:
        raise ConfigError(where, f"expected {size} decoded bytes")
    return raw


def _release_path(value: Any, where: str) -> str:
    text = _text(value, where, what="a relative file path")
    posix = PurePosixPath(text)
    if posix.is_absolute() or ".." in posix.parts or posix.as_posix() != text:
        raise ConfigError(where, "expected a normalized relative file path")
    return text


def _digest(value: Any, where: str) -> str:
    return _text(value, where, _HEX64, "a lowercase SHA-256")


def signature_payload(signed_file: str, signed_sha256: str) -> bytes:
    """The bytes an Ed25519 key signs for ``signed_file`` with digest ``signed_sha256``."""

    name = _release_path(signed_file, "signature.signed_file")
    return MESSAGE_PREFIX + name.encode("utf-8") + b"\x00" + _digest(signed_sha256, "signature.signed_sha256").encode("ascii")


# ----------------------------------------------------------------------------- keyring
@dataclass(frozen=True)
class TrustedKey:
    key_id: str
    public_key: bytes
    status: str
    created_at: str
    reason: str | None = None


class TrustedKeyring:
    """Public keys a signature may be made with, by key id."""

    _DOC = frozenset({"schema_version", "keys"})
    _ENTRY = frozenset({"key_id", "algorithm", "public_key", "status", "created_at"})

    def __init__(self, keys: Sequence[TrustedKey]) -> None:
        by_id = {key.key_id: key for key in keys}
        if not keys:
            raise ConfigError("trusted-keys.keys", "expected at least one key")
        if len(by_id) != len(keys):
            raise ConfigError("trusted-keys.keys", "key ids must be unique")
        self._by_id = by_id

    @classmethod
    def from_mapping(cls, value: Any, path: str = "trusted-keys") -> TrustedKeyring:
        doc = _check(value, path, cls._DOC)
        if doc["schema_version"] != "1.0":
            raise ConfigError(f"{path}.schema_version", "unsupported version")
        if not isinstance(doc["keys"], list):
            raise ConfigError(f"{path}.keys", "expected a list")
        keys = [cls._entry(item, f"{path}.keys[{i}]") for i, item in enumerate(doc["keys"])]
        return cls(keys)

    @classmethod
    def _entry(cls, value: Any, where: str) -> TrustedKey:
        item = _check(value, where, cls._ENTRY, frozenset({"reason"}))
        if item["algorithm"] != "ed25519":
            raise ConfigError(f"{where}.algorithm", "expected ed25519")
        if item["status"] not in ("active", "revoked"):
            raise ConfigError(f"{where}.status", "expected active or revoked")
        reason = item.get("reason")
        return TrustedKey(
            key_id=_text(item["key_id"], f"{where}.key_id", _IDENT, "a lowercase identifier"),
            public_key=_decoded(item["public_key"], f"{where}.public_key", 32),
            status=item["status"],
            created_at=_text(item["created_at"], f"{where}.created_at", what="a timestamp"),
            reason=None if reason is None else _text(reason, f"{where}.reason"),
        )

    @classmethod
    def from_file(cls, path: Path) -> TrustedKeyring:
        try:
            value = json.loads(Path(path).read_text(encoding="utf-8"))
        except (OSError, json.JSONDecodeError) as error:
            raise ConfigError(str(path), f"cannot read trusted keys: {error}") from error
        return cls.from_mapping(value, str(path))

    def active_public_key(self, key_id: str) -> Any:
        """The ``cryptography`` public-key object of an active key; raises for unknown or
        revoked keys."""

        key = self._by_id.get(key_id)
        if key is None:
            raise SignatureVerificationError(f"signature uses unknown key {key_id!r}")
        if key.status != "active":
            raise SignatureVerificationError(f"signature key {key_id!r} is not active")
        from cryptography.hazmat.primitives.asymmetric.ed25519 import Ed25519PublicKey

        return Ed25519PublicKey.from_public_bytes(key.public_key)


# --------------------------------------------------------------------------- envelope
@dataclass(frozen=True)
class DetachedSignature:
    key_id: str
    signed_file: str
    signed_sha256: str
    signature: bytes

    _FIELDS = frozenset({"schema_version", "algorithm", "key_id", "signed_file", "signed_sha256", "signature"})

    @classmethod
    def from_mapping(cls, value: Any, path: str = "signature") -> DetachedSignature:
        doc = _check(value, path, cls._FIELDS)
        if (doc["schema_version"], doc["algorithm"]) != ("1.0", "ed25519"):
            raise ConfigError(path, "unsupported signature version or algorithm")
        return cls(
            key_id=_text(doc["key_id"], f"{path}.key_id", _IDENT, "a lowercase identifier"),
            signed_file=_release_path(doc["signed_file"], f"{path}.signed_file"),
            signed_sha256=_digest(doc["signed_sha256"], f"{path}.signed_sha256"),
            signature=_decoded(doc["signature"], f"{path}.signature", 64),
        )

    @classmethod
    def from_file(cls, path: Path) -> DetachedSignature:
        try:
            return cls.from_mapping(json.loads(Path(path).read_text(encoding="utf-8")), str(path))
        except (OSError, json.JSONDecodeError) as error:
            raise SignatureVerificationError(f"cannot read detached signature {path}: {error}") from error
        except ConfigError as error:
            raise SignatureVerificationError(str(error)) from error

    def message(self) -> bytes:
        return signature_payload(self.signed_file, self.signed_sha256)

    def to_dict(self) -> dict[str, str]:
        return {
            "schema_version": "1.0",
            "algorithm": "ed25519",
            "key_id": self.key_id,
            "signed_file": self.signed_file,
            "signed_sha256": self.signed_sha256,
            "signature": base64.b64encode(self.signature).decode("ascii"),
        }

    def check(self, content: bytes, keyring: TrustedKeyring, expected_file: str) -> None:
        """Raises SignatureVerificationError unless this signs ``content`` as ``expected_file``."""

        expected = _release_path(expected_file, "signed_file")
        if self.signed_file != expected:
            raise SignatureVerificationError(f"signature names {self.signed_file!r}, expected {expected!r}")
        actual = hashlib.sha256(content).hexdigest()
        if not hmac.compare_digest(actual, self.signed_sha256):
            raise SignatureVerificationError(f"signed file SHA-256 mismatch: expected {self.signed_sha256}, got {actual}")
        from cryptography.exceptions import InvalidSignature

        try:
            keyring.active_public_key(self.key_id).verify(self.signature, self.message())
        except InvalidSignature as error:
            raise SignatureVerificationError("invalid Ed25519 signature") from error


def sign(private_key: Any, key_id: str, signed_file: str, content: bytes) -> DetachedSignature:
    """Signs ``content`` under the name ``signed_file`` with an Ed25519 private key."""

    return DetachedSignature.from_mapping(
        signature_document(private_key=private_key, key_id=key_id, signed_file=signed_file,
                           signed_sha256=hashlib.sha256(content).hexdigest())
    )


def signature_document(*, private_key: Any, key_id: str, signed_file: str, signed_sha256: str) -> dict[str, str]:
    """Signature document for a file known by its name and digest."""

    name = _release_path(signed_file, "signature.signed_file")
    digest = _digest(signed_sha256, "signature.signed_sha256")
    ident = _text(key_id, "signature.key_id", _IDENT, "a lowercase identifier")
    return DetachedSignature(ident, name, digest, private_key.sign(signature_payload(name, digest))).to_dict()


def verify_detached_content(
    content: bytes,
    signature: DetachedSignature | Mapping[str, Any],
    keyring: TrustedKeyring,
    *,
    signed_file: str,
) -> DetachedSignature:
    envelope = signature if isinstance(signature, DetachedSignature) else DetachedSignature.from_mapping(signature)
    envelope.check(content, keyring, signed_file)
    return envelope


def verify_detached_file(
    file_path: Path, signature_path: Path, keyring: TrustedKeyring, *, signed_file: str | None = None
) -> DetachedSignature:
    try:
        content = Path(file_path).read_bytes()
    except OSError as error:
        raise SignatureVerificationError(f"cannot read signed file {file_path}: {error}") from error
    envelope = DetachedSignature.from_file(signature_path)
    envelope.check(content, keyring, signed_file or Path(file_path).name)
    return envelope


def builtin_trusted_keyring() -> TrustedKeyring:
    """Release keys shipped with the package (``radeon_kernels/keys/trusted-keys.json``)."""

    return TrustedKeyring.from_file(Path(__file__).resolve().parents[1] / "keys" / "trusted-keys.json")


def sha256_file(path: Path) -> str:
    digest = hashlib.sha256()
    with Path(path).open("rb") as handle:
        for block in iter(lambda: handle.read(1 << 20), b""):
            digest.update(block)
    return digest.hexdigest()
