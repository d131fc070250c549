"""Pack discovery with Ed25519 signatures, and the built-in sm_100a pack (CPU)."""

from __future__ import annotations

import base64
import json

import pytest

from fakes import ENV, digest_of, fingerprint, write_pack
from radeon_kernels.runtime.loader import sha256_of
from radeon_kernels.runtime.packs import BUILTIN_PACK_ROOT, KernelPackRegistry, PackResolutionError
from radeon_kernels.runtime.registry import ArtifactSpec
from radeon_kernels.runtime.resources import builtin_dispatch_registry
from radeon_kernels.runtime.signing import (
    SignatureVerificationError,
    TrustedKeyring,
    builtin_trusted_keyring,
    signature_document,
    verify_detached_content,
)

ed25519 = pytest.importorskip("cryptography.hazmat.primitives.asymmetric.ed25519")


def _keyring(key, key_id="test-key", status="active"):
    from cryptography.hazmat.primitives import serialization

    public = key.public_key().public_bytes(serialization.Encoding.Raw, serialization.PublicFormat.Raw)
    return TrustedKeyring.from_mapping(
        {
            "schema_version": "1.0",
            "keys": [
                {
                    "key_id": key_id,
                    "algorithm": "ed25519",
                    "public_key": base64.b64encode(public).decode(),
                    "status": status,
                    "created_at": "2026-12-01T00:00:00+00:00",
                }
            ],
        }
    )


def _sign_pack(pack, key, key_id="test-key"):
    manifest = (pack / "manifest.json").read_bytes()
    doc = signature_document(
        private_key=key, key_id=key_id, signed_file="manifest.json", signed_sha256=digest_of(manifest)
    )
    (pack / "manifest.sig.json").write_text(json.dumps(doc), encoding="utf-8")


def test_signed_pack_is_discovered_and_resolved(tmp_path):
    key = ed25519.Ed25519PrivateKey.generate()
    payload = b"kernel"
    pack = write_pack(tmp_path, digest_of(payload), payload)
    _sign_pack(pack, key)
    registry = KernelPackRegistry.discover((tmp_path,), trusted_keys=_keyring(key))
    assert [p.pack_id for p in registry.packs] == ["test-pack"] and registry.rejected == ()
    spec = ArtifactSpec("native", "lib/test_kernel.so", "gemm_out", digest_of(payload))
    found = registry.resolve(
        fingerprint=fingerprint(), operator="gemm", semantic_version="1.0", artifact=spec, evidence_id="test-evidence"
    )
    assert found.pack.pack_id == "test-pack"
    # Only the pack built from the source tree is matched by location; an installed pack must
    # carry exactly the digest the dispatch entry pins.
    other = ArtifactSpec("native", "lib/test_kernel.so", "gemm_out", digest_of(b"other"))
    with pytest.raises(PackResolutionError):
        registry.resolve(fingerprint=fingerprint(), operator="gemm", semantic_version="1.0", artifact=other,
                         evidence_id="test-evidence")
    with pytest.raises(PackResolutionError):
        registry.resolve(
            fingerprint=fingerprint(), operator="gemm", semantic_version="1.0", artifact=spec, evidence_id="other"
        )


@pytest.mark.parametrize("tamper", ["manifest", "unsigned", "unknown-key", "revoked"])
def test_untrusted_packs_are_rejected(tmp_path, tamper):
    key = ed25519.Ed25519PrivateKey.generate()
    pack = write_pack(tmp_path, digest_of(b"k"), b"k")
    _sign_pack(pack, key)
    keyring = _keyring(key)
    if tamper == "manifest":
        (pack / "manifest.json").write_text((pack / "manifest.json").read_text().replace("0.1.0", "0.1.1"))
    elif tamper == "unsigned":
        (pack / "manifest.sig.json").unlink()
    elif tamper == "unknown-key":
        keyring = _keyring(ed25519.Ed25519PrivateKey.generate(), key_id="someone-else")
    elif tamper == "revoked":
        keyring = _keyring(key, status="revoked")
    registry = KernelPackRegistry.discover((tmp_path,), trusted_keys=keyring)
    assert registry.packs == () and len(registry.rejected) == 1


def test_signature_payload_binds_file_name_and_digest():
    key = ed25519.Ed25519PrivateKey.generate()
    content = b"{}"
    doc = signature_document(private_key=key, key_id="test-key", signed_file="manifest.json", signed_sha256=digest_of(content))
    verify_detached_content(content, doc, _keyring(key), signed_file="manifest.json")
    with pytest.raises(SignatureVerificationError, match="expected 'other.json'"):
        verify_detached_content(content, doc, _keyring(key), signed_file="other.json")
    with pytest.raises(SignatureVerificationError, match="SHA-256 mismatch"):
        verify_detached_content(b"{ }", doc, _keyring(key), signed_file="manifest.json")


def test_shipped_keyring_parses():
    ring = builtin_trusted_keyring()
    assert ring.active_public_key("rk-b200-release-2026-12b") is not None
    with pytest.raises(SignatureVerificationError, match="not active"):
        ring.active_public_key("rk-b200-release-2026-12")  # revoked: its private half was not kept


def test_builtin_pack_is_trusted_by_location_and_matches_dispatch():
    manifest_path = BUILTIN_PACK_ROOT / "rk-sm100a" / "manifest.json"
    if not manifest_path.is_file():
        pytest.skip("built-in pack not built yet")
    registry = KernelPackRegistry.discover((), builtin_roots=(BUILTIN_PACK_ROOT,))
    assert [p.pack_id for p in registry.packs] == ["rk-sm100a"]
    pack = registry.packs[0]
    assert pack.environment.architecture == "sm_100a"
    dispatch = builtin_dispatch_registry()
    for operator in ("gemm", "gemv", "swiglu", "rms_norm", "add_rms_norm", "gemm_swiglu", "paged_attention_decode"):
        item = pack.get(operator, "1.0")
        assert sha256_of(pack.root / item.artifact.artifact) == item.artifact.sha256
        for entry in dispatch.get(operator, "1.0").entries:
            if entry.environment.architecture != "sm_100a":
                continue  # the reference's own entries for its AMD packs
            winner, mine = entry.winner, item.artifact
            assert (winner.provider, winner.artifact, winner.format) == (mine.provider, mine.artifact, mine.format), entry.id
            assert entry.evidence_id == item.evidence_id
            # Trusted by location: resolved whatever digest the tracked entry pins, and loaded
            # against the digest this build's manifest records.
            resolved = registry.resolve(fingerprint=fingerprint(), operator=operator, semantic_version="1.0",
                                        artifact=winner, evidence_id=entry.evidence_id)
            assert resolved.load_spec.sha256 == mine.sha256 and resolved.load_spec.entrypoint == winner.entrypoint


def test_shipped_entries_pin_the_kernel_the_library_would_choose():
    """A pinned variant agrees with the library's own rule for that shape range.

    GEMV: the CUDA-core stream kernel (variant 2) only for M <= 2 -- from M = 3 it is
    FMA/L1-bound -- and the tensor-core kernel (variant 3) only from M = 3.  GEMM: the
    SM-pair kernel (variant 3) only with at least one 256 x 256 tile per SM pair of a
    148-SM B200, the 1-SM kernel (variant 2) below that.
    """

    from radeon_kernels import _native

    dispatch = builtin_dispatch_registry()
    gemv_stream, gemv_tc = _native.GEMV_VARIANTS["stream"], _native.GEMV_VARIANTS["tc"]
    for entry in dispatch.get("gemv", "1.0").entries:
        if entry.environment.architecture != "sm_100a":
            continue
        variant = entry.launch["variant"]
        m = entry.workload.values["m"]
        lo, hi = m.value if m.kind == "range" else (min(m.values()), max(m.values()))
        if variant == gemv_stream:
            assert hi <= 2, f"{entry.id}: stream kernel pinned for M up to {hi}"
        if variant == gemv_tc:
            assert lo >= 3, f"{entry.id}: tensor-core kernel pinned for M from {lo}"
    gemm_1sm, gemm_2sm = _native.GEMM_VARIANTS["tc_1sm"], _native.GEMM_VARIANTS["tc_2sm"]
    for entry in dispatch.get("gemm", "1.0").entries:
        if entry.environment.architecture != "sm_100a":
            continue
        variant = entry.launch["variant"]
        if variant not in (gemm_1sm, gemm_2sm):
            continue
        if "n" not in entry.workload.values:
            continue
        m_values = entry.workload.values["m"].values()
        n_values = entry.workload.values["n"].values()
        for m_ in m_values:  # both ends of a range
            for n_ in n_values:
                pair_tiles = (-(-m_ // 256)) * (-(-n_ // 256))
                assert (pair_tiles >= 74) == (variant == gemm_2sm), entry.id
