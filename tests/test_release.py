"""Signed releases of the sm_100a kernel pack, installed and verified the reference's way (CPU).

The release format is the reference's (src/radeon_kernels/runtime/installer.py): a tar.gz
of ``<pack_id>/{manifest.json, manifest.sig.json, lib/...}`` plus a signed pack-index record
carrying the manifest digest and signature and the archive's name, size and digest.
``install_release`` -> ``verify_installed_pack`` (installer.py:251-285) is the path a
reference install takes; here it runs on a release made from the pack this repository
builds, signed with a throwaway key, and on tampered variants of it.
"""

from __future__ import annotations

import base64
import io
import json
import shutil
import tarfile

import pytest

from fakes import fingerprint
from radeon_kernels.errors import ConfigError
from radeon_kernels.runtime.installer import PackInstallError, install_release, load_index, verify_installed_pack
from radeon_kernels.runtime.loader import ArtifactError, PrecompiledArtifactLoader
from radeon_kernels.runtime.packs import BUILTIN_PACK_ROOT
from radeon_kernels.runtime.publish import make_release, sign_manifest, write_index
from radeon_kernels.runtime.resources import builtin_dispatch_registry
from radeon_kernels.runtime.signing import SignatureVerificationError, TrustedKeyring, builtin_trusted_keyring, verify_detached_file

ed25519 = pytest.importorskip("cryptography.hazmat.primitives.asymmetric.ed25519")
PACK = BUILTIN_PACK_ROOT / "rk-sm100a"

# The reference's own dispatch entries (dispatch/*.json), which the shipped manifests keep
# beside the sm_100a entries so one manifest serves both packs.
REFERENCE_ENTRY_IDS = {
    "gemm": {"gemm-gfx1151-fp16-m256-n4096-k4096", "gemm-gfx1201-fp16-m512-n512-k512"},
    "gemv": {"gemv-gfx1201-decode-ffn-down-h4096-bf16", "gemv-gfx1201-decode-h8192-bf16", "gemv-gfx1201-decode-h8192-fp16"},
}


def _keyring(key, key_id="release-test"):
    from cryptography.hazmat.primitives import serialization

    public = key.public_key().public_bytes(serialization.Encoding.Raw, serialization.PublicFormat.Raw)
    return TrustedKeyring.from_mapping({"schema_version": "1.0", "keys": [{
        "key_id": key_id, "algorithm": "ed25519", "public_key": base64.b64encode(public).decode(),
        "status": "active", "created_at": "2026-12-02T00:00:00+00:00"}]})


KEEP = ("gemm", "gemv")  # the release under test carries these two operators of the built pack


@pytest.fixture(scope="module")
def signed_pack(tmp_path_factory):
    """(pack directory, key): the built pack's gemm and gemv artifacts (the real 38 MB shared
    object) under a manifest re-signed with a throwaway key.  Two operators keep the archive
    small enough for the CPU suite; the full pack has nine paths to the same object."""

    if not (PACK / "manifest.json").is_file() or not (PACK / "lib").is_dir():
        pytest.skip("built-in pack not built")
    key = ed25519.Ed25519PrivateKey.generate()
    pack = tmp_path_factory.mktemp("src") / "rk-sm100a"
    manifest = json.loads((PACK / "manifest.json").read_text())
    manifest["artifacts"] = [a for a in manifest["artifacts"] if a["operator"] in KEEP]
    for item in manifest["artifacts"]:
        target = pack / item["artifact"]
        target.parent.mkdir(parents=True, exist_ok=True)
        shutil.copyfile(PACK / item["artifact"], target)
    (pack / "manifest.json").write_text(json.dumps(manifest, indent=2) + "\n")
    assert sign_manifest(pack, key, "release-test")
    return pack, key


@pytest.fixture(scope="module")
def release(signed_pack, tmp_path_factory):
    """(archive, index, keyring, key): the signed pack released with a signed index."""

    pack, key = signed_pack
    out = tmp_path_factory.mktemp("out")
    record = make_release(pack, out, approval_id="approval-rk-sm100a-test")
    index_path = write_index([record], out / "gemm-1.0.json", key, "release-test")
    keyring = _keyring(key)
    index = load_index(index_path, trusted_keys=keyring)
    return out / record["release_file"], index, keyring, key


def _sm100a():
    import json as _json

    env = _json.loads((PACK / "manifest.json").read_text())["environment"]
    return fingerprint(rocm_abi=env["rocm_abi"], python_abi=env["python_abi"], pytorch_version=env["pytorch_version"])


def test_release_installs_and_verifies(release, tmp_path):
    archive, index, keyring, _ = release
    pack = install_release(archive, index, _sm100a(), tmp_path / "installed", trusted_keys=keyring)
    assert pack.pack_id == "rk-sm100a" and (tmp_path / "installed" / "rk-sm100a" / "manifest.sig.json").is_file()
    again = verify_installed_pack(tmp_path / "installed" / "rk-sm100a", trusted_keys=keyring)
    assert [a.operator for a in again.artifacts] == [a.operator for a in pack.artifacts]


def test_release_archive_is_reproducible(signed_pack, release, tmp_path):
    pack, _ = signed_pack
    again = make_release(pack, tmp_path / "again", approval_id="approval-rk-sm100a-test")
    assert again == release[1]["packs"][0]  # byte-identical archive, same record


def test_untrusted_key_is_rejected(release, tmp_path):
    archive, index, _, _ = release
    stranger = _keyring(ed25519.Ed25519PrivateKey.generate(), key_id="release-test")
    with pytest.raises(SignatureVerificationError):
        install_release(archive, index, _sm100a(), tmp_path / "installed", trusted_keys=stranger)
    assert not (tmp_path / "installed" / "rk-sm100a").exists()


def test_wrong_environment_finds_no_release(release, tmp_path):
    archive, index, keyring, _ = release
    with pytest.raises(PackInstallError, match="no indexed pack matches"):
        install_release(archive, index, fingerprint(architecture="gfx1201"), tmp_path / "i", trusted_keys=keyring)


def _rewrite(archive, tmp_path, mutate):
    """A copy of the release with its members passed through ``mutate(name, data) -> [(name, data)]``."""

    with tarfile.open(archive, "r:gz") as tar:
        members = [(m, tar.extractfile(m).read() if m.isfile() else None) for m in tar.getmembers()]
    out = tmp_path / "tampered" / archive.name
    out.parent.mkdir(parents=True, exist_ok=True)
    with tarfile.open(out, "w:gz", compresslevel=1) as tar:
        for member, data in members:
            for name, payload in mutate(member.name, data):
                info = tarfile.TarInfo(name)
                if payload is None:
                    info.type = tarfile.DIRTYPE
                    tar.addfile(info)
                else:
                    info.size = len(payload)
                    tar.addfile(info, io.BytesIO(payload))
    return out


def _reindex(index, archive):
    from radeon_kernels.runtime.loader import sha256_of

    record = dict(index["packs"][0], release_sha256=sha256_of(archive), release_size=archive.stat().st_size)
    return {"schema_version": "1.0", "packs": [record]}


@pytest.mark.parametrize("attack", ["artifact-bytes", "extra-member", "path-escape"])
def test_tampered_release_is_rejected(release, tmp_path, attack):
    archive, index, keyring, _ = release

    def mutate(name, data):
        if attack == "artifact-bytes" and name.endswith("gemv/rk_sm100a.so"):
            return [(name, data[:-1] + bytes([data[-1] ^ 1]))]
        if attack == "extra-member" and name.endswith("manifest.json"):
            return [(name, data), ("rk-sm100a/lib/extra.so", b"x")]
        if attack == "path-escape" and name.endswith("manifest.json"):
            return [(name, data), ("rk-sm100a/../escape.txt", b"x")]
        return [(name, data)]

    tampered = _rewrite(archive, tmp_path, mutate)
    with pytest.raises((PackInstallError, ConfigError, ArtifactError)):
        install_release(tampered, _reindex(index, tampered), _sm100a(), tmp_path / "installed", trusted_keys=keyring)
    assert not (tmp_path / "installed" / "rk-sm100a").exists()
    assert not (tmp_path / "escape.txt").exists()


def test_release_archive_must_match_the_index(release, tmp_path):
    archive, index, keyring, _ = release
    record = dict(index["packs"][0], release_size=index["packs"][0]["release_size"] + 1)
    with pytest.raises(PackInstallError, match="size mismatch"):
        install_release(archive, {"schema_version": "1.0", "packs": [record]}, _sm100a(), tmp_path / "i", trusted_keys=keyring)


def test_shipped_signature_verifies_with_the_shipped_keyring():
    """The tracked manifest.sig.json signs the tracked manifest with the shipped release key."""

    if not (PACK / "manifest.sig.json").is_file():
        pytest.skip("this build has no release key; the built-in pack is trusted by location only")
    verify_detached_file(PACK / "manifest.json", PACK / "manifest.sig.json", builtin_trusted_keyring(), signed_file="manifest.json")


def test_shipped_manifests_keep_the_reference_entries():
    dispatch = builtin_dispatch_registry()
    for operator, ids in REFERENCE_ENTRY_IDS.items():
        entries = {e.id: e for e in dispatch.get(operator, "1.0").entries}
        assert ids <= set(entries), f"{operator}: reference entries missing"
        assert {entries[i].environment.architecture for i in ids} <= {"gfx1151", "gfx1201"}
        assert any(e.environment.architecture == "sm_100a" for e in entries.values())


def test_reference_gemv_entrypoint_names_resolve_in_the_pack():
    if not (PACK / "lib" / "gemv" / "rk_sm100a.so").is_file():
        pytest.skip("built-in pack not built")
    import torch  # noqa: F401 -- the binding links libtorch, as in any process that calls it

    from radeon_kernels.runtime.pack import KernelPack

    pack = KernelPack.from_directory(PACK, verify_artifacts=False)
    spec = pack.get("gemv", "1.0").artifact
    loader = PrecompiledArtifactLoader(pack.root)
    for name in ("gemv_wave1", "gemv_wave2"):
        loaded = loader.load_entrypoint(type(spec)(spec.provider, spec.artifact, name, spec.sha256, spec.format))
        assert callable(loaded.callable)
