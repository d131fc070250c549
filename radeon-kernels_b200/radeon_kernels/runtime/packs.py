"""Kernel-pack discovery and resolution of a dispatch winner to an installed pack.

Discovery order and rules follow the reference (src/radeon_kernels/runtime/packs.py:33-147):
``RADEON_KERNELS_PACK_PATH`` entries first, then ``~/.local/share/radeon-kernels/packs``,
then ``<sys.prefix>/share/radeon-kernels/packs``; a root is either a pack itself or a
directory of packs; every ``manifest.json`` found there must carry a valid Ed25519
signature from the trusted keyring, and invalid packs are skipped but reported.

Addition for this build: the sm_100a pack compiled from this source tree lives inside the
package (``radeon_kernels/_packs``).  Like the dispatch manifests it ships with, it is part
of the installation rather than a downloaded release, so it is trusted by location and
checked by artifact SHA-256 only; it is consulted after the signed roots.
"""

from __future__ import annotations

import os
import sys
from dataclasses import dataclass, replace
from pathlib import Path
from typing import Iterable, Mapping, Sequence

from radeon_kernels.errors import ConfigError, RadeonKernelsError
from radeon_kernels.runtime.fingerprint import EnvironmentFingerprint
from radeon_kernels.runtime.pack import KernelPack, KernelPackArtifact
from radeon_kernels.runtime.registry import ArtifactSpec
from radeon_kernels.runtime.signing import (
    SignatureVerificationError,
    TrustedKeyring,
    builtin_trusted_keyring,
    verify_detached_file,
)

PACK_PATH_ENVIRONMENT_VARIABLE = "RADEON_KERNELS_PACK_PATH"
BUILTIN_PACK_ROOT = Path(__file__).resolve().parents[1] / "_packs"


class PackResolutionError(RadeonKernelsError):
    """No installed pack can satisfy an approved dispatch entry."""


@dataclass(frozen=True)
class ResolvedKernelPack:
    pack: KernelPack
    artifact: KernelPackArtifact
    # What to load: the dispatch winner, with the SHA-256 the pack vouches for (equal to the
    # winner's own digest for signed packs; the built-in pack's manifest digest otherwise).
    spec: ArtifactSpec | None = None

    @property
    def load_spec(self) -> ArtifactSpec:
        return self.spec if self.spec is not None else self.artifact.artifact


def default_pack_roots(
    *, environ: Mapping[str, str] | None = None, home: Path | None = None, prefix: Path | None = None
) -> tuple[Path, ...]:
    env = os.environ if environ is None else environ
    candidates = [Path(item).expanduser() for item in env.get(PACK_PATH_ENVIRONMENT_VARIABLE, "").split(os.pathsep) if item]
    candidates.append((home or Path.home()) / ".local" / "share" / "radeon-kernels" / "packs")
    candidates.append((prefix or Path(sys.prefix)) / "share" / "radeon-kernels" / "packs")
    ordered: dict[Path, None] = {}
    for root in candidates:
        ordered.setdefault(root.absolute(), None)
    return tuple(ordered)


def _pack_dirs(roots: Iterable[Path]) -> tuple[Path, ...]:
    found: dict[Path, None] = {}
    for root in roots:
        root = Path(root).expanduser()
        if (root / "manifest.json").is_file():
            candidates: Sequence[Path] = (root,)
        elif root.is_dir():
            candidates = [child for child in sorted(root.iterdir()) if (child / "manifest.json").is_file()]
        else:
            candidates = ()
        for candidate in candidates:
            found.setdefault(candidate.resolve(), None)
    return tuple(found)


class KernelPackRegistry:
    def __init__(
        self, packs: Sequence[KernelPack] = (), *, rejected: Sequence[str] = (), builtin: Iterable[Path] = ()
    ) -> None:
        self._packs = tuple(packs)
        self._rejected = tuple(rejected)
        self._builtin = frozenset(Path(root) for root in builtin)

    @classmethod
    def discover(
        cls,
        roots: Iterable[Path],
        *,
        require_signatures: bool = True,
        trusted_keys: TrustedKeyring | None = None,
        builtin_roots: Iterable[Path] = (),
    ) -> KernelPackRegistry:
        """Load every pack under ``roots`` (signed) and ``builtin_roots`` (trusted by location)."""

        packs: list[KernelPack] = []
        rejected: list[str] = []
        keyring = trusted_keys
        signed_dirs = _pack_dirs(roots)
        if require_signatures and keyring is None and signed_dirs:
            keyring = builtin_trusted_keyring()
        for directory in signed_dirs:
            try:
                if require_signatures:
                    verify_detached_file(
                        directory / "manifest.json", directory / "manifest.sig.json", keyring, signed_file="manifest.json"
                    )
                packs.append(KernelPack.from_directory(directory, verify_artifacts=False))
            except (ConfigError, SignatureVerificationError) as error:
                rejected.append(f"{directory}: {error}")
        builtin: list[Path] = []
        for directory in _pack_dirs(builtin_roots):
            if any(pack.root == directory for pack in packs):
                continue
            try:
                pack = KernelPack.from_directory(directory, verify_artifacts=False)
            except ConfigError as error:
                rejected.append(f"{directory}: {error}")
                continue
            packs.append(pack)
            builtin.append(pack.root)
        return cls(packs, rejected=rejected, builtin=builtin)

    @property
    def packs(self) -> tuple[KernelPack, ...]:
        return self._packs

    @property
    def rejected(self) -> tuple[str, ...]:
        return self._rejected

    def resolve(
        self,
        *,
        fingerprint: EnvironmentFingerprint,
        operator: str,
        semantic_version: str,
        artifact: ArtifactSpec,
        evidence_id: str,
    ) -> ResolvedKernelPack:
        for pack in self._packs:
            if not pack.matches(fingerprint):
                continue
            try:
                item = pack.get(operator, semantic_version)
            except ConfigError:
                continue
            if item.evidence_id != evidence_id:
                continue
            if item.artifact == artifact:
                return ResolvedKernelPack(pack=pack, artifact=item, spec=artifact)
            # The pack built from this source tree is trusted by location: the dispatch entry
            # names its file, format and entrypoint, and its own manifest (written by the same
            # build) supplies the digest the file is verified against -- a rebuild does not
            # rewrite the tracked manifests.
            mine = item.artifact
            if pack.root in self._builtin and (mine.provider, mine.artifact, mine.format) == (
                artifact.provider, artifact.artifact, artifact.format
            ):
                return ResolvedKernelPack(pack=pack, artifact=item, spec=replace(artifact, sha256=mine.sha256))
        note = f"; {len(self._rejected)} invalid pack(s) were ignored" if self._rejected else ""
        raise PackResolutionError(
            f"no installed kernel pack matches {operator} {semantic_version}, "
            f"{fingerprint.architecture}, toolkit ABI {fingerprint.rocm_abi}{note}"
        )
