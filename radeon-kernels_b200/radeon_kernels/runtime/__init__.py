"""Static dispatch runtime: manifests, fingerprints, packs, verified loading, explain."""

from radeon_kernels.runtime.dispatcher import DispatchDecision, Dispatcher, DispatchRequest
from radeon_kernels.runtime.explain import explain_last_dispatch, get_last_dispatch
from radeon_kernels.runtime.fingerprint import EnvironmentFingerprint
from radeon_kernels.runtime.loader import PrecompiledArtifactLoader
from radeon_kernels.runtime.pack import KernelPack
from radeon_kernels.runtime.packs import KernelPackRegistry, PackResolutionError, default_pack_roots
from radeon_kernels.runtime.registry import DispatchRegistry
from radeon_kernels.runtime.resources import builtin_dispatch_registry
from radeon_kernels.runtime.signing import (
    SignatureVerificationError,
    TrustedKeyring,
    builtin_trusted_keyring,
    verify_detached_content,
    verify_detached_file,
)

__all__ = [
    "DispatchDecision",
    "DispatchRegistry",
    "DispatchRequest",
    "Dispatcher",
    "EnvironmentFingerprint",
    "KernelPack",
    "KernelPackRegistry",
    "PackResolutionError",
    "PrecompiledArtifactLoader",
    "SignatureVerificationError",
    "TrustedKeyring",
    "builtin_dispatch_registry",
    "builtin_trusted_keyring",
    "default_pack_roots",
    "explain_last_dispatch",
    "get_last_dispatch",
    "verify_detached_content",
    "verify_detached_file",
]
