"""Fake torch / tensors / loaders for CPU tests of the dispatch runtime.

Same approach as the reference's tests/test_gemm_dispatch.py:21-177: tensors carry shape,
dtype, device and flags only; ``mm`` and the built-in provider just count calls.
"""

from __future__ import annotations

import hashlib
import json
from dataclasses import dataclass
from pathlib import Path
from types import SimpleNamespace

from radeon_kernels.runtime.fingerprint import EnvironmentFingerprint
from radeon_kernels.runtime.loader import PrecompiledArtifactLoader
from radeon_kernels.runtime.registry import DispatchManifest

ENV = {
    "architecture": "sm_100a",
    "wavefront_size": 32,
    "rocm_abi": "12.8",
    "python_abi": "cp312",
    "pytorch_version": "2.11.0+cu128",
}


@dataclass(frozen=True)
class FakeDevice:
    index: int = 0


class FakeTensor:
    _next = 1000

    def __init__(self, shape, *, dtype="float16", device=FakeDevice(), contiguous=True, requires_grad=False):
        self.shape = tuple(shape)
        self.dtype = dtype
        self.device = device
        self.is_cuda = True
        self.requires_grad = requires_grad
        self._contiguous = contiguous
        self._ptr = FakeTensor._next
        FakeTensor._next += 1

    def dim(self):
        return len(self.shape)

    def is_contiguous(self):
        return self._contiguous

    def new_empty(self, shape):
        return FakeTensor(shape, dtype=self.dtype, device=self.device)

    def data_ptr(self):
        return self._ptr


class FakeTorch:
    Tensor = FakeTensor
    float16 = "float16"
    bfloat16 = "bfloat16"
    int32 = "int32"
    int64 = "int64"

    def __init__(self):
        self.cuda = SimpleNamespace(current_device=lambda: 0)
        self.mm_calls = 0

    def mm(self, a, b, *, out=None):
        self.mm_calls += 1
        return out if out is not None else a.new_empty((a.shape[0], b.shape[1]))

    @staticmethod
    def is_grad_enabled():
        return True


class FakeCudaProvider:
    """Stands in for radeon_kernels.providers.cuda_builtin."""

    SELECTED_GEMM = "cuda/gemm"
    SELECTED_GEMV = "cuda/gemv"

    def __init__(self):
        self.gemm_calls = 0
        self.gemv_calls = 0

    def gemm(self, torch_module, a, b, output=None):
        self.gemm_calls += 1
        return output if output is not None else a.new_empty((a.shape[0], b.shape[1]))

    def gemv(self, torch_module, x, weight):
        self.gemv_calls += 1
        return x.new_empty((x.shape[0], weight.shape[0]))


def fingerprint(**overrides) -> EnvironmentFingerprint:
    values = dict(ENV, features=("tcgen05", "tma"))
    values.update(overrides)
    return EnvironmentFingerprint(**values)


def gemm_manifest(digest: str, *, fallbacks=("cuda",)) -> DispatchManifest:
    return DispatchManifest.from_mapping(
        {
            "schema_version": "1.0",
            "operator": "gemm",
            "semantic_version": "1.0",
            "default_fallbacks": list(fallbacks),
            "entries": [
                {
                    "id": "test-gemm-winner",
                    "priority": 100,
                    "environment": dict(ENV, features=["tcgen05"]),
                    "workload": {
                        "dtype": "fp16",
                        "layout": "nn",
                        "m": [2, 2],
                        "n": [4, 4],
                        "k": [3, 3],
                        "contiguous": True,
                        "requires_grad": False,
                    },
                    "winner": {
                        "provider": "native",
                        "artifact": "lib/test_kernel.so",
                        "entrypoint": "gemm_out",
                        "sha256": digest,
                        "format": "python_extension",
                    },
                    "launch": {"variant": 2},
                    "fallbacks": list(fallbacks),
                    "evidence_id": "test-evidence",
                }
            ],
        }
    )


def write_pack(root: Path, digest: str, payload: bytes, *, operator="gemm", entrypoint="gemm_out") -> Path:
    pack = root / "test-pack"
    (pack / "lib").mkdir(parents=True)
    (pack / "lib" / "test_kernel.so").write_bytes(payload)
    (pack / "manifest.json").write_text(
        json.dumps(
            {
                "schema_version": "1.0",
                "pack_id": "test-pack",
                "pack_version": "0.1.0",
                "environment": dict(ENV),
                "artifacts": [
                    {
                        "operator": operator,
                        "semantic_version": "1.0",
                        "provider": "native",
                        "artifact": "lib/test_kernel.so",
                        "entrypoint": entrypoint,
                        "sha256": digest,
                        "format": "python_extension",
                        "evidence_id": "test-evidence",
                    }
                ],
            }
        ),
        encoding="utf-8",
    )
    return pack


class FakeLoader:
    """Verifies the artifact digest for real, then returns a stub entrypoint."""

    variants: list[int] = []

    def __init__(self, root: Path):
        self._verifier = PrecompiledArtifactLoader(root)

    def load_entrypoint(self, artifact):
        self._verifier.resolve_and_verify(artifact)

        def call(a, b, output, variant):
            FakeLoader.variants.append(variant)
            return output

        return SimpleNamespace(callable=call)


def digest_of(payload: bytes) -> str:
    return hashlib.sha256(payload).hexdigest()
