"""rk.gemm dispatch control flow on CPU (fake tensors, real manifests, real digest checks).

Mirrors the reference's tests/test_gemm_dispatch.py cases, with the declared fallback
being this build's ``cuda`` provider instead of ``torch``.
"""

from __future__ import annotations

import os
from pathlib import Path

import pytest

from fakes import (
    FakeCudaProvider,
    FakeLoader,
    FakeTensor,
    FakeTorch,
    digest_of,
    fingerprint,
    gemm_manifest,
    write_pack,
)
from radeon_kernels.ops.gemm.api import GemmDispatchError, GemmRuntime
from radeon_kernels.runtime.explain import clear_last_dispatch, explain_last_dispatch, get_last_dispatch
from radeon_kernels.runtime.packs import KernelPackRegistry, default_pack_roots
from radeon_kernels.runtime.registry import DispatchRegistry
from radeon_kernels.runtime.resources import builtin_dispatch_registry

ARTIFACT = b"precompiled kernel"


@pytest.fixture(autouse=True)
def _reset():
    clear_last_dispatch()
    FakeLoader.variants.clear()


@pytest.fixture
def env(tmp_path):
    torch = FakeTorch()
    cuda = FakeCudaProvider()

    def make(root: Path = tmp_path, detector=None, fallbacks=("cuda",)):
        return GemmRuntime(
            registry=DispatchRegistry([gemm_manifest(digest_of(ARTIFACT), fallbacks=fallbacks)]),
            pack_roots=(root,),
            loader_factory=FakeLoader,
            fingerprint_detector=detector or (lambda **_: fingerprint()),
            require_pack_signatures=False,
            cuda_provider=cuda,
        )

    return torch, cuda, make


def test_executes_exact_precompiled_winner(env, tmp_path):
    torch, cuda, make = env
    write_pack(tmp_path, digest_of(ARTIFACT), ARTIFACT)
    result = make().execute(FakeTensor((2, 3)), FakeTensor((3, 4)), torch_module=torch)
    assert result.shape == (2, 4)
    assert FakeLoader.variants == [2]
    assert cuda.gemm_calls == 0 and torch.mm_calls == 0
    record = get_last_dispatch()
    assert record["selected"] == "native/gemm_out"
    assert "loaded pack test-pack 0.1.0" in record["reason"]
    assert record["architecture"] == "sm_100a"


def test_missing_pack_runs_declared_cuda_fallback(env):
    torch, cuda, make = env
    result = make().execute(FakeTensor((2, 3)), FakeTensor((3, 4)), torch_module=torch)
    assert result.shape == (2, 4)
    assert cuda.gemm_calls == 1 and torch.mm_calls == 0
    assert get_last_dispatch()["selected"] == "cuda/gemm"
    assert "winner unavailable" in get_last_dispatch()["reason"]
    assert "executed declared cuda fallback" in get_last_dispatch()["reason"]


def test_bf16_outside_the_entry_uses_the_fallback(env):
    torch, cuda, make = env
    make().execute(FakeTensor((2, 3), dtype="bfloat16"), FakeTensor((3, 4), dtype="bfloat16"), torch_module=torch)
    assert cuda.gemm_calls == 1
    assert get_last_dispatch()["selected"] == "cuda/gemm"


def test_toolkit_abi_mismatch_uses_the_fallback(env, tmp_path):
    torch, cuda, make = env
    write_pack(tmp_path, digest_of(ARTIFACT), ARTIFACT)
    make(detector=lambda **_: fingerprint(rocm_abi="12.9")).execute(
        FakeTensor((2, 3)), FakeTensor((3, 4)), torch_module=torch
    )
    assert cuda.gemm_calls == 1 and FakeLoader.variants == []


def test_missing_feature_uses_the_fallback(env, tmp_path):
    torch, cuda, make = env
    write_pack(tmp_path, digest_of(ARTIFACT), ARTIFACT)
    make(detector=lambda **_: fingerprint(features=("tma",))).execute(
        FakeTensor((2, 3)), FakeTensor((3, 4)), torch_module=torch
    )
    assert cuda.gemm_calls == 1 and FakeLoader.variants == []


def test_tampered_winner_falls_back_after_the_hash_check(env, tmp_path):
    torch, cuda, make = env
    pack = write_pack(tmp_path, digest_of(ARTIFACT), ARTIFACT)
    (pack / "lib" / "test_kernel.so").write_bytes(b"tampered")
    make().execute(FakeTensor((2, 3)), FakeTensor((3, 4)), torch_module=torch)
    assert cuda.gemm_calls == 1
    assert "SHA-256 mismatch" in get_last_dispatch()["reason"]


def test_unmatched_shape_skips_the_pack(env):
    torch, cuda, make = env
    result = make().execute(FakeTensor((1, 3)), FakeTensor((3, 4)), torch_module=torch)
    assert result.shape == (1, 4)
    assert FakeLoader.variants == []
    assert "no compatible" in get_last_dispatch()["reason"]


def test_autograd_inputs_never_take_the_inference_winner(env, tmp_path):
    torch, cuda, make = env
    write_pack(tmp_path, digest_of(ARTIFACT), ARTIFACT)
    make().execute(FakeTensor((2, 3), requires_grad=True), FakeTensor((3, 4)), torch_module=torch)
    assert FakeLoader.variants == []
    assert get_last_dispatch()["selected"] == "cuda/gemm"


def test_winner_writes_into_the_caller_output(env, tmp_path):
    torch, cuda, make = env
    write_pack(tmp_path, digest_of(ARTIFACT), ARTIFACT)
    out = FakeTensor((2, 4))
    assert make().execute(FakeTensor((2, 3)), FakeTensor((3, 4)), output=out, torch_module=torch) is out


@pytest.mark.parametrize(
    "args, message",
    [
        (((2, 3), (3, 4), (2, 5)), "output must have shape"),
        (((2, 3), (4, 4), None), "inner dimensions must match"),
    ],
)
def test_bad_arguments_raise_before_dispatch(env, args, message):
    torch, cuda, make = env
    a, b, out = args
    with pytest.raises(ValueError, match=message):
        make().execute(FakeTensor(a), FakeTensor(b), output=FakeTensor(out) if out else None, torch_module=torch)
    assert get_last_dispatch() is None


def test_type_errors_raise_before_dispatch(env):
    torch, cuda, make = env
    with pytest.raises(TypeError, match="same dtype"):
        make().execute(FakeTensor((2, 3)), FakeTensor((3, 4), dtype="bfloat16"), torch_module=torch)
    with pytest.raises(TypeError, match="float16 and torch.bfloat16"):
        make().execute(FakeTensor((2, 3), dtype="float32"), FakeTensor((3, 4), dtype="float32"), torch_module=torch)
    with pytest.raises(TypeError, match="PyTorch tensors"):
        make().execute([[1.0]], FakeTensor((3, 4)), torch_module=torch)
    assert get_last_dispatch() is None


def test_cpu_tensors_are_rejected(env):
    torch, cuda, make = env
    a = FakeTensor((2, 3))
    a.is_cuda = False
    with pytest.raises(ValueError, match="visible CUDA GPU"):
        make().execute(a, FakeTensor((3, 4)), torch_module=torch)


def test_torch_only_fallback_is_refused_not_executed(env):
    torch, cuda, make = env
    with pytest.raises(GemmDispatchError):
        make(fallbacks=("torch",)).execute(FakeTensor((1, 3)), FakeTensor((3, 4)), torch_module=torch)
    assert torch.mm_calls == 0 and cuda.gemm_calls == 0
    record = get_last_dispatch()
    assert record["selected"] == "none"
    assert "not available on this build" in record["reason"]


def test_explain_has_the_seven_reference_lines(env, tmp_path):
    torch, cuda, make = env
    write_pack(tmp_path, digest_of(ARTIFACT), ARTIFACT)
    make().execute(FakeTensor((2, 3)), FakeTensor((3, 4)), torch_module=torch)
    lines = explain_last_dispatch().splitlines()
    assert [line.split(":", 1)[0] for line in lines] == [
        "operator",
        "architecture",
        "selected",
        "artifact",
        "evidence",
        "fallbacks",
        "reason",
    ]
    assert lines[2] == "selected: native/gemm_out"
    assert lines[5] == "fallbacks: cuda"


def test_explain_without_dispatch():
    assert explain_last_dispatch() == "No Radeon kernel dispatch has been performed in this context."


def test_builtin_manifests_cover_every_shape_on_sm100a():
    registry = builtin_dispatch_registry()
    gemm = registry.get("gemm", "1.0")
    assert gemm.default_fallbacks == ("cuda",)
    # The reference's own gfx entries stay in the manifest beside the sm_100a ones; on a B200
    # only the sm_100a entries can match, and every one of them falls back to this library.
    assert {entry.environment.architecture for entry in gemm.entries} == {"sm_100a", "gfx1151", "gfx1201"}
    assert all(entry.fallbacks == ("cuda",) for entry in gemm.entries if entry.environment.architecture == "sm_100a")
    from radeon_kernels.runtime.dispatcher import Dispatcher, DispatchRequest

    dispatcher = Dispatcher(registry)
    for dtype in ("bf16", "fp16"):
        for m, n, k in ((1, 8, 8), (7, 13, 5), (4096, 14336, 4096), (16384, 7168, 8192)):
            signature = {"dtype": dtype, "layout": "nn", "m": m, "n": n, "k": k, "contiguous": True, "requires_grad": False}
            decision = dispatcher.select(DispatchRequest("gemm", "1.0", signature), fingerprint())
            assert decision.matched, signature
            assert decision.winner.entrypoint == "gemm_out"
    exact = dispatcher.select(
        DispatchRequest(
            "gemm",
            "1.0",
            {"dtype": "fp16", "layout": "nn", "m": 4096, "n": 14336, "k": 4096, "contiguous": True, "requires_grad": False},
        ),
        fingerprint(),
    )
    assert exact.entry_id == "gemm-sm100a-fp16-m4096-n14336-k4096"


def test_pack_roots_put_explicit_paths_first():
    roots = default_pack_roots(
        environ={"RADEON_KERNELS_PACK_PATH": f"/first{os.pathsep}/second"},
        home=Path("/home/tester"),
        prefix=Path("/runtime"),
    )
    assert roots[:2] == (Path("/first"), Path("/second"))
    assert roots[-2] == Path("/home/tester/.local/share/radeon-kernels/packs")
    assert roots[-1] == Path("/runtime/share/radeon-kernels/packs")


def test_invalid_packs_are_ignored_but_reported(tmp_path):
    (tmp_path / "invalid").mkdir()
    (tmp_path / "invalid" / "manifest.json").write_text("{}", encoding="utf-8")
    registry = KernelPackRegistry.discover((tmp_path,), require_signatures=False)
    assert registry.packs == ()
    assert len(registry.rejected) == 1


def test_repeated_calls_use_the_cached_decision(env, tmp_path):
    torch, cuda, make = env
    write_pack(tmp_path, digest_of(ARTIFACT), ARTIFACT)
    runtime = make()
    for _ in range(3):
        runtime.execute(FakeTensor((2, 3)), FakeTensor((3, 4)), torch_module=torch)
    assert FakeLoader.variants == [2, 2, 2]
    record = get_last_dispatch()
    assert record["selected"] == "native/gemm_out" and "loaded pack" in record["reason"]
    record["selected"] = "mutated"  # readers get copies; the cached record is untouched
    runtime.execute(FakeTensor((2, 3)), FakeTensor((3, 4)), torch_module=torch)
    assert get_last_dispatch()["selected"] == "native/gemm_out"
    # a different signature is decided afresh
    runtime.execute(FakeTensor((1, 3)), FakeTensor((3, 4)), torch_module=torch)
    assert get_last_dispatch()["selected"] == "cuda/gemm"
