"""Manifest parsing/validation, fingerprints, selection, loader integrity (CPU)."""

from __future__ import annotations

import copy
import hashlib
from pathlib import Path
from types import SimpleNamespace

import pytest

from fakes import ENV, fingerprint
from radeon_kernels.errors import ConfigError
from radeon_kernels.ops._runtime import OperatorRuntime
from radeon_kernels.runtime.dispatcher import Dispatcher, DispatchRequest
from radeon_kernels.runtime.explain import clear_last_dispatch, get_last_dispatch
from radeon_kernels.runtime.fingerprint import EnvironmentFingerprint, FingerprintError, cuda_architecture_name
from radeon_kernels.runtime.loader import (
    ArtifactIntegrityError,
    PrecompiledArtifactLoader,
    extension_module_name,
)
from radeon_kernels.runtime.registry import ArtifactSpec, DispatchManifest, DispatchRegistry, ValueConstraint


def entry(entry_id="a", priority=100, workload=None, features=None, launch=None):
    env = dict(ENV)
    if features is not None:
        env["features"] = features
    return {
        "id": entry_id,
        "priority": priority,
        "environment": env,
        "workload": workload or {"dtype": "fp16", "m": [1, 8]},
        "winner": {
            "provider": "native",
            "artifact": "lib/k.so",
            "entrypoint": "run",
            "sha256": "a" * 64,
            "format": "python_extension",
        },
        "launch": launch if launch is not None else {},
        "fallbacks": ["cuda"],
        "evidence_id": "ev",
    }


def manifest(*entries, **overrides):
    value = {
        "schema_version": "1.0",
        "operator": "op",
        "semantic_version": "1.0",
        "default_fallbacks": ["cuda"],
        "entries": list(entries),
    }
    value.update(overrides)
    return value


def test_same_priority_overlap_is_ambiguous():
    with pytest.raises(ConfigError, match="ambiguous"):
        DispatchManifest.from_mapping(manifest(entry("a"), entry("b", workload={"dtype": "fp16", "m": [4, 16]})))


def test_partial_shadow_is_rejected():
    with pytest.raises(ConfigError, match="strict subset"):
        DispatchManifest.from_mapping(
            manifest(entry("a", 100, {"dtype": "fp16", "m": [4, 16]}), entry("b", 10, {"dtype": "fp16", "m": [1, 8]}))
        )


def test_strict_subset_at_higher_priority_is_accepted_and_wins():
    parsed = DispatchManifest.from_mapping(
        manifest(entry("wide", 10, {"dtype": "fp16", "m": [1, 64]}), entry("narrow", 100, {"dtype": "fp16", "m": [4, 4]}))
    )
    dispatcher = Dispatcher(DispatchRegistry([parsed]))
    hit = dispatcher.select(DispatchRequest("op", "1.0", {"dtype": "fp16", "m": 4}), fingerprint())
    assert hit.entry_id == "narrow"
    miss = dispatcher.select(DispatchRequest("op", "1.0", {"dtype": "fp16", "m": 5}), fingerprint())
    assert miss.entry_id == "wide"
    none = dispatcher.select(DispatchRequest("op", "1.0", {"dtype": "bf16", "m": 5}), fingerprint())
    assert not none.matched and none.fallbacks == ("cuda",)
    assert get_last_dispatch()["reason"] == "no compatible environment and workload region matched"


def test_feature_subset_makes_an_environment_strictly_narrower():
    parsed = DispatchManifest.from_mapping(
        manifest(entry("plain", 10, features=[]), entry("tc", 100, features=["tcgen05"]))
    )
    dispatcher = Dispatcher(DispatchRegistry([parsed]))
    assert dispatcher.select(DispatchRequest("op", "1.0", {"dtype": "fp16", "m": 2}), fingerprint()).entry_id == "tc"
    no_tc = fingerprint(features=("tma",))
    assert dispatcher.select(DispatchRequest("op", "1.0", {"dtype": "fp16", "m": 2}), no_tc).entry_id == "plain"


@pytest.mark.parametrize(
    "mutate, message",
    [
        (lambda e: e.update(unexpected=1), "unknown fields"),
        (lambda e: e.pop("evidence_id"), "missing fields"),
        (lambda e: e.update(launch={"variant": [1]}), "expected a string, number or boolean"),
        (lambda e: e.update(priority=-1), "non-negative"),
        (lambda e: e.update(priority=True), "non-negative"),
        (lambda e: e["winner"].update(sha256="A" * 64), "lowercase SHA-256"),
        (lambda e: e["winner"].update(artifact="../escape.so"), "normalized relative path"),
        (lambda e: e["winner"].update(artifact="/abs.so"), "normalized relative path"),
        (lambda e: e["winner"].update(format="cubin"), "python_extension or hsaco"),
        (lambda e: e["environment"].update(architecture="hopper"), "architecture"),
        (lambda e: e["environment"].update(wavefront_size=48), "32 or 64"),
        (lambda e: e["environment"].update(rocm_abi="twelve"), "MAJOR.MINOR"),
        (lambda e: e.update(workload={"m": [0, 4]}), "integer ranges"),
        (lambda e: e.update(workload={"m": [4, 1]}), "integer ranges"),
        (lambda e: e.update(workload={"m": {"one_of": [1, 1]}}), "duplicate"),
        (lambda e: e.update(workload={}), "at least one constraint"),
        (lambda e: e.update(fallbacks=["cuda", "cuda"]), "duplicates"),
    ],
)
def test_entry_validation(mutate, message):
    value = entry()
    mutate(value)
    with pytest.raises(ConfigError, match=message):
        DispatchManifest.from_mapping(manifest(value))


def test_manifest_level_validation():
    with pytest.raises(ConfigError, match="unsupported dispatch schema version"):
        DispatchManifest.from_mapping(manifest(schema_version="2.0"))
    with pytest.raises(ConfigError, match="non-empty list"):
        DispatchManifest.from_mapping(manifest(default_fallbacks=[]))
    with pytest.raises(ConfigError, match="entry ids must be unique"):
        DispatchManifest.from_mapping(
            manifest(entry("a", 10, {"dtype": "fp16"}), entry("a", 20, {"dtype": "bf16"}))
        )
    with pytest.raises(ConfigError, match="duplicate manifest"):
        DispatchRegistry([DispatchManifest.from_mapping(manifest()), DispatchManifest.from_mapping(manifest())])


def test_value_constraints_are_type_exact():
    assert ValueConstraint.from_raw(True, "x").matches(True)
    assert not ValueConstraint.from_raw(True, "x").matches(1)
    assert not ValueConstraint.from_raw(1, "x").matches(True)
    rng = ValueConstraint.from_raw([2, 8], "x")
    assert rng.matches(2) and rng.matches(8) and not rng.matches(9) and not rng.matches(True)
    choice = ValueConstraint.from_raw({"one_of": ["fp16", "bf16"]}, "x")
    assert choice.matches("bf16") and not choice.matches("fp32")


def test_manifest_round_trips_through_to_dict():
    parsed = DispatchManifest.from_mapping(manifest(entry(launch={"variant": 3})))
    assert DispatchManifest.from_mapping(copy.deepcopy(parsed.to_dict())) == parsed


def test_fingerprint_validation_and_naming():
    assert cuda_architecture_name(10, 0) == "sm_100a"
    assert cuda_architecture_name(8, 9) == "sm_89"
    fp = EnvironmentFingerprint.from_mapping(
        {"architecture": "sm_100a", "wavefront_size": 32, "rocm_abi": "12.8.93", "python_abi": "cp312", "pytorch_version": "x"}
    )
    assert fp.rocm_abi == "12.8"
    with pytest.raises(FingerprintError):
        EnvironmentFingerprint("sm_100a", 16, "12.8", "cp312", "x")
    with pytest.raises(FingerprintError, match="unknown fingerprint fields"):
        EnvironmentFingerprint.from_mapping({"bogus": 1})


def test_fingerprint_detect_from_a_fake_cuda_torch():
    props = SimpleNamespace(major=10, minor=0, warp_size=32)
    fake = SimpleNamespace(
        cuda=SimpleNamespace(is_available=lambda: True, get_device_properties=lambda index: props),
        version=SimpleNamespace(cuda="12.8", hip=None),
        __version__="2.11.0+cu128",
    )
    fp = EnvironmentFingerprint.detect(torch_module=fake, device_index=0)
    assert (fp.architecture, fp.rocm_abi, fp.features) == ("sm_100a", "12.8", ("tcgen05", "tma"))
    fake.cuda.is_available = lambda: False
    with pytest.raises(FingerprintError, match="no visible CUDA GPU"):
        EnvironmentFingerprint.detect(torch_module=fake)


def _spec(path: str, payload: bytes) -> ArtifactSpec:
    return ArtifactSpec("native", path, "run", hashlib.sha256(payload).hexdigest())


def test_loader_verifies_digest_and_detects_later_tampering(tmp_path):
    (tmp_path / "lib").mkdir()
    target = tmp_path / "lib" / "k.so"
    target.write_bytes(b"one")
    loader = PrecompiledArtifactLoader(tmp_path)
    assert loader.resolve_and_verify(_spec("lib/k.so", b"one")) == target.resolve()
    # cached: the second call does not re-hash, but a changed file is re-hashed and rejected
    target.write_bytes(b"two!")
    with pytest.raises(ArtifactIntegrityError, match="SHA-256 mismatch"):
        loader.resolve_and_verify(_spec("lib/k.so", b"one"))


def test_loader_rejects_escapes_and_missing_files(tmp_path):
    outside = tmp_path / "outside.so"
    outside.write_bytes(b"x")
    root = tmp_path / "pack"
    (root / "lib").mkdir(parents=True)
    (root / "lib" / "link.so").symlink_to(outside)
    loader = PrecompiledArtifactLoader(root)
    with pytest.raises(ArtifactIntegrityError, match="escapes"):
        loader.resolve_and_verify(_spec("lib/link.so", b"x"))
    with pytest.raises(ArtifactIntegrityError, match="missing"):
        loader.resolve_and_verify(_spec("lib/none.so", b"x"))


def test_python_extension_module_name_comes_from_pyinit(tmp_path):
    blob = tmp_path / "renamed.cpython-312-x86_64-linux-gnu.so"
    blob.write_bytes(b"\x00junk\x00PyInit_rk_sm100a\x00more\x00")
    assert extension_module_name(blob) == "rk_sm100a"
    blob.write_bytes(b"\x00PyInit_one\x00PyInit_two\x00")
    with pytest.raises(Exception, match="multiple PyInit"):
        extension_module_name(blob)


class _Packs:
    def __init__(self, root):
        self.root = root
        self.calls = 0

    def resolve(self, *, artifact, **_):
        self.calls += 1
        return SimpleNamespace(pack=SimpleNamespace(root=self.root, pack_id="test-pack", pack_version="0.1.0"),
                               load_spec=artifact)


class _Loader:
    def __init__(self, _root):
        pass

    def load_entrypoint(self, _artifact):
        return SimpleNamespace(callable=lambda value, **launch: f"native:{value}:{launch}")


def _operator_runtime(tmp_path, *, winner: bool):
    entries = [entry("op-winner", 100, {"dtype": "fp16", "rows": [2, 2]}, launch={"variant": 2})] if winner else []
    packs = _Packs(tmp_path)
    runtime = OperatorRuntime(
        registry=DispatchRegistry([DispatchManifest.from_mapping(manifest(*entries))]),
        pack_registry=packs,
        loader_factory=_Loader,
        fingerprint_detector=lambda **_: fingerprint(),
    )
    return runtime, packs


def _run(runtime):
    return runtime.execute(
        operator="op",
        semantic_version="1.0",
        signature={"dtype": "fp16", "rows": 2},
        device_index=0,
        torch_module=object(),
        native_arguments=("input",),
        fallback=lambda: "cuda-result",
        fallback_selected="cuda/op",
    )


def test_operator_runtime_fallback_only_manifest(tmp_path):
    clear_last_dispatch()
    runtime, packs = _operator_runtime(tmp_path, winner=False)
    assert _run(runtime) == "cuda-result"
    assert packs.calls == 0
    assert get_last_dispatch()["selected"] == "cuda/op"


def test_operator_runtime_passes_launch_parameters_to_the_winner(tmp_path):
    clear_last_dispatch()
    runtime, packs = _operator_runtime(tmp_path, winner=True)
    assert _run(runtime) == "native:input:{'variant': 2}"
    assert packs.calls == 1
    assert get_last_dispatch()["selected"] == "native/run"
