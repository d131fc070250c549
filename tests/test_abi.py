"""The C ABI library: loads, exports every declared symbol, validates before touching a GPU.

No kernel is launched here (CPU-only suite); GPU behaviour is in test_gpu_*.py.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from radeon_kernels import _native

HEADER = Path(__file__).resolve().parents[1] / "include" / "rk_kernels.h"


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*RK_API\s+[a-z_][a-z0-9_ \*]*?\b(rk_[a-z0-9_]+)\s*\(", text, flags=re.M)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for required in ("rk_gemm", "rk_gemv", "rk_status_string", "rk_device_status", "rk_gather_column_blocks"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = _native.library()
    missing = [name for name in declared_functions() if not hasattr(lib, name)]
    assert missing == []


def test_builtin_binding_exports_the_reference_entrypoints():
    ext = _native.extension()
    for name in ("gemm_out", "gemm", "gemv", "gemv_out", "gemv_stream", "gemv_scalar", "gather_column_blocks", "device_status"):
        assert callable(getattr(ext, name))
    assert ext.abi_version() == 1


def test_pack_artifact_imports_and_exports_entrypoints():
    from radeon_kernels.runtime.packs import BUILTIN_PACK_ROOT, KernelPackRegistry
    from radeon_kernels.runtime.loader import PrecompiledArtifactLoader

    registry = KernelPackRegistry.discover((), builtin_roots=(BUILTIN_PACK_ROOT,))
    pack = registry.packs[0]
    loader = PrecompiledArtifactLoader(pack.root)
    for operator, entrypoint in (("gemm", "gemm_out"), ("gemv", "gemv")):
        loaded = loader.load_entrypoint(pack.get(operator, "1.0").artifact)
        assert loaded.entrypoint == entrypoint and callable(loaded.callable)


def test_status_strings_and_variant_names():
    lib = _native.library()
    assert lib.rk_abi_version() == 1
    assert lib.rk_status_string(_native.RK_OK) == b"ok"
    assert lib.rk_status_string(_native.RK_ERR_TIMEOUT) == b"device-side wait timed out"
    assert lib.rk_status_string(99) == b"unknown status"
    assert lib.rk_variant_name(0, 2) == b"gemm:tc_1sm"
    assert lib.rk_variant_name(1, 2) == b"gemv:stream"


def test_arguments_are_validated_before_any_device_work():
    lib = _native.library()
    null = ctypes.c_void_p(0)
    # negative sizes, bad dtype, bad variant: rejected without a GPU
    assert lib.rk_gemm(null, null, null, -1, 4, 4, 0, 0, null) == _native.RK_ERR_INVALID_ARGUMENT
    assert lib.rk_gemm(null, null, null, 4, 4, 4, 7, 0, null) == _native.RK_ERR_INVALID_ARGUMENT
    assert lib.rk_gemm(null, null, null, 4, 4, 4, 0, 99, null) == _native.RK_ERR_UNSUPPORTED
    assert lib.rk_gemm(null, null, null, 4, 4, 4, 0, 0, null) == _native.RK_ERR_INVALID_ARGUMENT  # null C
    assert lib.rk_gemm(null, null, null, 0, 4, 4, 0, 0, null) == _native.RK_OK  # empty: nothing to do
    # rk_gemm_layout: layouts 0-3 (nn, nt, tn, tt); anything else is rejected up front
    assert lib.rk_gemm_layout(null, null, null, 4, 4, 4, 4, 0, 0, null) == _native.RK_ERR_INVALID_ARGUMENT
    assert lib.rk_gemm_layout(null, null, null, 4, 4, 4, -1, 0, 0, null) == _native.RK_ERR_INVALID_ARGUMENT
    assert lib.rk_gemm_layout(null, null, null, 0, 4, 4, 2, 0, 0, null) == _native.RK_OK
    assert lib.rk_gemm_layout(null, null, null, 4, 4, 4, 1, 0, 99, null) == _native.RK_ERR_UNSUPPORTED
    assert lib.rk_gemv(null, null, null, 33, 4, 4, 0, 0, null) == _native.RK_ERR_INVALID_ARGUMENT
    assert lib.rk_gemv(null, null, null, 0, 4, 4, 0, 0, null) == _native.RK_ERR_INVALID_ARGUMENT
    assert lib.rk_gemv(null, null, null, 1, 4, 4, 0, 0, null) == _native.RK_ERR_INVALID_ARGUMENT  # null pointers
    assert lib.rk_gather_column_blocks(null, null, 3, 2, 8, 0, null) == _native.RK_ERR_INVALID_ARGUMENT  # 8 % 3
    assert lib.rk_gemv_workspace_size(1, 8, 8, 0, 0, None) == _native.RK_ERR_INVALID_ARGUMENT
    size = ctypes.c_size_t(7)
    assert lib.rk_gemv_workspace_size(40, 8, 8, 0, 0, ctypes.byref(size)) == _native.RK_ERR_INVALID_ARGUMENT
    assert size.value == 0
    assert lib.rk_gemv_ex(null, null, null, 1, 4, 4, 0, 0, null, 0, null) == _native.RK_ERR_INVALID_ARGUMENT


def test_gemv_allgather_control_area_size():
    """rk_gemv_allgather's control area: the control block, then 2 x world x M x N_block
    8-byte packets; radeon_kernels.distributed.peer rounds it up to whole 4 KiB pages in front
    of each output, and GEMM-only shapes (M > 32) keep the 4 KiB minimum."""

    from radeon_kernels.distributed.peer import CTL_REGION, RK_PEER_CTL_BYTES, control_region_bytes

    lib = _native.library()
    size = ctypes.c_size_t(0)
    assert lib.rk_gemv_allgather_ctl_bytes(1, 1024, 8, ctypes.byref(size)) == _native.RK_OK
    assert size.value == RK_PEER_CTL_BYTES + 2 * 8 * 1 * 1024 * 8
    assert lib.rk_gemv_allgather_ctl_bytes(32, 4096, 2, ctypes.byref(size)) == _native.RK_OK
    assert size.value == RK_PEER_CTL_BYTES + 2 * 2 * 32 * 4096 * 8
    for bad in ((0, 8, 2), (33, 8, 2), (1, 0, 2), (1, 8, 0), (1, 8, 9)):
        assert lib.rk_gemv_allgather_ctl_bytes(*bad, ctypes.byref(size)) == _native.RK_ERR_INVALID_ARGUMENT
        assert size.value == 0
    assert lib.rk_gemv_allgather_ctl_bytes(1, 8, 2, None) == _native.RK_ERR_INVALID_ARGUMENT
    assert control_region_bytes((1, 8192), 8) == 135168  # 512 + 131072 bytes -> 33 pages
    assert control_region_bytes((1, 16), 2) == CTL_REGION
    assert control_region_bytes((16384, 57344), 8) == CTL_REGION  # M > 32: the GEMM's exchange


def test_missing_binary_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_native, "_library", None)
    monkeypatch.setattr(_native, "LIBRARY_PATH", tmp_path / "librk_kernels.so")
    from radeon_kernels.errors import NativeLibraryError

    with pytest.raises(NativeLibraryError, match="build it with"):
        _native.library()
