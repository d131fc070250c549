"""Locate and load the compiled sm_100a library and its PyTorch binding.

Two handles onto the same kernels:

* :func:`extension` -- the PyTorch binding ``_lib/_rk_ext*.so`` (tensors in, current CUDA
  stream, RuntimeError on failure); used by the built-in ``cuda`` provider;
* :func:`library` -- ``_lib/librk_kernels.so`` through ``ctypes``: the raw C ABI of
  ``include/rk_kernels.h`` (pointers, sizes, stream), used by FFI callers and the parity
  tests.

There is no Python or CPU fallback: when the binaries are missing this raises
:class:`~radeon_kernels.errors.NativeLibraryError` and names the build command.
"""

from __future__ import annotations

import ctypes
import importlib.util
import sysconfig
import threading
from pathlib import Path
from types import ModuleType

from radeon_kernels.errors import NativeLibraryError

LIB_DIR = Path(__file__).resolve().parent / "_lib"
LIBRARY_PATH = LIB_DIR / "librk_kernels.so"
EXTENSION_PATH = LIB_DIR / f"_rk_ext{sysconfig.get_config_var('EXT_SUFFIX') or '.so'}"
BUILD_HINT = "build it with `python radeon-kernels_b200/csrc/build.py` (or __graft_entry__.build())"

# rk_status codes (include/rk_kernels.h)
RK_OK = 0
RK_ERR_INVALID_ARGUMENT = 1
RK_ERR_UNSUPPORTED = 2
RK_ERR_CUDA = 3
RK_ERR_TIMEOUT = 4
RK_ERR_NO_DEVICE = 5
RK_ERR_TOO_LARGE = 6
# rk_dtype
RK_DTYPE_FP16 = 0
RK_DTYPE_BF16 = 1
# variants
GEMM_VARIANTS = {"auto": 0, "simt": 1, "tc_1sm": 2, "tc_2sm": 3}
GEMV_VARIANTS = {"auto": 0, "scalar": 1, "stream": 2, "tc": 3}

_lock = threading.Lock()
_extension: ModuleType | None = None
_library: ctypes.CDLL | None = None


def extension() -> ModuleType:
    global _extension
    if _extension is None:
        with _lock:
            if _extension is None:
                if not EXTENSION_PATH.is_file():
                    raise NativeLibraryError(f"missing compiled binding {EXTENSION_PATH.name}; {BUILD_HINT}")
                import torch  # noqa: F401  -- the binding links libtorch; load it first

                spec = importlib.util.spec_from_file_location("_rk_ext", EXTENSION_PATH)
                if spec is None or spec.loader is None:
                    raise NativeLibraryError(f"cannot import {EXTENSION_PATH}")
                module = importlib.util.module_from_spec(spec)
                try:
                    spec.loader.exec_module(module)
                except ImportError as error:
                    raise NativeLibraryError(f"cannot load {EXTENSION_PATH.name}: {error}") from error
                _extension = module
    return _extension


def _declare(lib: ctypes.CDLL) -> None:
    i64, vp, cint = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int
    lib.rk_gemm.argtypes = [vp, vp, vp, i64, i64, i64, cint, cint, vp]
    lib.rk_gemm.restype = cint
    lib.rk_gemm_layout.argtypes = [vp, vp, vp, i64, i64, i64, cint, cint, cint, vp]
    lib.rk_gemm_layout.restype = cint
    lib.rk_gemv_allgather_ctl_bytes.argtypes = [i64, i64, ctypes.c_int32, ctypes.POINTER(ctypes.c_size_t)]
    lib.rk_gemv_allgather_ctl_bytes.restype = cint
    lib.rk_sdpa.argtypes = [vp] * 4 + [i64] * 5 + [cint, ctypes.c_float, cint, vp]
    lib.rk_sdpa.restype = cint
    lib.rk_silu_mul_backward.argtypes = [vp] * 5 + [i64, i64, cint, vp]
    lib.rk_silu_mul_backward.restype = cint
    lib.rk_rms_norm_backward_workspace_size.argtypes = [i64, i64, ctypes.POINTER(ctypes.c_size_t)]
    lib.rk_rms_norm_backward_workspace_size.restype = cint
    lib.rk_rms_norm_backward.argtypes = [vp] * 5 + [i64, i64, ctypes.c_float, cint, vp, ctypes.c_size_t, vp]
    lib.rk_rms_norm_backward.restype = cint
    lib.rk_add_rms_norm_backward.argtypes = [vp] * 7 + [i64, i64, ctypes.c_float, cint, vp, ctypes.c_size_t, vp]
    lib.rk_add_rms_norm_backward.restype = cint
    lib.rk_paged_attention_set_path.argtypes = [cint]
    lib.rk_paged_attention_set_path.restype = None
    lib.rk_norm_backward_set_ctas_per_sm.argtypes = [cint]
    lib.rk_norm_backward_set_ctas_per_sm.restype = None
    lib.rk_gemv.argtypes = [vp, vp, vp, i64, i64, i64, cint, cint, vp]
    lib.rk_gemv.restype = cint
    lib.rk_gemv_ex.argtypes = [vp, vp, vp, i64, i64, i64, cint, cint, vp, ctypes.c_size_t, vp]
    lib.rk_gemv_ex.restype = cint
    lib.rk_gemv_workspace_size.argtypes = [i64, i64, i64, cint, cint, ctypes.POINTER(ctypes.c_size_t)]
    lib.rk_gemv_workspace_size.restype = cint
    lib.rk_paged_attention_decode.argtypes = [vp] * 6 + [i64] * 7 + [ctypes.c_float, cint, cint, vp, ctypes.c_size_t, vp]
    lib.rk_paged_attention_decode.restype = cint
    lib.rk_paged_attention_workspace_size.argtypes = [i64] * 6 + [ctypes.POINTER(ctypes.c_size_t)]
    lib.rk_paged_attention_workspace_size.restype = cint
    lib.rk_gemm_swiglu.argtypes = [vp, vp, vp, i64, i64, i64, cint, cint, vp]
    lib.rk_gemm_swiglu.restype = cint
    lib.rk_silu_mul.argtypes = [vp, vp, vp, i64, i64, cint, vp]
    lib.rk_silu_mul.restype = cint
    lib.rk_rms_norm.argtypes = [vp, vp, vp, i64, i64, ctypes.c_float, cint, vp]
    lib.rk_rms_norm.restype = cint
    lib.rk_add_rms_norm.argtypes = [vp, vp, vp, vp, vp, i64, i64, ctypes.c_float, cint, vp]
    lib.rk_add_rms_norm.restype = cint
    lib.rk_gemv_fixed_scratch.argtypes = [vp, vp, vp, i64, i64, i64, cint, vp]
    lib.rk_gemv_fixed_scratch.restype = cint
    lib.rk_debug_fill_fixed_scratch.argtypes = [cint, vp]
    lib.rk_debug_fill_fixed_scratch.restype = cint
    lib.rk_debug_last_kernel.argtypes = []
    lib.rk_debug_last_kernel.restype = ctypes.c_char_p
    lib.rk_gemv_allgather.argtypes = [vp, vp, i64, i64, i64, cint, vp, vp]
    lib.rk_gemv_allgather.restype = cint
    lib.rk_gemm_allgather.argtypes = [vp, vp, i64, i64, i64, cint, vp, vp]
    lib.rk_gemm_allgather.restype = cint
    lib.rk_gather_column_blocks.argtypes = [vp, vp, i64, i64, i64, cint, vp]
    lib.rk_gather_column_blocks.restype = cint
    lib.rk_status_string.argtypes = [cint]
    lib.rk_status_string.restype = ctypes.c_char_p
    lib.rk_last_error.argtypes = []
    lib.rk_last_error.restype = ctypes.c_char_p
    lib.rk_device_status.argtypes = [vp]
    lib.rk_device_status.restype = cint
    lib.rk_set_wait_timeout_ns.argtypes = [ctypes.c_uint64]
    lib.rk_set_wait_timeout_ns.restype = None
    lib.rk_debug_inject_stall.argtypes = [cint]
    lib.rk_debug_inject_stall.restype = None
    lib.rk_gemv_set_tuning.argtypes = [cint, cint]
    lib.rk_gemv_set_tuning.restype = None
    lib.rk_gemm_set_tile_n.argtypes = [cint]
    lib.rk_gemm_set_tile_n.restype = None
    lib.rk_gemv_tc_set_cluster.argtypes = [cint]
    lib.rk_gemv_tc_set_cluster.restype = None
    lib.rk_gemv_tc_set_exchange.argtypes = [cint]
    lib.rk_gemv_tc_set_exchange.restype = None
    lib.rk_norm_set_threads.argtypes = [cint]
    lib.rk_norm_set_threads.restype = None
    lib.rk_set_programmatic_launch.argtypes = [cint]
    lib.rk_set_programmatic_launch.restype = cint
    lib.rk_variant_name.argtypes = [cint, cint]
    lib.rk_variant_name.restype = ctypes.c_char_p
    lib.rk_gemm_select_variant.argtypes = [vp, vp, vp, i64, i64, i64, cint]
    lib.rk_gemm_select_variant.restype = cint
    lib.rk_gemv_select_variant.argtypes = [vp, vp, vp, i64, i64, i64, cint]
    lib.rk_gemv_select_variant.restype = cint
    lib.rk_launch_count.argtypes = []
    lib.rk_launch_count.restype = ctypes.c_uint64
    lib.rk_abi_version.argtypes = []
    lib.rk_abi_version.restype = cint


def library() -> ctypes.CDLL:
    global _library
    if _library is None:
        with _lock:
            if _library is None:
                if not LIBRARY_PATH.is_file():
                    raise NativeLibraryError(f"missing {LIBRARY_PATH.name}; {BUILD_HINT}")
                try:
                    lib = ctypes.CDLL(str(LIBRARY_PATH))
                except OSError as error:
                    raise NativeLibraryError(f"cannot load {LIBRARY_PATH}: {error}") from error
                _declare(lib)
                _library = lib
    return _library


def status_text(code: int) -> str:
    text = library().rk_status_string(code).decode()
    if code == RK_ERR_CUDA:
        text += f" ({library().rk_last_error().decode()})"
    return text
