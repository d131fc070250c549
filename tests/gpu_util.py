"""Helpers for GPU tests: seeded BASELINE inputs, C-ABI calls through ctypes, bit views."""

from __future__ import annotations

import ctypes

import numpy as np

from radeon_kernels import _native

DTYPE_CODE = {"fp16": _native.RK_DTYPE_FP16, "bf16": _native.RK_DTYPE_BF16}


def torch_dtype(name):
    import torch

    return {"fp16": torch.float16, "bf16": torch.bfloat16}[name]


def to_device(bits: np.ndarray, dtype: str, device="cuda"):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16).copy())
    return t.view(torch_dtype(dtype)).to(device)


def to_bits(tensor) -> np.ndarray:
    import torch

    return tensor.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def stream_handle():
    import torch

    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def abi_gemm(a, b, c, variant: int, dtype: str) -> int:
    lib = _native.library()
    m, k = a.shape
    n = b.shape[1]
    return lib.rk_gemm(
        ctypes.c_void_p(a.data_ptr()),
        ctypes.c_void_p(b.data_ptr()),
        ctypes.c_void_p(c.data_ptr()),
        m,
        n,
        k,
        DTYPE_CODE[dtype],
        variant,
        stream_handle(),
    )


LAYOUT_CODE = {"nn": 0, "nt": 1, "tn": 2, "tt": 3}


def abi_gemm_layout(a_stored, b_stored, c, layout: str, variant: int, dtype: str) -> int:
    """rk_gemm_layout on stored operands: A is [M,K] ("n") or [K,M] ("t"), B is [K,N] or [N,K]."""

    lib = _native.library()
    m = a_stored.shape[1] if layout[0] == "t" else a_stored.shape[0]
    k = a_stored.shape[0] if layout[0] == "t" else a_stored.shape[1]
    n = b_stored.shape[0] if layout[1] == "t" else b_stored.shape[1]
    return lib.rk_gemm_layout(
        ctypes.c_void_p(a_stored.data_ptr()),
        ctypes.c_void_p(b_stored.data_ptr()),
        ctypes.c_void_p(c.data_ptr()),
        m,
        n,
        k,
        LAYOUT_CODE[layout],
        DTYPE_CODE[dtype],
        variant,
        stream_handle(),
    )


def abi_gemv(x, w, out, variant: int, dtype: str) -> int:
    lib = _native.library()
    m, k = x.shape
    n = w.shape[0]
    return lib.rk_gemv(
        ctypes.c_void_p(x.data_ptr()),
        ctypes.c_void_p(w.data_ptr()),
        ctypes.c_void_p(out.data_ptr()),
        m,
        n,
        k,
        DTYPE_CODE[dtype],
        variant,
        stream_handle(),
    )


def device_status() -> int:
    return _native.library().rk_device_status(stream_handle())


def seeded(shape, seed: int, dist: str, dtype: str, generator=None):
    """BASELINE.json inputs: fp32 from a seeded CPU torch.Generator, cast, copied to the GPU."""

    import torch

    gen = generator or torch.Generator().manual_seed(seed)
    if dist == "uniform":
        x = torch.rand(shape, generator=gen) * 2 - 1
    elif dist == "uniform16":
        x = (torch.rand(shape, generator=gen) * 2 - 1) / 16
    elif dist == "normal64":
        x = torch.randn(shape, generator=gen) / 64
    elif dist == "normal":
        x = torch.randn(shape, generator=gen)
    elif dist.startswith("normal/"):
        x = torch.randn(shape, generator=gen) / float(dist.split("/", 1)[1]) ** 0.5
    else:
        raise ValueError(dist)
    return x.to(torch_dtype(dtype))
