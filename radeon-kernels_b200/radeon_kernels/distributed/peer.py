"""Peer-mapped exchange buffers for the fused compute + all-gather kernels.

No counterpart in the reference (it is single-GPU).  A :class:`PeerExchange` is created
collectively by every rank of a process group (one process per GPU).  Each rank allocates
one device buffer -- a control region (the ``RK_PEER_CTL_BYTES`` control block and, for the
GEMV's packet exchange, the staging area ``rk_gemv_allgather_ctl_bytes`` sizes) followed by
its full output ``[M, N]`` -- exports it with ``rk_ipc_export``, and maps every other rank's buffer with
``rk_ipc_open`` (CUDA IPC; NVLink / NVSwitch peer access).  The kernels behind
``rk_gemv_allgather`` / ``rk_gemm_allgather`` then store every rank's column block straight
into every rank's output and order the calls through the control blocks, so a gathered
result needs no NCCL call and no permute pass.

The fused path is used only where it is safe: CUDA tensors, at most ``RK_PEER_MAX`` ranks,
every rank on a different physical GPU (two ranks on one GPU would run kernels that wait on
each other on the same device), and every mapping opened on every rank; the ranks agree on
the outcome collectively, so either all take it or all use the NCCL all-gather.
"""

from __future__ import annotations

import ctypes
import math
from typing import Any

RK_PEER_MAX = 8
RK_PEER_CTL_BYTES = 512
CTL_REGION = 4096  # smallest control region at the start of each buffer (keeps the output 4 KiB aligned)
GEMV_MAX_M = 32  # rk_gemv_allgather's row limit: shapes above it never need the staging area


class _IpcHandle(ctypes.Structure):
    _fields_ = [("bytes", ctypes.c_ubyte * 64), ("offset", ctypes.c_uint64)]


def _declare(lib: ctypes.CDLL) -> None:
    if getattr(lib, "_rk_ipc_declared", False):
        return
    lib.rk_ipc_export.argtypes = [ctypes.c_void_p, ctypes.POINTER(_IpcHandle)]
    lib.rk_ipc_export.restype = ctypes.c_int
    lib.rk_ipc_open.argtypes = [ctypes.POINTER(_IpcHandle), ctypes.POINTER(ctypes.c_void_p)]
    lib.rk_ipc_open.restype = ctypes.c_int
    lib.rk_ipc_close.argtypes = [ctypes.POINTER(_IpcHandle)]
    lib.rk_ipc_close.restype = ctypes.c_int
    lib._rk_ipc_declared = True


def _lib() -> ctypes.CDLL:
    from radeon_kernels import _native

    lib = _native.library()
    _declare(lib)
    return lib


def control_region_bytes(shape: tuple[int, int], world: int) -> int:
    """Bytes in front of each rank's output: the control block, plus, for shapes that
    ``rk_gemv_allgather`` can run (M <= 32), its packet staging area; a multiple of 4 KiB."""

    from radeon_kernels import _native

    m, n = int(shape[0]), int(shape[1])
    need = RK_PEER_CTL_BYTES
    if 1 <= m <= GEMV_MAX_M and world >= 1 and n % world == 0:
        size = ctypes.c_size_t(0)
        status = _lib().rk_gemv_allgather_ctl_bytes(m, n // world, world, ctypes.byref(size))
        if status != _native.RK_OK:
            raise RuntimeError(f"rk_gemv_allgather_ctl_bytes failed: {_native.status_text(status)}")
        need = int(size.value)
    return max(CTL_REGION, -(-need // CTL_REGION) * CTL_REGION)


def export_handle(ptr: int) -> bytes:
    """IPC handle (72 bytes) of the device allocation holding ``ptr``."""

    from radeon_kernels import _native

    handle = _IpcHandle()
    status = _lib().rk_ipc_export(ctypes.c_void_p(ptr), ctypes.byref(handle))
    if status != _native.RK_OK:
        raise RuntimeError(f"rk_ipc_export failed: {_native.status_text(status)}")
    return bytes(handle)


def open_handle(raw: bytes) -> int:
    """Maps another process's exported pointer into this process; returns its address here."""

    from radeon_kernels import _native

    handle = _IpcHandle.from_buffer_copy(raw)
    ptr = ctypes.c_void_p()
    status = _lib().rk_ipc_open(ctypes.byref(handle), ctypes.byref(ptr))
    if status != _native.RK_OK:
        raise RuntimeError(f"rk_ipc_open failed: {_native.status_text(status)}")
    return int(ptr.value or 0)


def close_handle(raw: bytes) -> None:
    handle = _IpcHandle.from_buffer_copy(raw)
    _lib().rk_ipc_close(ctypes.byref(handle))


def _dist() -> Any:
    import torch.distributed as dist

    return dist


def _all_gather(obj: Any, group: Any) -> list[Any]:
    dist = _dist()
    out: list[Any] = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, obj, group=group)
    return out


def _device_uuid(device: Any) -> str:
    import torch

    return str(torch.cuda.get_device_properties(device).uuid)


class PeerMappingError(RuntimeError):
    """Raised on every rank when some rank could not map a peer's buffer."""


class PeerExchange:
    """One full output ``[M, N]`` per rank, mapped into every rank, plus its control block.

    Collective: every rank of ``group`` constructs it with the same ``shape`` and ``dtype``.
    ``output`` is this rank's full output; it is rewritten by the next fused call on this
    exchange (the other ranks start writing only after this rank has issued that call).
    """

    def __init__(self, shape: tuple[int, int], dtype: Any, *, group: Any = None, timeout_s: float = 10.0) -> None:
        import torch

        dist = _dist()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if not 1 <= self.world <= RK_PEER_MAX:
            raise ValueError(f"a peer exchange spans 1 to {RK_PEER_MAX} ranks, not {self.world}")
        self.shape = (int(shape[0]), int(shape[1]))
        self.dtype = dtype
        self.timeout_ns = int(timeout_s * 1e9)
        device = torch.device("cuda", torch.cuda.current_device())
        nbytes = math.prod(self.shape) * torch.empty((), dtype=dtype).element_size()
        self.ctl_region = control_region_bytes(self.shape, self.world)
        self._storage = torch.zeros(self.ctl_region + nbytes, dtype=torch.uint8, device=device)
        self.output = self._storage[self.ctl_region:].view(dtype).view(self.shape)
        # The zeroed control block must be in memory before any rank's kernel can write it.
        torch.cuda.current_stream(device).synchronize()
        base = self._storage.data_ptr()
        handles = _all_gather(export_handle(base), group)
        self._opened: list[bytes] = []
        bases, error = [], ""
        try:
            for j, raw in enumerate(handles):
                if j == self.rank:
                    bases.append(base)
                else:
                    bases.append(open_handle(raw))
                    self._opened.append(raw)
        except RuntimeError as failure:
            error = str(failure)
        # Every rank learns whether every rank mapped every buffer, so all fail together.
        failures = [e for e in _all_gather(error, group) if e]
        if failures:
            for raw in self._opened:
                close_handle(raw)
            self._opened = []
            raise PeerMappingError(f"peer mapping failed on {len(failures)} rank(s): {failures[0]}")
        self.ctl_ptrs = bases
        self.out_ptrs = [b + self.ctl_region for b in bases]
        dist.barrier(group=group)

    def close(self) -> None:
        """Collective: unmaps the peers' buffers once no rank uses the exchange any more."""

        if self._opened:
            _dist().barrier(group=self.group)
            for raw in self._opened:
                close_handle(raw)
            self._opened = []


def fused_path_available(device_tensor: Any, *, group: Any = None) -> bool:
    """Collective check: may every rank of ``group`` take the fused peer-store path?

    Every rank must call it (it exchanges one small object); the answer is the same on all.
    """

    world = _dist().get_world_size(group)
    ok = bool(getattr(device_tensor, "is_cuda", False)) and 1 < world <= RK_PEER_MAX
    uuid = None
    if ok:
        try:
            from radeon_kernels import _native

            _native.extension()
            _lib()
            uuid = _device_uuid(device_tensor.device)
        except Exception:  # noqa: BLE001 -- any failure means "not on this rank"; decided collectively
            ok = False
    votes = _all_gather((ok, uuid), group)
    if not all(vote[0] for vote in votes):
        return False
    uuids = [vote[1] for vote in votes]
    return len(set(uuids)) == len(uuids)


__all__ = ["CTL_REGION", "PeerExchange", "control_region_bytes", "PeerMappingError", "RK_PEER_CTL_BYTES", "RK_PEER_MAX", "export_handle", "fused_path_available", "open_handle"]
