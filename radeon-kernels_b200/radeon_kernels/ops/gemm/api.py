"""Public GEMM: ``rk.gemm(a, b, *, out=None)`` computes ``a @ b`` on the GPU.

Drop-in for the reference's ``radeon_kernels.ops.gemm`` (src/radeon_kernels/ops/gemm/api.py):

* same validation, order and messages (api.py:56-101): rank-2 CUDA tensors on one device,
  one dtype (fp16/bf16), matching inner dimension, and a contiguous ``out`` of shape
  ``(m, n)`` with the input's device and dtype -- all checked before any dispatch;
* same dispatch signature ``{dtype, layout: "nn", m, n, k, contiguous, requires_grad}``;
* same control flow (api.py:158-237): exact-match manifest entry -> pack -> verified
  ``gemm_out(a, b, out, variant)`` writing into the caller's (or a new) output; any
  winner failure falls to the declared fallback with the reason recorded.

The fallback is this library's ``cuda`` provider (tcgen05 or generic CUDA kernel), never
``torch.mm``.  Autograd inputs never take an inference-only winner (the manifests pin
``requires_grad: false``) and run the fallback's differentiable path.
"""

from __future__ import annotations

from dataclasses import dataclass
from threading import Lock
from typing import Any

from radeon_kernels.errors import RadeonKernelsError
from radeon_kernels.ops._common import dtype_name, device_index_of
from radeon_kernels.ops._runtime import WINNER_FAILURES, DispatchingRuntime, record_execution
from radeon_kernels.runtime.explain import record_dispatch_shared
from radeon_kernels.providers import cuda_builtin, native

_SEMANTIC_VERSION = "1.0"


class GemmDispatchError(RadeonKernelsError):
    """Neither an approved GEMM winner nor a fallback can execute."""


@dataclass(frozen=True)
class _GemmCall:
    a: Any
    b: Any
    output: Any | None
    signature: dict[str, str | int | bool]
    device_index: int


def _torch() -> Any:
    try:
        import torch
    except ImportError as error:
        raise GemmDispatchError("GEMM requires a CUDA PyTorch installation") from error
    return torch


def _validate_call(torch_module: Any, a: Any, b: Any, output: Any | None) -> _GemmCall:
    tensor = getattr(torch_module, "Tensor", ())
    if not isinstance(a, tensor) or not isinstance(b, tensor):
        raise TypeError("gemm inputs must be PyTorch tensors")
    if a.dim() != 2 or b.dim() != 2:
        raise ValueError("gemm inputs must be rank-2 matrices")
    if not a.is_cuda or not b.is_cuda:
        raise ValueError("gemm inputs must be on a visible CUDA GPU")
    if a.device != b.device:
        raise ValueError("gemm inputs must be on the same device")
    if a.dtype != b.dtype:
        raise TypeError("gemm inputs must have the same dtype")
    if a.shape[1] != b.shape[0]:
        raise ValueError("gemm inner dimensions must match")
    dtype = dtype_name(torch_module, a.dtype, "gemm")
    m, k = (int(v) for v in a.shape)
    n = int(b.shape[1])
    if output is not None:
        if not isinstance(output, tensor):
            raise TypeError("gemm output must be a PyTorch tensor")
        if tuple(output.shape) != (m, n):
            raise ValueError(f"gemm output must have shape {(m, n)}")
        if output.device != a.device or output.dtype != a.dtype:
            raise ValueError("gemm output must match the input device and dtype")
        if not output.is_contiguous():
            raise ValueError("gemm output must be contiguous")
    return _GemmCall(
        a=a,
        b=b,
        output=output,
        signature={
            "dtype": dtype,
            "layout": "nn",
            "m": m,
            "n": n,
            "k": k,
            "contiguous": bool(a.is_contiguous() and b.is_contiguous()),
            "requires_grad": bool(a.requires_grad or b.requires_grad),
        },
        device_index=device_index_of(torch_module, a),
    )


class GemmRuntime(DispatchingRuntime):
    def execute(self, a: Any, b: Any, *, output: Any | None = None, torch_module: Any | None = None) -> Any:
        torch_runtime = torch_module or _torch()
        call = _validate_call(torch_runtime, a, b, output)
        key = self.fast_key("gemm", call.device_index, call.signature)
        cached = self.fast_lookup(key)
        if cached is not None:
            entry, variant, record = cached
            target = call.output
            if target is None:
                target = call.a.new_empty((call.signature["m"], call.signature["n"]))
            result = entry(call.a, call.b, target, variant)
            if result is None or (hasattr(result, "data_ptr") and result.data_ptr() != target.data_ptr()):
                raise native.NativeProviderError("native GEMM did not return the caller-provided output")
            record_dispatch_shared(record)
            return result
        fingerprint = self.fingerprint(torch_runtime, call.device_index)
        decision = self.decide("gemm", _SEMANTIC_VERSION, call.signature, fingerprint)
        failure: str | None = None
        if decision.matched:
            try:
                resolved = self.resolve(decision, fingerprint)
                target = call.output
                if target is None:
                    target = call.a.new_empty((call.signature["m"], call.signature["n"]))
                loader = self.loader(resolved.pack.root)
                result = native.gemm(loader, resolved.load_spec, decision.launch, call.a, call.b, target)
                reason = f"{decision.reason}; loaded pack {resolved.pack.pack_id} {resolved.pack.pack_version}"
                record_execution(
                    decision,
                    selected=f"{decision.winner.provider}/{decision.winner.entrypoint}",
                    artifact=decision.winner.artifact,
                    evidence_id=decision.evidence_id,
                    reason=reason,
                )
                entry = loader.load_entrypoint(resolved.load_spec).callable
                self.fast_store(key, entry, decision.launch["variant"], decision, reason)
                return result
            except WINNER_FAILURES as error:
                failure = str(error)
        return self.run_fallback(
            decision,
            failure,
            lambda: self.cuda_provider.gemm(torch_runtime, call.a, call.b, call.output),
            cuda_builtin.SELECTED_GEMM,
            GemmDispatchError,
            "no approved GEMM implementation is available",
        )


_DEFAULT_RUNTIME: GemmRuntime | None = None
_DEFAULT_RUNTIME_LOCK = Lock()


def _default_runtime() -> GemmRuntime:
    global _DEFAULT_RUNTIME
    if _DEFAULT_RUNTIME is None:
        with _DEFAULT_RUNTIME_LOCK:
            if _DEFAULT_RUNTIME is None:
                _DEFAULT_RUNTIME = GemmRuntime()
    return _DEFAULT_RUNTIME


def reset_runtime() -> None:
    """Reload dispatch manifests and installed packs before the next public GEMM call."""

    global _DEFAULT_RUNTIME
    with _DEFAULT_RUNTIME_LOCK:
        _DEFAULT_RUNTIME = None


def gemm(a: Any, b: Any, *, out: Any | None = None) -> Any:
    """Compute ``a @ b`` with the published sm_100a winner or the built-in CUDA kernels."""

    return _default_runtime().execute(a, b, output=out)


__all__ = ["GemmDispatchError", "GemmRuntime", "gemm", "reset_runtime"]
