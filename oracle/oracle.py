"""numpy front-end of the C oracle (``rk_oracle.c``) -- TEST INFRASTRUCTURE ONLY.

Arrays of 16-bit values are passed as ``numpy.uint16`` bit patterns (the exact bits of
the fp16/bf16 tensors), so no conversion happens outside the C code.  Each call returns
``(rounded_uint16, fp32_sums)``.

Parity pinned by ``tests/test_oracle.py`` against ``tests/golden/*.npz``, which hold the
outputs of the reference's own functions (see ``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIBRARY = ORACLE_DIR / "_build" / "librk_oracle.so"
FP16, BF16 = 0, 1
_lib: ctypes.CDLL | None = None


def build() -> Path:
    """Compile the oracle with the committed Makefile (needs gcc; seconds)."""

    subprocess.run(["make", "-s", "-C", str(ORACLE_DIR)], check=True)
    return LIBRARY


def _library() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIBRARY.is_file():
            build()
        lib = ctypes.CDLL(str(LIBRARY))
        u16p, f32p, i64, cint = (
            np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS"),
            np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS"),
            ctypes.c_int64,
            ctypes.c_int,
        )
        lib.rk_oracle_gemm.argtypes = [u16p, u16p, u16p, f32p, f32p, i64, i64, i64, cint]
        lib.rk_oracle_gemm.restype = None
        lib.rk_oracle_gemv.argtypes = [u16p, u16p, u16p, f32p, f32p, i64, i64, i64, cint]
        lib.rk_oracle_gemv.restype = None
        lib.rk_oracle_round.argtypes = [f32p, u16p, i64, cint]
        lib.rk_oracle_round.restype = None
        lib.rk_oracle_widen.argtypes = [u16p, f32p, i64, cint]
        lib.rk_oracle_widen.restype = None
        f32 = ctypes.c_float
        lib.rk_oracle_silu_mul.argtypes = [u16p, u16p, u16p, f32p, i64, cint]
        lib.rk_oracle_silu_mul.restype = None
        lib.rk_oracle_rms_norm.argtypes = [u16p, u16p, u16p, f32p, f32p, i64, i64, f32, cint]
        lib.rk_oracle_rms_norm.restype = None
        lib.rk_oracle_add_rms_norm.argtypes = [u16p, u16p, u16p, u16p, u16p, f32p, f32p, i64, i64, f32, cint]
        lib.rk_oracle_add_rms_norm.restype = None
        f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
        lib.rk_oracle_silu_mul_backward.argtypes = [u16p, u16p, u16p, u16p, u16p, f32p, f32p, f32p, i64, cint]
        lib.rk_oracle_silu_mul_backward.restype = None
        lib.rk_oracle_rms_norm_backward.argtypes = [
            u16p, u16p, u16p, ctypes.c_void_p, u16p, f32p, f32p, u16p, f32p, f32p, f64p, i64, i64, f32, cint, cint,
        ]
        lib.rk_oracle_rms_norm_backward.restype = None
        _lib = lib
    return _lib


def _code(dtype: str) -> int:
    if dtype not in ("fp16", "bf16"):
        raise ValueError(f"unsupported dtype {dtype!r}")
    return BF16 if dtype == "bf16" else FP16


def gemm(a_bits: np.ndarray, b_bits: np.ndarray, dtype: str) -> tuple[np.ndarray, np.ndarray]:
    """C = A @ B on 16-bit bit patterns: A [M,K], B [K,N]."""

    a = np.ascontiguousarray(a_bits, dtype=np.uint16)
    b = np.ascontiguousarray(b_bits, dtype=np.uint16)
    (m, k), (k2, n) = a.shape, b.shape
    if k != k2:
        raise ValueError("inner dimensions differ")
    c = np.empty((m, n), np.uint16)
    acc = np.empty((m, n), np.float32)
    work = np.empty(k * n + k + 1, np.float32)
    _library().rk_oracle_gemm(a, b, c, acc, work, m, n, k, _code(dtype))
    return c, acc


def gemv(x_bits: np.ndarray, w_bits: np.ndarray, dtype: str) -> tuple[np.ndarray, np.ndarray]:
    """out = x @ W^T on 16-bit bit patterns: x [M,K], W [N,K]."""

    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    w = np.ascontiguousarray(w_bits, dtype=np.uint16)
    (m, k), (n, k2) = x.shape, w.shape
    if k != k2:
        raise ValueError("K dimensions differ")
    out = np.empty((m, n), np.uint16)
    acc = np.empty((m, n), np.float32)
    work = np.empty(2 * k + 1, np.float32)
    _library().rk_oracle_gemv(x, w, out, acc, work, m, n, k, _code(dtype))
    return out, acc


def gemm_swiglu(a_bits: np.ndarray, b_bits: np.ndarray, dtype: str) -> tuple[np.ndarray, np.ndarray]:
    """silu(A @ B[:, :N]) * (A @ B[:, N:]) from the fp32 sums (B [K, 2N]); returns (bits, fp32).

    The fused operator has no counterpart in the reference; its definition is the
    reference's two operators composed in fp32 -- the GEMM sums (as rk_oracle_gemm forms
    them) fed to silu_mul_reference's arithmetic (ops/swiglu/reference.py:6-9) before any
    rounding.
    """

    _, acc = gemm(a_bits, b_bits, dtype)
    n = acc.shape[1] // 2
    g, u = acc[:, :n], acc[:, n:]
    with np.errstate(over="ignore", invalid="ignore"):
        s = (np.float32(1) / (np.float32(1) + np.exp(-g))).astype(np.float32)
        out32 = ((g * s).astype(np.float32) * u).astype(np.float32)
    return round_to(out32, dtype), out32


def silu_mul(gate_bits: np.ndarray, up_bits: np.ndarray, dtype: str) -> tuple[np.ndarray, np.ndarray]:
    """silu(gate) * up on 16-bit bit patterns [tokens, hidden]; returns (bits, fp32 before rounding)."""

    g = np.ascontiguousarray(gate_bits, dtype=np.uint16)
    u = np.ascontiguousarray(up_bits, dtype=np.uint16)
    if g.shape != u.shape:
        raise ValueError("gate and up shapes differ")
    out = np.empty(g.shape, np.uint16)
    exact = np.empty(g.shape, np.float32)
    _library().rk_oracle_silu_mul(g.reshape(-1), u.reshape(-1), out.reshape(-1), exact.reshape(-1), g.size, _code(dtype))
    return out, exact


def rms_norm(x_bits: np.ndarray, w_bits: np.ndarray, eps: float, dtype: str) -> tuple[np.ndarray, np.ndarray]:
    """Row RMS normalisation of x [tokens, hidden] by weight [hidden]; returns (bits, fp32)."""

    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    w = np.ascontiguousarray(w_bits, dtype=np.uint16)
    tokens, hidden = x.shape
    out = np.empty(x.shape, np.uint16)
    exact = np.empty(x.shape, np.float32)
    work = np.empty(hidden + 1, np.float32)
    _library().rk_oracle_rms_norm(x, w, out, exact, work, tokens, hidden, eps, _code(dtype))
    return out, exact


def add_rms_norm(
    x_bits: np.ndarray, r_bits: np.ndarray, w_bits: np.ndarray, eps: float, dtype: str
) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """(rms_norm(x + residual), x + residual) on bit patterns; also the fp32 normalised values."""

    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    r = np.ascontiguousarray(r_bits, dtype=np.uint16)
    w = np.ascontiguousarray(w_bits, dtype=np.uint16)
    tokens, hidden = x.shape
    out = np.empty(x.shape, np.uint16)
    residual_out = np.empty(x.shape, np.uint16)
    exact = np.empty(x.shape, np.float32)
    work = np.empty(hidden + 1, np.float32)
    _library().rk_oracle_add_rms_norm(x, r, w, out, residual_out, exact, work, tokens, hidden, eps, _code(dtype))
    return out, residual_out, exact


def silu_mul_backward(dy_bits: np.ndarray, gate_bits: np.ndarray, up_bits: np.ndarray, dtype: str) -> dict[str, np.ndarray]:
    """Gradients of silu(gate) * up (reference autograd order); bits, fp32 values and term scales."""

    dy, g, u = (np.ascontiguousarray(a, dtype=np.uint16) for a in (dy_bits, gate_bits, up_bits))
    if not (dy.shape == g.shape == u.shape):
        raise ValueError("dy, gate and up shapes differ")
    out = {
        "grad_gate": np.empty(g.shape, np.uint16),
        "grad_up": np.empty(g.shape, np.uint16),
        "grad_gate_fp32": np.empty(g.shape, np.float32),
        "grad_up_fp32": np.empty(g.shape, np.float32),
        "grad_gate_scale": np.empty(g.shape, np.float32),
    }
    _library().rk_oracle_silu_mul_backward(
        dy.reshape(-1), g.reshape(-1), u.reshape(-1), out["grad_gate"].reshape(-1), out["grad_up"].reshape(-1),
        out["grad_gate_fp32"].reshape(-1), out["grad_up_fp32"].reshape(-1), out["grad_gate_scale"].reshape(-1),
        g.size, _code(dtype),
    )
    out["grad_up_scale"] = np.abs(out["grad_up_fp32"])
    return out


def _norm_backward(dy_bits, x_bits, w_bits, dres_bits, eps: float, add: bool, dtype: str) -> dict[str, np.ndarray]:
    dy = np.ascontiguousarray(dy_bits, dtype=np.uint16)
    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    w = np.ascontiguousarray(w_bits, dtype=np.uint16)
    tokens, hidden = x.shape
    if dy.shape != x.shape or w.shape != (hidden,):
        raise ValueError("shapes of dy, x and weight do not match")
    dres = None if dres_bits is None else np.ascontiguousarray(dres_bits, dtype=np.uint16)
    out = {
        "grad_x": np.empty(x.shape, np.uint16),
        "grad_x_fp32": np.empty(x.shape, np.float32),
        "grad_x_scale": np.empty(x.shape, np.float32),
        "grad_weight": np.empty(hidden, np.uint16),
        "grad_weight_fp32": np.empty(hidden, np.float32),
        "grad_weight_scale": np.empty(hidden, np.float32),
    }
    work = np.empty(2 * hidden, np.float64)
    lib_call = _library().rk_oracle_rms_norm_backward
    lib_call(
        dy, x, w, None if dres is None else dres.ctypes.data_as(ctypes.c_void_p), out["grad_x"], out["grad_x_fp32"],
        out["grad_x_scale"], out["grad_weight"], out["grad_weight_fp32"], out["grad_weight_scale"], work,
        tokens, hidden, eps, 1 if add else 0, _code(dtype),
    )
    if add and dres is not None:
        # add_rms_norm rounds twice: round(round(dx) + dres).  One representable step of
        # the intermediate round(dx) -- an allowed difference on its own -- survives the
        # second rounding and, where dx and dres cancel, spans several steps of the result.
        dx_only = _norm_backward(dy_bits, x_bits, w_bits, None, eps, False, dtype)["grad_x"]
        out["grad_x_intermediate"] = np.abs(widen(dx_only, dtype))
    return out


def rms_norm_backward(dy_bits, x_bits, w_bits, eps: float, dtype: str) -> dict[str, np.ndarray]:
    """Gradients of rms_norm(x, weight) for the output gradient dy (reference autograd order)."""

    return _norm_backward(dy_bits, x_bits, w_bits, None, eps, False, dtype)


def add_rms_norm_backward(dy_bits, dres_bits, residual_out_bits, w_bits, eps: float, dtype: str) -> dict[str, np.ndarray]:
    """Gradients of add_rms_norm from the saved residual_out: grad_x (= the residual's gradient)
    and grad_weight; dres_bits is the residual_out gradient, or None when none flows."""

    return _norm_backward(dy_bits, residual_out_bits, w_bits, dres_bits, eps, True, dtype)


# Gradients: elementwise expressions whose terms can cancel (silu_mul's dgate at
# g ~ -1.28, rms_norm's dx where its two terms meet) and fp32 sums over a row or over the
# rows (rms_norm's c and dw) whose order differs between implementations.  The gate per
# element: NaN exactly where the reference has NaN; otherwise at most one representable
# step from the reference's rounded gradient, or -- where the value is much smaller than
# the terms that formed it -- within GRADIENT_REL x (the sum of the terms' magnitudes)
# plus one step of the value.  A wrong formula misses by a large fraction of the terms.
GRADIENT_REL = 2.0**-14
_STEP = {"bf16": 2.0**-7, "fp16": 2.0**-10}


def assert_gradient(
    result_bits, ref_bits, ref_fp32, ref_scale, dtype: str, rel: float = GRADIENT_REL, intermediate=None
) -> dict[str, float]:
    """Raise AssertionError unless a 16-bit gradient passes the gate above.  `intermediate`:
    magnitudes of a value rounded to the dtype before the last operation (one step of it
    is allowed as well)."""

    result = np.asarray(result_bits, np.uint16)
    ref = np.asarray(ref_bits, np.uint16)
    if result.shape != ref.shape:
        raise AssertionError(f"shape {result.shape} != {ref.shape}")
    nan_r, nan_ref = _is_nan(result, dtype), _is_nan(ref, dtype)
    if not np.array_equal(nan_r, nan_ref):
        raise AssertionError(f"NaN positions differ at {np.argwhere(nan_r != nan_ref)[:5].tolist()}")
    keep = ~nan_ref
    steps = ulp_distance(result[keep], ref[keep])
    value = widen(result[keep], dtype).astype(np.float64)
    ref32 = np.asarray(ref_fp32, np.float64)[keep]
    scale = np.asarray(ref_scale, np.float64)[keep]
    with np.errstate(invalid="ignore"):
        allowed = rel * scale + _STEP[dtype] * np.abs(ref32)
        if intermediate is not None:
            allowed = allowed + _STEP[dtype] * np.asarray(intermediate, np.float64)[keep]
        close = np.abs(value - ref32) <= allowed
    ok = (steps <= 1) | close
    if not ok.all():
        i = int(np.argmin(ok))
        where = np.argwhere(keep)[i].tolist()
        raise AssertionError(
            f"gradient at {where}: {value[i]!r} vs reference {ref32[i]!r} ({int(steps[i])} steps, "
            f"terms of magnitude {scale[i]:.3e})"
        )
    return {"max_steps": float(steps.max(initial=0)), "within_one_step": float(np.mean(steps <= 1)) if steps.size else 1.0}


def paged_attention_decode(
    q_bits: np.ndarray,
    k_bits: np.ndarray,
    v_bits: np.ndarray,
    block_tables: np.ndarray,
    context_lengths: np.ndarray,
    scale: float,
    dtype: str,
) -> tuple[np.ndarray, np.ndarray]:
    """Decode attention over a paged K/V cache; returns (bits, fp32 before rounding).

    Restates paged_attention_decode_reference (src/radeon_kernels/ops/paged_attention/
    reference.py:8-47) in numpy fp32: positions t < context_length map to cache slot
    block_tables[b, t // block_size] * block_size + t % block_size; query head h reads KV head
    h // (query_heads // kv_heads); scores q . k * scale, softmax with the maximum
    subtracted, probabilities times V.  A sequence with no position gives NaN (the
    reference's softmax of an all -inf row).
    """

    q = widen(q_bits, dtype)
    k = widen(k_bits, dtype)
    v = widen(v_bits, dtype)
    batch, heads, head_dim = q.shape
    _, block_size, kv_heads, _ = k.shape
    group = heads // kv_heads
    max_ctx = block_tables.shape[1] * block_size
    out = np.empty((batch, heads, head_dim), np.float32)
    sc = np.float32(scale)
    for b in range(batch):
        ctx = int(min(max(int(context_lengths[b]), 0), max_ctx))
        if ctx == 0:
            out[b] = np.nan
            continue
        t = np.arange(ctx)
        blocks = np.asarray(block_tables[b], np.int64)[t // block_size]
        keys = k[blocks, t % block_size]  # [ctx, kv_heads, head_dim]
        values = v[blocks, t % block_size]
        for h in range(heads):
            kvh = h // group
            scores = (keys[:, kvh, :] @ q[b, h]).astype(np.float32) * sc
            e = np.exp(scores - scores.max()).astype(np.float32)
            p = (e / e.sum(dtype=np.float32)).astype(np.float32)
            out[b, h] = (p @ values[:, kvh, :]).astype(np.float32)
    return round_to(out, dtype), out


def sdpa(q_bits: np.ndarray, k_bits: np.ndarray, v_bits: np.ndarray, is_causal: bool, scale: float, dtype: str) -> tuple[np.ndarray, np.ndarray]:
    """Self-attention over [batch, heads, sequence, head_dim]; returns (bits, fp32 before rounding).

    Restates sdpa_reference (src/radeon_kernels/ops/sdpa/reference.py:13-36) in numpy fp32:
    K and V expanded to the query heads (query head h reads KV head h // (Hq // Hkv)),
    scores = (Q K^T) * scale, keys after the query masked with -inf when causal, softmax in
    fp32 with the row maximum subtracted, probabilities times V, one rounding.
    """

    q = widen(q_bits, dtype)
    k = widen(k_bits, dtype)
    v = widen(v_bits, dtype)
    batch, heads, seq, _ = q.shape
    group = heads // k.shape[1]
    out = np.empty(q.shape, np.float32)
    sc = np.float32(scale)
    mask = np.triu(np.ones((seq, seq), dtype=bool), 1) if is_causal else None
    for b in range(batch):
        for h in range(heads):
            kvh = h // group
            scores = (q[b, h] @ k[b, kvh].T).astype(np.float32) * sc
            if mask is not None:
                scores = np.where(mask, np.float32(-np.inf), scores)
            with np.errstate(invalid="ignore"):
                e = np.exp(scores - scores.max(axis=1, keepdims=True)).astype(np.float32)
                p = (e / e.sum(axis=1, keepdims=True, dtype=np.float32)).astype(np.float32)
            out[b, h] = (p @ v[b, kvh]).astype(np.float32)
    return round_to(out, dtype), out


def assert_attention(
    result_bits: np.ndarray, ref_bits: np.ndarray, ref_fp32: np.ndarray, dtype: str, rounded_p: bool = False
) -> dict[str, float]:
    """NaN exactly where the reference has NaN; the GEMM parity gate on the rest.

    Attention outputs are fp32 sums over the context (q.k, then p.V) whose order differs
    between implementations, like a GEMM's, so the finite part gets assert_parity.
    rounded_p: the implementation rounds the probabilities to the dtype before the p.V
    product (tensor-core flash attention, as torch's flash SDPA does); each p then carries
    up to half a step of relative error, which moves small outputs by more than one step,
    so only the relative-to-max part of the gate (TOLERANCE) applies.
    """

    result = np.asarray(result_bits, np.uint16)
    ref = np.asarray(ref_bits, np.uint16)
    nan_r, nan_ref = _is_nan(result, dtype), _is_nan(ref, dtype)
    if not np.array_equal(nan_r, nan_ref):
        raise AssertionError(f"NaN positions differ at {np.argwhere(nan_r != nan_ref)[:5].tolist()}")
    keep = ~nan_ref
    if not keep.any():
        return {"parity_error": 0.0}
    if rounded_p:
        summary = compare(result[keep], ref[keep], np.asarray(ref_fp32)[keep], dtype)
        assert summary["parity"] <= TOLERANCE[dtype], f"parity {summary['parity']:.3e} > {TOLERANCE[dtype]} ({dtype})"
        return summary
    return assert_parity(result[keep], ref[keep], np.asarray(ref_fp32)[keep], dtype)


def widen(bits: np.ndarray, dtype: str) -> np.ndarray:
    src = np.ascontiguousarray(bits, dtype=np.uint16)
    dst = np.empty(src.shape, np.float32)
    _library().rk_oracle_widen(src.reshape(-1), dst.reshape(-1), src.size, _code(dtype))
    return dst


def round_to(values: np.ndarray, dtype: str) -> np.ndarray:
    src = np.ascontiguousarray(values, dtype=np.float32)
    dst = np.empty(src.shape, np.uint16)
    _library().rk_oracle_round(src.reshape(-1), dst.reshape(-1), src.size, _code(dtype))
    return dst


def parity_error(result: np.ndarray, reference: np.ndarray) -> float:
    """The north-star metric max|C - C_ref| / max|C_ref| (fp64 arithmetic)."""

    result = np.asarray(result, np.float64)
    reference = np.asarray(reference, np.float64)
    scale = float(np.max(np.abs(reference))) if reference.size else 0.0
    if reference.size == 0:
        return 0.0
    diff = float(np.max(np.abs(result - reference)))
    return diff / scale if scale > 0 else diff


# Tolerances of the parity gate, by output dtype (max|C - C_ref| / max|C_ref|).
TOLERANCE = {"bf16": 4e-3, "fp16": 1e-3}


def ulp_distance(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """Distance in representable steps between two arrays of 16-bit float bit patterns."""

    def ordered(bits: np.ndarray) -> np.ndarray:
        v = np.asarray(bits, np.int32)
        return np.where(v & 0x8000, 0x8000 - (v & 0x7FFF), 0x8000 + (v & 0x7FFF))

    return np.abs(ordered(a_bits) - ordered(b_bits))


def _is_nan(bits: np.ndarray, dtype: str) -> np.ndarray:
    v = np.asarray(bits, np.uint16)
    if dtype == "bf16":
        return ((v & 0x7F80) == 0x7F80) & ((v & 0x007F) != 0)
    return ((v & 0x7C00) == 0x7C00) & ((v & 0x03FF) != 0)


# Elementwise and row-normalisation operators (silu_mul, rms_norm, add_rms_norm): every
# output is a short fp32 expression of its inputs -- no long cancelling sum -- so the gate
# is per element: NaN exactly where the reference has NaN (any sign or payload), and at
# most one representable step from the reference's rounded value everywhere else.  One
# step covers the last-bit differences between libm implementations of exp (sigmoid) and
# between fp32 summation orders of the squares (RMS); it is below the reference
# contracts' atol/rtol of 0.01 (contracts/swiglu-1.0.json, add_rms_norm-1.0.json).
ELEMENTWISE_MAX_ULP = 1


def assert_elementwise(result_bits: np.ndarray, ref_bits: np.ndarray, dtype: str, max_ulp: int = ELEMENTWISE_MAX_ULP) -> int:
    """Raise AssertionError unless result matches ref per element (see above); returns the max step."""

    result = np.asarray(result_bits, np.uint16)
    ref = np.asarray(ref_bits, np.uint16)
    if result.shape != ref.shape:
        raise AssertionError(f"shape {result.shape} != {ref.shape}")
    nan_r, nan_ref = _is_nan(result, dtype), _is_nan(ref, dtype)
    if not np.array_equal(nan_r, nan_ref):
        raise AssertionError(f"NaN positions differ at {np.argwhere(nan_r != nan_ref)[:5].tolist()}")
    if result.size == 0 or nan_ref.all():
        return 0
    steps = ulp_distance(result[~nan_ref], ref[~nan_ref])
    worst = int(steps.max())
    if worst > max_ulp:
        where = np.argwhere(~nan_ref)[int(np.argmax(steps))].tolist()
        raise AssertionError(f"{worst} steps from the reference at {where} (max {max_ulp})")
    return worst


def compare(result_bits: np.ndarray, ref_bits: np.ndarray, ref_fp32: np.ndarray, dtype: str) -> dict[str, float]:
    """Parity summary of a 16-bit result against the reference's rounded and fp32 outputs.

    * ``parity``    -- max|C - C_ref32| / max|C_ref32| (the gate, TOLERANCE[dtype]);
    * ``max_steps`` -- largest distance in representable steps from the reference's rounded
      output over the elements with |C_ref| >= max|C_ref| / 64 (smaller elements are
      dominated by cancellation, where the fp32 summation order alone moves the result
      by several steps);
    * ``equal``     -- fraction of elements bit-identical to the reference's output.
    """

    if ref_bits.size == 0:
        return {"parity": 0.0, "max_steps": 0.0, "equal": 1.0}
    ref32 = np.asarray(ref_fp32, np.float32)
    big = np.abs(ref32) >= np.abs(ref32).max() / 64
    steps = ulp_distance(result_bits, ref_bits)
    return {
        "parity": parity_error(widen(result_bits, dtype), ref32),
        "max_steps": float(steps[big].max(initial=0)),
        "equal": float(np.mean(np.asarray(result_bits) == np.asarray(ref_bits))),
    }


def assert_parity(result_bits: np.ndarray, ref_bits: np.ndarray, ref_fp32: np.ndarray, dtype: str) -> dict[str, float]:
    summary = compare(result_bits, ref_bits, ref_fp32, dtype)
    assert summary["parity"] <= TOLERANCE[dtype], f"parity {summary['parity']:.3e} > {TOLERANCE[dtype]} ({dtype})"
    assert summary["max_steps"] <= 1, f"{summary['max_steps']} representable steps from the reference"
    return summary
