"""The CPU oracle, pinned against fixtures produced by the reference's own functions."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden_cases
from oracle import oracle


def _load(path):
    data = np.load(path)
    return {key: data[key] for key in data.files}


@pytest.mark.parametrize("path", golden_cases("gemm"), ids=lambda p: p.stem)
def test_oracle_gemm_matches_reference_fixtures(path):
    case = _load(path)
    dtype = str(case["dtype"])
    c, acc = oracle.gemm(case["a"], case["b"], dtype)
    # fp32 sums agree with the reference's fp32 product up to accumulation order.
    np.testing.assert_allclose(acc, case["c_fp32"], rtol=0, atol=2e-5 * max(1.0, np.abs(case["c_fp32"]).max()))
    # Rounded outputs: the reference's torch.mm result, to at most one representable step
    # on every element not dominated by cancellation, and within the parity gate.
    oracle.assert_parity(c, case["c_ref"], case["c_fp32"], dtype)


@pytest.mark.parametrize("path", golden_cases("gemv"), ids=lambda p: p.stem)
def test_oracle_gemv_matches_reference_fixtures(path):
    case = _load(path)
    dtype = str(case["dtype"])
    out, acc = oracle.gemv(case["x"], case["w"], dtype)
    np.testing.assert_allclose(acc, case["out_fp32"], rtol=0, atol=2e-5 * max(1.0, np.abs(case["out_fp32"]).max()))
    oracle.assert_parity(out, case["out_reference"], case["out_fp32"], dtype)
    oracle.assert_parity(out, case["out_fallback"], case["out_fp32"], dtype)


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_conversions_round_trip_every_finite_pattern(dtype):
    bits = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    wide = oracle.widen(bits, dtype)
    back = oracle.round_to(wide, dtype)
    finite = np.isfinite(wide)
    assert np.array_equal(back[finite], bits[finite])
    assert np.all(np.isnan(oracle.widen(back[np.isnan(wide)], dtype)))


def test_rounding_is_nearest_even_against_numpy_fp16():
    rng = np.random.default_rng(7)
    values = np.concatenate(
        [
            rng.standard_normal(200_000).astype(np.float32) * 1000,
            rng.standard_normal(50_000).astype(np.float32) * 1e-5,  # subnormal range of fp16
            np.array([65504.0, 65520.0, 65519.996, 6e-8, 3e-8, 2.98e-8, -0.0, 1e9], np.float32),
        ]
    )
    ours = oracle.round_to(values, "fp16")
    with np.errstate(over="ignore"):
        expected = values.astype(np.float16).view(np.uint16)
    assert np.array_equal(ours, expected)


def test_parity_check_detects_a_planted_error():
    # The mistake is planted in the oracle's own inputs on the CPU: one flipped mantissa
    # bit of one A element must push the metric past the tolerance against the fixture.
    case = _load(golden_cases("gemm_bf16_64x96x128")[0])
    a = case["a"].copy()
    a[5, 7] ^= np.uint16(0x0040)
    c, _ = oracle.gemm(a, case["b"], "bf16")
    assert oracle.ulp_distance(c, case["c_ref"]).max() > 1
    a = case["a"].copy()
    a[5] = 0x3F80  # a whole row set to 1.0
    c, _ = oracle.gemm(a, case["b"], "bf16")
    assert oracle.parity_error(oracle.widen(c, "bf16"), case["c_fp32"]) > oracle.TOLERANCE["bf16"]


def test_parity_metric_definition():
    ref = np.array([[1.0, -4.0], [2.0, 0.5]])
    assert oracle.parity_error(ref, ref) == 0.0
    assert oracle.parity_error(ref + 0.04, ref) == pytest.approx(0.01)


# ------------------------------------------------------------ decode neighbours


@pytest.mark.parametrize("path", golden_cases("silu"), ids=lambda p: p.stem)
def test_oracle_silu_mul_matches_reference_fixtures(path):
    case = _load(path)
    out, exact = oracle.silu_mul(case["gate"], case["up"], case["dtype"])
    oracle.assert_elementwise(out, case["out_ref"], case["dtype"])
    finite = np.isfinite(case["out_fp32"])
    np.testing.assert_allclose(exact[finite], case["out_fp32"][finite], rtol=2e-6, atol=0)


@pytest.mark.parametrize("path", golden_cases("rms"), ids=lambda p: p.stem)
def test_oracle_rms_norm_matches_reference_fixtures(path):
    case = _load(path)
    out, exact = oracle.rms_norm(case["x"], case["weight"], float(case["eps"]), case["dtype"])
    oracle.assert_elementwise(out, case["out_ref"], case["dtype"])
    np.testing.assert_allclose(exact, case["out_fp32"], rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("path", golden_cases("add_rms"), ids=lambda p: p.stem)
def test_oracle_add_rms_norm_matches_reference_fixtures(path):
    case = _load(path)
    out, residual_out, exact = oracle.add_rms_norm(
        case["x"], case["residual"], case["weight"], float(case["eps"]), case["dtype"]
    )
    assert np.array_equal(residual_out, case["residual_out_ref"])  # one rounded add: bit-exact
    oracle.assert_elementwise(out, case["out_ref"], case["dtype"])
    np.testing.assert_allclose(exact, case["out_fp32"], rtol=2e-6, atol=1e-7)


def test_elementwise_gate_detects_a_planted_error():
    case = _load(golden_cases("rms_bf16_t4")[0])
    out, _ = oracle.rms_norm(case["x"], case["weight"], float(case["eps"]), case["dtype"])
    planted = out.copy()
    planted[1, 7] += 2  # two representable steps
    with pytest.raises(AssertionError):
        oracle.assert_elementwise(planted, case["out_ref"], case["dtype"])
    nan = out.copy()
    nan[0, 0] = 0x7FC0  # a NaN where the reference is finite
    with pytest.raises(AssertionError):
        oracle.assert_elementwise(nan, case["out_ref"], case["dtype"])


@pytest.mark.parametrize("path", golden_cases("paged"), ids=lambda p: p.stem)
def test_oracle_paged_attention_matches_reference_fixtures(path):
    case = _load(path)
    dtype = str(case["dtype"])
    out, out32 = oracle.paged_attention_decode(
        case["q"], case["k"], case["v"], case["block_tables"], case["context_lengths"], float(case["scale"]), dtype
    )
    oracle.assert_attention(out, case["out_ref"], out32, dtype)


@pytest.mark.parametrize("path", golden_cases("sdpa"), ids=lambda p: p.stem)
def test_oracle_sdpa_matches_reference_fixtures(path):
    case = _load(path)
    dtype = str(case["dtype"])
    out, out32 = oracle.sdpa(case["q"], case["k"], case["v"], bool(case["is_causal"]), float(case["scale"]), dtype)
    oracle.assert_attention(out, case["out_ref"], out32, dtype)


@pytest.mark.parametrize("path", golden_cases("sdpa"), ids=lambda p: p.stem)
def test_reference_path_sdpa_reproduces_the_reference_bits(path):
    """oracle.reference_path.sdpa_reference (the contract's reference entrypoint) on CPU gives
    the reference function's own output bit for bit."""

    import torch

    from oracle import reference_path

    case = _load(path)
    dt = {"bf16": torch.bfloat16, "fp16": torch.float16}[str(case["dtype"])]
    t = lambda bits: torch.from_numpy(bits.view(np.int16).copy()).view(dt)  # noqa: E731
    out = reference_path.sdpa_reference(torch, t(case["q"]), t(case["k"]), t(case["v"]), bool(case["is_causal"]), float(case["scale"]))
    assert np.array_equal(out.view(torch.int16).numpy().view(np.uint16), case["out_ref"])


# ----------------------------------------------------------------- gradients
@pytest.mark.parametrize("path", golden_cases("grad_silu"), ids=lambda p: p.stem)
def test_oracle_silu_mul_backward_matches_reference_autograd(path):
    case = _load(path)
    dt = str(case["dtype"])
    got = oracle.silu_mul_backward(case["dy"], case["gate"], case["up"], dt)
    oracle.assert_gradient(got["grad_gate"], case["grad_gate_ref"], got["grad_gate_fp32"], got["grad_gate_scale"], dt)
    oracle.assert_gradient(got["grad_up"], case["grad_up_ref"], got["grad_up_fp32"], got["grad_up_scale"], dt)


@pytest.mark.parametrize("path", golden_cases("grad_rms"), ids=lambda p: p.stem)
def test_oracle_rms_norm_backward_matches_reference_autograd(path):
    case = _load(path)
    dt = str(case["dtype"])
    got = oracle.rms_norm_backward(case["dy"], case["x"], case["weight"], float(case["eps"]), dt)
    oracle.assert_gradient(got["grad_x"], case["grad_x_ref"], got["grad_x_fp32"], got["grad_x_scale"], dt)
    oracle.assert_gradient(
        got["grad_weight"], case["grad_weight_ref"], got["grad_weight_fp32"], got["grad_weight_scale"], dt
    )


@pytest.mark.parametrize("path", golden_cases("grad_add_rms"), ids=lambda p: p.stem)
def test_oracle_add_rms_norm_backward_matches_reference_autograd(path):
    case = _load(path)
    dt = str(case["dtype"])
    dres = case.get("dres")
    got = oracle.add_rms_norm_backward(case["dy"], dres, case["residual_out"], case["weight"], float(case["eps"]), dt)
    oracle.assert_gradient(got["grad_x"], case["grad_x_ref"], got["grad_x_fp32"], got["grad_x_scale"], dt)
    # both inputs of the add receive the same gradient
    assert np.array_equal(case["grad_x_ref"], case["grad_residual_ref"])
    oracle.assert_gradient(
        got["grad_weight"], case["grad_weight_ref"], got["grad_weight_fp32"], got["grad_weight_scale"], dt
    )


def test_gradient_gate_detects_planted_errors():
    case = _load(golden_cases("grad_rms_bf16_t4")[0])
    got = oracle.rms_norm_backward(case["dy"], case["x"], case["weight"], float(case["eps"]), "bf16")
    # An error of 1 % of the terms' magnitude (what a wrong term in the formula gives),
    # planted in the oracle's own output.
    wrong = oracle.round_to(got["grad_x_fp32"] + 0.01 * got["grad_x_scale"], "bf16")
    with pytest.raises(AssertionError):
        oracle.assert_gradient(wrong, case["grad_x_ref"], got["grad_x_fp32"], got["grad_x_scale"], "bf16")
    two_steps = got["grad_weight"].copy()
    two_steps[5] += 2
    with pytest.raises(AssertionError):
        oracle.assert_gradient(
            two_steps, case["grad_weight_ref"], got["grad_weight_fp32"], got["grad_weight_scale"], "bf16"
        )


def test_silu_backward_specials_follow_the_reference():
    """inf / -inf / NaN gates give NaN gradients where the reference's graph does, and the
    saturated ends of the sigmoid give the reference's zeros and signs."""

    case = _load(golden_cases("grad_silu_bf16_t8")[0])
    got = oracle.silu_mul_backward(case["dy"], case["gate"], case["up"], "bf16")
    for key in ("grad_gate", "grad_up"):
        mine, ref = got[key][0, :8], case[f"{key}_ref"][0, :8]
        nan = oracle._is_nan(ref, "bf16")
        assert np.array_equal(oracle._is_nan(mine, "bf16"), nan)  # NaN payloads may differ
        assert np.array_equal(mine[~nan], ref[~nan])
