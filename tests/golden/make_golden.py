"""Generate the golden parity fixtures from the reference's own functions.

Run in a container where the reference source tree is available (it is not on the GPU
boxes; the fixtures it writes are committed):

    python tests/golden/make_golden.py --reference-src <path to reference>/src

For every case the inputs are drawn exactly as BASELINE.json describes (fp32 from a
seeded ``torch.Generator``, then cast to the 16-bit dtype) and the outputs are produced
by calling the reference package itself:

* GEMM:  ``radeon_kernels.providers.torch_fallback.gemm(torch, a, b)``  (torch_fallback.py:6-9)
* GEMV:  ``radeon_kernels.ops.gemv.reference.gemv_fallback`` and ``gemv_reference``
  (ops/gemv/reference.py:6-15)
* paged decode attention: ``ops.paged_attention.reference.paged_attention_decode_reference``
  (paged_attention/reference.py:8-47)
* self-attention: ``ops.sdpa.reference.sdpa_reference`` (sdpa/reference.py:13-36), inputs
  drawn U[-0.125, 0.125) as the reference's SDPA benchmark draws them (benchmark.py:75-78)
* SwiGLU, RMSNorm, residual add + RMSNorm (the decode neighbours):
  ``ops.swiglu.reference.silu_mul_reference`` (swiglu/reference.py:6-9),
  ``ops.rms_norm.reference.rms_norm_reference`` (rms_norm/reference.py:6-10),
  ``ops.add_rms_norm.reference.add_rms_norm_reference`` (add_rms_norm/reference.py:8-12)
* gradients of those three (``grad_*`` fixtures): torch autograd run through the same
  reference functions, which is how the reference serves inputs that require gradients

plus the fp32 values before the final rounding.  16-bit arrays are stored as uint16 bit
patterns.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

# name, dtype, M, N, K, seed, distribution
GEMM_CASES = [
    ("gemm_bf16_64x96x128_uniform", "bf16", 64, 96, 128, 0, "uniform"),
    ("gemm_fp16_64x96x128_normal64", "fp16", 64, 96, 128, 3, "normal64"),
    ("gemm_bf16_7x13x5_ragged", "bf16", 7, 13, 5, 10, "uniform"),
    ("gemm_fp16_130x264x72_ragged_tiles", "fp16", 130, 264, 72, 11, "normal64"),
    ("gemm_bf16_200x520x136_ragged_tiles", "bf16", 200, 520, 136, 12, "uniform16"),
    ("gemm_bf16_1x8x8_tiny", "bf16", 1, 8, 8, 13, "uniform"),
    ("gemm_fp16_3x5x0_empty_k", "fp16", 3, 5, 0, 14, "uniform"),
    ("gemm_bf16_64x128x1024_k_deep", "bf16", 64, 128, 1024, 0, "uniform"),
]
# name, dtype, M, N, K, seed
GEMV_CASES = [
    ("gemv_bf16_m1_n256_k512", "bf16", 1, 256, 512, 1),
    ("gemv_fp16_m4_n96_k1024", "fp16", 4, 96, 1024, 2),
    ("gemv_bf16_m16_n64_k2048", "bf16", 16, 64, 2048, 1),
    ("gemv_fp16_m3_n37_k13_ragged", "fp16", 3, 37, 13, 2),
    ("gemv_bf16_m32_n40_k264", "bf16", 32, 40, 264, 1),
    ("gemv_fp16_m4_n8_k14336_ffn_down", "fp16", 4, 8, 14336, 2),
]


# name, dtype, tokens, hidden, seed, gate scale (silu_mul cases)
SILU_CASES = [
    ("silu_bf16_t4_h264", "bf16", 4, 264, 20, 1.0),
    ("silu_fp16_t1_h11008_decode", "fp16", 1, 11008, 21, 1.0),
    ("silu_bf16_t3_h13_ragged", "bf16", 3, 13, 22, 1.0),
    ("silu_fp16_t8_h96_wide_range", "fp16", 8, 96, 23, 12.0),
]
# name, operator, dtype, tokens, hidden, seed, eps
NORM_CASES = [
    ("rms_bf16_t4_h4096", "rms_norm", "bf16", 4, 4096, 30, 1e-6),
    ("rms_fp16_t1_h8192_decode", "rms_norm", "fp16", 1, 8192, 31, 1e-6),
    ("rms_bf16_t3_h13_ragged", "rms_norm", "bf16", 3, 13, 32, 1e-5),
    ("rms_fp16_t2_h20000_long_row", "rms_norm", "fp16", 2, 20000, 33, 1e-6),
    ("add_rms_bf16_t4_h4096", "add_rms_norm", "bf16", 4, 4096, 40, 1e-6),
    ("add_rms_fp16_t1_h8192_decode", "add_rms_norm", "fp16", 1, 8192, 41, 1e-6),
    ("add_rms_bf16_t5_h100_ragged", "add_rms_norm", "bf16", 5, 100, 42, 1e-5),
    ("add_rms_bf16_t2_h16392_long_row", "add_rms_norm", "bf16", 2, 16392, 43, 1e-6),
]

# Gradients (autograd through the reference's own fallback functions; the reference runs
# inputs that require gradients on exactly these graphs).
# name, operator, dtype, tokens, hidden, seed, eps (norms) / gate scale (silu_mul), flags
GRAD_CASES = [
    ("grad_silu_bf16_t4_h264", "silu_mul", "bf16", 4, 264, 70, 1.0, ""),
    ("grad_silu_fp16_t3_h13_ragged", "silu_mul", "fp16", 3, 13, 71, 1.0, ""),
    ("grad_silu_bf16_t8_h96_wide_range", "silu_mul", "bf16", 8, 96, 72, 12.0, "specials"),
    ("grad_rms_bf16_t4_h4096", "rms_norm", "bf16", 4, 4096, 73, 1e-6, ""),
    ("grad_rms_fp16_t3_h13_ragged", "rms_norm", "fp16", 3, 13, 74, 1e-5, ""),
    ("grad_rms_bf16_t2_h20000_long_row", "rms_norm", "bf16", 2, 20000, 75, 1e-6, ""),
    ("grad_add_rms_bf16_t4_h4096", "add_rms_norm", "bf16", 4, 4096, 76, 1e-6, ""),
    ("grad_add_rms_fp16_t5_h100_ragged_out_only", "add_rms_norm", "fp16", 5, 100, 77, 1e-5, "out_only"),
    ("grad_add_rms_bf16_t2_h16392_long_row", "add_rms_norm", "bf16", 2, 16392, 78, 1e-6, ""),
]

# Self-attention (ops.sdpa.reference.sdpa_reference): name, dtype, batch, query_heads,
# kv_heads, sequence, head_dim, causal, scale (None: 1/sqrt(head_dim)), seed
SDPA_CASES = [
    ("sdpa_bf16_b1_mha2_s37_d64_causal", "bf16", 1, 2, 2, 37, 64, True, None, 80),
    ("sdpa_fp16_b2_gqa4x2_s130_d128_causal", "fp16", 2, 4, 2, 130, 128, True, None, 81),
    ("sdpa_bf16_b1_gqa8x1_s200_d128_noncausal", "bf16", 1, 8, 1, 200, 128, False, 0.05, 82),
    ("sdpa_fp16_b1_mha2_s64_d256_causal", "fp16", 1, 2, 2, 64, 256, True, None, 83),
    ("sdpa_bf16_b1_gqa4x2_s260_d64_noncausal", "bf16", 1, 4, 2, 260, 64, False, None, 84),
]

# name, dtype, batch, query_heads, kv_heads, head_dim, block_size, num_blocks, max_blocks,
# context lengths, index dtype, scale (None: 1/sqrt(head_dim)), seed
PAGED_CASES = [
    ("paged_bf16_b2_gqa4x2_d64_p16", "bf16", 2, 4, 2, 64, 16, 12, 5, [37, 64], "int32", None, 60),
    ("paged_fp16_b1_mqa8x1_d128_p16", "fp16", 1, 8, 1, 128, 16, 9, 8, [113], "int64", None, 61),
    ("paged_bf16_b3_mha4_d256_p32_zero_len", "bf16", 3, 4, 4, 256, 32, 6, 3, [1, 70, 0], "int32", 0.05, 62),
    ("paged_fp16_b2_gqa32x8_d128_p16", "fp16", 2, 32, 8, 128, 16, 40, 16, [200, 256], "int32", None, 63),
]


def _bits(tensor):
    import torch

    return tensor.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def _draw(torch, shape, seed, dist, generator=None):
    gen = generator or torch.Generator().manual_seed(seed)
    if dist == "uniform":
        return torch.rand(shape, generator=gen) * 2 - 1
    if dist == "uniform16":
        return (torch.rand(shape, generator=gen) * 2 - 1) / 16
    if dist == "normal64":
        return torch.randn(shape, generator=gen) / 64
    raise ValueError(dist)


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--reference-src", required=True, type=Path)
    args = parser.parse_args(argv)
    sys.path.insert(0, str(args.reference_src.resolve()))
    import torch

    import radeon_kernels  # the reference package
    from radeon_kernels.ops.add_rms_norm.reference import add_rms_norm_reference
    from radeon_kernels.ops.gemv.reference import gemv_fallback, gemv_reference
    from radeon_kernels.ops.paged_attention.reference import paged_attention_decode_reference
    from radeon_kernels.ops.rms_norm.reference import rms_norm_reference
    from radeon_kernels.ops.sdpa.reference import sdpa_reference
    from radeon_kernels.ops.swiglu.reference import silu_mul_reference
    from radeon_kernels.providers import torch_fallback

    origin = Path(radeon_kernels.__file__).resolve()
    if not origin.is_relative_to(args.reference_src.resolve()):
        raise SystemExit(f"imported radeon_kernels from {origin}, not from the reference")
    dtypes = {"bf16": torch.bfloat16, "fp16": torch.float16}

    for name, dt, m, n, k, seed, dist in GEMM_CASES:
        gen = torch.Generator().manual_seed(seed)
        a = _draw(torch, (m, k), seed, dist, gen).to(dtypes[dt])
        b = _draw(torch, (k, n), seed, dist, gen).to(dtypes[dt])
        c = torch_fallback.gemm(torch, a, b)
        c32 = torch.mm(a.float(), b.float())
        np.savez_compressed(
            HERE / f"{name}.npz", dtype=dt, a=_bits(a), b=_bits(b), c_ref=_bits(c), c_fp32=c32.numpy()
        )
        print(name, tuple(c.shape))

    for name, dt, m, n, k, seed in GEMV_CASES:
        gen = torch.Generator().manual_seed(seed)
        x = torch.randn((m, k), generator=gen).to(dtypes[dt])
        w = (torch.randn((n, k), generator=gen) / k**0.5).to(dtypes[dt])
        out = gemv_fallback(torch, x, w)
        out_ref = gemv_reference(torch, x, w)
        out32 = torch.mm(x.float(), w.float().t())
        np.savez_compressed(
            HERE / f"{name}.npz",
            dtype=dt,
            x=_bits(x),
            w=_bits(w),
            out_fallback=_bits(out),
            out_reference=_bits(out_ref),
            out_fp32=out32.numpy(),
        )
        print(name, tuple(out.shape))

    for name, dt, batch, hq, hkv, d, bs, nb, maxb, lens, idx, scale, seed in PAGED_CASES:
        gen = torch.Generator().manual_seed(seed)
        q = torch.randn((batch, hq, d), generator=gen).to(dtypes[dt])
        k = torch.randn((nb, bs, hkv, d), generator=gen).to(dtypes[dt])
        v = torch.randn((nb, bs, hkv, d), generator=gen).to(dtypes[dt])
        # every sequence's logical blocks map to scattered physical blocks
        tables = torch.stack([torch.randperm(nb, generator=gen)[:maxb] for _ in range(batch)])
        itype = torch.int32 if idx == "int32" else torch.int64
        tables = tables.to(itype)
        lengths = torch.tensor(lens, dtype=itype)
        eff_scale = scale if scale is not None else 1.0 / d**0.5
        out = paged_attention_decode_reference(torch, q, k, v, tables, lengths, scale)
        np.savez_compressed(
            HERE / f"{name}.npz", dtype=dt, q=_bits(q), k=_bits(k), v=_bits(v), block_tables=tables.numpy(),
            context_lengths=lengths.numpy(), scale=np.float64(eff_scale), out_ref=_bits(out),
        )
        print(name, tuple(out.shape))

    for name, dt, tokens, hidden, seed, scale in SILU_CASES:
        gen = torch.Generator().manual_seed(seed)
        gate = (torch.randn((tokens, hidden), generator=gen) * scale).to(dtypes[dt])
        up = torch.randn((tokens, hidden), generator=gen).to(dtypes[dt])
        if name.endswith("wide_range"):
            # saturated sigmoid at both ends, signed zeros, infinities and a NaN
            specials = torch.tensor([60000.0, -60000.0, 0.0, -0.0, float("inf"), float("-inf"), float("nan"), 11.0])
            gate[0, : specials.numel()] = specials.to(dtypes[dt])
        out = silu_mul_reference(torch, gate, up)
        g32 = gate.float()
        exact = g32 * torch.sigmoid(g32) * up.float()
        np.savez_compressed(
            HERE / f"{name}.npz", dtype=dt, gate=_bits(gate), up=_bits(up), out_ref=_bits(out), out_fp32=exact.numpy()
        )
        print(name, tuple(out.shape))

    for name, operator, dt, tokens, hidden, seed, eps in NORM_CASES:
        gen = torch.Generator().manual_seed(seed)
        x = torch.randn((tokens, hidden), generator=gen).to(dtypes[dt])
        weight = (1.0 + 0.1 * torch.randn((hidden,), generator=gen)).to(dtypes[dt])
        fields = {"dtype": dt, "eps": np.float64(eps), "x": _bits(x), "weight": _bits(weight)}
        if operator == "rms_norm":
            source = x
            fields["out_ref"] = _bits(rms_norm_reference(torch, x, weight, eps))
        else:
            residual = torch.randn((tokens, hidden), generator=gen).to(dtypes[dt])
            out, residual_out = add_rms_norm_reference(torch, x, residual, weight, eps)
            fields.update(residual=_bits(residual), out_ref=_bits(out), residual_out_ref=_bits(residual_out))
            source = residual_out
        s32 = source.float()
        exact = s32 * torch.rsqrt(s32.square().mean(dim=-1, keepdim=True) + eps) * weight.float()
        fields["out_fp32"] = exact.numpy()
        np.savez_compressed(HERE / f"{name}.npz", **fields)
        print(name, (tokens, hidden))

    for name, dt, batch, hq, hkv, seq, d, causal, scale, seed in SDPA_CASES:
        gen = torch.Generator().manual_seed(seed)
        q = (torch.rand((batch, hq, seq, d), generator=gen) * 0.25 - 0.125).to(dtypes[dt])
        k = (torch.rand((batch, hkv, seq, d), generator=gen) * 0.25 - 0.125).to(dtypes[dt])
        v = (torch.rand((batch, hkv, seq, d), generator=gen) * 0.25 - 0.125).to(dtypes[dt])
        eff_scale = 1.0 / d**0.5 if scale is None else scale
        out = sdpa_reference(torch, q, k, v, causal, eff_scale)
        np.savez_compressed(
            HERE / f"{name}.npz", dtype=dt, q=_bits(q), k=_bits(k), v=_bits(v), is_causal=np.bool_(causal),
            scale=np.float64(eff_scale), out_ref=_bits(out),
        )
        print(name, tuple(out.shape))

    for name, operator, dt, tokens, hidden, seed, param, flags in GRAD_CASES:
        gen = torch.Generator().manual_seed(seed)
        dy = torch.randn((tokens, hidden), generator=gen).to(dtypes[dt])
        if operator == "silu_mul":
            gate = (torch.randn((tokens, hidden), generator=gen) * param).to(dtypes[dt])
            up = torch.randn((tokens, hidden), generator=gen).to(dtypes[dt])
            if flags == "specials":
                specials = torch.tensor([60000.0, -60000.0, 0.0, -0.0, float("inf"), float("-inf"), float("nan"), -1.28])
                gate[0, : specials.numel()] = specials.to(dtypes[dt])
            gate.requires_grad_(True)
            up.requires_grad_(True)
            silu_mul_reference(torch, gate, up).backward(dy)
            np.savez_compressed(
                HERE / f"{name}.npz", dtype=dt, dy=_bits(dy), gate=_bits(gate.detach()), up=_bits(up.detach()),
                grad_gate_ref=_bits(gate.grad), grad_up_ref=_bits(up.grad),
            )
        else:
            x = torch.randn((tokens, hidden), generator=gen).to(dtypes[dt]).requires_grad_(True)
            weight = (1.0 + 0.1 * torch.randn((hidden,), generator=gen)).to(dtypes[dt]).requires_grad_(True)
            fields = {"dtype": dt, "eps": np.float64(param), "dy": _bits(dy), "x": _bits(x.detach()),
                      "weight": _bits(weight.detach())}
            if operator == "rms_norm":
                rms_norm_reference(torch, x, weight, param).backward(dy)
            else:
                residual = torch.randn((tokens, hidden), generator=gen).to(dtypes[dt]).requires_grad_(True)
                dres = torch.randn((tokens, hidden), generator=gen).to(dtypes[dt])
                out, residual_out = add_rms_norm_reference(torch, x, residual, weight, param)
                if flags == "out_only":
                    torch.autograd.backward([out], [dy])
                else:
                    torch.autograd.backward([out, residual_out], [dy, dres])
                    fields["dres"] = _bits(dres)
                fields.update(residual=_bits(residual.detach()), residual_out=_bits(residual_out.detach()),
                              grad_residual_ref=_bits(residual.grad))
            fields.update(grad_x_ref=_bits(x.grad), grad_weight_ref=_bits(weight.grad))
            np.savez_compressed(HERE / f"{name}.npz", **fields)
        print(name, (tokens, hidden))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
