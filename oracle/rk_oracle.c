/*
 * rk_oracle.c -- CPU restatement of the reference's arithmetic for the GEMM/GEMV path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (radeon-kernels_b200/) links or
 * calls this file; only tests/, __graft_entry__.smoke() and bench.py's CPU baseline do,
 * as the checker.
 *
 * What is restated (the decode neighbours silu_mul / rms_norm / add_rms_norm are at the
 * end of the file).  The reference computes both operators with PyTorch:
 *   rk.gemm fallback:  torch.mm(a, b)                        providers/torch_fallback.py:6-9
 *   rk.gemv fallback:  torch.mm(x, weight.T)                 ops/gemv/reference.py:12-15
 *   rk.gemv oracle:    torch.mm(x.float(), weight.float().T).to(x.dtype)
 *                                                            ops/gemv/reference.py:6-9
 * i.e. 16-bit inputs widened exactly to fp32, products accumulated in fp32, the sum
 * rounded once to the input dtype with round-to-nearest-even.  PyTorch itself is a
 * third-party dependency (not vendored; the reference pins builds 2.14.0a0+rocm7.15 and
 * 2.11.0+rocm7.2.4 in dispatch/gemm-1.0.json:17,51); its CPU kernels accumulate in fp32
 * in a blocked order.  This file accumulates in fp32 in increasing k, so it agrees with
 * torch.mm to fp32 rounding of the sum -- the tests pin it against fixtures produced by
 * the reference's own functions (tests/golden/make_golden.py).
 *
 * Every function also returns the unrounded fp32 sums, the quantity the parity metric
 * max|C - C_ref| / max|C_ref| is measured against.
 *
 * Conversions are written from the IEEE 754 binary16 / bfloat16 definitions.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define RK_ORACLE_FP16 0
#define RK_ORACLE_BF16 1

static float bits_to_f32(uint32_t u) {
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

static uint32_t f32_to_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, sizeof u);
  return u;
}

/* bfloat16 is the upper half of binary32: widening is exact. */
static float bf16_to_f32(uint16_t h) { return bits_to_f32((uint32_t)h << 16); }

/* binary16: 1 sign, 5 exponent (bias 15), 10 fraction bits. */
static float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t frac = h & 0x3FFu;
  if (exp == 0x1Fu) return bits_to_f32(sign | 0x7F800000u | (frac << 13)); /* inf / nan */
  if (exp == 0) {
    if (frac == 0) return bits_to_f32(sign); /* signed zero */
    /* subnormal: value = frac * 2^-24, normalise into binary32 */
    int e = -14;
    while ((frac & 0x400u) == 0) {
      frac <<= 1;
      --e;
    }
    frac &= 0x3FFu;
    return bits_to_f32(sign | ((uint32_t)(e + 127) << 23) | (frac << 13));
  }
  return bits_to_f32(sign | ((exp + 112u) << 23) | (frac << 13)); /* rebias 15 -> 127 */
}

/* binary32 -> bfloat16, round to nearest, ties to even; NaN stays NaN. */
static uint16_t f32_to_bf16(float f) {
  uint32_t u = f32_to_bits(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x0040u);
  const uint32_t lsb = (u >> 16) & 1u;
  u += 0x7FFFu + lsb;
  return (uint16_t)(u >> 16);
}

/* binary32 -> binary16, round to nearest, ties to even, with subnormals and overflow to inf. */
static uint16_t f32_to_f16(float f) {
  const uint32_t u = f32_to_bits(f);
  const uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
  const uint32_t abs = u & 0x7FFFFFFFu;
  if (abs > 0x7F800000u) return (uint16_t)(sign | 0x7E00u);  /* nan */
  if (abs == 0x7F800000u) return (uint16_t)(sign | 0x7C00u); /* inf */
  const int exp = (int)(abs >> 23) - 127;
  uint32_t mant = (abs & 0x7FFFFFu) | 0x800000u; /* 24-bit significand with hidden bit */
  if (exp > 15) return (uint16_t)(sign | 0x7C00u);
  if (exp >= -14) {
    /* normal range: keep 11 significant bits, drop 13 */
    uint32_t keep = mant >> 13, rest = mant & 0x1FFFu;
    if (rest > 0x1000u || (rest == 0x1000u && (keep & 1u))) ++keep;
    /* keep may carry into bit 11 (0x800): the exponent field absorbs it */
    const uint32_t bits = ((uint32_t)(exp + 15) << 10) + (keep - 0x400u);
    if (bits >= 0x7C00u) return (uint16_t)(sign | 0x7C00u);
    return (uint16_t)(sign | bits);
  }
  if (abs == 0) return sign;
  /* subnormal result: value = q * 2^-24 with q = mant * 2^(exp - 23 + 24) */
  const int shift = -exp - 14 + 13; /* bits of mant dropped */
  if (shift > 24) return sign;      /* below half the smallest subnormal */
  uint32_t keep = mant >> shift;
  const uint32_t rest = mant & ((1u << shift) - 1u);
  const uint32_t half = 1u << (shift - 1);
  if (rest > half || (rest == half && (keep & 1u))) ++keep;
  return (uint16_t)(sign | keep); /* keep == 0x400 rounds up into the smallest normal */
}

static float load16(const uint16_t* p, int64_t i, int dtype) {
  return dtype == RK_ORACLE_BF16 ? bf16_to_f32(p[i]) : f16_to_f32(p[i]);
}

static uint16_t store16(float v, int dtype) {
  return dtype == RK_ORACLE_BF16 ? f32_to_bf16(v) : f32_to_f16(v);
}

void rk_oracle_round(const float* src, uint16_t* dst, int64_t count, int dtype) {
  for (int64_t i = 0; i < count; ++i) dst[i] = store16(src[i], dtype);
}

void rk_oracle_widen(const uint16_t* src, float* dst, int64_t count, int dtype) {
  for (int64_t i = 0; i < count; ++i) dst[i] = load16(src, i, dtype);
}

/*
 * C = A @ B with A [M,K], B [K,N], C [M,N] row-major 16-bit.  `acc` ([M,N] fp32) receives
 * the unrounded sums; `work` must hold K*N + K floats (widened B and one row of A).
 */
void rk_oracle_gemm(const uint16_t* A, const uint16_t* B, uint16_t* C, float* acc, float* work,
                    int64_t M, int64_t N, int64_t K, int dtype) {
  float* bw = work;
  float* arow = work + K * N;
  rk_oracle_widen(B, bw, K * N, dtype);
  for (int64_t i = 0; i < M; ++i) {
    float* crow = acc + i * N;
    for (int64_t j = 0; j < N; ++j) crow[j] = 0.0f;
    rk_oracle_widen(A + i * K, arow, K, dtype);
    for (int64_t k = 0; k < K; ++k) {
      const float a = arow[k];
      const float* brow = bw + k * N;
      for (int64_t j = 0; j < N; ++j) crow[j] += a * brow[j];
    }
    for (int64_t j = 0; j < N; ++j) C[i * N + j] = store16(crow[j], dtype);
  }
}

/*
 * out = x @ W^T with x [M,K], W [N,K] ("nk"), out [M,N].  `acc` receives the fp32 sums;
 * `work` must hold 2*K floats.
 */
void rk_oracle_gemv(const uint16_t* x, const uint16_t* W, uint16_t* out, float* acc, float* work,
                    int64_t M, int64_t N, int64_t K, int dtype) {
  float* xw = work;
  float* ww = work + K;
  for (int64_t m = 0; m < M; ++m) {
    rk_oracle_widen(x + m * K, xw, K, dtype);
    for (int64_t n = 0; n < N; ++n) {
      rk_oracle_widen(W + n * K, ww, K, dtype);
      float s = 0.0f;
      for (int64_t k = 0; k < K; ++k) s += xw[k] * ww[k];
      acc[m * N + n] = s;
      out[m * N + n] = store16(s, dtype);
    }
  }
}

/*
 * Decode neighbours of the GEMV/GEMM path (the reference's fp32 definitions):
 *   silu_mul_reference     ops/swiglu/reference.py:6-9
 *       g = float(gate); out = (g * sigmoid(g)) * float(up), rounded once
 *   rms_norm_reference     ops/rms_norm/reference.py:6-10
 *       v = float(x); var = mean(v * v); out = (v * rsqrt(var + eps)) * float(weight)
 *   add_rms_norm_reference ops/add_rms_norm/reference.py:8-12
 *       s = x + residual in the 16-bit dtype (one rounding); out = rms_norm(s)
 * sigmoid(g) = 1 / (1 + exp(-g)) with the C library's expf; rsqrt(v) = 1 / sqrtf(v).
 * The squares are rounded to fp32 (as torch's square() stores them) and summed in double;
 * PyTorch sums them in fp32 in a blocked order, so the two means agree to the last fp32
 * bit or two.  `exact` receives every output before its final rounding.
 */
void rk_oracle_silu_mul(const uint16_t* gate, const uint16_t* up, uint16_t* out, float* exact,
                        int64_t n, int dtype) {
  for (int64_t i = 0; i < n; ++i) {
    const float g = load16(gate, i, dtype);
    const float s = 1.0f / (1.0f + expf(-g));
    const float gs = g * s;
    const float v = gs * load16(up, i, dtype);
    exact[i] = v;
    out[i] = store16(v, dtype);
  }
}

static void rms_rows(const float* v, const uint16_t* weight, uint16_t* out, float* exact,
                     int64_t hidden, float eps, int dtype) {
  double sum = 0.0;
  for (int64_t j = 0; j < hidden; ++j) {
    const float sq = v[j] * v[j];
    sum += (double)sq;
  }
  const float mean = (float)sum / (float)hidden;
  const float r = 1.0f / sqrtf(mean + eps);
  for (int64_t j = 0; j < hidden; ++j) {
    const float normalized = v[j] * r;
    const float y = normalized * load16(weight, j, dtype);
    exact[j] = y;
    out[j] = store16(y, dtype);
  }
}

/* `work` must hold `hidden` floats. */
void rk_oracle_rms_norm(const uint16_t* x, const uint16_t* weight, uint16_t* out, float* exact,
                        float* work, int64_t tokens, int64_t hidden, float eps, int dtype) {
  for (int64_t t = 0; t < tokens; ++t) {
    rk_oracle_widen(x + t * hidden, work, hidden, dtype);
    rms_rows(work, weight, out + t * hidden, exact + t * hidden, hidden, eps, dtype);
  }
}

void rk_oracle_add_rms_norm(const uint16_t* x, const uint16_t* residual, const uint16_t* weight,
                            uint16_t* out, uint16_t* residual_out, float* exact, float* work,
                            int64_t tokens, int64_t hidden, float eps, int dtype) {
  for (int64_t t = 0; t < tokens; ++t) {
    for (int64_t j = 0; j < hidden; ++j) {
      const int64_t i = t * hidden + j;
      residual_out[i] = store16(load16(x, i, dtype) + load16(residual, i, dtype), dtype);
      work[j] = load16(residual_out, i, dtype);
    }
    rms_rows(work, weight, out + t * hidden, exact + t * hidden, hidden, eps, dtype);
  }
}

/*
 * Backward passes: what autograd computes through the three reference graphs above (the
 * reference sends inputs that require gradients to those fallbacks: ops/swiglu/api.py:49,
 * ops/rms_norm/api.py:53, ops/add_rms_norm/api.py:57), term for term in fp32:
 *   silu_mul:     s = sigmoid(g); du = dy*(g*s); t = dy*u; dg = t*s + ((t*g)*(1-s))*s
 *                 (mul backward twice, then sigmoid backward grad*(1-s)*s)
 *   rms_norm:     r as in the forward; c = sum_j (dy_j*w_j)*x_j (rsqrt's input gradient
 *                 source); q = ((-0.5*c)*(r*r*r))/H (rsqrt backward, then mean backward);
 *                 dx = (dy*w)*r + q*(2*x) (pow backward); dw = sum over rows of dy*(x*r)
 *   add_rms_norm: x is the saved residual_out s; ds = round(round(dx) + dres) when the
 *                 residual_out gradient dres is given (two 16-bit gradients of s added),
 *                 round(dx) otherwise; both inputs of the add receive ds
 * Row and column sums are taken in double (PyTorch sums in fp32 in its own order, so the
 * two agree to the last fp32 bits).  Every output also gets `scale`, the sum of the
 * magnitudes of the terms that form it, so a checker can tell cancellation (a result much
 * smaller than its terms) from a wrong value.
 */
void rk_oracle_silu_mul_backward(const uint16_t* dy, const uint16_t* gate, const uint16_t* up,
                                 uint16_t* dgate, uint16_t* dup, float* dgate32, float* dup32,
                                 float* dgate_scale, int64_t n, int dtype) {
  for (int64_t i = 0; i < n; ++i) {
    const float d = load16(dy, i, dtype), g = load16(gate, i, dtype), u = load16(up, i, dtype);
    const float s = 1.0f / (1.0f + expf(-g));
    const float du = d * (g * s);
    const float t = d * u;
    const float direct = t * s;
    const float through_sigmoid = ((t * g) * (1.0f - s)) * s;
    const float dg = direct + through_sigmoid;
    dgate32[i] = dg;
    dup32[i] = du;
    dgate_scale[i] = fabsf(direct) + fabsf(through_sigmoid);
    dgate[i] = store16(dg, dtype);
    dup[i] = store16(du, dtype);
  }
}

/* `work` must hold 2 * hidden doubles; dres may be NULL; add != 0 selects add_rms_norm. */
void rk_oracle_rms_norm_backward(const uint16_t* dy, const uint16_t* x, const uint16_t* weight,
                                 const uint16_t* dres, uint16_t* dx, float* dx32, float* dx_scale,
                                 uint16_t* dw, float* dw32, float* dw_scale, double* work,
                                 int64_t tokens, int64_t hidden, float eps, int add, int dtype) {
  double* dw_acc = work;
  double* dw_abs = work + hidden;
  for (int64_t j = 0; j < hidden; ++j) dw_acc[j] = dw_abs[j] = 0.0;
  for (int64_t t = 0; t < tokens; ++t) {
    const int64_t row = t * hidden;
    double sum_sq = 0.0, c = 0.0, c_abs = 0.0;
    for (int64_t j = 0; j < hidden; ++j) {
      const float v = load16(x, row + j, dtype);
      const float sq = v * v;
      sum_sq += (double)sq;
      const float term = (load16(dy, row + j, dtype) * load16(weight, j, dtype)) * v;
      c += (double)term;
      c_abs += fabs((double)term);
    }
    const float mean = (float)sum_sq / (float)hidden;
    const float r = 1.0f / sqrtf(mean + eps);
    const float q = ((-0.5f * (float)c) * (r * r * r)) / (float)hidden;
    const float q_abs = ((0.5f * (float)c_abs) * (r * r * r)) / (float)hidden;
    for (int64_t j = 0; j < hidden; ++j) {
      const float d = load16(dy, row + j, dtype), v = load16(x, row + j, dtype);
      const float w = load16(weight, j, dtype);
      const float direct = (d * w) * r;
      const float g = direct + q * (2.0f * v);
      float scale = fabsf(direct) + q_abs * fabsf(2.0f * v);
      uint16_t bits = store16(g, dtype);
      float exact = g;
      if (add && dres != NULL) {
        const float e = load16(dres, row + j, dtype);
        exact = load16(&bits, 0, dtype) + e;
        bits = store16(exact, dtype);
        scale += fabsf(e);
      }
      dx[row + j] = bits;
      dx32[row + j] = exact;
      dx_scale[row + j] = scale;
      const float contribution = d * (v * r);
      dw_acc[j] += (double)contribution;
      dw_abs[j] += fabs((double)contribution);
    }
  }
  for (int64_t j = 0; j < hidden; ++j) {
    dw32[j] = (float)dw_acc[j];
    dw_scale[j] = (float)dw_abs[j];
    dw[j] = store16((float)dw_acc[j], dtype);
  }
}
