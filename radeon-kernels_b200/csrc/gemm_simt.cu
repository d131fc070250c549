// gemm_simt.cu -- generic predicated CUDA-core GEMM (variant RK_GEMM_SIMT).
//
// The always-available kernel: any M, N, K, any element alignment.  It is the
// edge-case path (N or K not a multiple of 8, unaligned views) and the
// built-in "cuda" fallback of the dispatch manifests; shapes the tensor-core
// kernel accepts never come here under RK_GEMM_AUTO.  64x64 output tile per
// 256-thread CTA, 16-deep K panels staged in shared memory as fp32, 4x4
// outputs per thread, fp32 accumulation, round-to-nearest-even output.
// Operands are addressed through element strides, so every rk_layout runs here:
// A(m, k) = A[m * sam + k * sak], B(k, n) = B[k * sbk + n * sbn].
#include <cuda_runtime.h>

#include "rk_device.cuh"
#include "rk_internal.h"

namespace rk {
namespace {

constexpr int TM = 64, TN = 64, TK = 16;

template <typename T>
__global__ void __launch_bounds__(256)
    gemm_simt_kernel(const T* __restrict__ A, const T* __restrict__ B, T* __restrict__ C,
                     int64_t M, int64_t N, int64_t K, int64_t sam, int64_t sak, int64_t sbk,
                     int64_t sbn) {
  __shared__ float As[TK][TM + 4];
  __shared__ float Bs[TK][TN + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * TM;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * TN;
  float acc[4][4] = {};
  pdl_begin();
  for (int64_t k0 = 0; k0 < K; k0 += TK) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = threadIdx.x + i * 256;
      const int r = idx / TK, c = idx % TK;  // A tile: 64 rows x 16 k
      const int64_t m = m0 + r, k = k0 + c;
      As[c][r] = (m < M && k < K) ? to_f32(A[m * sam + k * sak]) : 0.f;
      const int rb = idx / TN, cb = idx % TN;  // B tile: 16 k x 64 cols
      const int64_t kb = k0 + rb, n = n0 + cb;
      Bs[rb][cb] = (kb < K && n < N) ? to_f32(B[kb * sbk + n * sbn]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = m0 + ty + 16 * i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t n = n0 + tx + 16 * j;
      if (n < N) C[m * N + n] = from_f32<T>(acc[i][j]);
    }
  }
}

}  // namespace

rk_status gemm_simt_launch(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                           rk_layout layout, rk_dtype dt, cudaStream_t s) {
  const int64_t gx = (N + TN - 1) / TN, gy = (M + TM - 1) / TM;
  if (gx > 0x7fffffffll || gy > 65535) return RK_ERR_UNSUPPORTED;
  const bool at = layout == RK_LAYOUT_TN || layout == RK_LAYOUT_TT;
  const bool bt = layout == RK_LAYOUT_NT || layout == RK_LAYOUT_TT;
  const int64_t sam = at ? 1 : K, sak = at ? M : 1;
  const int64_t sbk = bt ? 1 : N, sbn = bt ? K : 1;
  dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy));
  cudaError_t e;
  if (dt == RK_DTYPE_BF16)
    e = launch_kernel(gemm_simt_kernel<__nv_bfloat16>, grid, dim3(256), 0, s, 0,
                      static_cast<const __nv_bfloat16*>(A), static_cast<const __nv_bfloat16*>(B),
                      static_cast<__nv_bfloat16*>(C), M, N, K, sam, sak, sbk, sbn);
  else
    e = launch_kernel(gemm_simt_kernel<__half>, grid, dim3(256), 0, s, 0,
                      static_cast<const __half*>(A), static_cast<const __half*>(B),
                      static_cast<__half*>(C), M, N, K, sam, sak, sbk, sbn);
  note_launch("gemm_simt_kernel");
  return cuda_status(e);
}

}  // namespace rk
