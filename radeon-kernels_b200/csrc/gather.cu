// gather.cu -- column-block gather for N-sharded results.
//
// An all-gather of per-rank C blocks C_g[M, N/G] produces G contiguous blocks
// [G][M][N/G]; callers that need the full row-major C[M, N] run this HBM-bound
// permute (read + write of M*N elements).  16-byte copies when every block row
// is a multiple of 8 elements and both buffers are 16-byte aligned, else
// 2-byte copies.  Grid-stride, sized as a multiple of the SM count.
#include <cuda_runtime.h>

#include "rk_device.cuh"
#include "rk_internal.h"

namespace rk {
namespace {

template <typename V>
__global__ void __launch_bounds__(256)
    gather_blocks_kernel(const V* __restrict__ blocks, V* __restrict__ out, int64_t G, int64_t M,
                         int64_t nb /* block row length in V units */) {
  const int64_t total = G * M * nb;
  pdl_begin();
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    // i enumerates the destination: row m, block g, offset j.
    const int64_t j = i % nb;
    const int64_t t = i / nb;
    const int64_t g = t % G;
    const int64_t m = t / G;
    out[i] = blocks[(g * M + m) * nb + j];
  }
}

}  // namespace

rk_status gather_column_blocks_launch(const void* blocks, void* out, int64_t G, int64_t M,
                                      int64_t N, rk_dtype dt, cudaStream_t s) {
  (void)dt;  // a pure byte permute: fp16 and bf16 are both 2-byte elements
  const int64_t nb = N / G;
  const int64_t total = M * N;
  const int grid_cap = device_sm_count() * 8;
  if (nb % 8 == 0 && aligned16(blocks) && aligned16(out)) {
    const int64_t units = total / 8;
    const int grid = static_cast<int>(units / 256 + 1 < grid_cap ? units / 256 + 1 : grid_cap);
    const cudaError_t e = launch_kernel(gather_blocks_kernel<uint4>, dim3(grid), dim3(256), 0, s, 0,
                                        static_cast<const uint4*>(blocks), static_cast<uint4*>(out),
                                        G, M, nb / 8);
    note_launch();
    return cuda_status(e);
  }
  const int grid = static_cast<int>(total / 256 + 1 < grid_cap ? total / 256 + 1 : grid_cap);
  const cudaError_t e = launch_kernel(gather_blocks_kernel<uint16_t>, dim3(grid), dim3(256), 0, s, 0,
                                      static_cast<const uint16_t*>(blocks),
                                      static_cast<uint16_t*>(out), G, M, nb);
  note_launch();
  return cuda_status(e);
}

}  // namespace rk
