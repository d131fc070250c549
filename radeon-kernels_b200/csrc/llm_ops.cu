// llm_ops.cu -- the elementwise and row-normalisation neighbours of the decode GEMV/GEMM:
//   silu_mul(gate, up)                 out = silu(gate) * up
//   rms_norm(x, weight, eps)           out = x * rsqrt(mean(x^2) + eps) * weight
//   add_rms_norm(x, residual, w, eps)  s = x + residual (rounded to the dtype);
//                                      out = rms_norm(s, w, eps), residual_out = s
// fp16/bf16 in and out, fp32 arithmetic, one round-to-nearest-even per stored value.
//
// All three are HBM streams (no data reuse beyond a row), so the design is about
// bytes in flight and launch latency:
//   * 16-byte vector loads/stores (8 elements) when the hidden size is a multiple of 8
//     and every pointer is 16-byte aligned; a scalar path otherwise;
//   * silu_mul: one grid-stride loop over the flat tensor, grid = resident CTAs x SMs;
//   * (add_)rms_norm: one CTA per row (grid-stride over rows), each thread holding up to
//     4 16-byte vectors of the row in registers between the sum of squares and the scaled
//     store (longer rows are re-read from L2 for the second pass); the per-row sum is a
//     warp-shuffle tree plus a fixed-order sum over the warps (deterministic).  The CTA
//     size per row is chosen from the shape: few rows (decode) get 256 threads, many rows
//     (prefill) the fewest threads whose registers hold the row, so more rows are
//     resident per SM and fewer waves are needed.
// Arithmetic follows the reference's fp32 definitions (src/radeon_kernels/ops/swiglu/
// reference.py:6-9, ops/rms_norm/reference.py:6-10, ops/add_rms_norm/reference.py:8-12):
// silu(g) * u = (g * (1 / (1 + exp(-g)))) * u (exp and the reciprocal through the fast
// intrinsics, see silu_mul_f32), rsqrt(v) = 1 / sqrt(v) with IEEE sqrt and division, the
// mean as the fp32 sum divided by the hidden size.
//
// Role of the reference: silu_mul_kernel, rms_norm_kernel, add_rms_norm_kernel and their
// bindings (benchmarks/llm_ops/native_llm_ops.hip:51-94, :125-133, :306-353, :397-416).
#include <cuda_runtime.h>

#include <atomic>

#include "rk_device.cuh"
#include "rk_internal.h"

namespace rk {
namespace {

constexpr int ROW_CACHE = 4;  // 16-byte vectors per thread kept in registers

// Tuning override of the threads per row (64, 128, 256; 0 = built-in choice).
std::atomic<int> g_norm_threads{0};

// silu(g) * u: swiglu_f32 (rk_device.cuh), shared with the fused GEMM epilogue.
__device__ __forceinline__ float silu_mul_f32(float g, float u) { return swiglu_f32(g, u); }

template <typename T>
__device__ __forceinline__ uint32_t pack_silu(uint32_t g2, uint32_t u2) {
  const float2 g = Pack2<T>::to_floats(g2);
  const float2 u = Pack2<T>::to_floats(u2);
  return Pack2<T>::from_floats(silu_mul_f32(g.x, u.x), silu_mul_f32(g.y, u.y));
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(256)
    silu_mul_kernel(const T* __restrict__ gate, const T* __restrict__ up, T* __restrict__ out,
                    int64_t n) {
  pdl_begin();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (VEC) {
    const int64_t nv = n / 8;
    const uint4* g4 = reinterpret_cast<const uint4*>(gate);
    const uint4* u4 = reinterpret_cast<const uint4*>(up);
    uint4* o4 = reinterpret_cast<uint4*>(out);
    for (int64_t i = t0; i < nv; i += stride) {
      const uint4 g = ld_stream_v4(g4 + i);
      const uint4 u = ld_stream_v4(u4 + i);
      uint4 o;
      o.x = pack_silu<T>(g.x, u.x);
      o.y = pack_silu<T>(g.y, u.y);
      o.z = pack_silu<T>(g.z, u.z);
      o.w = pack_silu<T>(g.w, u.w);
      o4[i] = o;
    }
    for (int64_t i = nv * 8 + t0; i < n; i += stride)
      out[i] = from_f32<T>(silu_mul_f32(to_f32(gate[i]), to_f32(up[i])));
  } else {
    for (int64_t i = t0; i < n; i += stride)
      out[i] = from_f32<T>(silu_mul_f32(to_f32(gate[i]), to_f32(up[i])));
  }
}

// Sum over the CTA in a fixed order: shuffle tree inside each warp, then warp 0 adds the
// eight warp sums in warp order.  Every thread receives the total.
template <int ROW_THREADS>
__device__ __forceinline__ float row_sum(float v, float* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // scratch is reused row after row
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int w = 0; w < ROW_THREADS / 32; ++w) total += scratch[w];
  return total;
}

template <typename T>
__device__ __forceinline__ float2 add_round(uint32_t a2, uint32_t b2, uint32_t* rounded) {
  // s = x + residual in fp32, rounded once to the dtype (what a 16-bit tensor add stores).
  const float2 a = Pack2<T>::to_floats(a2);
  const float2 b = Pack2<T>::to_floats(b2);
  *rounded = Pack2<T>::from_floats(a.x + b.x, a.y + b.y);
  return Pack2<T>::to_floats(*rounded);
}

template <typename T>
__device__ __forceinline__ uint32_t scale_pack(uint32_t v2, uint32_t w2, float r) {
  const float2 v = Pack2<T>::to_floats(v2);
  const float2 w = Pack2<T>::to_floats(w2);
  return Pack2<T>::from_floats((v.x * r) * w.x, (v.y * r) * w.y);
}

// One CTA per row.  ADD: s = x + residual is formed, stored to residual_out and
// normalised; otherwise x is normalised.  VEC: 16-byte vectors (hidden % 8 == 0, aligned).
template <typename T, bool ADD, bool VEC, int ROW_THREADS>
__global__ void __launch_bounds__(ROW_THREADS)
    rms_norm_kernel(const T* __restrict__ x, const T* __restrict__ residual,
                    const T* __restrict__ weight, T* __restrict__ out, T* __restrict__ residual_out,
                    int64_t rows, int hidden, float eps) {
  __shared__ float scratch[ROW_THREADS / 32];
  pdl_begin();
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const size_t base = static_cast<size_t>(row) * hidden;
    float sq = 0.f;
    if (VEC) {
      const int nv = hidden / 8;
      const uint4* x4 = reinterpret_cast<const uint4*>(x + base);
      const uint4* r4 = ADD ? reinterpret_cast<const uint4*>(residual + base) : nullptr;
      uint4* s4 = ADD ? reinterpret_cast<uint4*>(residual_out + base) : nullptr;
      const uint4* w4 = reinterpret_cast<const uint4*>(weight);
      uint4* o4 = reinterpret_cast<uint4*>(out + base);
      uint4 cache[ROW_CACHE];
#pragma unroll
      for (int c = 0; c < ROW_CACHE; ++c) {
        const int v = threadIdx.x + c * ROW_THREADS;
        if (v < nv) {
          uint4 a = ld_stream_v4(x4 + v);
          if (ADD) {
            const uint4 b = ld_stream_v4(r4 + v);
            uint4 s;
            float2 f;
            f = add_round<T>(a.x, b.x, &s.x);
            sq += f.x * f.x + f.y * f.y;
            f = add_round<T>(a.y, b.y, &s.y);
            sq += f.x * f.x + f.y * f.y;
            f = add_round<T>(a.z, b.z, &s.z);
            sq += f.x * f.x + f.y * f.y;
            f = add_round<T>(a.w, b.w, &s.w);
            sq += f.x * f.x + f.y * f.y;
            s4[v] = s;
            a = s;
          } else {
            const uint32_t parts[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
            for (int p = 0; p < 4; ++p) {
              const float2 f = Pack2<T>::to_floats(parts[p]);
              sq += f.x * f.x + f.y * f.y;
            }
          }
          cache[c] = a;
        }
      }
      // Rows longer than the register cache: the rest is streamed once here and read
      // back (from L2) in the second pass.
      for (int v = threadIdx.x + ROW_CACHE * ROW_THREADS; v < nv; v += ROW_THREADS) {
        uint4 a = x4[v];
        if (ADD) {
          const uint4 b = r4[v];
          uint4 s;
          float2 f;
          f = add_round<T>(a.x, b.x, &s.x);
          sq += f.x * f.x + f.y * f.y;
          f = add_round<T>(a.y, b.y, &s.y);
          sq += f.x * f.x + f.y * f.y;
          f = add_round<T>(a.z, b.z, &s.z);
          sq += f.x * f.x + f.y * f.y;
          f = add_round<T>(a.w, b.w, &s.w);
          sq += f.x * f.x + f.y * f.y;
          s4[v] = s;
        } else {
          const uint32_t parts[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const float2 f = Pack2<T>::to_floats(parts[p]);
            sq += f.x * f.x + f.y * f.y;
          }
        }
      }
      const float total = row_sum<ROW_THREADS>(sq, scratch);
      const float r = 1.0f / sqrtf(total / static_cast<float>(hidden) + eps);
#pragma unroll
      for (int c = 0; c < ROW_CACHE; ++c) {
        const int v = threadIdx.x + c * ROW_THREADS;
        if (v < nv) {
          const uint4 a = cache[c];
          const uint4 w = __ldg(w4 + v);
          uint4 o;
          o.x = scale_pack<T>(a.x, w.x, r);
          o.y = scale_pack<T>(a.y, w.y, r);
          o.z = scale_pack<T>(a.z, w.z, r);
          o.w = scale_pack<T>(a.w, w.w, r);
          o4[v] = o;
        }
      }
      for (int v = threadIdx.x + ROW_CACHE * ROW_THREADS; v < nv; v += ROW_THREADS) {
        // The same thread stored residual_out[v] above, so the read sees it.
        const uint4 a = ADD ? s4[v] : x4[v];
        const uint4 w = __ldg(w4 + v);
        uint4 o;
        o.x = scale_pack<T>(a.x, w.x, r);
        o.y = scale_pack<T>(a.y, w.y, r);
        o.z = scale_pack<T>(a.z, w.z, r);
        o.w = scale_pack<T>(a.w, w.w, r);
        o4[v] = o;
      }
    } else {
      for (int i = threadIdx.x; i < hidden; i += ROW_THREADS) {
        float v = to_f32(x[base + i]);
        if (ADD) {
          const T s = from_f32<T>(v + to_f32(residual[base + i]));
          residual_out[base + i] = s;
          v = to_f32(s);
        }
        sq += v * v;
      }
      const float total = row_sum<ROW_THREADS>(sq, scratch);
      const float r = 1.0f / sqrtf(total / static_cast<float>(hidden) + eps);
      for (int i = threadIdx.x; i < hidden; i += ROW_THREADS) {
        const float v = to_f32(ADD ? residual_out[base + i] : x[base + i]);
        out[base + i] = from_f32<T>((v * r) * to_f32(weight[i]));
      }
    }
  }
}

// Prefill rows that fit the register cache: each CTA walks a few rows (grid-stride) and
// loads the next row before reducing and storing the current one, so the HBM reads of one
// row overlap the writes of the last (a single wave of one-row CTAs reads everything, then
// writes everything).  Same arithmetic as rms_norm_kernel's VEC path.
template <typename T, bool ADD, int ROW_THREADS>
__global__ void __launch_bounds__(ROW_THREADS)
    rms_norm_pipe_kernel(const T* __restrict__ x, const T* __restrict__ residual,
                         const T* __restrict__ weight, T* __restrict__ out, T* __restrict__ residual_out,
                         int64_t rows, int hidden, float eps) {
  __shared__ float scratch[ROW_THREADS / 32];
  pdl_begin();
  const int nv = hidden / 8;
  const uint4* w4 = reinterpret_cast<const uint4*>(weight);
  uint4 a[ROW_CACHE], b[ROW_CACHE];
  auto load = [&](int64_t row, uint4 (&xa)[ROW_CACHE], uint4 (&rb)[ROW_CACHE]) {
    const size_t base = static_cast<size_t>(row) * hidden;
    const uint4* x4 = reinterpret_cast<const uint4*>(x + base);
    const uint4* r4 = ADD ? reinterpret_cast<const uint4*>(residual + base) : nullptr;
#pragma unroll
    for (int c = 0; c < ROW_CACHE; ++c) {
      const int v = threadIdx.x + c * ROW_THREADS;
      if (v < nv) {
        xa[c] = ld_stream_v4(x4 + v);
        if (ADD) rb[c] = ld_stream_v4(r4 + v);
      }
    }
  };
  int64_t row = blockIdx.x;
  if (row < rows) load(row, a, b);
  for (; row < rows; row += gridDim.x) {
    uint4 na[ROW_CACHE], nb[ROW_CACHE];
    const int64_t next = row + gridDim.x;
    if (next < rows) load(next, na, nb);
    const size_t base = static_cast<size_t>(row) * hidden;
    uint4* s4 = ADD ? reinterpret_cast<uint4*>(residual_out + base) : nullptr;
    uint4* o4 = reinterpret_cast<uint4*>(out + base);
    float sq = 0.f;
#pragma unroll
    for (int c = 0; c < ROW_CACHE; ++c) {
      const int v = threadIdx.x + c * ROW_THREADS;
      if (v < nv) {
        if (ADD) {
          uint4 s;
          float2 f;
          f = add_round<T>(a[c].x, b[c].x, &s.x);
          sq += f.x * f.x + f.y * f.y;
          f = add_round<T>(a[c].y, b[c].y, &s.y);
          sq += f.x * f.x + f.y * f.y;
          f = add_round<T>(a[c].z, b[c].z, &s.z);
          sq += f.x * f.x + f.y * f.y;
          f = add_round<T>(a[c].w, b[c].w, &s.w);
          sq += f.x * f.x + f.y * f.y;
          s4[v] = s;
          a[c] = s;
        } else {
          const uint32_t parts[4] = {a[c].x, a[c].y, a[c].z, a[c].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 f = Pack2<T>::to_floats(parts[q]);
            sq += f.x * f.x + f.y * f.y;
          }
        }
      }
    }
    const float total = row_sum<ROW_THREADS>(sq, scratch);
    const float r = 1.0f / sqrtf(total / static_cast<float>(hidden) + eps);
#pragma unroll
    for (int c = 0; c < ROW_CACHE; ++c) {
      const int v = threadIdx.x + c * ROW_THREADS;
      if (v < nv) {
        const uint4 w = __ldg(w4 + v);
        uint4 o;
        o.x = scale_pack<T>(a[c].x, w.x, r);
        o.y = scale_pack<T>(a[c].y, w.y, r);
        o.z = scale_pack<T>(a[c].z, w.z, r);
        o.w = scale_pack<T>(a[c].w, w.w, r);
        o4[v] = o;
      }
    }
#pragma unroll
    for (int c = 0; c < ROW_CACHE; ++c) {
      a[c] = na[c];
      if (ADD) b[c] = nb[c];
    }
  }
}

int elementwise_grid(int64_t vectors) {
  const int64_t cap = static_cast<int64_t>(device_sm_count()) * 8;  // 8 x 256 threads per SM
  const int64_t want = (vectors + 255) / 256;
  return static_cast<int>(want < 1 ? 1 : (want < cap ? want : cap));
}

// Enough CTAs to fill every SM's thread slots (2048 threads per SM); more rows are
// walked grid-stride.
int row_grid(int64_t rows, int threads) {
  const int64_t cap = static_cast<int64_t>(device_sm_count()) * (2048 / threads);
  return static_cast<int>(rows < cap ? rows : cap);
}

template <typename T>
rk_status silu_mul_typed(const void* gate, const void* up, void* out, int64_t n, cudaStream_t s) {
  const bool vec = aligned16(gate) && aligned16(up) && aligned16(out);
  const int grid = elementwise_grid(vec ? n / 8 : n);
  const cudaError_t e =
      vec ? launch_kernel(silu_mul_kernel<T, true>, dim3(grid), dim3(256), 0, s, 0,
                          static_cast<const T*>(gate), static_cast<const T*>(up),
                          static_cast<T*>(out), n)
          : launch_kernel(silu_mul_kernel<T, false>, dim3(grid), dim3(256), 0, s, 0,
                          static_cast<const T*>(gate), static_cast<const T*>(up),
                          static_cast<T*>(out), n);
  note_launch();
  return cuda_status(e);
}

// Rows per CTA of the prefill pipeline.  Measured on B200 (bf16, CUDA graph, inputs larger
// than L2; one-row CTAs -> 2 / 4 / 8 rows): rms_norm 2048 x 4096 10.3 -> 8.4 / 11.4 / 15.2 us,
// 1024 x 8192 10.8 -> 8.1 / 11.9 / 16.9 us, 8192 x 4096 31.1 -> 24.9 / 24.8 / 25.6 us;
// add_rms_norm within 1 % at 2 rows.  Two rows keep enough rows in flight per SM and still
// overlap each CTA's second read with its first write.
constexpr int NORM_PIPE_RPC = 2;

template <typename T, bool ADD, int THREADS>
cudaError_t launch_rows(bool vec, int64_t rows, const void* x, const void* residual,
                        const void* weight, void* out, void* residual_out, int64_t hidden,
                        float eps, cudaStream_t s) {
  // rms_norm only: add_rms_norm already overlaps its reads with the residual_out stores of
  // the first pass, and measured no faster (slower at 1024 x 8192) with two rows per CTA.
  if (!ADD && vec && hidden / 8 <= static_cast<int64_t>(ROW_CACHE) * THREADS &&
      rows >= 4ll * device_sm_count()) {
    // Prefill: at least NORM_PIPE_RPC rows per CTA, within the resident capacity.
    const int64_t cap = static_cast<int64_t>(device_sm_count()) * (2048 / THREADS);
    int64_t rpc = NORM_PIPE_RPC;
    if ((rows + rpc - 1) / rpc > cap) rpc = (rows + cap - 1) / cap;
    const int grid = static_cast<int>((rows + rpc - 1) / rpc);
    return launch_kernel(rms_norm_pipe_kernel<T, ADD, THREADS>, dim3(grid), dim3(THREADS), 0, s, 0,
                         static_cast<const T*>(x), static_cast<const T*>(residual), static_cast<const T*>(weight),
                         static_cast<T*>(out), static_cast<T*>(residual_out), rows, static_cast<int>(hidden), eps);
  }
  const int grid = row_grid(rows, THREADS);
  auto kernel = vec ? rms_norm_kernel<T, ADD, true, THREADS> : rms_norm_kernel<T, ADD, false, THREADS>;
  return launch_kernel(kernel, dim3(grid), dim3(THREADS), 0, s, 0, static_cast<const T*>(x),
                       static_cast<const T*>(residual), static_cast<const T*>(weight),
                       static_cast<T*>(out), static_cast<T*>(residual_out), rows,
                       static_cast<int>(hidden), eps);
}

template <typename T, bool ADD>
rk_status rms_norm_typed(const void* x, const void* residual, const void* weight, void* out,
                         void* residual_out, int64_t rows, int64_t hidden, float eps,
                         cudaStream_t s) {
  bool vec = hidden % 8 == 0 && aligned16(x) && aligned16(weight) && aligned16(out);
  if (ADD) vec = vec && aligned16(residual) && aligned16(residual_out);
  int threads = g_norm_threads.load();
  if (threads != 64 && threads != 128 && threads != 256) {
    // Few rows (decode): 256 threads per row, the shortest latency per row.  Many rows
    // (prefill): the fewest threads whose register cache still holds the whole row, so
    // more rows are resident per SM (measured on B200: 2048 x 4096 add_rms_norm 10.7 us
    // with 128 threads vs 11.5 us with 256; 1024 x 8192 best with 256).
    threads = 256;
    if (rows >= 2ll * device_sm_count()) {
      const int64_t per_thread = (hidden / 8 + ROW_CACHE - 1) / ROW_CACHE;
      threads = 64;
      while (threads < 256 && threads < per_thread) threads *= 2;
    }
  }
  cudaError_t e;
  if (threads == 64)
    e = launch_rows<T, ADD, 64>(vec, rows, x, residual, weight, out, residual_out, hidden, eps, s);
  else if (threads == 128)
    e = launch_rows<T, ADD, 128>(vec, rows, x, residual, weight, out, residual_out, hidden, eps, s);
  else
    e = launch_rows<T, ADD, 256>(vec, rows, x, residual, weight, out, residual_out, hidden, eps, s);
  note_launch();
  return cuda_status(e);
}

}  // namespace

rk_status silu_mul_launch(const void* gate, const void* up, void* out, int64_t tokens,
                          int64_t hidden, rk_dtype dt, cudaStream_t s) {
  const int64_t n = tokens * hidden;
  if (n == 0) return RK_OK;
  return dt == RK_DTYPE_BF16 ? silu_mul_typed<__nv_bfloat16>(gate, up, out, n, s)
                             : silu_mul_typed<__half>(gate, up, out, n, s);
}

void norm_set_threads(int threads) { g_norm_threads.store(threads); }

rk_status rms_norm_launch(const void* x, const void* residual, const void* weight, void* out,
                          void* residual_out, int64_t tokens, int64_t hidden, float eps,
                          rk_dtype dt, cudaStream_t s) {
  if (tokens == 0) return RK_OK;
  if (hidden > (1ll << 30)) return RK_ERR_UNSUPPORTED;
  const bool add = residual != nullptr;
  if (dt == RK_DTYPE_BF16)
    return add ? rms_norm_typed<__nv_bfloat16, true>(x, residual, weight, out, residual_out, tokens,
                                                      hidden, eps, s)
               : rms_norm_typed<__nv_bfloat16, false>(x, residual, weight, out, residual_out,
                                                       tokens, hidden, eps, s);
  return add ? rms_norm_typed<__half, true>(x, residual, weight, out, residual_out, tokens, hidden,
                                            eps, s)
             : rms_norm_typed<__half, false>(x, residual, weight, out, residual_out, tokens,
                                             hidden, eps, s);
}

}  // namespace rk
