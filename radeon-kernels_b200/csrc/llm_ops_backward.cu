// llm_ops_backward.cu -- backward passes of silu_mul, rms_norm and add_rms_norm.
//
// The reference serves inputs that require gradients through its torch fallbacks, so a
// reference user's gradients are the autograd of those fp32 graphs
// (src/radeon_kernels/ops/swiglu/reference.py:6-9, ops/rms_norm/reference.py:6-10,
// ops/add_rms_norm/reference.py:8-12).  These kernels evaluate the same chain-rule terms
// in the same fp32 order and round once to the dtype:
//
//   silu_mul   out = (g * s) * u, s = sigmoid(g):
//              du = dy * (g * s);   t = dy * u;   dg = t * s + ((t * g) * (1 - s)) * s
//   rms_norm   r = rsqrt(mean(x^2) + eps), y = (x * r) * w:
//              c = sum_j (dy_j * w_j) * x_j;   q = ((-0.5 * c) * (r * r * r)) / H
//              dx = (dy * w) * r + q * (2 * x);   dw = sum_rows dy * (x * r)
//   add_rms_norm  s = x + residual (saved as residual_out), out = rms_norm(s):
//              ds = round(dx of rms_norm at s) + d(residual_out), rounded again (the two
//              gradients of s are 16-bit tensors that autograd adds); dx = dresidual = ds
//
// All three are HBM streams.  silu_mul's backward is one grid-stride loop over 16-byte
// vectors (reads dy, g, u; writes dg, du).  The normalisations use a CTA per row
// (grid-stride over rows) with dy and x of the row held in registers between the two
// row sums (sum of squares, sum of dy*w*x) and the gradient stores.  The weight gradient
// is a column sum over rows: each CTA accumulates its rows' dy * (x * r) in shared memory
// (one fp32 slot per column, each owned by one thread, so no atomics); the CTAs of a
// thread-block cluster of 8 then add their accumulators through distributed shared memory
// (rank r sums column slice r over the 8 CTAs in rank order) and write one fp32 partial
// row per cluster to the caller's workspace, and a second kernel adds the partial rows in
// cluster order -- deterministic for a given shape and device.  (One partial row per CTA
// made the second kernel the larger of the two: 24 us for 1184 partial rows of 4096.)
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>

#include "rk_device.cuh"
#include "rk_internal.h"

namespace rk {
namespace {

constexpr int BWD_CACHE = 4;          // 16-byte vectors of dy and of x per thread in registers
constexpr int MAX_DW_HIDDEN = 49152;  // shared-memory weight-gradient accumulators (192 KiB)
constexpr int DW_CLUSTER = 8;         // CTAs whose accumulators are added before the write-out

std::atomic<int> g_bwd_ctas_per_sm{0};  // tuning override of the row kernel's CTAs per SM

// -------------------------------------------------------------------- silu_mul
__device__ __forceinline__ void silu_mul_grad(float dy, float g, float u, float& dg, float& du) {
  const float s = __fdividef(1.0f, 1.0f + __expf(-g));  // the forward's sigmoid (swiglu_f32)
  du = dy * (g * s);
  const float t = dy * u;  // gradient of g * s
  dg = t * s + ((t * g) * (1.0f - s)) * s;
}

template <typename T>
__device__ __forceinline__ void silu_grad_pack(uint32_t dy2, uint32_t g2, uint32_t u2,
                                               uint32_t& dg2, uint32_t& du2) {
  const float2 dy = Pack2<T>::to_floats(dy2);
  const float2 g = Pack2<T>::to_floats(g2);
  const float2 u = Pack2<T>::to_floats(u2);
  float dga, dua, dgb, dub;
  silu_mul_grad(dy.x, g.x, u.x, dga, dua);
  silu_mul_grad(dy.y, g.y, u.y, dgb, dub);
  dg2 = Pack2<T>::from_floats(dga, dgb);
  du2 = Pack2<T>::from_floats(dua, dub);
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(256)
    silu_mul_backward_kernel(const T* __restrict__ dy, const T* __restrict__ gate,
                             const T* __restrict__ up, T* __restrict__ dgate, T* __restrict__ dup,
                             int64_t n) {
  pdl_begin();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  int64_t done = 0;
  if (VEC) {
    const int64_t nv = n / 8;
    const uint4* d4 = reinterpret_cast<const uint4*>(dy);
    const uint4* g4 = reinterpret_cast<const uint4*>(gate);
    const uint4* u4 = reinterpret_cast<const uint4*>(up);
    uint4* dg4 = reinterpret_cast<uint4*>(dgate);
    uint4* du4 = reinterpret_cast<uint4*>(dup);
    for (int64_t i = t0; i < nv; i += stride) {
      const uint4 d = ld_stream_v4(d4 + i);
      const uint4 g = ld_stream_v4(g4 + i);
      const uint4 u = ld_stream_v4(u4 + i);
      uint4 og, ou;
      silu_grad_pack<T>(d.x, g.x, u.x, og.x, ou.x);
      silu_grad_pack<T>(d.y, g.y, u.y, og.y, ou.y);
      silu_grad_pack<T>(d.z, g.z, u.z, og.z, ou.z);
      silu_grad_pack<T>(d.w, g.w, u.w, og.w, ou.w);
      dg4[i] = og;
      du4[i] = ou;
    }
    done = nv * 8;
  }
  for (int64_t i = done + t0; i < n; i += stride) {
    float dg, du;
    silu_mul_grad(to_f32(dy[i]), to_f32(gate[i]), to_f32(up[i]), dg, du);
    dgate[i] = from_f32<T>(dg);
    dup[i] = from_f32<T>(du);
  }
}

// ------------------------------------------------------------- (add_)rms_norm
// Two row sums in one pass, fixed order: shuffle tree per warp, then the warp sums added
// in warp order.  Every thread receives both totals.
template <int ROW_THREADS>
__device__ __forceinline__ float2 row_sum2(float a, float b, float2* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // scratch is reused row after row
  if (lane == 0) scratch[warp] = make_float2(a, b);
  __syncthreads();
  float2 t = make_float2(0.f, 0.f);
#pragma unroll
  for (int w = 0; w < ROW_THREADS / 32; ++w) {
    t.x += scratch[w].x;
    t.y += scratch[w].y;
  }
  return t;
}

// Accumulates x^2 and (dy * w) * x of one packed pair.
template <typename T>
__device__ __forceinline__ void pass1_pair(uint32_t dy2, uint32_t x2, uint32_t w2, float& sq,
                                           float& c) {
  const float2 d = Pack2<T>::to_floats(dy2);
  const float2 x = Pack2<T>::to_floats(x2);
  const float2 w = Pack2<T>::to_floats(w2);
  sq += x.x * x.x + x.y * x.y;
  c += (d.x * w.x) * x.x + (d.y * w.y) * x.y;
}

// Input gradient of one element (fp32, before rounding).
__device__ __forceinline__ float grad_x(float dy, float x, float w, float r, float q) {
  return (dy * w) * r + q * (2.0f * x);
}

// Gradients of one packed pair: the rounded input gradient, plus (ADD with a
// residual_out gradient) that gradient, rounded again; adds dy * (x * r) to the pair's
// weight-gradient slots.  Without a residual_out gradient nothing is added (autograd adds
// no term, so a -0 input gradient stays -0).
template <typename T, bool ADD, bool DW>
__device__ __forceinline__ uint32_t pass2_pair(uint32_t dy2, uint32_t x2, uint32_t w2,
                                               uint32_t dres2, bool has_dres, float r, float q,
                                               float* dw_a, float* dw_b) {
  const float2 d = Pack2<T>::to_floats(dy2);
  const float2 x = Pack2<T>::to_floats(x2);
  const float2 w = Pack2<T>::to_floats(w2);
  uint32_t out = Pack2<T>::from_floats(grad_x(d.x, x.x, w.x, r, q), grad_x(d.y, x.y, w.y, r, q));
  if (ADD && has_dres) {
    const float2 g = Pack2<T>::to_floats(out);
    const float2 e = Pack2<T>::to_floats(dres2);
    out = Pack2<T>::from_floats(g.x + e.x, g.y + e.y);
  }
  if (DW) {
    *dw_a += d.x * (x.x * r);
    *dw_b += d.y * (x.y * r);
  }
  return out;
}

// One CTA per row, grid-stride.  x is the normalised tensor's input (rms_norm) or
// residual_out (add_rms_norm).  ADD: dres (nullable: no residual_out gradient) is added to
// the rounded input gradient and the sum is stored to dx and, when non-null, dres_out.
// DW (launched in clusters of DW_CLUSTER CTAs, grid a multiple of it): shared memory holds
// `hidden` fp32 accumulators in column order; after the rows, the cluster's sum goes to
// dw_partial[(blockIdx.x / DW_CLUSTER) * hidden ...].  Every thread reaches both cluster
// barriers (no early exit), and the second keeps each CTA's shared memory alive until the
// other CTAs of its cluster have read it.
template <typename T, bool ADD, bool VEC, bool DW, int ROW_THREADS>
__global__ void __launch_bounds__(ROW_THREADS)
    rms_norm_backward_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                             const T* __restrict__ weight, const T* __restrict__ dres,
                             T* __restrict__ dx, T* __restrict__ dres_out,
                             float* __restrict__ dw_partial, int64_t rows, int hidden, float eps) {
  extern __shared__ __align__(16) float sdw[];
  __shared__ float2 scratch[ROW_THREADS / 32];
  const int nv = hidden / 8;
  // Weight-gradient accumulators: registers for the register-cached vectors of a row
  // (columns 8 v .. 8 v + 7 of vector v = threadIdx.x + k * ROW_THREADS), shared memory for
  // the rest (longer rows, scalar path), which therefore starts at zero.
  float dwreg[BWD_CACHE][8];
#pragma unroll
  for (int k = 0; k < BWD_CACHE; ++k)
#pragma unroll
    for (int j = 0; j < 8; ++j) dwreg[k][j] = 0.f;
  const int cached_cols = VEC ? 8 * BWD_CACHE * ROW_THREADS : 0;
  if (DW)
    for (int i = cached_cols + threadIdx.x; i < hidden; i += ROW_THREADS) sdw[i] = 0.f;
  pdl_begin();
  const float inv_h = 1.0f / static_cast<float>(hidden);
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const size_t base = static_cast<size_t>(row) * hidden;
    float sq = 0.f, c = 0.f;
    if (VEC) {
      const uint4* d4 = reinterpret_cast<const uint4*>(dy + base);
      const uint4* x4 = reinterpret_cast<const uint4*>(x + base);
      const uint4* w4 = reinterpret_cast<const uint4*>(weight);
      uint4 dcache[BWD_CACHE], xcache[BWD_CACHE];
#pragma unroll
      for (int k = 0; k < BWD_CACHE; ++k) {
        const int v = threadIdx.x + k * ROW_THREADS;
        if (v < nv) {
          dcache[k] = ld_stream_v4(d4 + v);
          xcache[k] = ld_stream_v4(x4 + v);
        }
      }
#pragma unroll
      for (int k = 0; k < BWD_CACHE; ++k) {
        const int v = threadIdx.x + k * ROW_THREADS;
        if (v < nv) {
          const uint4 w = __ldg(w4 + v);
          pass1_pair<T>(dcache[k].x, xcache[k].x, w.x, sq, c);
          pass1_pair<T>(dcache[k].y, xcache[k].y, w.y, sq, c);
          pass1_pair<T>(dcache[k].z, xcache[k].z, w.z, sq, c);
          pass1_pair<T>(dcache[k].w, xcache[k].w, w.w, sq, c);
        }
      }
      // Rows longer than the register cache: streamed once here, read back from L2 below.
      for (int v = threadIdx.x + BWD_CACHE * ROW_THREADS; v < nv; v += ROW_THREADS) {
        const uint4 d = d4[v], xv = x4[v], w = __ldg(w4 + v);
        pass1_pair<T>(d.x, xv.x, w.x, sq, c);
        pass1_pair<T>(d.y, xv.y, w.y, sq, c);
        pass1_pair<T>(d.z, xv.z, w.z, sq, c);
        pass1_pair<T>(d.w, xv.w, w.w, sq, c);
      }
      const float2 tot = row_sum2<ROW_THREADS>(sq, c, scratch);
      const float r = 1.0f / sqrtf(tot.x * inv_h + eps);
      const float q = ((-0.5f * tot.y) * (r * r * r)) / static_cast<float>(hidden);
      const uint4* e4 = ADD && dres != nullptr ? reinterpret_cast<const uint4*>(dres + base) : nullptr;
      uint4* o4 = reinterpret_cast<uint4*>(dx + base);
      uint4* ro4 = ADD && dres_out != nullptr ? reinterpret_cast<uint4*>(dres_out + base) : nullptr;
      auto store = [&](int v, const uint4& d, const uint4& xv, float* acc) {
        const uint4 w = __ldg(w4 + v);
        const bool has = e4 != nullptr;
        const uint4 e = has ? ld_stream_v4(e4 + v) : make_uint4(0u, 0u, 0u, 0u);
        uint4 o;
        o.x = pass2_pair<T, ADD, DW>(d.x, xv.x, w.x, e.x, has, r, q, acc + 0, acc + 1);
        o.y = pass2_pair<T, ADD, DW>(d.y, xv.y, w.y, e.y, has, r, q, acc + 2, acc + 3);
        o.z = pass2_pair<T, ADD, DW>(d.z, xv.z, w.z, e.z, has, r, q, acc + 4, acc + 5);
        o.w = pass2_pair<T, ADD, DW>(d.w, xv.w, w.w, e.w, has, r, q, acc + 6, acc + 7);
        o4[v] = o;
        if (ro4 != nullptr) ro4[v] = o;
      };
#pragma unroll
      for (int k = 0; k < BWD_CACHE; ++k) {
        const int v = threadIdx.x + k * ROW_THREADS;
        if (v < nv) store(v, dcache[k], xcache[k], dwreg[k]);
      }
      for (int v = threadIdx.x + BWD_CACHE * ROW_THREADS; v < nv; v += ROW_THREADS) {
        float acc[8];
        float4* s4 = reinterpret_cast<float4*>(sdw) + 2 * v;  // columns 8 v .. 8 v + 7
        if (DW) {
          const float4 lo = s4[0], hi = s4[1];
          acc[0] = lo.x, acc[1] = lo.y, acc[2] = lo.z, acc[3] = lo.w;
          acc[4] = hi.x, acc[5] = hi.y, acc[6] = hi.z, acc[7] = hi.w;
        }
        store(v, d4[v], x4[v], acc);
        if (DW) {
          s4[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
          s4[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
        }
      }
    } else {
      for (int i = threadIdx.x; i < hidden; i += ROW_THREADS) {
        const float d = to_f32(dy[base + i]), xv = to_f32(x[base + i]);
        sq += xv * xv;
        c += (d * to_f32(weight[i])) * xv;
      }
      const float2 tot = row_sum2<ROW_THREADS>(sq, c, scratch);
      const float r = 1.0f / sqrtf(tot.x * inv_h + eps);
      const float q = ((-0.5f * tot.y) * (r * r * r)) / static_cast<float>(hidden);
      for (int i = threadIdx.x; i < hidden; i += ROW_THREADS) {
        const float d = to_f32(dy[base + i]), xv = to_f32(x[base + i]);
        T g = from_f32<T>(grad_x(d, xv, to_f32(weight[i]), r, q));
        if (ADD) {
          if (dres != nullptr) g = from_f32<T>(to_f32(g) + to_f32(dres[base + i]));
          if (dres_out != nullptr) dres_out[base + i] = g;
        }
        dx[base + i] = g;
        if (DW) sdw[i] += d * (xv * r);
      }
    }
  }
  if (DW) {
    if (VEC) {
#pragma unroll
      for (int k = 0; k < BWD_CACHE; ++k) {
        const int v = threadIdx.x + k * ROW_THREADS;
        if (v < nv) {
          float4* s4 = reinterpret_cast<float4*>(sdw) + 2 * v;
          s4[0] = make_float4(dwreg[k][0], dwreg[k][1], dwreg[k][2], dwreg[k][3]);
          s4[1] = make_float4(dwreg[k][4], dwreg[k][5], dwreg[k][6], dwreg[k][7]);
        }
      }
    }
    cluster_sync_all();  // every CTA of the cluster has finished accumulating
    const uint32_t rank = cluster_ctarank();
    float* part = dw_partial + static_cast<size_t>(blockIdx.x / DW_CLUSTER) * hidden;
    const uint32_t base = smem_u32(sdw);
    if (VEC) {
      // hidden % 8 == 0: float4 slices, rank r takes float4 columns [r * per, (r + 1) * per).
      const int n4 = hidden / 4;
      const int per = (n4 + DW_CLUSTER - 1) / DW_CLUSTER;
      const int end = min(n4, static_cast<int>(rank + 1) * per);
      for (int i = static_cast<int>(rank) * per + threadIdx.x; i < end; i += ROW_THREADS) {
        float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int q = 0; q < DW_CLUSTER; ++q) {
          const float4 v = ld_cluster_v4(map_to_rank(base + 16u * i, q));
          t.x += v.x, t.y += v.y, t.z += v.z, t.w += v.w;
        }
        reinterpret_cast<float4*>(part)[i] = t;
      }
    } else {
      const int per = (hidden + DW_CLUSTER - 1) / DW_CLUSTER;
      const int end = min(hidden, static_cast<int>(rank + 1) * per);
      for (int i = static_cast<int>(rank) * per + threadIdx.x; i < end; i += ROW_THREADS) {
        float t = 0.f;
#pragma unroll
        for (int q = 0; q < DW_CLUSTER; ++q) t += ld_cluster_f32(map_to_rank(base + 4u * i, q));
        part[i] = t;
      }
    }
    cluster_sync_all();  // peers are done reading this CTA's accumulators
  }
}

// dw[col] = sum over the partial rows in cluster order, rounded once.  32 columns x
// REDUCE_GROUPS groups per CTA: group g adds a fixed contiguous range of partial rows
// (all its loads independent, so they are in flight together), then the group sums are
// added in group order.
constexpr int REDUCE_GROUPS = 32;

template <typename T>
__global__ void __launch_bounds__(32 * REDUCE_GROUPS)
    weight_grad_reduce_kernel(const float* __restrict__ partial, int parts, int hidden,
                              T* __restrict__ dw) {
  __shared__ float acc[REDUCE_GROUPS][33];
  const int lane = threadIdx.x & 31, grp = threadIdx.x >> 5;
  const int col = blockIdx.x * 32 + lane;
  pdl_begin();
  const int per = (parts + REDUCE_GROUPS - 1) / REDUCE_GROUPS;
  float s = 0.f;
  if (col < hidden) {
    const int p0 = grp * per, p1 = min(parts, p0 + per);
#pragma unroll 8
    for (int p = p0; p < p1; ++p) s += partial[static_cast<size_t>(p) * hidden + col];
  }
  acc[grp][lane] = s;
  __syncthreads();
  if (grp == 0 && col < hidden) {
    float t = 0.f;
#pragma unroll
    for (int g = 0; g < REDUCE_GROUPS; ++g) t += acc[g][lane];
    dw[col] = from_f32<T>(t);
  }
}

int elementwise_grid(int64_t vectors) {
  const int64_t cap = static_cast<int64_t>(device_sm_count()) * 8;  // 8 x 256 threads per SM
  const int64_t want = (vectors + 255) / 256;
  return static_cast<int>(want < 1 ? 1 : (want < cap ? want : cap));
}

template <typename T>
rk_status silu_mul_backward_typed(const void* dy, const void* gate, const void* up, void* dgate,
                                  void* dup, int64_t n, cudaStream_t s) {
  const bool vec = aligned16(dy) && aligned16(gate) && aligned16(up) && aligned16(dgate) &&
                   aligned16(dup);
  const int grid = elementwise_grid(vec ? n / 8 : n);
  auto kernel = vec ? silu_mul_backward_kernel<T, true> : silu_mul_backward_kernel<T, false>;
  const cudaError_t e = launch_kernel(kernel, dim3(grid), dim3(256), 0, s, 0,
                                      static_cast<const T*>(dy), static_cast<const T*>(gate),
                                      static_cast<const T*>(up), static_cast<T*>(dgate),
                                      static_cast<T*>(dup), n);
  note_launch();
  return cuda_status(e);
}

// Threads per row: 256 for few rows; from two rows per SM, the fewest threads whose
// register cache holds the row (as the forward kernels).
int bwd_threads(int64_t rows, int64_t hidden) {
  if (rows < 2ll * device_sm_count()) return 256;
  const int64_t per_thread = (hidden / 8 + BWD_CACHE - 1) / BWD_CACHE;
  int threads = 64;
  while (threads < 256 && threads < per_thread) threads *= 2;
  return threads;
}

// CTAs of the row kernel: up to 2048 threads per SM, one row each, more rows walked
// grid-stride.  With a weight gradient the grid is a multiple of the cluster size (CTAs
// past the last row only add zeros).
int bwd_grid(int64_t rows, int threads, bool dw) {
  const int sms = device_sm_count();
  int per_sm = g_bwd_ctas_per_sm.load();
  if (per_sm <= 0) per_sm = 2048 / threads;
  const int64_t cap = static_cast<int64_t>(sms) * per_sm;
  int64_t grid = rows < cap ? rows : cap;
  if (dw) {
    // About four rows per CTA once there are enough rows for every SM: the cluster
    // sum and the partial-row write are paid once per CTA.
    if (g_bwd_ctas_per_sm.load() <= 0) {
      const int64_t quarter = (rows + 3) / 4;
      const int64_t floor_rows = rows < sms ? rows : sms;
      grid = std::min(grid, std::max(quarter, floor_rows));
    }
    grid = (grid + DW_CLUSTER - 1) / DW_CLUSTER * DW_CLUSTER;
  }
  return static_cast<int>(grid);
}

template <typename T, bool ADD, bool DW, int THREADS>
cudaError_t launch_bwd_rows(bool vec, int grid, const void* dy, const void* x, const void* w,
                            const void* dres, void* dx, void* dres_out, float* partial,
                            int64_t rows, int64_t hidden, float eps, cudaStream_t s) {
  auto kernel = vec ? rms_norm_backward_kernel<T, ADD, true, DW, THREADS>
                    : rms_norm_backward_kernel<T, ADD, false, DW, THREADS>;
  const size_t smem = DW ? static_cast<size_t>(hidden) * sizeof(float) : 0;
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  return launch_kernel(kernel, dim3(grid), dim3(THREADS), smem, s, DW ? DW_CLUSTER : 0,
                       static_cast<const T*>(dy),
                       static_cast<const T*>(x), static_cast<const T*>(w),
                       static_cast<const T*>(dres), static_cast<T*>(dx), static_cast<T*>(dres_out),
                       partial, rows, static_cast<int>(hidden), eps);
}

template <typename T, bool ADD, bool DW>
cudaError_t launch_bwd_threads(int threads, bool vec, int grid, const void* dy, const void* x,
                               const void* w, const void* dres, void* dx, void* dres_out,
                               float* partial, int64_t rows, int64_t hidden, float eps,
                               cudaStream_t s) {
  if (threads == 64)
    return launch_bwd_rows<T, ADD, DW, 64>(vec, grid, dy, x, w, dres, dx, dres_out, partial, rows,
                                           hidden, eps, s);
  if (threads == 128)
    return launch_bwd_rows<T, ADD, DW, 128>(vec, grid, dy, x, w, dres, dx, dres_out, partial,
                                            rows, hidden, eps, s);
  return launch_bwd_rows<T, ADD, DW, 256>(vec, grid, dy, x, w, dres, dx, dres_out, partial, rows,
                                          hidden, eps, s);
}

template <typename T, bool ADD>
rk_status rms_norm_backward_typed(const void* dy, const void* x, const void* w, const void* dres,
                                  void* dx, void* dres_out, void* dw, int64_t rows, int64_t hidden,
                                  float eps, void* workspace, size_t workspace_bytes,
                                  cudaStream_t s) {
  bool vec = hidden % 8 == 0 && aligned16(dy) && aligned16(x) && aligned16(w) && aligned16(dx);
  if (ADD) vec = vec && aligned16(dres) && aligned16(dres_out);
  const bool want_dw = dw != nullptr;
  const int threads = bwd_threads(rows, hidden);
  const int grid = bwd_grid(rows, threads, want_dw);
  float* partial = static_cast<float*>(workspace);
  const int parts = grid / DW_CLUSTER;
  if (want_dw) {
    if (hidden > MAX_DW_HIDDEN) return RK_ERR_UNSUPPORTED;
    if (workspace == nullptr ||
        workspace_bytes < static_cast<size_t>(parts) * static_cast<size_t>(hidden) * sizeof(float) ||
        !aligned16(workspace))
      return RK_ERR_INVALID_ARGUMENT;
  }
  cudaError_t e = want_dw ? launch_bwd_threads<T, ADD, true>(threads, vec, grid, dy, x, w, dres, dx,
                                                             dres_out, partial, rows, hidden, eps, s)
                          : launch_bwd_threads<T, ADD, false>(threads, vec, grid, dy, x, w, dres, dx,
                                                              dres_out, nullptr, rows, hidden, eps, s);
  note_launch();
  if (e != cudaSuccess || !want_dw) return cuda_status(e);
  e = launch_kernel(weight_grad_reduce_kernel<T>, dim3(static_cast<unsigned>((hidden + 31) / 32)),
                    dim3(32 * REDUCE_GROUPS), 0, s, 0, static_cast<const float*>(partial), parts,
                    static_cast<int>(hidden), static_cast<T*>(dw));
  note_launch();
  return cuda_status(e);
}

}  // namespace

void norm_backward_set_ctas_per_sm(int ctas) { g_bwd_ctas_per_sm.store(ctas); }

size_t rms_norm_backward_workspace_bytes(int64_t tokens, int64_t hidden) {
  if (tokens <= 0 || hidden <= 0) return 0;
  const int grid = bwd_grid(tokens, bwd_threads(tokens, hidden), true);
  return static_cast<size_t>(grid / DW_CLUSTER) * static_cast<size_t>(hidden) * sizeof(float);
}

rk_status silu_mul_backward_launch(const void* dy, const void* gate, const void* up, void* dgate,
                                   void* dup, int64_t tokens, int64_t hidden, rk_dtype dt,
                                   cudaStream_t s) {
  const int64_t n = tokens * hidden;
  if (n == 0) return RK_OK;
  return dt == RK_DTYPE_BF16
             ? silu_mul_backward_typed<__nv_bfloat16>(dy, gate, up, dgate, dup, n, s)
             : silu_mul_backward_typed<__half>(dy, gate, up, dgate, dup, n, s);
}

rk_status rms_norm_backward_launch(const void* dy, const void* x, const void* w, bool add,
                                   const void* dres, void* dx, void* dres_out, void* dw,
                                   int64_t tokens, int64_t hidden, float eps, rk_dtype dt,
                                   void* workspace, size_t workspace_bytes, cudaStream_t s) {
  if (hidden > (1ll << 30)) return RK_ERR_UNSUPPORTED;
  if (tokens == 0) {
    // The weight gradient of no rows is zero.
    return dw == nullptr ? RK_OK
                         : cuda_status(cudaMemsetAsync(dw, 0, static_cast<size_t>(hidden) * 2, s));
  }
  if (dt == RK_DTYPE_BF16)
    return add ? rms_norm_backward_typed<__nv_bfloat16, true>(dy, x, w, dres, dx, dres_out, dw, tokens,
                                                               hidden, eps, workspace, workspace_bytes, s)
               : rms_norm_backward_typed<__nv_bfloat16, false>(dy, x, w, dres, dx, dres_out, dw, tokens,
                                                                hidden, eps, workspace, workspace_bytes, s);
  return add ? rms_norm_backward_typed<__half, true>(dy, x, w, dres, dx, dres_out, dw, tokens, hidden,
                                                     eps, workspace, workspace_bytes, s)
             : rms_norm_backward_typed<__half, false>(dy, x, w, dres, dx, dres_out, dw, tokens, hidden,
                                                      eps, workspace, workspace_bytes, s);
}

}  // namespace rk
