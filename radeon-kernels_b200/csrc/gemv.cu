// gemv.cu -- decode GEMV / skinny GEMM: out[M,N] = x[M,K] @ W[N,K]^T, M <= 32.
//
// The weight is the only large operand (N*K*2 bytes, read exactly once), so
// the kernel is an HBM stream.  Design for B200:
//   * each warp owns ROWS weight rows and a contiguous slice of K; every lane
//     issues 128-bit `ld.global.nc.L1::no_allocate` loads, a warp covers 512
//     contiguous bytes of a row per load, UNROLL x ROWS loads are in flight
//     per lane before the first FMA (Little's law: ~5 MB must be in flight
//     across 148 SMs to cover HBM latency);
//   * x (at most 32 x K x 2 bytes) stays in L2/L1 and is read with __ldg;
//     one 16-byte x vector feeds ROWS rows;
//   * M >= 2: each weight word is widened to fp32 once and feeds every row of x
//     through packed FMAs (fma.rn.f32x2), so the work per weight element grows by
//     one FMA lane per row of x, not by a widening and a scalar FMA;
//   * fp32 accumulation, warp-shuffle tree reduction;
//   * split-K inside the CTA: the 8 warps form (8/KS) row groups x KS K-slices
//     and the KS partial sums are added in a fixed order through shared
//     memory -- deterministic, no workspace, no second launch.  KS grows when
//     N is too small to give every SM enough rows.
// No tensor cores.  HBM-bound at M = 1; from M = 3 the automatic choice is the tcgen05
// skinny kernel (gemv_tcgen05.cu), which keeps the weight stream at HBM speed while the
// FMA work here grows with M.
//
// Role of the reference: replaces gemv_wave_kernel / gemv_packed_kernel /
// gemv_lds_kernel (benchmarks/gemv/native_gemv.hip:30-203), whose lanes
// stride K one element at a time (native_gemv.hip:49-58).
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <map>
#include <mutex>
#include <tuple>

#include "rk_device.cuh"
#include "rk_internal.h"
#include "rk_peer.cuh"

namespace rk {

static std::atomic<int> g_gemv_rows_override{0};
static std::atomic<int> g_gemv_ks_override{0};

namespace {

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T, int MB, int ROWS>
__device__ __forceinline__ void fma_vec(float (&acc)[MB][ROWS], const uint4 (&w)[ROWS],
                                        const uint4& xv, int m) {
  const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const float2 xf = Pack2<T>::to_floats(xs[p]);
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const uint32_t ws[4] = {w[r].x, w[r].y, w[r].z, w[r].w};
      const float2 wf = Pack2<T>::to_floats(ws[p]);
      acc[m][r] = fmaf(wf.x, xf.x, acc[m][r]);
      acc[m][r] = fmaf(wf.y, xf.y, acc[m][r]);
    }
  }
}

// M >= 2: one 16-byte vector of each of ROWS weight rows against the x vectors of every
// row m < M at the same k.  Each weight word is widened once and feeds all M rows through
// packed fp32 FMAs (fma.rn.f32x2: even and odd k accumulate in the two halves of acc, added
// at the end), so the per-element work is one FMA lane per row of x plus a shared widening.
template <typename T, int MB, int ROWS>
__device__ __forceinline__ void fma_rows(float2 (&acc)[MB][ROWS], const uint4 (&w)[ROWS],
                                         const uint4 (&xv)[MB], int M) {
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    float2 wf[ROWS];
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const uint32_t ws[4] = {w[r].x, w[r].y, w[r].z, w[r].w};
      wf[r] = Pack2<T>::to_floats(ws[p]);
    }
#pragma unroll
    for (int m = 0; m < MB; ++m) {
      if (m < M) {
        const uint32_t xs[4] = {xv[m].x, xv[m].y, xv[m].z, xv[m].w};
        const float2 xf = Pack2<T>::to_floats(xs[p]);
#pragma unroll
        for (int r = 0; r < ROWS; ++r) acc[m][r] = ffma2(wf[r], xf, acc[m][r]);
      }
    }
  }
}

// Reduce V = MB*ROWS per-lane partial sums across the warp with a transposed
// butterfly (V-1 + 5-log2(V) shuffles instead of 5*V): afterwards lane L holds
// the full sum of value index (L >> (5 - log2 V)).
template <int V>
__device__ __forceinline__ float warp_reduce_scatter(float (&vals)[V], int lane) {
  static_assert((V & (V - 1)) == 0 && V >= 1 && V <= 32, "V must be a power of two <= 32");
  int count = V;
#pragma unroll
  for (int offset = 16; offset >= 1; offset >>= 1) {
    if (count > 1) {
      const bool upper = (lane & offset) != 0;
      const int half = count / 2;
#pragma unroll
      for (int i = 0; i < V / 2; ++i) {
        if (i < half) {
          const float send = upper ? vals[i] : vals[i + half];
          const float keep = upper ? vals[i + half] : vals[i];
          vals[i] = keep + __shfl_xor_sync(0xffffffffu, send, offset);
        }
      }
      count = half;
    } else {
      vals[0] += __shfl_xor_sync(0xffffffffu, vals[0], offset);
    }
  }
  return vals[0];
}

template <int V>
struct Log2 {
  static constexpr int value = V <= 1 ? 0 : 1 + Log2<V / 2>::value;
};
template <>
struct Log2<1> {
  static constexpr int value = 0;
};

// Balanced streaming GEMV.  CTA c owns a contiguous block of rows (the grid is
// sized to the GPU's resident-CTA capacity and rows are dealt out so no CTA has
// more than one row more than another: no second-wave tail).  Inside the CTA
// the 8 warps form (8/KS) row groups x KS K-slices; a warp streams ROWS rows of
// its K-slice at a time with UNROLL 16-byte loads per row per lane in flight
// (out-of-range vectors are predicated off, never loaded).  Per-warp partial
// sums go to shared memory [KS][rows][MB] and are added in ks order.
//
// PEER: the fused all-gather form (rk_gemv_allgather).  W holds this rank's block of
// weight rows; the output (peer.out[rank], row stride peer.ldo) is gathered into every
// rank's full output at the end of the kernel as rk_peer.cuh describes, the push done by
// the grid's last CTA (the block is at most 32 x N elements).  CTA 0 announces the call at
// the start.
template <typename T, int MB, int ROWS, int KS, bool PEER = false>
__global__ void __launch_bounds__(GEMV_THREADS)
    gemv_stream_kernel(const T* __restrict__ x, const T* __restrict__ W, T* __restrict__ out,
                       int M, int N, int K, int rows_base, int rows_rem, int rows_max,
                       const __grid_constant__ PeerOut<T> peer) {
  constexpr int RG = GEMV_WARPS / KS;
  constexpr int UNROLL = ROWS >= 4 ? 2 : 4;
  constexpr int V = MB * ROWS;
  constexpr int LOGV = Log2<V>::value;
  extern __shared__ float red[];  // [KS][rows_max][MB]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rg = warp / KS, ks = warp % KS;
  const int cta = blockIdx.x;
  const int row_begin = cta * rows_base + min(cta, rows_rem);
  const int rows = rows_base + (cta < rows_rem ? 1 : 0);
  const int KV = K >> 3;  // 16-byte vectors per row
  const int v0 = static_cast<int>(static_cast<int64_t>(KV) * ks / KS);
  const int v1 = static_cast<int>(static_cast<int64_t>(KV) * (ks + 1) / KS);
  // Warm L2 with this warp's first step of weight loads (ROWS rows x up to 32 x UNROLL
  // vectors) while the previous kernel of the stream drains: a prefetch has no result and
  // L2 is coherent, so it may precede the dependency wait.  The weight only.
  if (lane < ROWS && rg * ROWS + lane < rows && v1 > v0) {
    const int row = row_begin + rg * ROWS + lane;
    const int vecs = min(v1 - v0, 32 * UNROLL);
    prefetch_l2_bulk(W + static_cast<size_t>(row) * K + static_cast<size_t>(v0) * 8,
                     static_cast<uint32_t>(vecs) * 16u);
  }

  pdl_begin();
  uint32_t epoch = 0;
  if constexpr (PEER) {
    epoch = peer_call_epoch(peer);
    if (blockIdx.x == 0 && threadIdx.x == 0) peer_announce(peer, epoch);
  }
  const uint4* xrow = reinterpret_cast<const uint4*>(x);

  // Row chunks of ROWS rows are dealt to the RG row groups round-robin.
  for (int i0 = rg * ROWS; i0 < rows; i0 += RG * ROWS) {
    const uint4* wrow[ROWS];
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const int row = row_begin + min(i0 + r, rows - 1);  // duplicates are never stored
      wrow[r] = reinterpret_cast<const uint4*>(W + static_cast<size_t>(row) * K);
    }
    float acc[MB][ROWS];    // M = 1
    float2 acc2[MB][ROWS];  // M >= 2 (even / odd k)
#pragma unroll
    for (int m = 0; m < MB; ++m)
#pragma unroll
      for (int r = 0; r < ROWS; ++r) {
        acc[m][r] = 0.f;
        acc2[m][r] = make_float2(0.f, 0.f);
      }

    for (int v = v0 + lane; v < v1; v += 32 * UNROLL) {
      uint4 w[UNROLL][ROWS];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const bool in = v + 32 * u < v1;
#pragma unroll
        for (int r = 0; r < ROWS; ++r)
          w[u][r] = in ? ld_stream_v4(wrow[r] + v + 32 * u) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        if (v + 32 * u < v1) {
          if constexpr (MB == 1) {
            fma_vec<T, MB, ROWS>(acc, w[u], __ldg(xrow + v + 32 * u), 0);
          } else {
            uint4 xv[MB];
#pragma unroll
            for (int m = 0; m < MB; ++m)
              xv[m] = m < M ? __ldg(xrow + static_cast<size_t>(m) * KV + v + 32 * u) : make_uint4(0, 0, 0, 0);
            fma_rows<T, MB, ROWS>(acc2, w[u], xv, M);
          }
        }
      }
    }

    float vals[V];
#pragma unroll
    for (int m = 0; m < MB; ++m)
#pragma unroll
      for (int r = 0; r < ROWS; ++r) vals[m * ROWS + r] = MB == 1 ? acc[m][r] : acc2[m][r].x + acc2[m][r].y;
    const float sum = warp_reduce_scatter<V>(vals, lane);
    const int idx = lane >> (5 - LOGV);  // value index this lane now holds
    if ((lane & ((1 << (5 - LOGV)) - 1)) == 0) {
      const int m = idx / ROWS, r = idx % ROWS;
      if (i0 + r < rows) red[(ks * rows_max + i0 + r) * MB + m] = sum;
    }
  }
  __syncthreads();
  if constexpr (PEER) {
    // Every CTA stores its rows into this rank's own full output and sends them to every
    // other rank as packets {value bits, call number} in that rank's staging slot of this
    // call's parity (rk_peer.cuh); then it polls its rows of every other rank's block from
    // this rank's staging and writes them into the local output.
    const int W = peer.world, R = peer.rank;
    T* const mine = peer.out[R];  // this rank's block inside its own full output
    const uint32_t par = epoch & 1u;
    const size_t sect = static_cast<size_t>(M) * N;  // packets per (parity, source rank)
    __shared__ int may_send;
    if (threadIdx.x == 0) {
      may_send = (W == 1 || peer_wait_all(peer.ctl[R]->ready, W, epoch - 1u, peer.timeout_ns)) ? 1 : 0;
      if (!may_send) atomicOr(peer.status, RK_DEV_ERR_TIMEOUT_PEER);
    }
    __syncthreads();
    for (int t = threadIdx.x; t < rows * M; t += GEMV_THREADS) {
      const int i = t / M, m = t % M;
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < KS; ++k) s += red[(k * rows_max + i) * MB + m];
      const T v = from_f32<T>(s);
      mine[static_cast<size_t>(m) * peer.ldo + row_begin + i] = v;
      if (may_send) {
        const uint64_t pkt = (static_cast<uint64_t>(epoch) << 32) | bits_of(v);
        const size_t at = (par * W + R) * sect + static_cast<size_t>(m) * N + row_begin + i;
        for (int j = 0; j < W; ++j)
          if (j != R) st_relaxed_sys_u64(peer_stage(peer.ctl[j]) + at, pkt);
      }
    }
    const uint64_t* stage = peer_stage(peer.ctl[R]);
    const int per_peer = rows * M;
    bool timed_out = false;
    for (int t = threadIdx.x; t < (W - 1) * per_peer && !timed_out; t += GEMV_THREADS) {
      const int jj = t / per_peer, rem = t - jj * per_peer;
      const int j = jj + (jj >= R ? 1 : 0);
      const int i = rem / M, m = rem - i * M;
      const uint64_t* src = stage + (par * W + j) * sect + static_cast<size_t>(m) * N + row_begin + i;
      uint64_t pkt = ld_relaxed_sys_u64(src);
      if (static_cast<uint32_t>(pkt >> 32) != epoch) {
        const uint64_t t0 = globaltimer_ns();
        for (uint32_t it = 0;; ++it) {
          pkt = ld_relaxed_sys_u64(src);
          if (static_cast<uint32_t>(pkt >> 32) == epoch) break;
          if ((it & 15u) == 15u && (globaltimer_ns() - t0 > peer.timeout_ns || it >= (1u << 30))) {
            timed_out = true;
            break;
          }
        }
      }
      // Rank j's block of this rank's full output: columns [j N, (j + 1) N).
      if (!timed_out)
        mine[static_cast<ptrdiff_t>(m) * peer.ldo + static_cast<ptrdiff_t>(j - R) * N + row_begin + i] =
            from_bits<T>(static_cast<uint32_t>(pkt));
    }
    if (timed_out) atomicOr(peer.status, RK_DEV_ERR_TIMEOUT_PEER);
    // The call number advances once every CTA has read it: the grid's last CTA to finish.
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      if (atomicAdd(&peer.ctl[R]->done_ctas, 1u) == gridDim.x - 1u) {
        peer.ctl[R]->done_ctas = 0u;  // the next call starts after this kernel completes
        *reinterpret_cast<volatile uint32_t*>(&peer.ctl[R]->epoch) = epoch;
      }
    }
  } else {
    for (int t = threadIdx.x; t < rows * M; t += GEMV_THREADS) {
      const int i = t / M, m = t % M;
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < KS; ++k) s += red[(k * rows_max + i) * MB + m];
      out[static_cast<size_t>(m) * N + row_begin + i] = from_f32<T>(s);
    }
  }
}

// Generic GEMV: any K, any alignment.  One warp per output row, lanes stride K.
template <typename T, int MB>
__global__ void __launch_bounds__(256)
    gemv_scalar_kernel(const T* __restrict__ x, const T* __restrict__ W, T* __restrict__ out,
                       int M, int N, int K) {
  pdl_begin();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  if (row >= N) return;
  const T* w = W + static_cast<size_t>(row) * K;
  float acc[MB];
#pragma unroll
  for (int m = 0; m < MB; ++m) acc[m] = 0.f;
  for (int k = lane; k < K; k += 32) {
    const float wf = to_f32(w[k]);
#pragma unroll
    for (int m = 0; m < MB; ++m)
      if (m < M) acc[m] = fmaf(wf, to_f32(x[static_cast<size_t>(m) * K + k]), acc[m]);
  }
#pragma unroll
  for (int m = 0; m < MB; ++m) {
    const float s = warp_sum(acc[m]);
    if (lane == 0 && m < M) out[static_cast<size_t>(m) * N + row] = from_f32<T>(s);
  }
}

struct StreamLaunch {
  const void* kernel;
  // `peer` is null for the plain kernel, the fused all-gather targets otherwise.
  void (*launch)(const void*, const void*, void*, int, int, int, int, int, int, int, size_t,
                 cudaStream_t, const PeerTargets*, const LaunchCtl*);
};

template <typename T>
PeerOut<T> peer_out(const PeerTargets* t, const LaunchCtl* lc) {
  PeerOut<T> p{};
  if (t != nullptr) {
    for (int j = 0; j < t->world; ++j) {
      p.out[j] = static_cast<T*>(t->out[j]);
      p.ctl[j] = static_cast<PeerCtl*>(t->ctl[j]);
    }
    p.ldo = t->ldo;
    p.rank = t->rank;
    p.world = t->world;
    p.timeout_ns = t->timeout_ns;
    p.status = lc->status;
  }
  return p;
}

template <typename T, int MB, int ROWS, int KS, bool PEER>
void launch_stream(const void* x, const void* W, void* out, int M, int N, int K, int grid,
                   int rows_base, int rows_rem, int rows_max, size_t smem, cudaStream_t s,
                   const PeerTargets* peer, const LaunchCtl* lc) {
  // Launch errors are left for the caller's cudaGetLastError().
  (void)launch_kernel(gemv_stream_kernel<T, MB, ROWS, KS, PEER>, dim3(grid), dim3(GEMV_THREADS), smem,
                      s, 0, static_cast<const T*>(x), static_cast<const T*>(W), static_cast<T*>(out),
                      M, N, K, rows_base, rows_rem, rows_max, peer_out<T>(peer, lc));
}

template <typename T, int MB, int ROWS, int KS, bool PEER>
StreamLaunch make_stream() {
  return {reinterpret_cast<const void*>(&gemv_stream_kernel<T, MB, ROWS, KS, PEER>),
          &launch_stream<T, MB, ROWS, KS, PEER>};
}

template <typename T, int MB, int ROWS, bool PEER>
StreamLaunch pick_ks(int ks) {
  switch (ks) {
    case 1: return make_stream<T, MB, ROWS, 1, PEER>();
    case 2: return make_stream<T, MB, ROWS, 2, PEER>();
    case 4: return make_stream<T, MB, ROWS, 4, PEER>();
    default: return make_stream<T, MB, ROWS, 8, PEER>();
  }
}

template <typename T, int MB, bool PEER>
StreamLaunch pick_rows(int rows, int ks) {
  if constexpr (MB <= 4) {
    if (rows >= 4) return pick_ks<T, MB, 4, PEER>(ks);
  }
  if constexpr (MB <= 16) {
    if (rows >= 2) return pick_ks<T, MB, 2, PEER>(ks);
  }
  return pick_ks<T, MB, 1, PEER>(ks);
}

template <typename T, bool PEER = false>
StreamLaunch pick(int mb, int rows, int ks) {
  switch (mb) {
    case 1: return pick_rows<T, 1, PEER>(rows, ks);
    case 2: return pick_rows<T, 2, PEER>(rows, ks);
    case 4: return pick_rows<T, 4, PEER>(rows, ks);
    case 8: return pick_rows<T, 8, PEER>(rows, ks);
    case 16: return pick_rows<T, 16, PEER>(rows, ks);
    default: return pick_rows<T, 32, PEER>(rows, ks);
  }
}

int bucket_m(int64_t M) {
  int mb = 1;
  while (mb < M) mb <<= 1;
  return mb;
}

// Rows per warp the kernel instantiations actually provide for an M bucket.
int clamp_rows(int mb, int rows) {
  const int cap = mb <= 4 ? 4 : (mb <= 16 ? 2 : 1);
  int r = 1;
  while (r * 2 <= rows && r * 2 <= cap) r *= 2;
  return r;
}

// Resident CTAs per SM for a kernel (cached per device and kernel).
int resident_ctas(const void* kernel, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, const void*, size_t>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(dev, kernel, smem);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, GEMV_THREADS, smem) != cudaSuccess ||
      n < 1)
    n = 1;
  cache.emplace(key, n);
  return n;
}

}  // namespace

bool gemv_stream_supported(const void* x, const void* W, const void* out, int64_t M, int64_t N,
                           int64_t K) {
  (void)out;
  if (M < 1 || M > 32 || N < 1 || K < 8) return false;
  if (K % 8 != 0) return false;
  if (!aligned16(x) || !aligned16(W)) return false;
  if (N > (1ll << 31) - 64 || K > (1ll << 31) - 64) return false;
  return true;
}

namespace {

// The streaming launch shared by rk_gemv (peer == nullptr: out is [M, N]) and
// rk_gemv_allgather (out unused: the kernel stores into every rank's output).  Both take
// the same rows / K-split choice from (M, K), so every output element is reduced in the
// same order and the fused form reproduces the plain kernel bit for bit.
rk_status stream_run(const void* x, const void* W, void* out, int64_t M, int64_t N, int64_t K,
                     rk_dtype dt, cudaStream_t s, const PeerTargets* peer) {
  const int mb = bucket_m(M);
  int rows = g_gemv_rows_override.load();
  if (rows <= 0) rows = mb <= 2 ? 2 : (mb <= 4 ? 4 : (mb <= 16 ? 2 : 1));
  rows = clamp_rows(mb, rows);
  const int64_t kv = K / 8;
  int ks = g_gemv_ks_override.load();
  if (ks <= 0) {
    // Split K across the CTA's warps while each slice keeps >= 2 vectors per lane.
    ks = 8;
    while (ks > 1 && kv / ks < 64) ks /= 2;
    if (ks == 8) {
      // A lane walks its slice in steps of 32 x UNROLL vectors; a short slice that leaves
      // much of its last step empty keeps fewer loads in flight.  Take 4 slices instead of 8
      // when 8 would give at most two steps and 4 fill them clearly better (K = 4096: 64 of
      // 128 vectors with 8 slices, measured 7-17 % slower; K = 11008: 172 of 256, 3-9 %);
      // otherwise 8 (K = 8192, 14336: as fast; K = 28672, four steps: 8 measured 3.5 %
      // faster at M = 1 although 4 slices would fill their steps exactly).
      const int64_t step = 32 * (rows >= 4 ? 2 : 4);
      auto idle = [&](int64_t c) {
        const int64_t per = (kv + c - 1) / c, cap = (per + step - 1) / step * step;
        return static_cast<double>(cap - per) / static_cast<double>(cap);
      };
      if ((kv / 8 + step - 1) / step <= 2 && idle(4) < idle(8) - 0.02) ks = 4;
    }
  }
  ks = ks >= 8 ? 8 : (ks >= 4 ? 4 : (ks >= 2 ? 2 : 1));
  StreamLaunch L = peer != nullptr
                       ? (dt == RK_DTYPE_BF16 ? pick<__nv_bfloat16, true>(mb, rows, ks)
                                              : pick<__half, true>(mb, rows, ks))
                       : (dt == RK_DTYPE_BF16 ? pick<__nv_bfloat16>(mb, rows, ks)
                                              : pick<__half>(mb, rows, ks));
  LaunchCtl lc{};
  if (peer != nullptr) {
    const rk_status st = launch_ctl(&lc);
    if (st != RK_OK) return st;
  }
  // Grid: every resident CTA slot of the GPU, rows dealt out evenly; more CTAs only
  // when the per-CTA partial-sum buffer would exceed 32 KiB.
  const int rows_per_group = (GEMV_WARPS / ks) * rows;
  int64_t grid = static_cast<int64_t>(device_sm_count()) *
                 resident_ctas(L.kernel, static_cast<size_t>(ks) * 64 * mb * sizeof(float));
  const int64_t cap_rows = 32768 / (static_cast<int64_t>(ks) * mb * sizeof(float));
  if ((N + grid - 1) / grid > cap_rows) grid = (N + cap_rows - 1) / cap_rows;
  if (grid > N) grid = N;
  // Keep at least one row chunk per row group where N allows it.
  if (grid > 1 && N / grid < rows_per_group && N >= rows_per_group)
    grid = std::max<int64_t>(1, N / rows_per_group);
  const int rows_base = static_cast<int>(N / grid);
  const int rows_rem = static_cast<int>(N % grid);
  const int rows_max = rows_base + (rows_rem ? 1 : 0);
  const size_t smem = static_cast<size_t>(ks) * rows_max * mb * sizeof(float);
  L.launch(x, W, out, static_cast<int>(M), static_cast<int>(N), static_cast<int>(K),
           static_cast<int>(grid), rows_base, rows_rem, rows_max, smem, s, peer, &lc);
  note_launch(peer != nullptr ? "gemv_stream_kernel<PEER>" : "gemv_stream_kernel");
  return cuda_status(cudaGetLastError());
}

}  // namespace

rk_status gemv_stream_launch(const void* x, const void* W, void* out, int64_t M, int64_t N,
                             int64_t K, rk_dtype dt, cudaStream_t s) {
  if (!gemv_stream_supported(x, W, out, M, N, K)) return RK_ERR_UNSUPPORTED;
  return stream_run(x, W, out, M, N, K, dt, s, nullptr);
}

rk_status gemv_stream_allgather_launch(const void* x, const void* W, int64_t M, int64_t N_block,
                                       int64_t K, rk_dtype dt, const PeerTargets& t,
                                       cudaStream_t s) {
  if (!gemv_stream_supported(x, W, nullptr, M, N_block, K)) return RK_ERR_UNSUPPORTED;
  return stream_run(x, W, nullptr, M, N_block, K, dt, s, &t);
}

rk_status gemv_scalar_launch(const void* x, const void* W, void* out, int64_t M, int64_t N,
                             int64_t K, rk_dtype dt, cudaStream_t s) {
  if (M < 1 || M > 32 || N < 1 || K < 1) return RK_ERR_INVALID_ARGUMENT;
  if (N > (1ll << 31) - 64 || K > (1ll << 31) - 64) return RK_ERR_UNSUPPORTED;
  const unsigned grid = static_cast<unsigned>((N + 7) / 8);
  const int mb = bucket_m(M);
#define RK_SCALAR_CASE(MBV)                                                                       \
  case MBV:                                                                                       \
    if (dt == RK_DTYPE_BF16)                                                                      \
      (void)launch_kernel(gemv_scalar_kernel<__nv_bfloat16, MBV>, dim3(grid), dim3(256), 0, s, 0, \
                          static_cast<const __nv_bfloat16*>(x),                                   \
                          static_cast<const __nv_bfloat16*>(W),                                   \
                          static_cast<__nv_bfloat16*>(out), int(M), int(N), int(K));              \
    else                                                                                          \
      (void)launch_kernel(gemv_scalar_kernel<__half, MBV>, dim3(grid), dim3(256), 0, s, 0,        \
                          static_cast<const __half*>(x), static_cast<const __half*>(W),           \
                          static_cast<__half*>(out), int(M), int(N), int(K));                     \
    break;
  switch (mb) {
    RK_SCALAR_CASE(1)
    RK_SCALAR_CASE(2)
    RK_SCALAR_CASE(4)
    RK_SCALAR_CASE(8)
    RK_SCALAR_CASE(16)
    RK_SCALAR_CASE(32)
    default: return RK_ERR_INVALID_ARGUMENT;
  }
#undef RK_SCALAR_CASE
  note_launch("gemv_scalar_kernel");
  return cuda_status(cudaGetLastError());
}

void gemv_set_tuning(int rows, int ks) {
  g_gemv_rows_override.store(rows);
  g_gemv_ks_override.store(ks);
}

}  // namespace rk
