// paged_attention.cu -- decode attention over a paged K/V cache (one query token per
// sequence), the B200 counterpart of rk.paged_attention_decode:
//
//   out[b, h, :] = softmax_t(scale * q[b, h, :] . K[b, t, kvh, :]) @ V[b, t, kvh, :]
//   t < context_lengths[b], kvh = h / (query_heads / kv_heads),
//   K[b, t] = key_cache[block_tables[b, t / block_size], t % block_size]   (same for V)
//
// Arithmetic follows the reference's fp32 definition (src/radeon_kernels/ops/
// paged_attention/reference.py:8-47): fp32 scores, fp32 softmax, fp32 weighted sum, one
// rounding of the output.  A sequence with no valid position gives NaN, as torch's softmax
// of an all -inf row does.
//
// Design (an HBM stream over the K/V bytes of every sequence, "flash decoding"):
//   * grid (partition, kv head x head group, sequence): a CTA walks one contiguous range
//     of positions of one sequence for one KV head and the G (1, 2, 4 or 8) query heads
//     that share it (GQA), so every K/V vector is read from HBM once per group of up to
//     8 query heads;
//   * 128 threads; a position's 16-byte K and V vectors (8 elements) are spread over
//     D/8 threads, so 128*8/D positions are processed side by side, 4 deep in flight per
//     thread; the dot product of a position is a shuffle tree over its D/8 threads;
//   * online softmax per head and position group in fp32 (running max, running sum,
//     rescaled accumulator), merged across the groups of the CTA in shared memory in a
//     fixed order;
//   * several partitions per sequence: the partial (max, sum, accumulator) of each goes to
//     the caller's workspace and a second kernel merges them in partition order; a
//     single partition writes the output directly.
// Block-table entries outside [0, num_blocks) are never dereferenced: the position is
// skipped and RK_DEV_ERR_BAD_INDEX is set in the device status word.
//
// Role of the reference: attention_wave1/4/8 and paged_attention_impl
// (benchmarks/paged_attention/native_paged_attention.hip:192-283).
#include <cuda_runtime.h>

#include <atomic>

#include <cmath>

#include "rk_device.cuh"
#include "rk_internal.h"

namespace rk {
namespace pa {

constexpr int THREADS = 128;
constexpr int GMAX = 8;    // query heads per CTA at most
constexpr int UNROLL = 4;  // positions in flight per thread

struct Params {
  const void* q;
  const void* k;
  const void* v;
  const void* tables;
  const void* lens;
  void* out;
  float* part_acc;  // [batch, hq, partitions, D]
  float* part_ml;   // [batch, hq, partitions, 2] (max, sum)
  int batch, hq, hkv, group, head_groups;
  int num_blocks, block_size, max_blocks;
  int block_shift;  // log2(block_size) when it is a power of two, else -1
  int partitions, part_tokens;
  float scale;
};

// G: query heads handled per CTA (the GQA group size rounded up to 1, 2, 4 or 8).
template <typename T, typename Index, int D, int G>
__global__ void __launch_bounds__(THREADS)
    paged_partition_kernel(Params p, KernelCtl ctl) {
  constexpr int TPT = D / 8;             // threads per position
  constexpr int GROUPS = THREADS / TPT;  // positions side by side
  __shared__ float s_m[GROUPS][G];
  __shared__ float s_l[GROUPS][G];
  __shared__ float s_acc[GROUPS][G][D];

  pdl_begin();
  const int part = blockIdx.x;
  const int kvh = blockIdx.y / p.head_groups;
  const int hg = blockIdx.y - kvh * p.head_groups;
  const int b = blockIdx.z;
  const int tg = threadIdx.x / TPT, ti = threadIdx.x - tg * TPT;
  const int h0 = kvh * p.group + hg * G;
  const int nh = min(G, p.group - hg * G);

  const Index* tables = static_cast<const Index*>(p.tables) + static_cast<int64_t>(b) * p.max_blocks;
  int64_t ctx = static_cast<int64_t>(static_cast<const Index*>(p.lens)[b]);
  const int64_t max_ctx = static_cast<int64_t>(p.max_blocks) * p.block_size;
  ctx = ctx < 0 ? 0 : (ctx > max_ctx ? max_ctx : ctx);
  const int64_t t_begin = static_cast<int64_t>(part) * p.part_tokens;
  const int t_end = static_cast<int>(min(t_begin + p.part_tokens, ctx));

  // This thread's 8 dims of each query head, in fp32.
  float q[G][8];
  const T* qb = static_cast<const T*>(p.q) + (static_cast<int64_t>(b) * p.hq + h0) * D + ti * 8;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (g < nh) {
      const uint4 raw = *reinterpret_cast<const uint4*>(qb + static_cast<int64_t>(g) * D);
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = Pack2<T>::to_floats(w[j]);
        q[g][2 * j] = f.x;
        q[g][2 * j + 1] = f.y;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) q[g][j] = 0.f;
    }
  }
  float m[G], l[G], acc[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[g][j] = 0.f;
  }

  const int64_t row_stride = static_cast<int64_t>(p.hkv) * D;  // elements between slots
  const T* kbase = static_cast<const T*>(p.k) + static_cast<int64_t>(kvh) * D + ti * 8;
  const T* vbase = static_cast<const T*>(p.v) + static_cast<int64_t>(kvh) * D + ti * 8;

  // The trip count is the same for every thread of the CTA (the shuffles below are
  // warp-wide); a thread's positions are tb + tg + u * GROUPS.
  for (int64_t tb = t_begin; tb < t_end; tb += GROUPS * UNROLL) {
    uint4 kv[UNROLL], vv[UNROLL];
    bool use[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      // Positions fit in 32 bits (max_blocks * block_size < 2^31, checked by the host).
      const int t = static_cast<int>(tb) + tg + u * GROUPS;
      use[u] = false;
      kv[u] = make_uint4(0, 0, 0, 0);
      vv[u] = make_uint4(0, 0, 0, 0);
      if (t < t_end) {
        const int lb = p.block_shift >= 0 ? t >> p.block_shift : t / p.block_size;
        const int off = p.block_shift >= 0 ? t & (p.block_size - 1) : t - lb * p.block_size;
        const int64_t blk = static_cast<int64_t>(tables[lb]);
        if (blk >= 0 && blk < p.num_blocks) {
          const int64_t slot = blk * p.block_size + off;
          kv[u] = ld_stream_v4(kbase + slot * row_stride);
          vv[u] = ld_stream_v4(vbase + slot * row_stride);
          use[u] = true;
        } else if (ti == 0) {
          atomicOr(ctl.status, RK_DEV_ERR_BAD_INDEX);
        }
      }
    }
    // Scores of the UNROLL positions first (warp-wide shuffles run for every lane, used
    // position or not: a warp holds several position groups that can reach the end of the
    // range at different u), then one online-softmax step per head for the whole chunk.
    float sc[G][UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      float kf[8];
      const uint32_t kw[4] = {kv[u].x, kv[u].y, kv[u].z, kv[u].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 a = Pack2<T>::to_floats(kw[j]);
        kf[2 * j] = a.x;
        kf[2 * j + 1] = a.y;
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) s = fmaf(q[g][j], kf[j], s);
#pragma unroll
        for (int o = TPT / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        sc[g][u] = use[u] ? s * p.scale : -INFINITY;
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      if (g < nh && use[0]) {  // use[0] is false only when the whole chunk is past the end
        float cm = m[g];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) cm = fmaxf(cm, sc[g][u]);
        const float alpha = __expf(m[g] - cm);  // 0 when m was -inf
        float beta[UNROLL];
        float bsum = 0.f;
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
          beta[u] = __expf(sc[g][u] - cm);  // 0 for unused positions (-inf)
          bsum += beta[u];
        }
        l[g] = l[g] * alpha + bsum;
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[g][j] *= alpha;
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
          const uint32_t vw[4] = {vv[u].x, vv[u].y, vv[u].z, vv[u].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 c = Pack2<T>::to_floats(vw[j]);
            acc[g][2 * j] = fmaf(beta[u], c.x, acc[g][2 * j]);
            acc[g][2 * j + 1] = fmaf(beta[u], c.y, acc[g][2 * j + 1]);
          }
        }
        m[g] = cm;
      }
    }
  }

  // Merge the position groups of this CTA in group order.
  if (ti == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      s_m[tg][g] = m[g];
      s_l[tg][g] = l[g];
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < 8; ++j) s_acc[tg][g][ti * 8 + j] = acc[g][j];
  __syncthreads();

  for (int idx = threadIdx.x; idx < nh * D; idx += THREADS) {
    const int g = idx / D, d = idx - g * D;
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < GROUPS; ++j) mx = fmaxf(mx, s_m[j][g]);
    float sum = 0.f, a = 0.f;
    if (mx != -INFINITY) {
#pragma unroll
      for (int j = 0; j < GROUPS; ++j) {
        if (s_m[j][g] != -INFINITY) {
          const float w = __expf(s_m[j][g] - mx);
          sum += s_l[j][g] * w;
          a += s_acc[j][g][d] * w;
        }
      }
    }
    const int64_t head = static_cast<int64_t>(b) * p.hq + h0 + g;
    if (p.partitions == 1) {
      static_cast<T*>(p.out)[head * D + d] = from_f32<T>(a / sum);  // 0/0 = NaN for ctx 0
    } else {
      const int64_t slot = head * p.partitions + part;
      p.part_acc[slot * D + d] = a;
      if (d == 0) {
        p.part_ml[2 * slot] = mx;
        p.part_ml[2 * slot + 1] = sum;
      }
    }
  }
}

// One CTA per (sequence, query head), one thread per output element: merges the
// partitions in partition order.  Loads are issued 8 partitions at a time so a long
// partition list costs a few L2 round trips, not one per partition.
template <typename T, int D>
__global__ void __launch_bounds__(D) paged_merge_kernel(Params p) {
  constexpr int B8 = 8;
  pdl_begin();
  const int64_t head = blockIdx.x;
  const int d = threadIdx.x;
  const float* ml = p.part_ml + head * p.partitions * 2;
  const float* acc = p.part_acc + head * p.partitions * D + d;
  float mx = -INFINITY;
  for (int j0 = 0; j0 < p.partitions; j0 += B8) {
    float v[B8];
#pragma unroll
    for (int i = 0; i < B8; ++i) v[i] = j0 + i < p.partitions ? ml[2 * (j0 + i)] : -INFINITY;
#pragma unroll
    for (int i = 0; i < B8; ++i) mx = fmaxf(mx, v[i]);
  }
  float sum = 0.f, a = 0.f;
  if (mx != -INFINITY) {
    for (int j0 = 0; j0 < p.partitions; j0 += B8) {
      float pm[B8], pl[B8], pa[B8];
#pragma unroll
      for (int i = 0; i < B8; ++i) {
        const int j = j0 + i;
        const bool in = j < p.partitions;
        pm[i] = in ? ml[2 * j] : -INFINITY;
        pl[i] = in ? ml[2 * j + 1] : 0.f;
        pa[i] = in ? acc[static_cast<int64_t>(j) * D] : 0.f;
      }
#pragma unroll
      for (int i = 0; i < B8; ++i) {
        if (pm[i] != -INFINITY) {
          const float w = __expf(pm[i] - mx);
          sum += pl[i] * w;
          a += pa[i] * w;
        }
      }
    }
  }
  static_cast<T*>(p.out)[head * D + d] = from_f32<T>(a / sum);
}

struct Plan {
  int g, head_groups, partitions, part_tokens;
};

Plan plan(int64_t batch, int64_t hq, int64_t hkv, int64_t head_dim, int64_t max_ctx, int sms) {
  Plan pl{};
  const int64_t group = hq / hkv;
  pl.g = 1;
  while (pl.g < GMAX && pl.g < group) pl.g *= 2;
  pl.head_groups = static_cast<int>((group + pl.g - 1) / pl.g);
  const int64_t base = batch * hkv * pl.head_groups;
  // Enough partitions for eight CTAs (32 warps) per SM, each at least 32 KiB of K and V
  // per head (128 positions; 64 at head_dim 256): a CTA's positions are walked a few deep
  // per thread, so latency is hidden by the number of CTAs in flight, and shorter
  // partitions only add merge work.  At head_dim 256 a CTA keeps only 4 x 4 positions in
  // flight, so 128-position partitions left too few CTAs for short contexts (batch 4,
  // GQA 32 x 8, context 1024: 28.7 us with 128, 20.8 with 64, 25.4 with 32).
  int64_t parts = (8ll * sms + base - 1) / base;
  const int64_t min_len = head_dim >= 256 ? 64 : 128;
  const int64_t cap = (max_ctx + min_len - 1) / min_len;
  if (parts > cap) parts = cap;
  if (parts < 1) parts = 1;
  pl.partitions = static_cast<int>(parts);
  pl.part_tokens = static_cast<int>((max_ctx + parts - 1) / parts);
  return pl;
}

template <typename T, typename Index, int D, int G>
rk_status launch(Params prm, const Plan& pl, cudaStream_t s) {
  LaunchCtl lc;
  rk_status st = launch_ctl(&lc);
  if (st != RK_OK) return st;
  const KernelCtl ctl{lc.status, lc.timeout_ns, 0};
  const dim3 grid(static_cast<unsigned>(pl.partitions),
                  static_cast<unsigned>(prm.hkv * pl.head_groups), static_cast<unsigned>(prm.batch));
  cudaError_t e = launch_kernel(paged_partition_kernel<T, Index, D, G>, grid, dim3(THREADS), 0, s, 0,
                                prm, ctl);
  note_launch();
  if (e == cudaSuccess && pl.partitions > 1) {
    e = launch_kernel(paged_merge_kernel<T, D>, dim3(static_cast<unsigned>(prm.batch * prm.hq)),
                      dim3(D), 0, s, 0, prm);
    note_launch();
  }
  return cuda_status(e);
}

template <typename T, typename Index, int D>
rk_status launch_g(Params prm, const Plan& pl, cudaStream_t s) {
  switch (pl.g) {
    case 1: return launch<T, Index, D, 1>(prm, pl, s);
    case 2: return launch<T, Index, D, 2>(prm, pl, s);
    case 4: return launch<T, Index, D, 4>(prm, pl, s);
    default: return launch<T, Index, D, 8>(prm, pl, s);
  }
}

template <typename T, typename Index>
rk_status launch_d(Params prm, const Plan& pl, int64_t head_dim, cudaStream_t s) {
  switch (head_dim) {
    case 64: return launch_g<T, Index, 64>(prm, pl, s);
    case 128: return launch_g<T, Index, 128>(prm, pl, s);
    case 256: return launch_g<T, Index, 256>(prm, pl, s);
  }
  return RK_ERR_UNSUPPORTED;
}

}  // namespace pa

namespace {
std::atomic<int> g_paged_path{0};  // 0 automatic, 1 CUDA cores, 2 tensor cores
}  // namespace

void paged_attention_set_path(int path) { g_paged_path.store(path >= 0 && path <= 2 ? path : 0); }

// The larger of the two kernels' needs: which kernel runs also depends on pointers and
// dtype, which this query does not see.
size_t paged_attention_workspace_bytes(int64_t batch, int64_t hq, int64_t hkv, int64_t head_dim,
                                       int64_t max_blocks, int64_t block_size) {
  if (batch <= 0 || hq <= 0 || hkv <= 0 || hq % hkv != 0 || max_blocks <= 0 || block_size <= 0)
    return 0;
  const int64_t max_ctx = max_blocks * block_size;
  const pa::Plan pl = pa::plan(batch, hq, hkv, head_dim, max_ctx, device_sm_count());
  int tc_parts = 1, tc_tokens = 0;
  paged_attention_tc_plan(batch, hkv, max_ctx, device_sm_count(), &tc_parts, &tc_tokens);
  const int parts = pl.partitions > tc_parts ? pl.partitions : tc_parts;
  if (parts == 1) return 0;
  return static_cast<size_t>(batch) * hq * parts * (head_dim + 2) * sizeof(float);
}

rk_status paged_attention_launch(const void* query, const void* key_cache, const void* value_cache,
                                 const void* block_tables, const void* context_lengths, void* out,
                                 int64_t batch, int64_t hq, int64_t hkv, int64_t head_dim,
                                 int64_t num_blocks, int64_t block_size, int64_t max_blocks,
                                 float scale, rk_dtype dt, int index_bits, void* workspace,
                                 size_t workspace_bytes, cudaStream_t s) {
  const pa::Plan pl = pa::plan(batch, hq, hkv, head_dim, max_blocks * block_size, device_sm_count());
  const size_t need = paged_attention_workspace_bytes(batch, hq, hkv, head_dim, max_blocks, block_size);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need)) return RK_ERR_INVALID_ARGUMENT;
  if (batch > 65535 || hkv * pl.head_groups > 65535) return RK_ERR_UNSUPPORTED;
  pa::Params prm{};
  prm.q = query;
  prm.k = key_cache;
  prm.v = value_cache;
  prm.tables = block_tables;
  prm.lens = context_lengths;
  prm.out = out;
  prm.part_acc = static_cast<float*>(workspace);
  prm.part_ml = need > 0 ? static_cast<float*>(workspace) + batch * hq * pl.partitions * head_dim : nullptr;
  prm.batch = static_cast<int>(batch);
  prm.hq = static_cast<int>(hq);
  prm.hkv = static_cast<int>(hkv);
  prm.group = static_cast<int>(hq / hkv);
  prm.head_groups = pl.head_groups;
  prm.num_blocks = static_cast<int>(num_blocks);
  prm.block_size = static_cast<int>(block_size);
  prm.max_blocks = static_cast<int>(max_blocks);
  prm.block_shift = -1;
  for (int sh = 0; sh < 31; ++sh)
    if ((int64_t{1} << sh) == block_size) prm.block_shift = sh;
  prm.partitions = pl.partitions;
  prm.part_tokens = pl.part_tokens;
  prm.scale = scale;
  const bool bf16 = dt == RK_DTYPE_BF16;
  const int path = g_paged_path.load();
  const bool tc_ok = paged_attention_tc_supported(query, key_cache, value_cache, hq, hkv, head_dim, block_size);
  if (path == 2 && !tc_ok) return RK_ERR_UNSUPPORTED;
  // Automatic choice: the tensor-core kernel wherever it applies except head_dim-64 MHA, where
  // the CUDA-core kernel measured faster (no query heads share a K/V tile, and V^T is padded
  // to the MMA's 128 rows).
  const bool tc_auto = tc_ok && !(hq == hkv && head_dim == 64);
  if (path == 2 || (path == 0 && tc_auto)) {
    // Tensor-core kernel; its partitions (whole 128-position tiles) go through the same
    // workspace layout and merge kernel.
    PagedTcArgs a{};
    a.q = query;
    a.k = key_cache;
    a.v = value_cache;
    a.tables = block_tables;
    a.lens = context_lengths;
    a.out = out;
    a.batch = batch;
    a.hq = hq;
    a.hkv = hkv;
    a.head_dim = head_dim;
    a.num_blocks = num_blocks;
    a.block_size = block_size;
    a.max_blocks = max_blocks;
    a.index_bits = index_bits;
    a.scale = scale;
    a.dt = dt;
    paged_attention_tc_plan(batch, hkv, max_blocks * block_size, device_sm_count(), &a.partitions,
                            &a.part_tokens);
    if (a.partitions > 1) {
      a.part_acc = static_cast<float*>(workspace);
      a.part_ml = static_cast<float*>(workspace) + batch * hq * a.partitions * head_dim;
    }
    if (batch > 65535 || hkv > 65535) return RK_ERR_UNSUPPORTED;
    rk_status st = paged_attention_tc_launch(a, s);
    if (st != RK_OK || a.partitions == 1) return st;
    prm.partitions = a.partitions;
    prm.part_acc = a.part_acc;
    prm.part_ml = a.part_ml;
    cudaError_t e = cudaSuccess;
    switch (head_dim) {
      case 64:
        e = bf16 ? launch_kernel(pa::paged_merge_kernel<__nv_bfloat16, 64>, dim3(static_cast<unsigned>(batch * hq)), dim3(64), 0, s, 0, prm)
                 : launch_kernel(pa::paged_merge_kernel<__half, 64>, dim3(static_cast<unsigned>(batch * hq)), dim3(64), 0, s, 0, prm);
        break;
      default:
        e = bf16 ? launch_kernel(pa::paged_merge_kernel<__nv_bfloat16, 128>, dim3(static_cast<unsigned>(batch * hq)), dim3(128), 0, s, 0, prm)
                 : launch_kernel(pa::paged_merge_kernel<__half, 128>, dim3(static_cast<unsigned>(batch * hq)), dim3(128), 0, s, 0, prm);
    }
    note_launch();
    return cuda_status(e);
  }
  if (index_bits == 32)
    return bf16 ? pa::launch_d<__nv_bfloat16, int32_t>(prm, pl, head_dim, s)
                : pa::launch_d<__half, int32_t>(prm, pl, head_dim, s);
  return bf16 ? pa::launch_d<__nv_bfloat16, int64_t>(prm, pl, head_dim, s)
              : pa::launch_d<__half, int64_t>(prm, pl, head_dim, s);
}

}  // namespace rk
