// paged_attention_tc.cu -- paged decode attention on the tcgen05 tensor cores.
//
// Same operator and result format as paged_attention.cu (the reference's
// paged_attention_decode, src/radeon_kernels/ops/paged_attention/api.py:38-157,
// reference.py:8-47), for head_dim 64 / 128, GQA groups up to 16 query heads per KV head and
// block sizes 8, 16, 32, 64, 128.  The CUDA-core kernel spends ~65 warp instructions per
// cached position on dot products, shuffles and the per-position softmax bookkeeping; here
// the two products run on the tensor cores with positions as the 128-row M dimension:
//
//   S^T [128 positions x 16 heads] = K_tile [128 x D] . Q^T [D x 16]      (K-major A and B)
//   O^T [D x 16 heads]            += V_tile^T [D x 128] . P^T [128 x 16]  (MN-major A, K-major B)
//
// so each thread owns one position (TMEM lane) for the softmax -- a handful of exponentials
// per tile -- and one output dimension (O^T lane) for the rescaling and the epilogue.
//
// One CTA per (context partition, KV head, sequence) serves every query head of the GQA
// group (padded to N = 16; the padding rows of Q are zero): four softmax warps, a load warp
// and an MMA warp that meet on mbarriers only.  The load warp streams the partition's
// 128-position tiles: one TMA box per cache block and 64-dim chunk, through a
// 4-D tensor map over [num_blocks, block_size, kv_heads, head_dim]; a block index that is out
// of range, or a block past the context, is loaded from the out-of-range coordinate
// num_blocks, which reads as zero (no fault, no stale bytes, full byte count), and its
// positions are masked; an out-of-range index inside the context is reported through the
// status word (RK_DEV_ERR_BAD_INDEX), as the CUDA-core kernel does.  A ring of STAGES tiles
// keeps the HBM stream going while the softmax runs.  (A first version with the loads and
// MMAs issued from the softmax warps between CTA barriers took 4-5 us per tile, slower than
// the CUDA-core kernel.)  Online softmax per head in fp32
// (base 2, hardware ex2), lazy rescaling of O^T (only when a head's maximum grows by more
// than 2^8); bf16 probabilities as P_hi + P_lo (two MMAs) so they keep ~16 significant bits.
// Partition results go to the workspace in the CUDA-core kernel's format (natural-log
// maximum, sum, unnormalised accumulator) and the same merge kernel combines them.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <mutex>
#include <string>
#include <type_traits>

#include "rk_device.cuh"
#include "rk_internal.h"
#include "rk_tma.h"

namespace rk {

namespace patc {

constexpr int TILE = 128;  // positions per tile (TMEM lanes, MMA M)
constexpr int NG = 16;     // query heads per CTA, padded (MMA N)
constexpr int THREADS = 192;  // 4 softmax warps, a load warp, an MMA warp
constexpr int UMMA_K = 16;
constexpr float LN2 = 0.6931471805599453f;

template <typename T, int D>
struct Cfg {
  static constexpr bool SPLIT = std::is_same<T, __nv_bfloat16>::value;
  static constexpr int CHUNKS = D / 64;                // real 64-dim chunks
  static constexpr int K_BYTES = CHUNKS * TILE * 128;  // CHUNKS x [128 positions x 128 B]
  static constexpr int V_BYTES = 2 * TILE * 128;       // 2 chunks (M = 128); D = 64: chunk 1 zero
  static constexpr int LOAD_BYTES = 2 * K_BYTES;       // bytes the TMA delivers per tile (K + V)
  static constexpr int STAGES = D == 64 ? 4 : 3;
  static constexpr int Q_BYTES = CHUNKS * NG * 128;    // Q^T: CHUNKS x [16 heads x 128 B]
  static constexpr int P_BYTES = 2 * NG * 128;         // P^T: 2 position chunks x [16 x 128 B]
  static constexpr int TMEM_COLS = 64;                 // S^T x 2 (16 each), O^T (16)
  static constexpr int SMEM = 1024 + STAGES * (K_BYTES + V_BYTES) + Q_BYTES +
                              2 * (SPLIT ? 2 : 1) * P_BYTES + 2048;  // P^T by tile parity
  static_assert(D == 64 || D == 128, "head_dim");
  static_assert(SMEM <= 232448, "shared memory per CTA");
};

struct Params {
  const void* q;
  const void* tables;
  const void* lens;
  void* out;
  float* part_acc;  // [batch, hq, partitions, D]
  float* part_ml;   // [batch, hq, partitions, 2] (natural-log max, sum)
  int batch, hq, hkv, group;
  int num_blocks, block_size, max_blocks;
  int partitions, part_tokens;  // part_tokens: a multiple of TILE
  float scale_log2;
};

struct __align__(8) Bars {
  uint64_t kv_full[4];   // TMA: tile in the stage
  uint64_t kv_empty[4];  // MMA commit: the stage's tile is no longer read
  uint64_t s_done[2];    // MMA commit: S^T buffer holds the tile's scores
  uint64_t p_full[2];    // one arrival per softmax warp: P^T_t written (buffer t & 1)
  uint64_t o_done[2];    // MMA commit: O^T += V^T P^T_t done (t & 1)
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  float red[2][4][NG];  // per-warp per-head maxima, by tile parity
  float red_l[4][NG];   // per-warp per-head sums (epilogue)
};

// Named barrier of the four softmax warps (id 1).
__device__ __forceinline__ void softmax_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Warps 0-3: softmax (thread = position = TMEM lane; for O^T, thread = output dimension);
// warp 4: bulk loads; warp 5: MMA issue.  They meet on mbarriers only, so the loads run
// STAGES - 1 tiles ahead of the softmax and nothing waits on a CTA-wide barrier per tile.
template <typename T, typename Index, int D>
__global__ void __launch_bounds__(THREADS, 1)
    paged_tc_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                    Params p, KernelCtl ctl) {
  using C = Cfg<T, D>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sk = smem;                          // STAGES x K tile
  uint8_t* sv = sk + STAGES * C::K_BYTES;      // STAGES x V tile
  uint8_t* sq = sv + STAGES * C::V_BYTES;      // Q^T
  uint8_t* sp = sq + C::Q_BYTES;  // P^T buffers: [parity][hi, lo]
  constexpr int P_SET = (C::SPLIT ? 2 : 1) * C::P_BYTES;
  Bars* bars = reinterpret_cast<Bars*>(sp + 2 * P_SET);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int part = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int h0 = kvh * p.group;
  const int G = p.group;  // real heads of this CTA (<= NG)
  const int bs = p.block_size;
  const Index* tables = static_cast<const Index*>(p.tables) + static_cast<int64_t>(b) * p.max_blocks;
  const int t_begin = part * p.part_tokens;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&bars->kv_full[s]), 1);
      mbar_init(smem_u32(&bars->kv_empty[s]), 1);
    }
    mbar_init(smem_u32(&bars->s_done[0]), 1);
    mbar_init(smem_u32(&bars->s_done[1]), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&bars->p_full[s]), 4);
      mbar_init(smem_u32(&bars->o_done[s]), 1);
    }
    mbar_init(smem_u32(&bars->drain), 1);
    bars->abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmap_k);
    tma_prefetch_desc(&tmap_v);
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&bars->tmem_base), C::TMEM_COLS);
    tmem_relinquish();
  }
  if (D == 64) {
    // V^T is the M = 128 operand: its second 64-row chunk stays zero in every stage.
    for (int i = tid; i < STAGES * TILE * 128 / 16; i += THREADS) {
      const int st = i / (TILE * 128 / 16), r = i - st * (TILE * 128 / 16);
      reinterpret_cast<uint4*>(sv + st * C::V_BYTES + TILE * 128)[r] = make_uint4(0, 0, 0, 0);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  constexpr int O_COL = 2 * NG;
  pdl_begin();  // global memory is touched only after this
  int64_t ctx64 = static_cast<int64_t>(static_cast<const Index*>(p.lens)[b]);
  const int64_t max_ctx = static_cast<int64_t>(p.max_blocks) * bs;
  ctx64 = ctx64 < 0 ? 0 : (ctx64 > max_ctx ? max_ctx : ctx64);
  const int t_end = min(t_begin + p.part_tokens, static_cast<int>(ctx64));
  const int n_tiles = t_end > t_begin ? (t_end - t_begin + TILE - 1) / TILE : 0;

  // Q^T operand: rows = heads (zero past the group), K-major with the 128-byte swizzle.
  {
    const T* qb = static_cast<const T*>(p.q) + (static_cast<int64_t>(b) * p.hq + h0) * D;
    for (int i = tid; i < NG * D / 8; i += THREADS) {
      const int g = i / (D / 8), dv = i - g * (D / 8);  // head, 16-byte unit of the row
      const uint4 v = g < G ? *reinterpret_cast<const uint4*>(qb + static_cast<int64_t>(g) * D + dv * 8)
                            : make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(sq + (dv >> 3) * (NG * 128) + g * 128 + (((dv & 7) ^ (g & 7)) << 4)) = v;
    }
  }
  fence_proxy_async_smem();
  __syncthreads();

  int never = 0;
  volatile int* abort = &bars->abort;
  auto fail = [&](uint32_t code) {
    *abort = 1;
    atomicOr(ctl.status, code);
  };

  if (warp == 4) {
    // ------------------------------------------------------------ loads
    uint32_t issued[4] = {0, 0, 0, 0};
    const int blocks_per_tile = TILE / bs;
    for (int t = 0; t < n_tiles; ++t) {
      const int st = t % STAGES;
      bool ok = true;
      if (lane == 0 && t >= STAGES)
        ok = mbar_wait_bounded(smem_u32(&bars->kv_empty[st]), ((t / STAGES) - 1) & 1, ctl.timeout_ns, abort);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) fail(RK_DEV_ERR_TIMEOUT_PRODUCER);
        break;
      }
      const uint32_t bar = smem_u32(&bars->kv_full[st]);
      if (lane == 0) {
        mbar_arrive_expect_tx(bar, C::LOAD_BYTES);
        ++issued[st];
      }
      __syncwarp();
      if (lane < blocks_per_tile) {
        const int pos = t_begin + t * TILE + lane * bs;  // first position of block `lane`
        int blk = p.num_blocks;                           // out of range: reads as zero
        if (pos < t_end) {
          const int64_t idx = static_cast<int64_t>(tables[pos / bs]);
          if (idx >= 0 && idx < p.num_blocks)
            blk = static_cast<int>(idx);
          else
            atomicOr(ctl.status, RK_DEV_ERR_BAD_INDEX);
        }
#pragma unroll
        for (int c = 0; c < C::CHUNKS; ++c) {
          const uint32_t off = c * (TILE * 128) + lane * bs * 128;
          tma_load_4d(smem_u32(sk + st * C::K_BYTES + off), &tmap_k, bar, c * 64, kvh, 0, blk);
          tma_load_4d(smem_u32(sv + st * C::V_BYTES + off), &tmap_v, bar, c * 64, kvh, 0, blk);
        }
      }
    }
    // No bulk copy may still be landing when the CTA exits: wait for the last load of
    // each stage (earlier ones completed before that stage was refilled).
    if (lane == 0)
      for (int s = 0; s < STAGES; ++s)
        if (issued[s] > 0 &&
            !mbar_wait_bounded(smem_u32(&bars->kv_full[s]), (issued[s] - 1) & 1u, ctl.timeout_ns, &never))
          atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_DRAIN);
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t IDESC_S = umma_idesc_f16(std::is_same<T, __nv_bfloat16>::value, TILE, NG, false, false);
      constexpr uint32_t IDESC_O = umma_idesc_f16(std::is_same<T, __nv_bfloat16>::value, TILE, NG, true, false);
      int issued_mma = 0;
      auto issue_s = [&](int t) -> bool {  // S^T_t = K_t Q^T into buffer t & 1
        const int st = t % STAGES;
        if (!mbar_wait_bounded(smem_u32(&bars->kv_full[st]), (t / STAGES) & 1, ctl.timeout_ns, abort)) {
          fail(RK_DEV_ERR_TIMEOUT_PRODUCER);
          return false;
        }
        tc_fence_after();
        const uint64_t dk = umma_desc_sw128(smem_u32(sk + st * C::K_BYTES), 16, 1024);
        const uint64_t dq = umma_desc_sw128(smem_u32(sq), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < D / UMMA_K; ++kk) {
          const uint32_t off_k = (kk >> 2) * (TILE * 128) + (kk & 3) * 32;
          const uint32_t off_q = (kk >> 2) * (NG * 128) + (kk & 3) * 32;
          tc_mma_f16(tmem + (t & 1) * NG, umma_desc_advance(dk, off_k), umma_desc_advance(dq, off_q),
                     IDESC_S, kk > 0 ? 1u : 0u);
        }
        tc_commit(smem_u32(&bars->s_done[t & 1]));
        ++issued_mma;
        return true;
      };
      bool ok = issue_s(0);
      for (int j = 0; j < n_tiles && ok; ++j) {
        // S^T_{j+1} into the buffer of S^T_{j-1}, which the softmax warps read before P_{j-1}.
        if (j + 1 < n_tiles && !issue_s(j + 1)) break;
        if (!mbar_wait_bounded(smem_u32(&bars->p_full[j & 1]), (j >> 1) & 1, ctl.timeout_ns, abort)) {
          fail(RK_DEV_ERR_TIMEOUT_PRODUCER);
          break;
        }
        tc_fence_after();
        const int st = j % STAGES;
        const uint64_t dv = umma_desc_sw128(smem_u32(sv + st * C::V_BYTES), TILE * 128, 1024);
        const uint64_t dp = umma_desc_sw128(smem_u32(sp + (j & 1) * P_SET), 16, 1024);
        const uint64_t dplo = umma_desc_sw128(smem_u32(sp + (j & 1) * P_SET + C::P_BYTES), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < TILE / UMMA_K; ++kk) {
          const uint64_t a = umma_desc_advance(dv, kk * 2048);
          const uint32_t off_p = (kk >> 2) * (NG * 128) + (kk & 3) * 32;
          tc_mma_f16(tmem + O_COL, a, umma_desc_advance(dp, off_p), IDESC_O, (j > 0 || kk > 0) ? 1u : 0u);
          if (C::SPLIT) tc_mma_f16(tmem + O_COL, a, umma_desc_advance(dplo, off_p), IDESC_O, 1u);
        }
        tc_commit(smem_u32(&bars->o_done[j & 1]));
        tc_commit(smem_u32(&bars->kv_empty[st]));
        ++issued_mma;
      }
      // Every MMA completes before TMEM is released.
      tc_commit(smem_u32(&bars->drain));
      if (!mbar_wait_bounded(smem_u32(&bars->drain), 0, ctl.timeout_ns, &never))
        atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_DRAIN);
      (void)issued_mma;
    }
  } else {
    // ------------------------------------------------------------ softmax
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    // Per-head state (identical in every softmax thread): the maximum the exponentials use.
    float m_use[NG], l_part[NG];
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      m_use[g] = -INFINITY;
      l_part[g] = 0.f;
    }
    // Block-table entry of this thread's position, fetched one tile ahead.
    auto entry_ok = [&](int pos) -> bool {
      if (pos >= t_end) return false;
      const int64_t idx = static_cast<int64_t>(tables[pos / bs]);
      return idx >= 0 && idx < p.num_blocks;
    };
    bool ok_next = n_tiles > 0 && entry_ok(t_begin + tid);
    for (int j = 0; j < n_tiles; ++j) {
      const bool attended = ok_next;
      if (j + 1 < n_tiles) ok_next = entry_ok(t_begin + (j + 1) * TILE + tid);
      if (!mbar_wait_bounded(smem_u32(&bars->s_done[j & 1]), (j >> 1) & 1, ctl.timeout_ns, abort))
        fail(RK_DEV_ERR_TIMEOUT_MMA);
      tc_fence_after();
      float s[NG];
      {
        uint32_t r[16];
        tmem_ld_32x32b_x16(t_lane + (j & 1) * NG, r);
        tmem_ld_wait();
#pragma unroll
        for (int g = 0; g < NG; ++g) s[g] = attended && g < G ? __uint_as_float(r[g]) * p.scale_log2 : -INFINITY;
      }
      // Per-head maximum over the tile: warp shuffles, then the four warps in order (slots
      // of this tile's parity: a warp rewrites them two tiles on, after the barrier of the
      // tile between, which its peers reach only once they have read them).
      float (*red)[NG] = bars->red[j & 1];
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        if (g < G) {  // G is uniform over the CTA
          float v = s[g];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
          if (lane == 0) red[warp][g] = v;
        }
      }
      softmax_sync();
      float alpha[NG];
      bool rescale = false;
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        alpha[g] = 1.f;
        if (g < G) {
          const float mt = fmaxf(fmaxf(red[0][g], red[1][g]), fmaxf(red[2][g], red[3][g]));
          if (mt > m_use[g] + 8.f) {  // lazy rescaling: P <= 256
            alpha[g] = ex2_approx(m_use[g] - mt);
            m_use[g] = mt;
            rescale = true;
          }
        }
      }
      // P for this position (zero for padding heads and masked positions).
      uint32_t hi[NG / 2], lo[NG / 2];
#pragma unroll
      for (int g = 0; g < NG; g += 2) {
        float e[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float m = m_use[g + h] == -INFINITY ? 0.f : m_use[g + h];
          e[h] = ex2_approx(s[g + h] - m);
          l_part[g + h] = l_part[g + h] * alpha[g + h] + e[h];
        }
        hi[g / 2] = Pack2<T>::from_floats(e[0], e[1]);
        if (C::SPLIT) {
          const float2 h2 = Pack2<T>::to_floats(hi[g / 2]);
          lo[g / 2] = Pack2<T>::from_floats(e[0] - h2.x, e[1] - h2.y);
        }
      }
      // P^T buffer j & 1 was read by P V_{j-2}; a rescaling of O^T needs every earlier
      // P V done (they complete in order: P V_{j-1} is enough).  Neither usually waits:
      // the softmax of tile j does not depend on P V_{j-1} otherwise.
      if (j >= 2) {
        if (!mbar_wait_bounded(smem_u32(&bars->o_done[j & 1]), ((j - 2) >> 1) & 1, ctl.timeout_ns, abort))
          fail(RK_DEV_ERR_TIMEOUT_MMA);
      }
      if (j > 0 && rescale) {  // uniform: every softmax thread holds the same maxima
        if (!mbar_wait_bounded(smem_u32(&bars->o_done[(j - 1) & 1]), ((j - 1) >> 1) & 1, ctl.timeout_ns, abort))
          fail(RK_DEV_ERR_TIMEOUT_MMA);
        tc_fence_after();
        {
          uint32_t r[16];
          tmem_ld_32x32b_x16(t_lane + O_COL, r);
          tmem_ld_wait();
#pragma unroll
          for (int g = 0; g < NG; ++g) r[g] = __float_as_uint(__uint_as_float(r[g]) * alpha[g]);
          tmem_st_32x32b_x16(t_lane + O_COL, r);
          tmem_st_wait();
        }
      }
      tc_fence_after();
      // P^T: row g = head, positions along K; this thread writes position `tid` of each row.
      {
        uint8_t* sp_hi = sp + (j & 1) * P_SET;
        uint8_t* sp_lo = sp_hi + C::P_BYTES;
        const int c = tid >> 6, within = tid & 63;
#pragma unroll
        for (int g = 0; g < NG; ++g) {
          const uint32_t off = c * (NG * 128) + g * 128 + (((within >> 3) ^ (g & 7)) << 4) + (within & 7) * 2;
          const uint32_t hv = (g & 1) ? (hi[g / 2] >> 16) : (hi[g / 2] & 0xffffu);
          *reinterpret_cast<uint16_t*>(sp_hi + off) = static_cast<uint16_t>(hv);
          if (C::SPLIT) {
            const uint32_t lv = (g & 1) ? (lo[g / 2] >> 16) : (lo[g / 2] & 0xffffu);
            *reinterpret_cast<uint16_t*>(sp_lo + off) = static_cast<uint16_t>(lv);
          }
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars->p_full[j & 1]));
    }

    // ---- epilogue: per-head sums over the 128 positions, then O^T row d = tid.
    if (n_tiles > 0 &&
        !mbar_wait_bounded(smem_u32(&bars->o_done[(n_tiles - 1) & 1]), ((n_tiles - 1) >> 1) & 1,
                           ctl.timeout_ns, abort))
      fail(RK_DEV_ERR_TIMEOUT_EPILOGUE);
    tc_fence_after();
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      if (g < G) {
        float v = l_part[g];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) bars->red_l[warp][g] = v;
      }
    }
    softmax_sync();
    float o_row[NG];
    if (n_tiles > 0) {
      uint32_t r[16];
      tmem_ld_32x32b_x16(t_lane + O_COL, r);
      tmem_ld_wait();
#pragma unroll
      for (int g = 0; g < NG; ++g) o_row[g] = __uint_as_float(r[g]);
    } else {
#pragma unroll
      for (int g = 0; g < NG; ++g) o_row[g] = 0.f;
    }
    if (tid < D && !*abort) {
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        if (g < G) {
          const float l = ((bars->red_l[0][g] + bars->red_l[1][g]) + bars->red_l[2][g]) + bars->red_l[3][g];
          const int64_t head = static_cast<int64_t>(b) * p.hq + h0 + g;
          if (p.partitions == 1) {
            static_cast<T*>(p.out)[head * D + tid] = from_f32<T>(o_row[g] / l);  // 0/0 = NaN for ctx 0
          } else {
            const int64_t slot = head * p.partitions + part;
            p.part_acc[slot * D + tid] = o_row[g];
            if (tid == 0) {
              p.part_ml[2 * slot] = m_use[g] == -INFINITY ? -INFINITY : m_use[g] * LN2;
              p.part_ml[2 * slot + 1] = l;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace patc

namespace {

// 4-D map over the cache [num_blocks, block_size, kv_heads, head_dim], boxes of one block's
// positions x 64 dims of one head (128-byte swizzle).  Block coordinates past num_blocks
// read as zero.
rk_status encode_cache_map(CUtensorMap* map, const void* base, rk_dtype dt, int64_t head_dim,
                           int64_t kv_heads, int64_t block_size, int64_t num_blocks) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (fn == nullptr) return RK_ERR_CUDA;
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(head_dim), static_cast<cuuint64_t>(kv_heads),
                              static_cast<cuuint64_t>(block_size), static_cast<cuuint64_t>(num_blocks)};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(head_dim * 2),
                                 static_cast<cuuint64_t>(kv_heads * head_dim * 2),
                                 static_cast<cuuint64_t>(block_size * kv_heads * head_dim * 2)};
  const cuuint32_t box[4] = {64, 1, static_cast<cuuint32_t>(block_size), 1};
  const cuuint32_t estride[4] = {1, 1, 1, 1};
  const CUtensorMapDataType t =
      dt == RK_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = fn(map, t, 4, const_cast<void*>(base), dims, strides, box, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r == CUDA_SUCCESS) return RK_OK;
  note_error("cuTensorMapEncodeTiled failed (CUresult " + std::to_string(static_cast<int>(r)) +
             ") for the paged K/V cache map");
  return RK_ERR_UNSUPPORTED;
}

template <typename T, typename Index, int D>
rk_status launch_tc(const PagedTcArgs& a, cudaStream_t s) {
  using C = patc::Cfg<T, D>;
  CUtensorMap tk, tv;
  rk_status st = encode_cache_map(&tk, a.k, a.dt, D, a.hkv, a.block_size, a.num_blocks);
  if (st != RK_OK) return st;
  if ((st = encode_cache_map(&tv, a.v, a.dt, D, a.hkv, a.block_size, a.num_blocks)) != RK_OK) return st;
  LaunchCtl lc;
  if ((st = launch_ctl(&lc)) != RK_OK) return st;
  const KernelCtl ctl{lc.status, lc.timeout_ns, 0};
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [&] {
    attr_err[dev & 63] = cudaFuncSetAttribute(patc::paged_tc_kernel<T, Index, D>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  });
  if (attr_err[dev & 63] != cudaSuccess) return cuda_status(attr_err[dev & 63]);
  patc::Params p{};
  p.q = a.q;
  p.tables = a.tables;
  p.lens = a.lens;
  p.out = a.out;
  p.part_acc = a.part_acc;
  p.part_ml = a.part_ml;
  p.batch = static_cast<int>(a.batch);
  p.hq = static_cast<int>(a.hq);
  p.hkv = static_cast<int>(a.hkv);
  p.group = static_cast<int>(a.hq / a.hkv);
  p.num_blocks = static_cast<int>(a.num_blocks);
  p.block_size = static_cast<int>(a.block_size);
  p.max_blocks = static_cast<int>(a.max_blocks);
  p.partitions = a.partitions;
  p.part_tokens = a.part_tokens;
  p.scale_log2 = static_cast<float>(static_cast<double>(a.scale) * 1.4426950408889634);
  const dim3 grid(static_cast<unsigned>(a.partitions), static_cast<unsigned>(a.hkv),
                  static_cast<unsigned>(a.batch));
  const cudaError_t e = launch_kernel(patc::paged_tc_kernel<T, Index, D>, grid, dim3(patc::THREADS),
                                      C::SMEM, s, 0, tk, tv, p, ctl);
  note_launch();
  return cuda_status(e);
}

}  // namespace

bool paged_attention_tc_supported(const void* key_cache, const void* value_cache, int64_t hq,
                                  int64_t hkv, int64_t head_dim, int64_t block_size) {
  if (device_cc_major() != 10) return false;
  if (head_dim != 64 && head_dim != 128) return false;
  if (hq / hkv > patc::NG) return false;
  if (block_size != 8 && block_size != 16 && block_size != 32 && block_size != 64 && block_size != 128)
    return false;
  return aligned16(key_cache) && aligned16(value_cache);
}

// Context partitions of the tensor-core kernel: about two CTAs per SM, whole 128-position
// tiles each.
void paged_attention_tc_plan(int64_t batch, int64_t hkv, int64_t max_ctx, int sms, int* partitions,
                             int* part_tokens) {
  const int64_t base = batch * hkv;
  int64_t parts = (2ll * sms + base - 1) / base;
  const int64_t tiles = (max_ctx + patc::TILE - 1) / patc::TILE;
  if (parts > tiles) parts = tiles;
  if (parts < 1) parts = 1;
  int64_t tokens = (max_ctx + parts - 1) / parts;
  tokens = (tokens + patc::TILE - 1) / patc::TILE * patc::TILE;
  *part_tokens = static_cast<int>(tokens);
  *partitions = static_cast<int>((max_ctx + tokens - 1) / tokens);
}

rk_status paged_attention_tc_launch(const PagedTcArgs& a, cudaStream_t s) {
  const bool bf16 = a.dt == RK_DTYPE_BF16;
  if (a.head_dim == 64) {
    if (a.index_bits == 32)
      return bf16 ? launch_tc<__nv_bfloat16, int32_t, 64>(a, s) : launch_tc<__half, int32_t, 64>(a, s);
    return bf16 ? launch_tc<__nv_bfloat16, int64_t, 64>(a, s) : launch_tc<__half, int64_t, 64>(a, s);
  }
  if (a.index_bits == 32)
    return bf16 ? launch_tc<__nv_bfloat16, int32_t, 128>(a, s) : launch_tc<__half, int32_t, 128>(a, s);
  return bf16 ? launch_tc<__nv_bfloat16, int64_t, 128>(a, s) : launch_tc<__half, int64_t, 128>(a, s);
}

}  // namespace rk
