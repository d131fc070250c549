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
constexpr int THREADS = 224;  // 4 softmax warps, a K load warp, an MMA warp, a V load warp
constexpr int UMMA_K = 16;
constexpr float LN2 = 0.6931471805599453f;

template <typename T, int D>
struct Cfg {
  static constexpr bool SPLIT = std::is_same<T, __nv_bfloat16>::value;
  static constexpr int CHUNKS = D / 64;                // real 64-dim chunks
  static constexpr int K_BYTES = CHUNKS * TILE * 128;  // CHUNKS x [128 positions x 128 B]
  static constexpr int V_BYTES = 2 * TILE * 128;       // 2 chunks (M = 128); D = 64: chunk 1 zero
  static constexpr int LOAD_BYTES = K_BYTES;           // bytes the TMA delivers per tile, K or V
  static constexpr int STAGES = D == 64 ? 4 : 3;
  static constexpr int Q_BYTES = CHUNKS * NG * 128;    // Q^T: CHUNKS x [16 heads x 128 B], x 2
  // bf16: P^T = [P_hi; P_lo] stacked as one N = 32 operand, so P V is one MMA per K step
  // into 32 accumulator columns (V P_hi, V P_lo) that the epilogue adds.
  static constexpr int PN = SPLIT ? 2 * NG : NG;       // rows of the P^T operand
  static constexpr int P_BYTES = 2 * PN * 128;         // P^T: 2 position chunks x [PN x 128 B]
  static constexpr int O_W = PN;                       // O^T columns per buffer
  static constexpr int TMEM_COLS = SPLIT ? 128 : 64;   // S^T x 2 (16 columns each), O^T x 2
  static constexpr int SMEM = 1024 + STAGES * (K_BYTES + V_BYTES) + 2 * Q_BYTES +
                              2 * P_BYTES + 2048;  // P^T by tile parity
  static_assert(D == 64 || D == 128, "head_dim");
  static_assert(SMEM <= 232448, "shared memory per CTA");
};

struct Params {
  const void* tables;
  const void* lens;
  void* out;
  float* part_acc;  // [batch, hq, partitions, D]
  float* part_ml;   // [batch, hq, partitions, 2] (natural-log max, sum)
  int batch, hq, hkv, group;
  int num_blocks, block_size, max_blocks;
  int partitions, part_tokens;  // part_tokens: a multiple of TILE
  int items;                    // batch * hkv * partitions
  int q_rows;                   // rows of one Q^T box: min(NG, hq)
  float scale_log2;
};

struct __align__(16) Bars {
  uint64_t k_full[4];    // TMA: K tile in the stage
  uint64_t k_empty[4];   // MMA commit: the score MMAs no longer read the stage's K tile
  uint64_t v_full[4];    // TMA: V tile in the stage
  uint64_t v_empty[4];   // MMA commit: P V no longer reads the stage's V tile
  uint64_t q_full[2];    // TMA: Q^T of the n-th non-empty item in buffer n & 1
  uint64_t q_empty[2];   // MMA commit: that item's S MMAs no longer read the buffer
  uint64_t s_done[2];    // MMA commit: S^T buffer t & 1 holds tile t's scores
  uint64_t p_full[2];    // one arrival per softmax warp: P^T_t written (buffer t & 1)
  uint64_t o_done[2];    // MMA commit: O^T += V^T P^T_t done (t & 1)
  uint64_t o_free[2];    // one arrival per softmax warp: O^T buffer n & 1 read out
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  alignas(16) float red[2][4][NG];    // per-warp per-head maxima, by tile parity
  alignas(16) float red_l[2][4][NG];  // per-warp per-head sums (epilogue), by item parity
};

// Reduce-scatter of N per-lane values (N = 1, 2, 4, 8, 16) over the warp: log2(N) halving
// steps (N/2 + N/4 + ... shuffles), then a butterfly over the remaining lane bits, leave in
// lane l the reduction over all 32 lanes of value head_of_lane<N>(l).  Each halving step
// keeps half of the values and folds in the partner's copy of that half, so N reductions
// share N + 4 - log2(N) shuffles instead of taking 5 dependent ones each.  The pairing
// order (lane bits 4, 3, 2, 1, 0) is the plain butterfly's, so results are the same.
template <int N>
__device__ __forceinline__ int head_of_lane(int lane) {
  constexpr int L = N >= 16 ? 4 : N >= 8 ? 3 : N >= 4 ? 2 : N >= 2 ? 1 : 0;
  return (lane >> (5 - L)) & (N - 1);
}
template <int N>
__device__ __forceinline__ bool scatter_writer(int lane) {  // one lane per head
  constexpr int L = N >= 16 ? 4 : N >= 8 ? 3 : N >= 4 ? 2 : N >= 2 ? 1 : 0;
  return (lane & ((1 << (5 - L)) - 1)) == 0;
}

template <int N, typename Op>
__device__ __forceinline__ float warp_reduce_scatter(const float (&v)[N], int lane, Op op) {
  static_assert(N == 1 || N == 2 || N == 4 || N == 8 || N == 16, "heads per item");
  float cur[N];
#pragma unroll
  for (int i = 0; i < N; ++i) cur[i] = v[i];
  int offset = 16;
#pragma unroll
  for (int n = N; n > 1; n >>= 1, offset >>= 1) {
    const bool up = lane & offset;
#pragma unroll
    for (int i = 0; i < n / 2; ++i)
      cur[i] = op(up ? cur[i + n / 2] : cur[i], __shfl_xor_sync(0xffffffffu, up ? cur[i] : cur[i + n / 2], offset));
  }
  float r = cur[0];
#pragma unroll
  for (; offset > 0; offset >>= 1) r = op(r, __shfl_xor_sync(0xffffffffu, r, offset));
  return r;
}

struct MaxOp {
  __device__ __forceinline__ float operator()(float a, float b) const { return fmaxf(a, b); }
};
struct AddOp {
  __device__ __forceinline__ float operator()(float a, float b) const { return a + b; }
};

// Combination of the four softmax warps' values of heads 0..N-1 (slots [4][NG]) in warp order.
template <int N, typename Op>
__device__ __forceinline__ void combine_warps(const float (*slots)[NG], float (&out)[N], Op op) {
  if constexpr (N >= 4) {
    float4 x[4][N / 4];
#pragma unroll
    for (int w = 0; w < 4; ++w)
#pragma unroll
      for (int i = 0; i < N / 4; ++i) x[w][i] = reinterpret_cast<const float4*>(slots[w])[i];
#pragma unroll
    for (int i = 0; i < N / 4; ++i) {
      out[4 * i + 0] = op(op(op(x[0][i].x, x[1][i].x), x[2][i].x), x[3][i].x);
      out[4 * i + 1] = op(op(op(x[0][i].y, x[1][i].y), x[2][i].y), x[3][i].y);
      out[4 * i + 2] = op(op(op(x[0][i].z, x[1][i].z), x[2][i].z), x[3][i].z);
      out[4 * i + 3] = op(op(op(x[0][i].w, x[1][i].w), x[2][i].w), x[3][i].w);
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = op(op(op(slots[0][i], slots[1][i]), slots[2][i]), slots[3][i]);
  }
}

// Named barrier of the four softmax warps (id 1).
__device__ __forceinline__ void softmax_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Work item = (sequence, KV head, context partition); items are numbered with the partition
// fastest, and CTA c takes items c, c + gridDim.x, ...
struct Item {
  int b, kvh, part;
  int t_begin, t_end, n_tiles;
};

__device__ __forceinline__ int item_sequence(const Params& p, int item) {
  return item / (p.hkv * p.partitions);
}

template <typename Index>
__device__ __forceinline__ Item make_item(const Params& p, int item, Index len_raw) {
  Item it;
  it.b = item / (p.hkv * p.partitions);
  const int rest = item - it.b * (p.hkv * p.partitions);
  it.kvh = rest / p.partitions;
  it.part = rest - it.kvh * p.partitions;
  const int64_t max_ctx = static_cast<int64_t>(p.max_blocks) * p.block_size;
  int64_t ctx = static_cast<int64_t>(len_raw);
  ctx = ctx < 0 ? 0 : (ctx > max_ctx ? max_ctx : ctx);
  it.t_begin = it.part * p.part_tokens;
  it.t_end = static_cast<int>(min(static_cast<int64_t>(it.t_begin) + p.part_tokens, ctx));
  it.n_tiles = it.t_end > it.t_begin ? (it.t_end - it.t_begin + TILE - 1) / TILE : 0;
  return it;
}

// Persistent: one CTA per SM walks its work items.  Warps 0-3: softmax (thread = position =
// TMEM lane; for O^T, thread = output dimension); warp 4: bulk loads of Q^T and K; warp 6:
// bulk loads of V; warp 5: MMA issue.  They meet on mbarriers only, so the loads run up to
// STAGES tiles ahead of their consumers across item boundaries, and an item's epilogue
// overlaps the next item's loads and score MMAs (O^T is double-buffered in TMEM by item
// parity).
template <typename T, typename Index, int D, int NGE>
__global__ void __launch_bounds__(THREADS, 1)
    paged_tc_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                    const __grid_constant__ CUtensorMap tmap_q, Params p, KernelCtl ctl) {
  using C = Cfg<T, D>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sk = smem;                          // STAGES x K tile
  uint8_t* sv = sk + STAGES * C::K_BYTES;      // STAGES x V tile
  uint8_t* sq = sv + STAGES * C::V_BYTES;      // 2 x Q^T (item parity)
  uint8_t* sp = sq + 2 * C::Q_BYTES;           // P^T buffers: [tile parity][hi, lo]
  constexpr int P_SET = C::P_BYTES;
  Bars* bars = reinterpret_cast<Bars*>(sp + 2 * P_SET);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bs = p.block_size;
  const int max_ctx = p.max_blocks * bs;
  const Index* lens = static_cast<const Index*>(p.lens);

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&bars->k_full[s]), 1);
      mbar_init(smem_u32(&bars->k_empty[s]), 1);
      mbar_init(smem_u32(&bars->v_full[s]), 1);
      mbar_init(smem_u32(&bars->v_empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&bars->q_full[s]), 1);
      mbar_init(smem_u32(&bars->q_empty[s]), 1);
      mbar_init(smem_u32(&bars->s_done[s]), 1);
      mbar_init(smem_u32(&bars->p_full[s]), 4);
      mbar_init(smem_u32(&bars->o_done[s]), 1);
      mbar_init(smem_u32(&bars->o_free[s]), 4);
    }
    mbar_init(smem_u32(&bars->drain), 1);
    bars->abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmap_k);
    tma_prefetch_desc(&tmap_v);
    tma_prefetch_desc(&tmap_q);
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&bars->tmem_base), C::TMEM_COLS);
    tmem_relinquish();
  }
  // P^T rows past NGE are never written: zero both buffers once.
  for (int i = tid; i < 2 * P_SET / 16; i += THREADS)
    reinterpret_cast<uint4*>(sp)[i] = make_uint4(0, 0, 0, 0);
  if (D == 64) {
    // V^T is the M = 128 operand: its second 64-row chunk stays zero in every stage.
    for (int i = tid; i < STAGES * TILE * 128 / 16; i += THREADS) {
      const int st = i / (TILE * 128 / 16), r = i - st * (TILE * 128 / 16);
      reinterpret_cast<uint4*>(sv + st * C::V_BYTES + TILE * 128)[r] = make_uint4(0, 0, 0, 0);
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  constexpr int O_COL = 2 * NG;  // O^T buffers at O_COL and O_COL + O_W
  pdl_begin();  // global memory is touched only after this

  int never = 0;
  volatile int* abort = &bars->abort;
  auto fail = [&](uint32_t code) {
    *abort = 1;
    atomicOr(ctl.status, code);
  };

  if (warp == 4 || warp == 6) {
    // ------------------------------------------------------------ loads
    // Warp 4 streams Q^T and the K tiles, warp 6 the V tiles, each through its own ring:
    // a K stage is free again once the tile's score MMAs are done, a V stage once its P V is,
    // so neither ring waits for the other operand's consumer.
    const bool is_k = warp == 4;
    uint8_t* ring = is_k ? sk : sv;
    const int ring_bytes = is_k ? C::K_BYTES : C::V_BYTES;
    uint64_t* full = is_k ? bars->k_full : bars->v_full;
    uint64_t* empty = is_k ? bars->k_empty : bars->v_empty;
    const CUtensorMap* tmap = is_k ? &tmap_k : &tmap_v;
    uint32_t issued[4] = {0, 0, 0, 0}, q_issued[2] = {0, 0};
    const int blocks_per_tile = TILE / bs;
    const uint32_t q_tx = static_cast<uint32_t>(C::CHUNKS * p.q_rows * 128);
    int g = 0, ne = 0;
    bool ok = true;
    int item = blockIdx.x;
    Index len_next = item < p.items ? lens[item_sequence(p, item)] : Index(0);
    for (; ok && item < p.items; item += gridDim.x) {
      const Index len_raw = len_next;
      const int b = item_sequence(p, item);
      const Index* tab = static_cast<const Index*>(p.tables) + static_cast<int64_t>(b) * p.max_blocks;
      // Block-table entry of this lane's block in the item's first tile, read before the
      // context length is known (any position below max_ctx has a table slot).
      const int t0 = (item - b * (p.hkv * p.partitions)) % p.partitions * p.part_tokens;
      Index ent = 0;
      if (lane < blocks_per_tile && t0 + lane * bs < max_ctx) ent = tab[(t0 + lane * bs) / bs];
      if (item + static_cast<int>(gridDim.x) < p.items)
        len_next = lens[item_sequence(p, item + gridDim.x)];
      const Item it = make_item(p, item, len_raw);
      if (it.n_tiles == 0) continue;
      if (is_k && lane == 0) {
        const int qb = ne & 1;
        if (ne >= 2) ok = mbar_wait_bounded(smem_u32(&bars->q_empty[qb]), ((ne - 2) >> 1) & 1, ctl.timeout_ns, abort);
        if (ok) {
          const uint32_t bar = smem_u32(&bars->q_full[qb]);
          mbar_arrive_expect_tx(bar, q_tx);
          ++q_issued[qb];
#pragma unroll
          for (int c = 0; c < C::CHUNKS; ++c)
            tma_load_3d(smem_u32(sq + qb * C::Q_BYTES + c * (NG * 128)), &tmap_q, bar, c * 64,
                        it.kvh * p.group, it.b);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) fail(RK_DEV_ERR_TIMEOUT_PRODUCER);
        break;
      }
      for (int t = 0; t < it.n_tiles; ++t, ++g) {
        const int st = g % STAGES;
        const int pos = it.t_begin + t * TILE + lane * bs;  // first position of block `lane`
        Index ent_next = 0;  // next tile's entry, fetched while this tile waits for its stage
        if (t + 1 < it.n_tiles && lane < blocks_per_tile && pos + TILE < it.t_end)
          ent_next = tab[(pos + TILE) / bs];
        bool okw = true;
        if (lane == 0 && g >= STAGES)
          okw = mbar_wait_bounded(smem_u32(&empty[st]), ((g / STAGES) - 1) & 1, ctl.timeout_ns, abort);
        okw = __shfl_sync(0xffffffffu, okw, 0);
        if (!okw) {
          if (lane == 0) fail(RK_DEV_ERR_TIMEOUT_PRODUCER);
          ok = false;
          break;
        }
        const uint32_t bar = smem_u32(&full[st]);
        if (lane == 0) {
          mbar_arrive_expect_tx(bar, C::LOAD_BYTES);
          ++issued[st];
        }
        __syncwarp();
        if (lane < blocks_per_tile) {
          int blk = p.num_blocks;  // out of range: reads as zero
          if (pos < it.t_end) {
            const int64_t idx = static_cast<int64_t>(ent);
            if (idx >= 0 && idx < p.num_blocks)
              blk = static_cast<int>(idx);
            else if (is_k)
              atomicOr(ctl.status, RK_DEV_ERR_BAD_INDEX);
          }
#pragma unroll
          for (int c = 0; c < C::CHUNKS; ++c) {
            const uint32_t off = c * (TILE * 128) + lane * bs * 128;
            tma_load_4d(smem_u32(ring + st * ring_bytes + off), tmap, bar, c * 64, it.kvh, 0, blk);
          }
        }
        ent = ent_next;
      }
      ++ne;
    }
    // No bulk copy may still be landing when the CTA exits: wait for the last load of
    // each stage and Q^T buffer (earlier ones completed before the buffer was refilled).
    if (lane == 0) {
      for (int s = 0; s < STAGES; ++s)
        if (issued[s] > 0 &&
            !mbar_wait_bounded(smem_u32(&full[s]), (issued[s] - 1) & 1u, ctl.timeout_ns, &never))
          atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_DRAIN);
      for (int s = 0; s < 2; ++s)
        if (q_issued[s] > 0 &&
            !mbar_wait_bounded(smem_u32(&bars->q_full[s]), (q_issued[s] - 1) & 1u, ctl.timeout_ns, &never))
          atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_DRAIN);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      constexpr uint32_t IDESC_S = umma_idesc_f16(std::is_same<T, __nv_bfloat16>::value, TILE, NG, false, false);
      constexpr uint32_t IDESC_O = umma_idesc_f16(std::is_same<T, __nv_bfloat16>::value, TILE, C::PN, true, false);
      // Cursor over this CTA's tiles: item, its tile count, tile j in it, non-empty item
      // count ne, tile count g, and the context length of the item after (read one item
      // ahead, so moving to the next item does not wait for a global load).
      struct Cur {
        int item, n, j, ne, g;
        Index len_next;
      };
      auto seek = [&](Cur& c) {  // from c.item on, to the first item with tiles
        for (; c.item < p.items; c.item += gridDim.x) {
          const Index len = c.len_next;
          const int nxt = c.item + static_cast<int>(gridDim.x);
          c.len_next = nxt < p.items ? lens[item_sequence(p, nxt)] : Index(0);
          c.n = make_item(p, c.item, len).n_tiles;
          if (c.n > 0) return;
        }
      };
      auto step = [&](Cur& c) {
        ++c.g;
        if (++c.j < c.n) return;
        c.j = 0;
        ++c.ne;
        c.item += gridDim.x;
        seek(c);
      };
      // S^T_t = K_t Q^T into buffer t & 1
      auto issue_s = [&](const Cur& c) -> bool {
        const int st = c.g % STAGES, qb = c.ne & 1;
        if (c.j == 0 &&
            !mbar_wait_bounded(smem_u32(&bars->q_full[qb]), (c.ne >> 1) & 1, ctl.timeout_ns, abort)) {
          fail(RK_DEV_ERR_TIMEOUT_PRODUCER);
          return false;
        }
        if (!mbar_wait_bounded(smem_u32(&bars->k_full[st]), (c.g / STAGES) & 1, ctl.timeout_ns, abort)) {
          fail(RK_DEV_ERR_TIMEOUT_PRODUCER);
          return false;
        }
        tc_fence_after();
        const uint64_t dk = umma_desc_sw128(smem_u32(sk + st * C::K_BYTES), 16, 1024);
        const uint64_t dq = umma_desc_sw128(smem_u32(sq + qb * C::Q_BYTES), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < D / UMMA_K; ++kk) {
          const uint32_t off_k = (kk >> 2) * (TILE * 128) + (kk & 3) * 32;
          const uint32_t off_q = (kk >> 2) * (NG * 128) + (kk & 3) * 32;
          tc_mma_f16(tmem + (c.g & 1) * NG, umma_desc_advance(dk, off_k), umma_desc_advance(dq, off_q),
                     IDESC_S, kk > 0 ? 1u : 0u);
        }
        tc_commit(smem_u32(&bars->s_done[c.g & 1]));
        tc_commit(smem_u32(&bars->k_empty[st]));
        if (c.j + 1 == c.n) tc_commit(smem_u32(&bars->q_empty[qb]));
        return true;
      };
      Cur cs{static_cast<int>(blockIdx.x), 0, 0, 0, 0,
             static_cast<int>(blockIdx.x) < p.items ? lens[item_sequence(p, blockIdx.x)] : Index(0)};
      seek(cs);
      Cur cp = cs;
      bool ok = true;
      if (cs.item < p.items) {
        ok = issue_s(cs);
        step(cs);
      }
      while (ok && cp.item < p.items) {
        // S^T of the next tile into the buffer of the tile before this one, which the
        // softmax warps read before they released P^T of it.
        if (cs.item < p.items) {
          if (!issue_s(cs)) break;
          step(cs);
        }
        if (!mbar_wait_bounded(smem_u32(&bars->p_full[cp.g & 1]), (cp.g >> 1) & 1, ctl.timeout_ns, abort)) {
          fail(RK_DEV_ERR_TIMEOUT_PRODUCER);
          break;
        }
        const int ob = cp.ne & 1;
        if (cp.j == 0 && cp.ne >= 2 &&
            !mbar_wait_bounded(smem_u32(&bars->o_free[ob]), ((cp.ne - 2) >> 1) & 1, ctl.timeout_ns, abort)) {
          fail(RK_DEV_ERR_TIMEOUT_EPILOGUE);
          break;
        }
        const int st = cp.g % STAGES;
        if (!mbar_wait_bounded(smem_u32(&bars->v_full[st]), (cp.g / STAGES) & 1, ctl.timeout_ns, abort)) {
          fail(RK_DEV_ERR_TIMEOUT_PRODUCER);
          break;
        }
        tc_fence_after();
        const uint64_t dv = umma_desc_sw128(smem_u32(sv + st * C::V_BYTES), TILE * 128, 1024);
        const uint64_t dp = umma_desc_sw128(smem_u32(sp + (cp.g & 1) * P_SET), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < TILE / UMMA_K; ++kk) {
          const uint32_t off_p = (kk >> 2) * (C::PN * 128) + (kk & 3) * 32;
          tc_mma_f16(tmem + O_COL + ob * C::O_W, umma_desc_advance(dv, kk * 2048), umma_desc_advance(dp, off_p),
                     IDESC_O, (cp.j > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(smem_u32(&bars->o_done[cp.g & 1]));
        tc_commit(smem_u32(&bars->v_empty[st]));
        step(cp);
      }
      // Every MMA completes before TMEM is released.
      tc_commit(smem_u32(&bars->drain));
      if (!mbar_wait_bounded(smem_u32(&bars->drain), 0, ctl.timeout_ns, &never))
        atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_DRAIN);
    }
  } else {
    // ------------------------------------------------------------ softmax
    // NGE = the group's heads rounded up to 1, 4, 8 or 16: only those rows of P^T are
    // written (the rest stay zero from the start), so a small group pays for its own heads.
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const int G = p.group;  // real heads per item (<= NGE), uniform over the CTA
    int g = 0, ne = 0;
    int item = blockIdx.x;
    Index len_next = item < p.items ? lens[item_sequence(p, item)] : Index(0);
    for (; item < p.items; item += gridDim.x) {
      const Index len_raw = len_next;
      const int b = item_sequence(p, item);
      const Index* tab = static_cast<const Index*>(p.tables) + static_cast<int64_t>(b) * p.max_blocks;
      const int t0 = (item - b * (p.hkv * p.partitions)) % p.partitions * p.part_tokens;
      // Block-table entry of this thread's first position, read before the length is known.
      Index e_cur = -1;
      if (t0 + tid < max_ctx) e_cur = tab[(t0 + tid) / bs];
      if (item + static_cast<int>(gridDim.x) < p.items)
        len_next = lens[item_sequence(p, item + gridDim.x)];
      const Item it = make_item(p, item, len_raw);
      const int h0 = it.kvh * G;
      // Per-head state (identical in every softmax thread): the maximum the exponentials use.
      float m_use[NGE], l_part[NGE];
#pragma unroll
      for (int gg = 0; gg < NGE; ++gg) {
        m_use[gg] = -INFINITY;
        l_part[gg] = 0.f;
      }
      for (int j = 0; j < it.n_tiles; ++j, ++g) {
        const int pos = it.t_begin + j * TILE + tid;
        const bool attended =
            pos < it.t_end && static_cast<int64_t>(e_cur) >= 0 && static_cast<int64_t>(e_cur) < p.num_blocks;
        if (j + 1 < it.n_tiles) e_cur = pos + TILE < it.t_end ? tab[(pos + TILE) / bs] : Index(-1);
        if (!mbar_wait_bounded(smem_u32(&bars->s_done[g & 1]), (g >> 1) & 1, ctl.timeout_ns, abort))
          fail(RK_DEV_ERR_TIMEOUT_MMA);
        tc_fence_after();
        float s[NGE];
        {
          uint32_t r[NGE <= 4 ? 4 : 16];
          if constexpr (NGE <= 4)
            tmem_ld_32x32b_x4(t_lane + (g & 1) * NG, r);
          else
            tmem_ld_32x32b_x16(t_lane + (g & 1) * NG, r);
          tmem_ld_wait();
#pragma unroll
          for (int gg = 0; gg < NGE; ++gg)
            s[gg] = attended && gg < G ? __uint_as_float(r[gg]) * p.scale_log2 : -INFINITY;
        }
        // Per-head maximum over the tile: a reduce-scatter within the warp, then the four
        // warps (slots of this tile's parity: a warp rewrites them two tiles on, after the
        // barrier of the tile between, which its peers reach only once they have read them).
        // Padding heads and masked positions are -inf, so no head needs a branch.
        float(*red)[NG] = bars->red[g & 1];
        {
          const float v = warp_reduce_scatter<NGE>(s, lane, MaxOp());
          if (scatter_writer<NGE>(lane)) red[warp][head_of_lane<NGE>(lane)] = v;
        }
        softmax_sync();
        float mt[NGE];
        combine_warps<NGE>(red, mt, MaxOp());
        float alpha[NGE];
        bool rescale = false;  // uniform: every softmax thread holds the same maxima
#pragma unroll
        for (int gg = 0; gg < NGE; ++gg) {
          alpha[gg] = 1.f;
          rescale |= mt[gg] > m_use[gg] + 8.f;  // lazy rescaling: P <= 256
        }
        if (rescale) {
#pragma unroll
          for (int gg = 0; gg < NGE; ++gg) {
            if (mt[gg] > m_use[gg] + 8.f) {
              alpha[gg] = ex2_approx(m_use[gg] - mt[gg]);
              m_use[gg] = mt[gg];
            }
          }
        }
        // P for this position (zero for padding heads and masked positions).
        constexpr int NP = (NGE + 1) / 2;  // packed pairs
        uint32_t hi[NP], lo[NP];
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          float e[2] = {0.f, 0.f};
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int gg = 2 * i + h;
            if (gg < NGE) {
              const float m = m_use[gg] == -INFINITY ? 0.f : m_use[gg];
              e[h] = ex2_approx(s[gg] - m);
              l_part[gg] = l_part[gg] * alpha[gg] + e[h];
            }
          }
          hi[i] = Pack2<T>::from_floats(e[0], e[1]);
          if (C::SPLIT) {
            const float2 h2 = Pack2<T>::to_floats(hi[i]);
            lo[i] = Pack2<T>::from_floats(e[0] - h2.x, e[1] - h2.y);
          }
        }
        // P^T buffer g & 1 was read by the P V of tile g - 2; a rescaling of O^T needs every
        // earlier P V of the item done (they complete in order: tile g - 1 is enough).
        // Neither usually waits: the softmax of a tile does not otherwise depend on P V.
        if (g >= 2 &&
            !mbar_wait_bounded(smem_u32(&bars->o_done[g & 1]), ((g - 2) >> 1) & 1, ctl.timeout_ns, abort))
          fail(RK_DEV_ERR_TIMEOUT_MMA);
        if (j > 0 && rescale) {  // uniform: every softmax thread holds the same maxima
          if (!mbar_wait_bounded(smem_u32(&bars->o_done[(g - 1) & 1]), ((g - 1) >> 1) & 1, ctl.timeout_ns, abort))
            fail(RK_DEV_ERR_TIMEOUT_MMA);
          tc_fence_after();
          if constexpr (C::SPLIT) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(t_lane + O_COL + (ne & 1) * C::O_W, r);
            tmem_ld_wait();
#pragma unroll
            for (int gg = 0; gg < NGE; ++gg) {
              r[gg] = __float_as_uint(__uint_as_float(r[gg]) * alpha[gg]);
              r[NG + gg] = __float_as_uint(__uint_as_float(r[NG + gg]) * alpha[gg]);
            }
            tmem_st_32x32b_x32(t_lane + O_COL + (ne & 1) * C::O_W, r);
          } else {
            uint32_t r[16];
            tmem_ld_32x32b_x16(t_lane + O_COL + (ne & 1) * C::O_W, r);
            tmem_ld_wait();
#pragma unroll
            for (int gg = 0; gg < NGE; ++gg) r[gg] = __float_as_uint(__uint_as_float(r[gg]) * alpha[gg]);
            tmem_st_32x32b_x16(t_lane + O_COL + (ne & 1) * C::O_W, r);
          }
          tmem_st_wait();
        }
        tc_fence_after();
        // P^T: row gg = head, positions along K; this thread writes position `tid` of each row.
        {
          // Rows 0..15: P (bf16: P_hi), rows 16..31: P_lo; row r of chunk c at
          // c * PN * 128 + r * 128, 16-byte units swizzled by r & 7.
          uint8_t* pb = sp + (g & 1) * P_SET;
          const int c = tid >> 6, within = tid & 63;
          const uint32_t base = c * (C::PN * 128) + (within & 7) * 2;
#pragma unroll
          for (int gg = 0; gg < NGE; ++gg) {
            const uint32_t off = base + gg * 128 + (((within >> 3) ^ (gg & 7)) << 4);
            const uint32_t hv = (gg & 1) ? (hi[gg / 2] >> 16) : (hi[gg / 2] & 0xffffu);
            *reinterpret_cast<uint16_t*>(pb + off) = static_cast<uint16_t>(hv);
            if (C::SPLIT) {
              const uint32_t lv = (gg & 1) ? (lo[gg / 2] >> 16) : (lo[gg / 2] & 0xffffu);
              *reinterpret_cast<uint16_t*>(pb + off + NG * 128) = static_cast<uint16_t>(lv);
            }
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&bars->p_full[g & 1]));
      }

      // ---- epilogue: per-head sums over the 128 positions, then O^T row d = tid.
      float o_row[NGE];
      float l_sum[NGE];
      if (it.n_tiles > 0) {
        if (!mbar_wait_bounded(smem_u32(&bars->o_done[(g - 1) & 1]), ((g - 1) >> 1) & 1, ctl.timeout_ns, abort))
          fail(RK_DEV_ERR_TIMEOUT_EPILOGUE);
        tc_fence_after();
        float(*red_l)[NG] = bars->red_l[ne & 1];
        {
          const float v = warp_reduce_scatter<NGE>(l_part, lane, AddOp());
          if (scatter_writer<NGE>(lane)) red_l[warp][head_of_lane<NGE>(lane)] = v;
        }
        softmax_sync();
        combine_warps<NGE>(red_l, l_sum, AddOp());
        const uint32_t o_addr = t_lane + O_COL + (ne & 1) * C::O_W;
        uint32_t r[NGE <= 4 ? 4 : 16], r_lo[NGE <= 4 ? 4 : 16];
        if constexpr (NGE <= 4) {
          tmem_ld_32x32b_x4(o_addr, r);
          if constexpr (C::SPLIT) tmem_ld_32x32b_x4(o_addr + NG, r_lo);
        } else {
          tmem_ld_32x32b_x16(o_addr, r);
          if constexpr (C::SPLIT) tmem_ld_32x32b_x16(o_addr + NG, r_lo);
        }
        tmem_ld_wait();
#pragma unroll
        for (int gg = 0; gg < NGE; ++gg)
          o_row[gg] = C::SPLIT ? __uint_as_float(r[gg]) + __uint_as_float(r_lo[gg]) : __uint_as_float(r[gg]);
        // O^T buffer ne & 1 is free for the item after next.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&bars->o_free[ne & 1]));
        ++ne;
      } else {
#pragma unroll
        for (int gg = 0; gg < NGE; ++gg) {
          o_row[gg] = 0.f;
          l_sum[gg] = 0.f;
        }
      }
      if (tid < D && !*abort) {
#pragma unroll
        for (int gg = 0; gg < NGE; ++gg) {
          if (gg < G) {
            const int64_t head = static_cast<int64_t>(it.b) * p.hq + h0 + gg;
            if (p.partitions == 1) {
              static_cast<T*>(p.out)[head * D + tid] = from_f32<T>(o_row[gg] / l_sum[gg]);  // 0/0 = NaN for ctx 0
            } else {
              const int64_t slot = head * p.partitions + it.part;
              p.part_acc[slot * D + tid] = o_row[gg];
              if (tid == 0) {
                p.part_ml[2 * slot] = m_use[gg] == -INFINITY ? -INFINITY : m_use[gg] * LN2;
                p.part_ml[2 * slot + 1] = l_sum[gg];
              }
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

template <typename T, typename Index, int D, int NGE>
rk_status launch_tc(const PagedTcArgs& a, cudaStream_t s) {
  using C = patc::Cfg<T, D>;
  const int64_t items = a.batch * a.hkv * a.partitions;
  if (items <= 0) return RK_OK;
  if (items > INT32_MAX) return RK_ERR_UNSUPPORTED;
  CUtensorMap tk, tv, tq;
  rk_status st = encode_cache_map(&tk, a.k, a.dt, D, a.hkv, a.block_size, a.num_blocks);
  if (st != RK_OK) return st;
  if ((st = encode_cache_map(&tv, a.v, a.dt, D, a.hkv, a.block_size, a.num_blocks)) != RK_OK) return st;
  // Q [batch, hq, D]: one box = 64 dims of the item's query heads (rows past the group are
  // other heads' queries or zero past hq; their score columns are masked).
  const int q_rows = a.hq < patc::NG ? static_cast<int>(a.hq) : patc::NG;
  if ((st = encode_tmap_3d(&tq, a.q, a.dt, D, a.hq, a.batch, 64, static_cast<uint32_t>(q_rows))) != RK_OK)
    return st;
  LaunchCtl lc;
  if ((st = launch_ctl(&lc)) != RK_OK) return st;
  const KernelCtl ctl{lc.status, lc.timeout_ns, 0};
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [&] {
    attr_err[dev & 63] = cudaFuncSetAttribute(patc::paged_tc_kernel<T, Index, D, NGE>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  });
  if (attr_err[dev & 63] != cudaSuccess) return cuda_status(attr_err[dev & 63]);
  patc::Params p{};
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
  p.items = static_cast<int>(items);
  p.q_rows = q_rows;
  p.scale_log2 = static_cast<float>(static_cast<double>(a.scale) * 1.4426950408889634);
  // Persistent: one CTA per SM (the stage ring takes most of the shared memory).
  const int sms = device_sm_count();
  const unsigned grid = static_cast<unsigned>(items < sms ? items : sms);
  const cudaError_t e = launch_kernel(patc::paged_tc_kernel<T, Index, D, NGE>, dim3(grid), dim3(patc::THREADS),
                                      C::SMEM, s, 0, tk, tv, tq, p, ctl);
  note_launch();
  return cuda_status(e);
}

// Heads per item rounded up to 1, 4, 8 or 16 (the softmax warps' per-head work).
template <typename T, typename Index, int D>
rk_status launch_tc_heads(const PagedTcArgs& a, cudaStream_t s) {
  const int64_t group = a.hq / a.hkv;
  if (group <= 1) return launch_tc<T, Index, D, 1>(a, s);
  if (group <= 4) return launch_tc<T, Index, D, 4>(a, s);
  if (group <= 8) return launch_tc<T, Index, D, 8>(a, s);
  return launch_tc<T, Index, D, 16>(a, s);
}

}  // namespace

bool paged_attention_tc_supported(const void* query, const void* key_cache, const void* value_cache,
                                  int64_t hq, int64_t hkv, int64_t head_dim, int64_t block_size) {
  if (device_cc_major() != 10) return false;
  if (head_dim != 64 && head_dim != 128) return false;
  if (hq / hkv > patc::NG) return false;
  if (block_size != 8 && block_size != 16 && block_size != 32 && block_size != 64 && block_size != 128)
    return false;
  return aligned16(query) && aligned16(key_cache) && aligned16(value_cache);
}

// Context partitions of the tensor-core kernel (whole 128-position tiles each).  The
// persistent CTAs (one per SM) take items round-robin, so the kernel lasts about
// ceil(items / SMs) x (tiles per item + a per-item epilogue) tile times, plus the merge
// kernel when there is more than one partition; the partition count minimising that
// estimate wins (fewest partitions on ties).  Costs in tile times; tiles per item are tried
// for every partition count up to 2 x SMs (a handful of integer operations each).
void paged_attention_tc_plan(int64_t batch, int64_t hkv, int64_t max_ctx, int sms, int* partitions,
                             int* part_tokens) {
  constexpr double ITEM_COST = 0.5, MERGE_COST = 2.0;
  // Decode loops ask for the same shape every step (twice: workspace size and launch).
  thread_local int64_t last_key[4] = {-1, -1, -1, -1};
  thread_local int last_parts = 1, last_tokens = patc::TILE;
  if (last_key[0] == batch && last_key[1] == hkv && last_key[2] == max_ctx && last_key[3] == sms) {
    *partitions = last_parts;
    *part_tokens = last_tokens;
    return;
  }
  const int64_t base = batch * hkv;
  const int64_t tiles = max_ctx > 0 ? (max_ctx + patc::TILE - 1) / patc::TILE : 1;
  const int64_t units = sms > 0 ? sms : 1;
  int64_t best_tpi = tiles;
  double best = 0.0;
  int64_t last_tpi = 0;
  const int64_t p_max = tiles < 2 * units ? tiles : 2 * units;
  for (int64_t p = 1; p <= p_max; ++p) {
    const int64_t tpi = (tiles + p - 1) / p;
    if (tpi == last_tpi) continue;
    last_tpi = tpi;
    const int64_t parts = (tiles + tpi - 1) / tpi;
    const int64_t waves = (base * parts + units - 1) / units;
    const double cost = static_cast<double>(waves) * (static_cast<double>(tpi) + ITEM_COST) +
                        (parts > 1 ? MERGE_COST : 0.0);
    if (p == 1 || cost < best) {
      best = cost;
      best_tpi = tpi;
    }
  }
  const int64_t tokens = best_tpi * patc::TILE;
  *part_tokens = static_cast<int>(tokens);
  *partitions = static_cast<int>(max_ctx > 0 ? (max_ctx + tokens - 1) / tokens : 1);
  last_key[0] = batch;
  last_key[1] = hkv;
  last_key[2] = max_ctx;
  last_key[3] = sms;
  last_parts = *partitions;
  last_tokens = *part_tokens;
}

rk_status paged_attention_tc_launch(const PagedTcArgs& a, cudaStream_t s) {
  const bool bf16 = a.dt == RK_DTYPE_BF16;
  if (a.head_dim == 64) {
    if (a.index_bits == 32)
      return bf16 ? launch_tc_heads<__nv_bfloat16, int32_t, 64>(a, s) : launch_tc_heads<__half, int32_t, 64>(a, s);
    return bf16 ? launch_tc_heads<__nv_bfloat16, int64_t, 64>(a, s) : launch_tc_heads<__half, int64_t, 64>(a, s);
  }
  if (a.index_bits == 32)
    return bf16 ? launch_tc_heads<__nv_bfloat16, int32_t, 128>(a, s) : launch_tc_heads<__half, int32_t, 128>(a, s);
  return bf16 ? launch_tc_heads<__nv_bfloat16, int64_t, 128>(a, s) : launch_tc_heads<__half, int64_t, 128>(a, s);
}

}  // namespace rk
