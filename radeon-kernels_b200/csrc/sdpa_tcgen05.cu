// sdpa_tcgen05.cu -- scaled dot-product self-attention (prefill) on the tcgen05 tensor cores.
//
//   out[b, h, q, :] = softmax_k(scale * Q[b,h,q,:] . K[b,g(h),k,:], causal mask) @ V[b,g(h)]
//
// Semantics of the reference's operator (src/radeon_kernels/ops/sdpa/api.py:22-118,
// reference.py:13-36): [batch, heads, sequence, head_dim] tensors, equal query and key
// lengths, GQA head g(h) = h / (Hq / Hkv), optional causal mask (key <= query), fp32 softmax
// and accumulation, output rounded once to the input dtype.  The reference computes it
// with torch's SDPA (its dispatch manifest has no native entry, dispatch/sdpa-1.0.json); its
// HIP candidate walks keys one at a time per query row (benchmarks/sdpa/native_sdpa.hip).
//
// One CTA per (128-row query tile, query head, batch), 352 threads (8 softmax warps, an
// MMA-issue warp and two load warps), flash-style:
//   * TMA loads -- the Q tile once, K and V tiles of BN keys (128; 64 for head_dim 256, to fit
//     shared memory) in rings of three (K) and two (V) stages (two and two at head_dim 256),
//     through 3-D tensor maps over the [batch*heads, S, D] stacks, so rows past the sequence
//     read as zero instead of the next head's;
//   * S = Q K^T (M = 128, N = BN keys, K = head_dim) into one of three TMEM buffers at
//     head_dim 64, two otherwise: Q and K are K-major 128-byte-swizzled tiles from TMA;
//   * two warps share each 32-row TMEM lane quarter, each thread half of its row's scores:
//     masks on the raw scores (skipped when every row of the warp attends every key of its
//     slice), tree maximum, the scale folded into one FMA before the hardware ex2, online
//     softmax in fp32 that rescales O in TMEM only when the maximum grew by more than 2^8
//     (lazy rescaling).  P = 2^(s - m) is rounded to fp16, or for bf16 kept as two bf16
//     terms P_hi + P_lo (see Cfg::SPLIT);
//   * 128-key tiles: each warp keeps its own maximum, sum and O accumulator over its half of
//     the keys (Cfg::SPLIT_O), so the two warps of a quarter never wait for each other in the
//     key loop; P is written over the warp's own S columns in TMEM (tcgen05.st, two 16-bit
//     values per column) and O += P V takes A from TMEM, so the softmax never waits for the
//     previous tile's P V except to rescale O.  64-key tiles (head_dim 256) exchange the row
//     maximum every tile, share one O and write P to shared memory in the K-major swizzled
//     layout;
//   * O += P V (M = 128, N = head_dim, K = BN keys) into TMEM columns past the S buffers: V
//     is an MN-major operand (row-major [keys, head_dim] tiles, as a GEMM's B);
//   * epilogue: the warps' partial results merged in slice order (O = sum w_q O_q, l = sum
//     w_q l_q, w_q = 2^(m_q - m)), O / l rounded to the dtype.
// The row sum l adds the fp32 exponentials.  Three more warps feed them, meeting on
// mbarriers only: one loads Q and the K ring, one the V ring (each stage refilled as soon as
// its consumer MMAs complete), one issues the MMAs -- S_{j+1} as soon as its K tile has
// landed and its TMEM buffer's last P V has completed, then P V_j once the eight softmax
// warps have written P_j.  Back-to-back tcgen05.mma instructions of M = 128, K = 16 run at
// 64 cycles for N = 128 (the tensor pipe's full rate), so a 128 x 128 bf16 tile's 24 MMAs
// need ~0.8 us; the softmax warps (~1.4 us per tile, most of it the 16 K hardware ex2 at 16
// per clock per SM) set the pace.  Every wait is bounded (status word on expiry) and made
// CTA-uniform; before TMEM is released every MMA and bulk copy this CTA issued has completed.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <mutex>
#include <type_traits>

#include "rk_device.cuh"
#include "rk_internal.h"
#include "rk_tma.h"

namespace rk {
namespace sdpa {

constexpr int BM = 128;  // query rows per CTA
// Two softmax warps per TMEM lane quarter (64 score columns per thread at 128-key tiles):
// measured 2-5 % faster than four (32 columns each) on every benchmark shape -- half the
// cross-warp exchange, and each thread's per-tile bookkeeping spread over twice the scores.
constexpr int SOFTMAX_WARPS = 8;
constexpr int NSL = SOFTMAX_WARPS / 4;  // warps (column slices) per TMEM lane quarter
static_assert(NSL == 2 || NSL == 4, "softmax warps");
// + an MMA-issue warp, a K (and Q) load warp and a V load warp, meeting on mbarriers only.
constexpr int MMA_WARP = SOFTMAX_WARPS, K_WARP = SOFTMAX_WARPS + 1, V_WARP = SOFTMAX_WARPS + 2;
constexpr int THREADS = 32 * (SOFTMAX_WARPS + 3);
constexpr int UMMA_K = 16;

// SPLIT (bf16): P is stored as P_hi + P_lo, both bf16 (P_hi: P with its low 16 bits
// cleared; P_lo: the rest, rounded), and O += P_hi V + P_lo V, so the probabilities keep ~16
// significant bits instead of bf16's 8.  Rounding P alone measured 4.5e-3 of the output's
// maximum on near-uniform attention, and 4.45e-3 on two of the reference fixtures even with
// the row sum taken over the rounded values; the gate is 4e-3.  fp16 P keeps 11 bits and is
// used as is.
template <typename T, int D>
struct Cfg {
  static constexpr bool SPLIT = std::is_same<T, __nv_bfloat16>::value;
  static constexpr int BN = D == 256 ? 64 : 128;      // keys per tile (shared-memory budget)
  static constexpr int CHUNKS = D / 64;              // 64-element (128-byte) column chunks
  static constexpr int Q_BYTES = CHUNKS * BM * 128;  // Q tile: CHUNKS x [128 rows x 128 B]
  static constexpr int K_BYTES = CHUNKS * BN * 128;  // K tile: same layout, BN keys
  static constexpr int V_BYTES = BN * D * 2;         // V tile: [BN/64 key blocks][CHUNKS][64 x 128 B]
  // 128-key tiles: P overwrites S in TMEM and P V reads it from there (no shared-memory
  // P, no proxy fence, and the softmax does not wait for the previous P V).  64-key tiles
  // (head_dim 256) keep P in shared memory in the K-major swizzled layout.
  static constexpr bool P_TMEM = BN == 128;
  static constexpr int P_BYTES = P_TMEM ? 0 : BM * BN * 2;  // P: BN/64 key chunks x [128 rows x 128 B]
  // SPLIT_O (128-key tiles): each column slice (warp) of a lane quarter keeps its own O
  // accumulator in TMEM and its own running maximum and sum over its keys, and the slices
  // are combined once, in the epilogue (as split-K partitions are merged).  The warps of a
  // quarter then never wait for each other inside the key loop (no per-tile exchange of the
  // row maximum); the P V MMAs are the same, each K step adding into its slice's O.
  // head_dim 256 (no TMEM for a second O) exchanges the maximum every tile.
  static constexpr bool SPLIT_O = P_TMEM;
  static constexpr int N_O = SPLIT_O ? NSL : 1;  // O accumulators
  // S / P buffers in TMEM: tile t uses buffer t % NBUF, so S_{t+1} needs P V_{t+1-NBUF}
  // done; K_t's stage is free once S_{t-KSTAGES} has completed, V_t's once P V_{t-VSTAGES}
  // has.  Three buffers where TMEM holds them next to the O accumulators (head_dim 64),
  // else two.
  static constexpr int NBUF = P_TMEM && 3 * BN + N_O * D <= 512 ? 3 : 2;
  static constexpr int KSTAGES = P_TMEM ? 3 : 2;
  static constexpr int VSTAGES = 2;
  // The per-row maximum and sum: 128-key tiles exchange them once, in the epilogue, in
  // shared memory; head_dim 256 (no shared memory to spare) every tile, in TMEM columns
  // past O.
  static constexpr bool X_SMEM = P_TMEM;
  static constexpr int X_BYTES = X_SMEM ? 2 * NSL * BM * 4 : 0;  // [max, sum][slice][row] floats
  static constexpr int TMEM_COLS = 512;
  static constexpr int SMEM = 1024 + Q_BYTES + KSTAGES * K_BYTES + VSTAGES * V_BYTES +
                              (SPLIT ? 2 : 1) * P_BYTES + X_BYTES + 256;
  static_assert(D == 64 || D == 128 || D == 256, "head_dim");
  static_assert(SMEM <= 232448, "shared memory per CTA");
};

struct __align__(8) Bars {
  uint64_t q_full;
  uint64_t k_full[3];
  uint64_t k_empty[3];  // MMA commit: the score MMAs no longer read the stage's K tile
  uint64_t v_full[3];
  uint64_t v_empty[3];  // MMA commit: P V no longer reads the stage's V tile
  uint64_t s_done[3];   // S_t complete (barrier t % NBUF)
  uint64_t pv_done[3];  // P V_t complete (barrier t % NBUF)
  uint64_t p_full[2];   // one arrival per softmax warp: P_t written (barrier t & 1)
  uint64_t drain;
  uint32_t tmem_base;
  int abort;  // set when a wait gave up; every later wait returns at once
};

struct Params {
  int seq;          // S (query and key length)
  int hq, hkv;      // heads
  int group;        // hq / hkv
  int q_tiles;      // ceil(S / BM)
  int causal;
  float scale_log2;  // scale * log2(e)
};

// Named barrier of the NSL softmax warps that share TMEM lane quarter q (ids 1..4).
__device__ __forceinline__ void quarter_sync(int q) {
  asm volatile("bar.sync %0, %1;" ::"r"(q + 1), "n"(32 * NSL) : "memory");
}

template <typename T, int D>
__global__ void __launch_bounds__(THREADS, 1)
    sdpa_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                const __grid_constant__ CUtensorMap tmap_v, T* __restrict__ out, Params p,
                KernelCtl ctl) {
  using C = Cfg<T, D>;
  constexpr int KSTAGES = C::KSTAGES, VSTAGES = C::VSTAGES, NBUF = C::NBUF;
  constexpr int BN = C::BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sq = smem;
  uint8_t* sk = sq + C::Q_BYTES;
  uint8_t* sv_s = sk + KSTAGES * C::K_BYTES;
  uint8_t* sp = sv_s + VSTAGES * C::V_BYTES;  // shared-memory P (64-key tiles only)
  uint8_t* sp_lo = sp + C::P_BYTES;           // SPLIT only
  float* xch = reinterpret_cast<float*>(sp + (C::SPLIT ? 2 : 1) * C::P_BYTES);  // X_SMEM only
  Bars* bars = reinterpret_cast<Bars*>(reinterpret_cast<uint8_t*>(xch) + C::X_BYTES);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Softmax warps: four share each 32-row TMEM lane quarter, each a quarter of the columns.
  const int quarter = warp & 3, slice = warp >> 2;
  constexpr int SLICE = BN / NSL;  // score columns per thread
  constexpr int OSL = D / NSL;     // output columns per thread
  // Heavier (later, under the causal mask) query tiles first.
  const int qtile = p.q_tiles - 1 - static_cast<int>(blockIdx.x);
  const int head = blockIdx.y, batch = blockIdx.z;
  const int kv_head = head / p.group;
  const int q_mat = batch * p.hq + head;      // matrix index in the [B*Hq, S, D] stack
  const int kv_mat = batch * p.hkv + kv_head;  // and in the [B*Hkv, S, D] stacks
  const int k_tiles_all = (p.seq + BN - 1) / BN;
  // Causal: the key tiles up to this query tile's last row.
  const int n_tiles = p.causal ? min(k_tiles_all, (qtile + 1) * (BM / BN)) : k_tiles_all;
  const int row = quarter * 32 + lane;  // TMEM lane and query row within the tile
  const int q_pos = qtile * BM + row;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bars->q_full), 1);
    for (int s = 0; s < KSTAGES; ++s) {
      mbar_init(smem_u32(&bars->k_full[s]), 1);
      mbar_init(smem_u32(&bars->k_empty[s]), 1);
    }
    for (int s = 0; s < VSTAGES; ++s) {
      mbar_init(smem_u32(&bars->v_full[s]), 1);
      mbar_init(smem_u32(&bars->v_empty[s]), 1);
    }
    for (int s = 0; s < NBUF; ++s) {
      mbar_init(smem_u32(&bars->s_done[s]), 1);
      mbar_init(smem_u32(&bars->pv_done[s]), 1);
    }
    for (int s = 0; s < 2; ++s) mbar_init(smem_u32(&bars->p_full[s]), SOFTMAX_WARPS);
    mbar_init(smem_u32(&bars->drain), 1);
    bars->abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmap_q);
    tma_prefetch_desc(&tmap_k);
    tma_prefetch_desc(&tmap_v);
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&bars->tmem_base), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  // TMEM columns: S / P buffers [b BN, (b + 1) BN) for b < NBUF, O accumulator o at
  // [O_COL + o D, O_COL + (o + 1) D), and with the exchange in TMEM, slots [X_COL, X_COL +
  // 12): row maxima by tile parity (2 x 4) and the row-sum shares (4).
  constexpr int O_COL = NBUF * BN, X_COL = O_COL + C::N_O * D;
  static_assert(X_COL + (C::X_SMEM ? 0 : 12) <= C::TMEM_COLS, "TMEM column plan");
  const uint32_t t_lane = tmem + (static_cast<uint32_t>(quarter * 32) << 16);  // this warp's lanes
  const uint32_t t_o = t_lane + O_COL;
  const uint32_t t_x = t_lane + X_COL;
  pdl_begin();  // global memory is touched only after this

  constexpr uint32_t IDESC_S =
      umma_idesc_f16(std::is_same<T, __nv_bfloat16>::value, BM, BN, false, false);
  constexpr uint32_t IDESC_O =
      umma_idesc_f16(std::is_same<T, __nv_bfloat16>::value, BM, D, false, true);
  int never = 0;
  volatile int* abort = &bars->abort;
  // A wait that gives up records why and sets the abort flag; every later wait returns at
  // once and no more work is issued, so every thread still reaches every barrier, and the
  // output is not written.
  auto fail = [&](uint32_t code) {
    *abort = 1;
    atomicOr(ctl.status, code);
  };
  // Completion of S_t / P V_t: barrier t % NBUF, its (t / NBUF)-th phase.  Every wait below
  // is for a tile whose barrier's next completion cannot happen before the wait returns.
  auto wait_s = [&](int t, volatile int* ab) {
    return mbar_wait_bounded(smem_u32(&bars->s_done[t % NBUF]), (t / NBUF) & 1, ctl.timeout_ns, ab);
  };
  auto wait_pv = [&](int t, volatile int* ab) {
    return mbar_wait_bounded(smem_u32(&bars->pv_done[t % NBUF]), (t / NBUF) & 1, ctl.timeout_ns, ab);
  };

  if (warp == K_WARP || warp == V_WARP) {
    if (lane == 0) {
      // ------------------------------------------------------------ loads
      // K (and Q) through one warp, V through another, each ring refilled as soon as its
      // consumer MMAs have completed: a K stage after S_{t-KSTAGES}, a V stage after
      // P V_{t-VSTAGES}.
      const bool is_k = warp == K_WARP;
      const int stages = is_k ? KSTAGES : VSTAGES;
      uint64_t* full = is_k ? bars->k_full : bars->v_full;
      uint64_t* empty = is_k ? bars->k_empty : bars->v_empty;
      uint32_t issued[3] = {0, 0, 0};
      if (is_k) {
        const uint32_t bar = smem_u32(&bars->q_full);
        mbar_arrive_expect_tx(bar, C::Q_BYTES);
#pragma unroll
        for (int c = 0; c < C::CHUNKS; ++c)
          tma_load_3d(smem_u32(sq + c * BM * 128), &tmap_q, bar, c * 64, qtile * BM, q_mat);
      }
      for (int t = 0; t < n_tiles; ++t) {
        const int st = t % stages;
        if (t >= stages &&
            !mbar_wait_bounded(smem_u32(&empty[st]), ((t / stages) - 1) & 1, ctl.timeout_ns, abort)) {
          fail(RK_DEV_ERR_TIMEOUT_PRODUCER);
          break;
        }
        const uint32_t bar = smem_u32(&full[st]);
        if (is_k) {
          mbar_arrive_expect_tx(bar, C::K_BYTES);
#pragma unroll
          for (int c = 0; c < C::CHUNKS; ++c)
            tma_load_3d(smem_u32(sk + st * C::K_BYTES + c * BN * 128), &tmap_k, bar, c * 64, t * BN, kv_mat);
        } else {
          mbar_arrive_expect_tx(bar, C::V_BYTES);
#pragma unroll
          for (int kb = 0; kb < BN / 64; ++kb)
#pragma unroll
            for (int c = 0; c < C::CHUNKS; ++c)
              tma_load_3d(smem_u32(sv_s + st * C::V_BYTES + (kb * C::CHUNKS + c) * 8192), &tmap_v, bar,
                          c * 64, t * BN + kb * 64, kv_mat);
        }
        ++issued[st];
      }
      // No bulk copy may still be landing when the CTA exits: wait for the last load of each
      // stage (earlier ones completed before the stage was refilled) and for Q.
      for (int st = 0; st < stages; ++st)
        if (issued[st] > 0 &&
            !mbar_wait_bounded(smem_u32(&full[st]), (issued[st] - 1) & 1u, ctl.timeout_ns, &never))
          atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_DRAIN);
      if (is_k && !mbar_wait_bounded(smem_u32(&bars->q_full), 0, ctl.timeout_ns, &never))
        atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_DRAIN);
    }
  } else if (warp == MMA_WARP) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issue
      int issued_mma = 0;
      // S_t = Q K_t^T into S buffer t % NBUF.
      auto issue_s = [&](int t) -> bool {
        const int st = t % KSTAGES;
        if ((t == 0 && !mbar_wait_bounded(smem_u32(&bars->q_full), 0, ctl.timeout_ns, abort)) ||
            !mbar_wait_bounded(smem_u32(&bars->k_full[st]), (t / KSTAGES) & 1, ctl.timeout_ns, abort)) {
          fail(RK_DEV_ERR_TIMEOUT_PRODUCER);
          return false;
        }
        tc_fence_after();
        const uint64_t dq = umma_desc_sw128(smem_u32(sq), 16, 1024);
        const uint64_t dk = umma_desc_sw128(smem_u32(sk + st * C::K_BYTES), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < D / UMMA_K; ++kk) {
          const uint32_t off_q = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          const uint32_t off_k = (kk >> 2) * (BN * 128) + (kk & 3) * 32;
          tc_mma_f16(tmem + (t % NBUF) * BN, umma_desc_advance(dq, off_q), umma_desc_advance(dk, off_k),
                     IDESC_S, kk > 0 ? 1u : 0u);
        }
        tc_commit(smem_u32(&bars->s_done[t % NBUF]));
        tc_commit(smem_u32(&bars->k_empty[st]));
        ++issued_mma;
        return true;
      };
      // O += P_t V_t.  128-key tiles: P_t read from TMEM where the softmax warps wrote it over
      // S_t, each slice within its own SLICE score columns (P_hi in the first SLICE/2, P_lo in
      // the next SLICE/2), each K step adding into its slice's O.
      auto issue_pv = [&](int t) -> bool {
        const int st = t % VSTAGES;
        if (!mbar_wait_bounded(smem_u32(&bars->v_full[st]), (t / VSTAGES) & 1, ctl.timeout_ns, abort)) {
          fail(RK_DEV_ERR_TIMEOUT_PRODUCER);
          return false;
        }
        tc_fence_after();
        const uint32_t t_p = tmem + (t % NBUF) * BN;
        const uint64_t dv = umma_desc_sw128(smem_u32(sv_s + st * C::V_BYTES), 8192, 1024);
        const uint64_t dp = umma_desc_sw128(smem_u32(sp), 16, 1024);
        const uint64_t dplo = umma_desc_sw128(smem_u32(sp_lo), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < BN / UMMA_K; ++kk) {
          const uint64_t b = umma_desc_advance(dv, (kk >> 2) * (C::CHUNKS * 8192) + (kk & 3) * 2048);
          if constexpr (C::P_TMEM) {
            constexpr int STEPS = SLICE / UMMA_K;  // K steps per slice
            const int sl = kk / STEPS, u = kk % STEPS;
            const uint32_t o = tmem + O_COL + sl * D, a = t_p + sl * SLICE + u * (UMMA_K / 2);
            const uint32_t acc = (t > 0 || u > 0) ? 1u : 0u;
            tc_mma_f16_ts(o, a, b, IDESC_O, acc);
            if (C::SPLIT) tc_mma_f16_ts(o, a + SLICE / 2, b, IDESC_O, 1u);
          } else {
            const uint32_t acc = (t > 0 || kk > 0) ? 1u : 0u;
            const uint32_t a_off = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
            tc_mma_f16(tmem + O_COL, umma_desc_advance(dp, a_off), b, IDESC_O, acc);
            if (C::SPLIT) tc_mma_f16(tmem + O_COL, umma_desc_advance(dplo, a_off), b, IDESC_O, 1u);
          }
        }
        tc_commit(smem_u32(&bars->pv_done[t % NBUF]));
        tc_commit(smem_u32(&bars->v_empty[st]));
        ++issued_mma;
        return true;
      };
      bool ok = issue_s(0);
      for (int j = 0; j < n_tiles && ok && !*abort; ++j) {
        // S_{j+1} into buffer (j+1) % NBUF once P V_{j+1-NBUF}, the last reader of that
        // buffer's P, has completed (the softmax warps read S before writing P over it).
        if (j + 1 < n_tiles) {
          if (j + 1 >= NBUF && !wait_pv(j + 1 - NBUF, abort)) {
            fail(RK_DEV_ERR_TIMEOUT_MMA);
            break;
          }
          if (!issue_s(j + 1)) break;
        }
        // P_j from all eight softmax warps, then O += P_j V_j.
        if (!mbar_wait_bounded(smem_u32(&bars->p_full[j & 1]), (j >> 1) & 1, ctl.timeout_ns, abort)) {
          fail(RK_DEV_ERR_TIMEOUT_PRODUCER);
          break;
        }
        if (!issue_pv(j)) break;
      }
      // ---- drain: every MMA this CTA issued completes before TMEM is released.
      if (issued_mma > 0) {
        tc_commit(smem_u32(&bars->drain));
        if (!mbar_wait_bounded(smem_u32(&bars->drain), 0, ctl.timeout_ns, &never))
          atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_DRAIN);
      }
    }
  } else {
    // -------------------------------------------------------------- softmax
    // Row state: the maximum the exponentials are taken against (SPLIT_O: of this warp's
    // keys; otherwise of the row, identical in the warps that share it) and this warp's share
    // of the row sum.
    float m_use = -INFINITY, l_part = 0.f;
    const int key_limit = p.causal ? min(p.seq, q_pos + 1) : p.seq;  // keys this row attends
    for (int j = 0; j < n_tiles; ++j) {
      if (!wait_s(j, abort)) fail(RK_DEV_ERR_TIMEOUT_MMA);
      tc_fence_after();
      const uint32_t t_s = t_lane + (j % NBUF) * BN;
      const int valid = key_limit - (j * BN + slice * SLICE);  // keys i < valid are attended
      // Raw scores (the scale is applied with the maximum below); masked keys are -inf.  A
      // warp whose rows all attend every key of its slice skips the mask.
      float sv[SLICE];
      {
        uint32_t r[SLICE];
#pragma unroll
        for (int c = 0; c < SLICE / 16; ++c)
          tmem_ld_32x32b_x16(t_s + slice * SLICE + c * 16, *reinterpret_cast<uint32_t(*)[16]>(r + c * 16));
        tmem_ld_wait();
        if (__all_sync(0xffffffffu, valid >= SLICE)) {
#pragma unroll
          for (int i = 0; i < SLICE; ++i) sv[i] = __uint_as_float(r[i]);
        } else {
#pragma unroll
          for (int i = 0; i < SLICE; ++i) sv[i] = i < valid ? __uint_as_float(r[i]) : -INFINITY;
        }
      }
      float mx;
      {
        // Four independent chains of three-input maxima (about half the instructions of a
        // two-input tree; the maximum is exact in any order).
        float a4[4] = {sv[0], sv[1], sv[2], sv[3]};
#pragma unroll
        for (int i = 4; i < SLICE; i += 2) a4[(i / 2) % 4] = fmax3(a4[(i / 2) % 4], sv[i], sv[i + 1]);
        mx = fmax3(fmaxf(a4[0], a4[1]), a4[2], a4[3]);
      }
      // SPLIT_O: this slice's own maximum.  Otherwise the row maximum over the warps of the
      // lane quarter, through TMEM slots of this tile's parity (a warp writes tile j+2's slots
      // only after the barrier of tile j+1, which its peers reach after reading tile j's).
      float m_raw;
      if constexpr (C::SPLIT_O) {
        m_raw = mx;
      } else {
        const uint32_t xs = t_x + (j & 1) * 4;
        tmem_st_32x32b_x1(xs + slice, __float_as_uint(mx));
        tmem_st_wait();
        tc_fence_before();
        quarter_sync(quarter);
        tc_fence_after();
        uint32_t r[4];
        tmem_ld_32x32b_x4(xs, r);
        tmem_ld_wait();
        m_raw = __uint_as_float(r[0]);  // only the NSL slots written this tile
#pragma unroll
        for (int q = 1; q < NSL; ++q) m_raw = fmaxf(m_raw, __uint_as_float(r[q]));
      }
      // The scale is positive, so the maximum of the scaled scores is the scaled maximum.
      const float m_tile = m_raw * p.scale_log2;
      // Lazy rescaling: the exponentials keep the old maximum until the row maximum
      // exceeds it by more than 2^8 (P <= 256, exact enough in fp16 and in bf16 hi + lo).
      float alpha = 1.f;
      if (m_tile > m_use + 8.f) {
        alpha = ex2_approx(m_use - m_tile);  // 0 for the first keys of the row
        m_use = m_tile;
      }
      const float m_sub = m_use == -INFINITY ? 0.f : m_use;

      // P = 2^(s scale - m) (one FMA, hardware ex2), packed two keys per 32-bit word.  bf16:
      // P_hi = P with the low 16 bits cleared (exact), P_lo = P - P_hi rounded to bf16, so
      // P_hi + P_lo keeps ~16 significant bits; fp16: P rounded once.  The row sum adds the
      // fp32 values.
      // Packed fp32 pairs (fma.rn.f32x2, add.rn.f32x2) for the scale and the sums: the loop
      // is issue-bound, and each lane rounds as the scalar operation would.
      uint32_t hi[SLICE / 2], lo[SLICE / 2];
      float e[SLICE];
      const float2 sc2 = make_float2(p.scale_log2, p.scale_log2), nm2 = make_float2(-m_sub, -m_sub);
#pragma unroll
      for (int i = 0; i < SLICE; i += 2) {
        const float2 x = ffma2(make_float2(sv[i], sv[i + 1]), sc2, nm2);
        e[i] = ex2_approx(x.x);
        e[i + 1] = ex2_approx(x.y);
      }
#pragma unroll
      for (int i = 0; i < SLICE; i += 2) {
        if constexpr (C::SPLIT) {
          const uint32_t b0 = __float_as_uint(e[i]), b1 = __float_as_uint(e[i + 1]);
          hi[i / 2] = __byte_perm(b0, b1, 0x7632);
          const float2 r = fadd2(make_float2(e[i], e[i + 1]), make_float2(-__uint_as_float(b0 & 0xFFFF0000u),
                                                                          -__uint_as_float(b1 & 0xFFFF0000u)));
          lo[i / 2] = Pack2<T>::from_floats(r.x, r.y);
        } else {
          hi[i / 2] = Pack2<T>::from_floats(e[i], e[i + 1]);
        }
      }
      float psum;
      {
        float2 t[SLICE / 4];
#pragma unroll
        for (int i = 0; i < SLICE / 4; ++i)
          t[i] = fadd2(make_float2(e[2 * i], e[2 * i + 1]), make_float2(e[2 * i + SLICE / 2], e[2 * i + 1 + SLICE / 2]));
#pragma unroll
        for (int w = SLICE / 8; w >= 1; w >>= 1)
#pragma unroll
          for (int i = 0; i < w; ++i) t[i] = fadd2(t[i], t[i + w]);
        psum = t[0].x + t[0].y;
      }
      l_part = l_part * alpha + psum;

      // O is rescaled (rarely, with lazy rescaling) once P V_{j-1} has completed; with P in
      // TMEM nothing else here waits for the previous tile's P V (a shared-memory P buffer
      // is free only once P V_{j-1} has read it).
      const bool rescale = j > 0 && __any_sync(0xffffffffu, alpha != 1.f);
      if (j > 0 && (rescale || !C::P_TMEM)) {
        if (!wait_pv(j - 1, abort)) fail(RK_DEV_ERR_TIMEOUT_MMA);
        tc_fence_after();
      }
      if (rescale) {
        // SPLIT_O: this slice's whole O; otherwise its OSL columns of the shared O.
        constexpr int RCOLS = C::SPLIT_O ? D : OSL;
        const uint32_t t_r = t_o + slice * RCOLS;
#pragma unroll
        for (int c = 0; c < RCOLS / 16; ++c) {
          uint32_t r[16];
          tmem_ld_32x32b_x16(t_r + c * 16, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          tmem_st_32x32b_x16(t_r + c * 16, r);
        }
      }
      if constexpr (C::P_TMEM) {
        // P_j over S_j in TMEM, within this warp's own score columns [slice * SLICE, +
        // SLICE), all read above: keys k, k + 1 packed in column slice * SLICE + k / 2 (P_hi),
        // P_lo SLICE / 2 columns further.  No other warp reads or writes these columns.
        static_assert(SLICE == 32 || SLICE == 64, "score columns per thread");
        if constexpr (SLICE == 32) {
          tmem_st_32x32b_x16(t_s + slice * SLICE, hi);
          if (C::SPLIT) tmem_st_32x32b_x16(t_s + slice * SLICE + SLICE / 2, lo);
        } else {
          tmem_st_32x32b_x32(t_s + slice * SLICE, hi);
          if (C::SPLIT) tmem_st_32x32b_x32(t_s + slice * SLICE + SLICE / 2, lo);
        }
      } else {
        // This thread's keys: 64-key chunk kf / 64, 16-byte units (kf % 64) / 8 onwards,
        // swizzled by row.
        const int kf = slice * SLICE;
        const int chunk_off = (kf >> 6) * (BM * 128) + row * 128;
#pragma unroll
        for (int u = 0; u < SLICE / 8; ++u) {
          const int unit_off = chunk_off + (((((kf & 63) >> 3) + u) ^ (row & 7)) << 4);
          *reinterpret_cast<uint4*>(sp + unit_off) =
              make_uint4(hi[4 * u], hi[4 * u + 1], hi[4 * u + 2], hi[4 * u + 3]);
          if (C::SPLIT)
            *reinterpret_cast<uint4*>(sp_lo + unit_off) =
                make_uint4(lo[4 * u], lo[4 * u + 1], lo[4 * u + 2], lo[4 * u + 3]);
        }
        fence_proxy_async_smem();
      }
      tmem_st_wait();
      // P_j (and O's rescaling) of this warp is in place: one arrival per warp.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars->p_full[j & 1]));
    }

    // ---- epilogue: O / l  (SPLIT_O: O = sum_q w_q O_q and l = sum_q w_q l_q over the
    // slices q in order, w_q = 2^(m_q - m) with m the row maximum; otherwise l = the warps'
    // shares added in slice order)
    if (!wait_pv(n_tiles - 1, abort)) fail(RK_DEV_ERR_TIMEOUT_EPILOGUE);
    tc_fence_after();
    float l;
    float w[C::N_O];
    if constexpr (C::X_SMEM) {
      // Shared-memory slots [max | sum][slice][row], written only here.
      xch[slice * BM + row] = m_use;
      xch[(NSL + slice) * BM + row] = l_part;
      quarter_sync(quarter);
      float m = xch[row];
#pragma unroll
      for (int q = 1; q < NSL; ++q) m = fmaxf(m, xch[q * BM + row]);
      l = 0.f;
#pragma unroll
      for (int q = 0; q < NSL; ++q) {
        const float mq = xch[q * BM + row];
        w[q] = mq == -INFINITY ? 0.f : ex2_approx(mq - m);  // a slice with no attended key adds 0
        l += w[q] * xch[(NSL + q) * BM + row];
      }
    } else {
      tmem_st_32x32b_x1(t_x + 8 + slice, __float_as_uint(l_part));
      tmem_st_wait();
      tc_fence_before();
      quarter_sync(quarter);
      tc_fence_after();
      uint32_t lr[4];
      tmem_ld_32x32b_x4(t_x + 8, lr);
      tmem_ld_wait();
      l = __uint_as_float(lr[0]);
#pragma unroll
      for (int q = 1; q < NSL; ++q) l += __uint_as_float(lr[q]);
      w[0] = 1.f;
    }
    const float inv = l > 0.f ? 1.0f / l : 0.f;
    const bool store = q_pos < p.seq && !*abort;
    T* orow = out + (static_cast<size_t>(q_mat) * p.seq + q_pos) * D + slice * OSL;
    // Two 16-column chunks per TMEM round trip (their loads issued together, one wait).
    constexpr int CPW = OSL / 16 >= 2 ? 2 : 1;
#pragma unroll
    for (int c0 = 0; c0 < OSL / 16; c0 += CPW) {
      uint32_t r[CPW][16];
      uint32_t r2[C::SPLIT_O ? CPW * (NSL - 1) : 1][16];
#pragma unroll
      for (int u = 0; u < CPW; ++u) {
        tmem_ld_32x32b_x16(t_o + slice * OSL + (c0 + u) * 16, r[u]);
        if constexpr (C::SPLIT_O) {
#pragma unroll
          for (int q = 1; q < NSL; ++q)
            tmem_ld_32x32b_x16(t_o + q * D + slice * OSL + (c0 + u) * 16, r2[u * (NSL - 1) + q - 1]);
        }
      }
      tmem_ld_wait();
#pragma unroll
      for (int u = 0; u < CPW; ++u) {
        if constexpr (C::SPLIT_O) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float v = w[0] * __uint_as_float(r[u][i]);
#pragma unroll
            for (int q = 1; q < NSL; ++q) v = fmaf(w[q], __uint_as_float(r2[u * (NSL - 1) + q - 1][i]), v);
            r[u][i] = __float_as_uint(v);
          }
        }
        if (store) {
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            uint4 v;
            v.x = Pack2<T>::from_floats(__uint_as_float(r[u][8 * q + 0]) * inv, __uint_as_float(r[u][8 * q + 1]) * inv);
            v.y = Pack2<T>::from_floats(__uint_as_float(r[u][8 * q + 2]) * inv, __uint_as_float(r[u][8 * q + 3]) * inv);
            v.z = Pack2<T>::from_floats(__uint_as_float(r[u][8 * q + 4]) * inv, __uint_as_float(r[u][8 * q + 5]) * inv);
            v.w = Pack2<T>::from_floats(__uint_as_float(r[u][8 * q + 6]) * inv, __uint_as_float(r[u][8 * q + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + (c0 + u) * 16 + 8 * q) = v;
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

}  // namespace sdpa

namespace {
template <typename T, int D>
rk_status launch_sdpa(const void* q, const void* k, const void* v, void* out, int64_t B,
                      int64_t Hq, int64_t Hkv, int64_t S, bool causal, float scale, rk_dtype dt,
                      cudaStream_t s) {
  using C = sdpa::Cfg<T, D>;
  CUtensorMap tq, tk, tv;
  rk_status st = encode_tmap_3d(&tq, q, dt, D, S, B * Hq, 64, sdpa::BM);
  if (st != RK_OK) return st;
  if ((st = encode_tmap_3d(&tk, k, dt, D, S, B * Hkv, 64, C::BN)) != RK_OK) return st;
  if ((st = encode_tmap_3d(&tv, v, dt, D, S, B * Hkv, 64, 64)) != RK_OK) return st;
  LaunchCtl lc;
  if ((st = launch_ctl(&lc)) != RK_OK) return st;
  KernelCtl ctl{lc.status, lc.timeout_ns, 0};

  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [&] {
    attr_err[dev & 63] = cudaFuncSetAttribute(sdpa::sdpa_kernel<T, D>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  });
  if (attr_err[dev & 63] != cudaSuccess) return cuda_status(attr_err[dev & 63]);

  sdpa::Params p;
  p.seq = static_cast<int>(S);
  p.hq = static_cast<int>(Hq);
  p.hkv = static_cast<int>(Hkv);
  p.group = static_cast<int>(Hq / Hkv);
  p.q_tiles = static_cast<int>((S + sdpa::BM - 1) / sdpa::BM);
  p.causal = causal ? 1 : 0;
  p.scale_log2 = static_cast<float>(static_cast<double>(scale) * 1.4426950408889634);
  const dim3 grid(static_cast<unsigned>(p.q_tiles), static_cast<unsigned>(Hq),
                  static_cast<unsigned>(B));
  const cudaError_t e = launch_kernel(sdpa::sdpa_kernel<T, D>, grid, dim3(sdpa::THREADS), C::SMEM, s,
                                      0, tq, tk, tv, static_cast<T*>(out), p, ctl);
  note_launch();
  return cuda_status(e);
}

template <typename T>
rk_status launch_sdpa_d(const void* q, const void* k, const void* v, void* out, int64_t B,
                        int64_t Hq, int64_t Hkv, int64_t S, int64_t D, bool causal, float scale,
                        rk_dtype dt, cudaStream_t s) {
  switch (D) {
    case 64: return launch_sdpa<T, 64>(q, k, v, out, B, Hq, Hkv, S, causal, scale, dt, s);
    case 128: return launch_sdpa<T, 128>(q, k, v, out, B, Hq, Hkv, S, causal, scale, dt, s);
    case 256: return launch_sdpa<T, 256>(q, k, v, out, B, Hq, Hkv, S, causal, scale, dt, s);
  }
  return RK_ERR_UNSUPPORTED;
}
}  // namespace

rk_status sdpa_launch(const void* q, const void* k, const void* v, void* out, int64_t B,
                      int64_t Hq, int64_t Hkv, int64_t S, int64_t D, bool causal, float scale,
                      rk_dtype dt, cudaStream_t s) {
  if (device_cc_major() != 10) return RK_ERR_UNSUPPORTED;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out)) return RK_ERR_UNSUPPORTED;
  // TMA coordinates and the kernel's matrix and row indices are 32-bit.
  if (S + 2 * sdpa::BM > (1ll << 31) || B * Hq > (1ll << 31)) return RK_ERR_UNSUPPORTED;
  if (Hq > 65535 || B > 65535) return RK_ERR_UNSUPPORTED;
  if (dt == RK_DTYPE_BF16)
    return launch_sdpa_d<__nv_bfloat16>(q, k, v, out, B, Hq, Hkv, S, D, causal, scale, dt, s);
  return launch_sdpa_d<__half>(q, k, v, out, B, Hq, Hkv, S, D, causal, scale, dt, s);
}

}  // namespace rk
