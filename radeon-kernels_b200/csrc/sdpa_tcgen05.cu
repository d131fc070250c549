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
// One CTA per (128-row query tile, query head, batch), 512 threads (16 warps), flash-style:
//   * thread 0 issues the TMA loads -- the Q tile once, K and V tiles of BN keys (128; 64
//     for head_dim 256, to fit shared memory) in a ring
//     of STAGES buffers, through 3-D tensor maps over the [batch*heads, S, D] stacks, so rows
//     past the sequence read as zero instead of the next head's -- and the MMAs;
//   * S = Q K^T (M = 128, N = BN keys, K = head_dim) into TMEM columns [0, BN): Q and K
//     are K-major 128-byte-swizzled tiles straight from TMA;
//   * four warps share each 32-row TMEM lane quarter, each thread a quarter of its row's
//     scores: it applies the scale (in base 2) and the masks, the row maximum is combined
//     through four spare TMEM columns in a fixed order, and the online softmax (fp32) rescales the
//     thread's quarter of the O row in TMEM only when the maximum grew by more than 2^8
//     (lazy rescaling); P = 2^(s - m) (hardware ex2) goes to shared memory in the K-major
//     swizzled layout the next MMA reads: rounded to fp16, or for bf16 as two bf16 terms
//     P_hi + P_lo (see Cfg::SPLIT).  (One warp per lane quarter, 128 scores per thread,
//     spent about 9 us per key tile on the dependent softmax chain.);
//   * O += P V (M = 128, N = head_dim, K = BN keys) into TMEM columns [128, 128 + D): V is
//     an MN-major operand (row-major [keys, head_dim] tiles, as a GEMM's B);
//   * epilogue: O / l rounded to the dtype; l is the four warps' shares added in order.
// The row sum l adds the fp32 exponentials.  Two S buffers in TMEM: thread 0 issues S_{j+1}
// as soon as S_j has landed, so the scores of the next tile are computed during this tile's
// softmax, and P V_j overlaps the next tile's exponentials.  Every wait is bounded (status word on
// expiry) and made CTA-uniform; before TMEM is released every MMA and bulk copy this CTA
// issued has completed.
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
constexpr int SOFTMAX_WARPS = 16;
constexpr int THREADS = 32 * (SOFTMAX_WARPS + 1);  // + the producer warp
constexpr int UMMA_K = 16;

// SPLIT (bf16): P is stored as P_hi + P_lo, both bf16, and O += P_hi V + P_lo V, so the
// probabilities keep ~16 significant bits instead of bf16's 8 (rounding P alone moved the
// output by up to 4.5e-3 of its maximum on near-uniform attention); fp16 P keeps 11 bits
// and is used as is.
template <typename T, int D>
struct Cfg {
  static constexpr bool SPLIT = std::is_same<T, __nv_bfloat16>::value;
  static constexpr int BN = D == 256 ? 64 : 128;      // keys per tile (shared-memory budget)
  static constexpr int CHUNKS = D / 64;              // 64-element (128-byte) column chunks
  static constexpr int Q_BYTES = CHUNKS * BM * 128;  // Q tile: CHUNKS x [128 rows x 128 B]
  static constexpr int K_BYTES = CHUNKS * BN * 128;  // K tile: same layout, BN keys
  static constexpr int V_BYTES = BN * D * 2;         // V tile: [BN/64 key blocks][CHUNKS][64 x 128 B]
  static constexpr int P_BYTES = BM * BN * 2;        // P: BN/64 key chunks x [128 rows x 128 B]
  static constexpr int STAGES = 2;
  static constexpr int TMEM_COLS = 512;  // S, O and the row-exchange columns
  static constexpr int SMEM =
      1024 + Q_BYTES + STAGES * (K_BYTES + V_BYTES) + (SPLIT ? 2 : 1) * P_BYTES + 256;
  static_assert(D == 64 || D == 128 || D == 256, "head_dim");
  static_assert(SMEM <= 232448, "shared memory per CTA");
};

struct __align__(8) Bars {
  uint64_t q_full;
  uint64_t k_full[2];
  uint64_t v_full[2];
  uint64_t s_done[2];  // one per S buffer (tile t: buffer t & 1)
  uint64_t o_done;
  uint64_t p_full;  // one arrival per softmax warp: P_t is in shared memory
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

// Named barrier of the four softmax warps that share TMEM lane quarter q (ids 1..4).
__device__ __forceinline__ void quarter_sync(int q) {
  asm volatile("bar.sync %0, 128;" ::"r"(q + 1) : "memory");
}

template <typename T, int D>
__global__ void __launch_bounds__(THREADS, 1)
    sdpa_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                const __grid_constant__ CUtensorMap tmap_v, T* __restrict__ out, Params p,
                KernelCtl ctl) {
  using C = Cfg<T, D>;
  constexpr int STAGES = C::STAGES;
  constexpr int BN = C::BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sq = smem;
  uint8_t* sk = sq + C::Q_BYTES;
  uint8_t* sv_s = sk + STAGES * C::K_BYTES;
  uint8_t* sp = sv_s + STAGES * C::V_BYTES;
  uint8_t* sp_lo = sp + C::P_BYTES;  // SPLIT only
  Bars* bars = reinterpret_cast<Bars*>(sp + (C::SPLIT ? 2 : 1) * C::P_BYTES);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool producer = warp == SOFTMAX_WARPS;  // TMA + MMA issue (one lane)
  // Softmax warps: four share each 32-row TMEM lane quarter, each a quarter of the columns.
  const int quarter = warp & 3, slice = (warp >> 2) & 3;
  constexpr int SLICE = BN / 4;  // score columns per thread
  constexpr int OSL = D / 4;     // output columns per thread
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
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&bars->k_full[s]), 1);
      mbar_init(smem_u32(&bars->v_full[s]), 1);
      mbar_init(smem_u32(&bars->s_done[s]), 1);
    }
    mbar_init(smem_u32(&bars->o_done), 1);
    mbar_init(smem_u32(&bars->p_full), SOFTMAX_WARPS);
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
  // TMEM columns: S buffers [0, BN) and [BN, 2 BN), O [O_COL, O_COL + D), exchange slots
  // [X_COL, X_COL + 12): row maxima by tile parity (2 x 4) and the row-sum shares (4).
  constexpr int O_COL = 2 * BN, X_COL = 384;
  static_assert(O_COL + D <= X_COL, "TMEM column plan");
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

  if (producer) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      // Bulk-copy bookkeeping: loads issued into each stage, and those waited for.
      uint32_t k_issued[2] = {0, 0}, v_issued[2] = {0, 0}, k_used[2] = {0, 0}, v_used[2] = {0, 0};
      bool q_used = false;
      int issued_mma = 0;
      auto load_k = [&](int t) {
        const int st = t % STAGES;
        const uint32_t bar = smem_u32(&bars->k_full[st]);
        mbar_arrive_expect_tx(bar, C::K_BYTES);
#pragma unroll
        for (int c = 0; c < C::CHUNKS; ++c)
          tma_load_3d(smem_u32(sk + st * C::K_BYTES + c * BN * 128), &tmap_k, bar, c * 64, t * BN,
                      kv_mat);
        ++k_issued[st];
      };
      auto load_v = [&](int t) {
        const int st = t % STAGES;
        const uint32_t bar = smem_u32(&bars->v_full[st]);
        mbar_arrive_expect_tx(bar, C::V_BYTES);
#pragma unroll
        for (int kb = 0; kb < BN / 64; ++kb)
#pragma unroll
          for (int c = 0; c < C::CHUNKS; ++c)
            tma_load_3d(smem_u32(sv_s + st * C::V_BYTES + (kb * C::CHUNKS + c) * 8192), &tmap_v, bar,
                        c * 64, t * BN + kb * 64, kv_mat);
        ++v_issued[st];
      };
      // S_t = Q K_t^T into S buffer t & 1.
      auto issue_s = [&](int t) {
        const int st = t % STAGES;
        bool got = true;
        if (t == 0) got = q_used = mbar_wait_bounded(smem_u32(&bars->q_full), 0, ctl.timeout_ns, abort);
        got = got && mbar_wait_bounded(smem_u32(&bars->k_full[st]), k_used[st] & 1u, ctl.timeout_ns, abort);
        if (!got) return fail(RK_DEV_ERR_TIMEOUT_PRODUCER);
        ++k_used[st];
        tc_fence_after();
        const uint64_t dq = umma_desc_sw128(smem_u32(sq), 16, 1024);
        const uint64_t dk = umma_desc_sw128(smem_u32(sk + st * C::K_BYTES), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < D / UMMA_K; ++kk) {
          const uint32_t off_q = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          const uint32_t off_k = (kk >> 2) * (BN * 128) + (kk & 3) * 32;
          tc_mma_f16(tmem + (t & 1) * BN, umma_desc_advance(dq, off_q), umma_desc_advance(dk, off_k),
                     IDESC_S, kk > 0 ? 1u : 0u);
        }
        tc_commit(smem_u32(&bars->s_done[t & 1]));
        ++issued_mma;
      };
      // O += P_t V_t.
      auto issue_pv = [&](int t) {
        const int st = t % STAGES;
        if (!mbar_wait_bounded(smem_u32(&bars->v_full[st]), v_used[st] & 1u, ctl.timeout_ns, abort))
          return fail(RK_DEV_ERR_TIMEOUT_PRODUCER);
        ++v_used[st];
        tc_fence_after();
        const uint64_t dp = umma_desc_sw128(smem_u32(sp), 16, 1024);
        const uint64_t dplo = umma_desc_sw128(smem_u32(sp_lo), 16, 1024);
        const uint64_t dv = umma_desc_sw128(smem_u32(sv_s + st * C::V_BYTES), 8192, 1024);
#pragma unroll
        for (int kk = 0; kk < BN / UMMA_K; ++kk) {
          const uint32_t a_off = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          const uint64_t b = umma_desc_advance(dv, (kk >> 2) * (C::CHUNKS * 8192) + (kk & 3) * 2048);
          tc_mma_f16(tmem + O_COL, umma_desc_advance(dp, a_off), b, IDESC_O, (t > 0 || kk > 0) ? 1u : 0u);
          if (C::SPLIT) tc_mma_f16(tmem + O_COL, umma_desc_advance(dplo, a_off), b, IDESC_O, 1u);
        }
        tc_commit(smem_u32(&bars->o_done));
        ++issued_mma;
      };

      {
        const uint32_t bar = smem_u32(&bars->q_full);
        mbar_arrive_expect_tx(bar, C::Q_BYTES);
#pragma unroll
        for (int c = 0; c < C::CHUNKS; ++c)
          tma_load_3d(smem_u32(sq + c * BM * 128), &tmap_q, bar, c * 64, qtile * BM, q_mat);
      }
      for (int t = 0; t < STAGES && t < n_tiles; ++t) {
        load_k(t);
        load_v(t);
      }
      issue_s(0);
      for (int j = 0; j < n_tiles && !*abort; ++j) {
        // V_{j+1} into the stage of V_{j-1}, once P V_{j-1} has completed.
        if (j >= 1 && j + 1 < n_tiles) {
          if (!mbar_wait_bounded(smem_u32(&bars->o_done), (j - 1) & 1, ctl.timeout_ns, abort)) {
            fail(RK_DEV_ERR_TIMEOUT_MMA);
            break;
          }
          load_v(j + 1);
        }
        // S_{j+1} into the buffer of S_{j-1}: every softmax warp has read it (they wrote
        // P_{j-1}, which P V_{j-1} consumed before this iteration).
        if (j + 1 < n_tiles) issue_s(j + 1);
        // K_{j+2} into the stage of K_j, once S_j has completed.
        if (j + 2 < n_tiles && !*abort) {
          if (!mbar_wait_bounded(smem_u32(&bars->s_done[j & 1]), (j >> 1) & 1, ctl.timeout_ns, abort)) {
            fail(RK_DEV_ERR_TIMEOUT_MMA);
            break;
          }
          load_k(j + 2);
        }
        // P_j from all sixteen softmax warps, then O += P_j V_j.
        if (*abort) break;
        if (!mbar_wait_bounded(smem_u32(&bars->p_full), j & 1, ctl.timeout_ns, abort)) {
          fail(RK_DEV_ERR_TIMEOUT_PRODUCER);
          break;
        }
        issue_pv(j);
      }
      // ---- drain: every MMA and bulk copy issued by this CTA completes before exit.
      if (issued_mma > 0) {
        tc_commit(smem_u32(&bars->drain));
        if (!mbar_wait_bounded(smem_u32(&bars->drain), 0, ctl.timeout_ns, &never))
          atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_DRAIN);
      }
      if (!q_used && !mbar_wait_bounded(smem_u32(&bars->q_full), 0, ctl.timeout_ns, &never))
        atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_DRAIN);
      for (int s = 0; s < STAGES; ++s) {
        // Loads issued but never waited for: wait for the last one of each stage.
        if (k_issued[s] > k_used[s] &&
            !mbar_wait_bounded(smem_u32(&bars->k_full[s]), (k_issued[s] - 1) & 1u, ctl.timeout_ns, &never))
          atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_DRAIN);
        if (v_issued[s] > v_used[s] &&
            !mbar_wait_bounded(smem_u32(&bars->v_full[s]), (v_issued[s] - 1) & 1u, ctl.timeout_ns, &never))
          atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_DRAIN);
      }
    }
  } else {
    // -------------------------------------------------------------- softmax
    // Row state (identical in the four warps that share a row): the maximum the
    // exponentials are taken against, and this warp's share of the row sum.
    float m_use = -INFINITY, l_part = 0.f;
    const int key_limit = p.causal ? min(p.seq, q_pos + 1) : p.seq;  // keys this row attends
    for (int j = 0; j < n_tiles; ++j) {
      if (!mbar_wait_bounded(smem_u32(&bars->s_done[j & 1]), (j >> 1) & 1, ctl.timeout_ns, abort))
        fail(RK_DEV_ERR_TIMEOUT_MMA);
      tc_fence_after();
      const uint32_t t_s = t_lane + (j & 1) * BN;
      const int valid = key_limit - (j * BN + slice * SLICE);  // keys i < valid are attended
      float sv[SLICE];
      float mx = -INFINITY;
      {
        uint32_t r[SLICE];
#pragma unroll
        for (int c = 0; c < SLICE / 16; ++c)
          tmem_ld_32x32b_x16(t_s + slice * SLICE + c * 16, *reinterpret_cast<uint32_t(*)[16]>(r + c * 16));
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < SLICE; ++i) {
          sv[i] = i < valid ? __uint_as_float(r[i]) * p.scale_log2 : -INFINITY;
          mx = fmaxf(mx, sv[i]);
        }
      }
      // Row maximum over the four warps of the lane quarter, through TMEM slots of this
      // tile's parity (a warp writes tile j+2's slots only after the barrier of tile j+1,
      // which its peers reach after reading tile j's).
      const uint32_t xs = t_x + (j & 1) * 4;
      tmem_st_32x32b_x1(xs + slice, __float_as_uint(mx));
      tmem_st_wait();
      tc_fence_before();
      quarter_sync(quarter);
      tc_fence_after();
      float m_tile;
      {
        uint32_t r[4];
        tmem_ld_32x32b_x4(xs, r);
        tmem_ld_wait();
        m_tile = fmaxf(fmaxf(__uint_as_float(r[0]), __uint_as_float(r[1])),
                       fmaxf(__uint_as_float(r[2]), __uint_as_float(r[3])));
      }
      // Lazy rescaling: the exponentials keep the old maximum until the row maximum
      // exceeds it by more than 2^8 (P <= 256, exact enough in fp16 and in bf16 hi + lo).
      float alpha = 1.f;
      if (m_tile > m_use + 8.f) {
        alpha = ex2_approx(m_use - m_tile);  // 0 for the first keys of the row
        m_use = m_tile;
      }
      const float m_sub = m_use == -INFINITY ? 0.f : m_use;

      // P = 2^(s - m), rounded (SPLIT: hi + lo), in registers until P V_{j-1} is done.  The
      // row sum adds the fp32 values (within 2^-16 of hi + lo; fp16 P within 2^-11).
      float psum = 0.f;
      uint32_t hi[SLICE / 2], lo[SLICE / 2];
#pragma unroll
      for (int i = 0; i < SLICE; i += 2) {
        const float e0 = ex2_approx(sv[i] - m_sub), e1 = ex2_approx(sv[i + 1] - m_sub);
        psum += e0 + e1;
        hi[i / 2] = Pack2<T>::from_floats(e0, e1);
        if (C::SPLIT) {
          const float2 h2 = Pack2<T>::to_floats(hi[i / 2]);
          lo[i / 2] = Pack2<T>::from_floats(e0 - h2.x, e1 - h2.y);
        }
      }
      l_part = l_part * alpha + psum;

      if (j > 0) {
        if (!mbar_wait_bounded(smem_u32(&bars->o_done), (j - 1) & 1, ctl.timeout_ns, abort))
          fail(RK_DEV_ERR_TIMEOUT_MMA);
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
          for (int c = 0; c < OSL / 16; ++c) {
            uint32_t r[16];
            tmem_ld_32x32b_x16(t_o + slice * OSL + c * 16, r);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st_32x32b_x16(t_o + slice * OSL + c * 16, r);
          }
          tmem_st_wait();
        }
      }
      {
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
      }
      // P_j (and O's rescaling) of this warp is in place: one arrival per warp.
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars->p_full));
    }

    // ---- epilogue: O / l  (l = the four warps' shares, added in slice order)
    if (!mbar_wait_bounded(smem_u32(&bars->o_done), (n_tiles - 1) & 1, ctl.timeout_ns, abort))
      fail(RK_DEV_ERR_TIMEOUT_EPILOGUE);
    tc_fence_after();
    tmem_st_32x32b_x1(t_x + 8 + slice, __float_as_uint(l_part));
    tmem_st_wait();
    tc_fence_before();
    quarter_sync(quarter);
    tc_fence_after();
    uint32_t lr[4];
    tmem_ld_32x32b_x4(t_x + 8, lr);
    tmem_ld_wait();
    const float l = ((__uint_as_float(lr[0]) + __uint_as_float(lr[1])) + __uint_as_float(lr[2])) +
                    __uint_as_float(lr[3]);
    const float inv = l > 0.f ? 1.0f / l : 0.f;
    const bool store = q_pos < p.seq && !*abort;
    T* orow = out + (static_cast<size_t>(q_mat) * p.seq + q_pos) * D + slice * OSL;
#pragma unroll
    for (int c = 0; c < OSL / 16; ++c) {
      uint32_t r[16];
      tmem_ld_32x32b_x16(t_o + slice * OSL + c * 16, r);
      tmem_ld_wait();
      if (store) {
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          uint4 v;
          v.x = Pack2<T>::from_floats(__uint_as_float(r[8 * q + 0]) * inv, __uint_as_float(r[8 * q + 1]) * inv);
          v.y = Pack2<T>::from_floats(__uint_as_float(r[8 * q + 2]) * inv, __uint_as_float(r[8 * q + 3]) * inv);
          v.z = Pack2<T>::from_floats(__uint_as_float(r[8 * q + 4]) * inv, __uint_as_float(r[8 * q + 5]) * inv);
          v.w = Pack2<T>::from_floats(__uint_as_float(r[8 * q + 6]) * inv, __uint_as_float(r[8 * q + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + c * 16 + 8 * q) = v;
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
