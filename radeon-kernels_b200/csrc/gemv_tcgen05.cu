// gemv_tcgen05.cu -- skinny GEMM / multi-row decode GEMV on the 5th-generation tensor
// cores: out[M,N] = x[M,K] @ W[N,K]^T for 1 <= M <= 32.
//
// Why tensor cores here: with CUDA cores every weight element costs M fused
// multiply-adds plus an x operand fetch, so at M >= 4 a CUDA-core kernel is bound by
// FMA issue and L1 traffic long before HBM (measured: 3.8 TB/s at M=4, 0.6 TB/s at
// M=16).  The tensor core does the M-fold reuse for free, leaving the kernel what it
// should be -- a pure HBM stream of W.
//
// Formulation (operands swapped so the tiny M becomes the UMMA N dimension):
//   D[128 rows of W, MN] += W_tile[128, 64] (A, K-major) * x_tile[MN, 64]^T (B, K-major)
// with MN = M rounded up to 16 or 32; x rows >= M are zero-filled by TMA.
//   * warp 0: TMA producer -- a 6- or 8-stage ring of {W 128x64 (16 KiB), x MNx64} boxes,
//     128-byte swizzle, completion on mbarriers;
//   * warp 1: TMEM allocation (32 columns) and one thread issuing tcgen05.mma
//     (M=128, N=MN, K=16), tcgen05.commit releases ring slots;
//   * warps 2..5: epilogue, tcgen05.ld of the 128 x MN fp32 accumulator.
// Split-K over a thread-block cluster of C CTAs (C = 1..8, one cluster per 128-row
// tile, CTA rank r owns K blocks [r*KB/C, (r+1)*KB/C)): the non-leader CTAs hand their
// partial accumulators to the leader, which adds them to its own in rank order, rounds
// once, and stores.  The hand-over is either pulled (a non-leader parks its partial in
// its own idle ring and signals the leader's mbarrier remotely; the leader reads it
// through distributed shared memory, ld.shared::cluster) or, for grids of at most one
// CTA per SM, pushed (non-leaders store straight into a receive area of the leader's
// shared memory, st.shared::cluster, and signal; the leader reads locally and its ring
// is 8 stages deep).  Same additions in the same order either way.
// Deterministic, no global workspace.  Every wait is bounded; the only unbounded
// waits are the two cluster barriers every thread reaches unconditionally (after
// barrier initialisation and before exit, so no CTA leaves while its shared memory
// may still be read).
//
// Role of the reference: the skinny-GEMM half of gemv_wave/packed/lds kernels
// (benchmarks/gemv/native_gemv.hip:30-203), which accept M <= 32 rows of x.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>
#include <type_traits>

#include "rk_device.cuh"
#include "rk_internal.h"
#include "rk_tma.h"

namespace rk {

// Tuning override of the split-K strategy: 0 = automatic, 1/2/4/8 = cluster size,
// -1 = stream-K through the workspace whenever one is supplied.
static std::atomic<int> g_gemv_tc_cluster{0};
// Tuning override of the cluster exchange: 0 = automatic, 1 = pulled, 2 = pushed.
static std::atomic<int> g_gemv_tc_exchange{0};

namespace gtc {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int UMMA_K = 16;
constexpr int W_STAGE = BM * BK * 2;  // 16 KiB
constexpr int THREADS = 192;
constexpr int STAGES = 6;       // ring depth of the pulled exchange (two CTAs per SM)
constexpr int PUSH_STAGES = 8;  // ring depth of the pushed exchange (one CTA per SM)
constexpr int TMEM_COLS = 32;
constexpr int MAX_CLUSTER = 8;
constexpr int PUSH_MAX_CLUSTER = 4;

// Two ways to combine a cluster's partial sums (the sum is the same, in the same order):
//  * pulled -- each non-leader parks its partial in its own idle ring and arrives on the
//    leader's barrier; the leader reads the partials through DSMEM.  No extra shared
//    memory, so two 6-stage CTAs fit an SM.
//  * pushed -- each non-leader stores its partial straight into a receive area of the
//    leader's shared memory (st.shared::cluster) and arrives; the leader reads them
//    locally.  The DSMEM round trips leave the leader's critical path, at the cost of
//    (cluster - 1) partial tiles of shared memory, so one CTA per SM -- which also
//    leaves room for an 8-stage ring.
template <int MN, bool PUSH>
struct Cfg {
  static constexpr int NST = PUSH ? PUSH_STAGES : STAGES;
  static constexpr int X_STAGE = MN * BK * 2;
  static constexpr int STAGE = W_STAGE + X_STAGE;  // multiple of 1024
  static constexpr int RING = NST * STAGE;
  static constexpr int SLOT = BM * MN * 4;  // one fp32 partial tile
  static constexpr int RECV = PUSH ? (PUSH_MAX_CLUSTER - 1) * SLOT : 0;
  static_assert(STAGE % 1024 == 0, "stage bases stay 1024-byte aligned");
  static_assert(SLOT <= RING, "the partial tile is parked in the idle ring");
};

template <int NST>
struct __align__(8) Bars {
  uint64_t full[NST];
  uint64_t empty[NST];
  uint64_t tmem_full;
  uint64_t drain;
  uint64_t partials;  // leader: one remote arrival per non-leader CTA
  uint32_t tmem_base;
  int abort;
};

template <int MN, bool PUSH>
constexpr int smem_bytes() {
  using C = Cfg<MN, PUSH>;
  return 1024 + C::RING + C::RECV + int(sizeof(Bars<C::NST>));
}

__device__ __forceinline__ uint32_t cluster_rank() { return cluster_ctarank(); }

__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void remote_arrive(uint32_t cluster_addr) { mbar_arrive_cluster(cluster_addr); }

__device__ __forceinline__ bool try_wait_cluster(uint32_t bar, uint32_t parity) {
  return mbar_try_wait_cluster(bar, parity);
}

__device__ __forceinline__ void epilogue_bar_sync() {
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

template <int MN>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[MN]);

template <>
__device__ __forceinline__ void tmem_ld_cols<16>(uint32_t taddr, uint32_t (&r)[16]) {
  tmem_ld_32x32b_x16(taddr, r);
}

template <>
__device__ __forceinline__ void tmem_ld_cols<32>(uint32_t taddr, uint32_t (&r)[32]) {
  tmem_ld_32x32b_x32(taddr, r);
}

template <typename T, int MN, bool PUSH>
__global__ void __launch_bounds__(THREADS, PUSH ? 1 : 2)
    gemv_tc_kernel(const __grid_constant__ CUtensorMap tmap_w,
                   const __grid_constant__ CUtensorMap tmap_x, T* __restrict__ out, int M, int N,
                   int K, int csize, KernelCtl ctl) {
  using C = Cfg<MN, PUSH>;
  constexpr int NST = C::NST;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  float* recv = reinterpret_cast<float*>(ring + C::RING);  // pushed exchange only
  auto* bars = reinterpret_cast<Bars<NST>*>(ring + C::RING + C::RECV);
  if (PUSH && csize > PUSH_MAX_CLUSTER) {  // the receive area holds PUSH_MAX_CLUSTER - 1 slots
    if (threadIdx.x == 0) atomicOr(ctl.status, RK_DEV_ERR_BAD_INDEX);
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int tile = blockIdx.x / csize;
  const int num_kb = (K + BK - 1) / BK;
  const int kb0 = static_cast<int>(static_cast<int64_t>(num_kb) * rank / csize);
  const int kb1 = static_cast<int>(static_cast<int64_t>(num_kb) * (rank + 1) / csize);
  volatile int* abort_flag = &bars->abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(smem_u32(&bars->full[s]), 1);
      mbar_init(smem_u32(&bars->empty[s]), 1);
    }
    mbar_init(smem_u32(&bars->tmem_full), 1);
    mbar_init(smem_u32(&bars->drain), 1);
    // Pulled: one arrival per non-leader CTA.  Pushed: one per epilogue thread of each
    // non-leader, each releasing its own stores into the receive area.
    mbar_init(smem_u32(&bars->partials), csize > 1 ? (PUSH ? 128 : 1) * (csize - 1) : 1);
    bars->abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_x);
    // Warm L2 with the weight boxes of this CTA's first ring fill while the previous kernel
    // of the stream drains (before the dependency wait: a prefetch has no result).  Only
    // the weight: x is what the previous kernel typically produces.
    for (int kb = kb0; kb < kb1 && kb < kb0 + NST; ++kb) tma_prefetch_l2_2d(&tmap_w, kb * BK, tile * BM);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&bars->tmem_base), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Announce "barriers initialised" to the cluster without waiting: the matching wait
  // comes right before the first remote access (the partial-sum exchange), so the
  // weight stream starts without a cluster-wide handshake on its critical path.
  cluster_arrive();
  const uint32_t tmem_base = bars->tmem_base;
  pdl_begin();  // global memory is touched only after this

  if (warp == 0) {
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, issued = 0, issued_parity = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait_bounded(smem_u32(&bars->empty[stage]), phase ^ 1, ctl.timeout_ns,
                               abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t full = smem_u32(&bars->full[stage]);
        uint8_t* base = ring + stage * C::STAGE;
        mbar_arrive_expect_tx(full, C::STAGE);
        tma_load_2d(smem_u32(base), &tmap_w, full, kb * BK, tile * BM);
        tma_load_2d(smem_u32(base + W_STAGE), &tmap_x, full, kb * BK, 0);
        issued |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == NST) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_PRODUCER);
      }
      int never = 0;
      for (int s = 0; s < NST; ++s)
        if ((issued >> s) & 1u)
          if (!mbar_wait_bounded(smem_u32(&bars->full[s]), (issued_parity >> s) & 1u,
                                 ctl.timeout_ns, &never))
            atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_DRAIN);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc =
          umma_idesc_f16(std::is_same<T, __nv_bfloat16>::value, BM, MN, false, false);
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait_bounded(smem_u32(&bars->full[stage]), phase, ctl.timeout_ns, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t w0 = smem_u32(ring + stage * C::STAGE);
        const uint32_t x0 = w0 + W_STAGE;
#pragma unroll
        for (int k = 0; k < BK / UMMA_K; ++k) {
          // Both operands K-major with the 128-byte swizzle: 8-row core groups
          // 1024 B apart; K advances 32 B inside the swizzle row.
          const uint64_t adesc = umma_desc_sw128(w0 + k * UMMA_K * 2, 16, 1024);
          const uint64_t bdesc = umma_desc_sw128(x0 + k * UMMA_K * 2, 16, 1024);
          tc_mma_f16(tmem_base, adesc, bdesc, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
        }
        tc_commit(smem_u32(&bars->empty[stage]));
        if (++stage == NST) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (ok) tc_commit(smem_u32(&bars->tmem_full));
      if (!ok) {
        *abort_flag = 1;
        atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_MMA);
      }
      tc_commit(smem_u32(&bars->drain));
      int never = 0;
      if (!mbar_wait_bounded(smem_u32(&bars->drain), 0, ctl.timeout_ns, &never))
        atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_DRAIN);
    }
  } else {
    // ------------------------------------------------------------- epilogue
    const int quarter = warp & 3;
    const int row_local = quarter * 32 + lane;
    const bool got = mbar_wait_bounded(smem_u32(&bars->tmem_full), 0, ctl.timeout_ns, abort_flag);
    const bool ok = __all_sync(0xffffffffu, got);
    float acc[MN];
    if (ok) {
      tc_fence_after();
      uint32_t r[MN];
      tmem_ld_cols<MN>(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16), r);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < MN; ++j) acc[j] = __uint_as_float(r[j]);
    } else {
      *abort_flag = 1;
      if (lane == 0) atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_EPILOGUE);
#pragma unroll
      for (int j = 0; j < MN; ++j) acc[j] = 0.f;
    }
    float* slot = reinterpret_cast<float*>(ring);  // the ring is idle once tmem_full fired
    cluster_wait();  // every CTA of the cluster has initialised its barriers
    if (rank != 0) {
      if constexpr (PUSH) {
        // Into the leader's receive area, slot rank - 1 (zeros if this CTA failed: the
        // leader still gets every slot and the status word carries the error).
        const uint32_t dst = map_to_rank(smem_u32(recv + (rank - 1) * (BM * MN) + row_local * MN), 0);
#pragma unroll
        for (int j = 0; j < MN; j += 4) st_cluster_v4(dst + j * 4, acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
        remote_arrive(map_to_rank(smem_u32(&bars->partials), 0));  // release.cluster: after the stores
      } else {
        if (ok) {
          // The async proxy (TMA, MMA) is done with the ring; order our generic writes after it.
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
#pragma unroll
          for (int j = 0; j < MN; j += 4)
            *reinterpret_cast<float4*>(slot + row_local * MN + j) =
                make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
        }
        epilogue_bar_sync();
        if (warp == 2 && lane == 0) {
          asm volatile("fence.acq_rel.cluster;" ::: "memory");
          remote_arrive(map_to_rank(smem_u32(&bars->partials), 0));
        }
      }
    } else {
      if (csize > 1) {
        bool ready = false;
        if (PUSH || ok) {
          const uint64_t t0 = globaltimer_ns();
          for (uint32_t it = 0;; ++it) {
            if (try_wait_cluster(smem_u32(&bars->partials), 0)) {
              ready = true;
              break;
            }
            if ((it & 63u) == 63u && globaltimer_ns() - t0 > ctl.timeout_ns) break;
          }
        }
        ready = __all_sync(0xffffffffu, ready);
        if (ready) {
          if constexpr (PUSH) {
            const float* mine = recv + row_local * MN;
            for (int c = 1; c < csize; ++c) {
#pragma unroll
              for (int j = 0; j < MN; j += 4) {
                const float4 v = *reinterpret_cast<const float4*>(mine + (c - 1) * (BM * MN) + j);
                acc[j] += v.x;
                acc[j + 1] += v.y;
                acc[j + 2] += v.z;
                acc[j + 3] += v.w;
              }
            }
          } else {
            const uint32_t mine = smem_u32(slot + row_local * MN);
            for (int c = 1; c < csize; ++c) {
              const uint32_t remote = map_to_rank(mine, static_cast<uint32_t>(c));
#pragma unroll
              for (int j = 0; j < MN; j += 4) {
                const float4 v = ld_cluster_v4(remote + j * 4);
                acc[j] += v.x;
                acc[j + 1] += v.y;
                acc[j + 2] += v.z;
                acc[j + 3] += v.w;
              }
            }
          }
        } else if (lane == 0) {
          atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_EPILOGUE);
        }
      }
      const int row = tile * BM + row_local;
      const bool store = ok;
      if (store && row < N) {
#pragma unroll
        for (int m = 0; m < MN; ++m)
          if (m < M) out[static_cast<size_t>(m) * N + row] = from_f32<T>(acc[m]);
      }
    }
  }

  if (warp < 2) {
    __syncwarp();
    cluster_wait();  // pairs with the arrive after initialisation (epilogue warps waited above)
  }
  tc_fence_before();
  __syncthreads();
  // No CTA leaves while another may still touch its shared memory: the leader reading a
  // parked partial (pulled), or a partial still landing in the leader's receive area
  // (pushed: the stores are released before each non-leader's arrival here).
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}


// ---------------------------------------------------------------------------
// Stream-K variant (used when the caller provides a workspace).  Two persistent CTAs
// per SM (one CTA's TMA stream tops out near 25 GB/s, two reach the ~45 GB/s an SM
// can pull); the (128-row tile, 64-deep K block) work units are dealt out as equal
// contiguous ranges, so every SM streams the same number of weight bytes for the
// whole call.  A range
// covers whole tiles (stored directly) plus at most a partial tile at each end; a
// shared tile's partials go to the workspace and the last CTA to finish it (atomic
// ticket) adds them in CTA order and re-zeroes the ticket.  Accumulators are double
// buffered in TMEM so the epilogue of one segment overlaps the MMAs of the next.
template <int MN>
struct Sk {
  static constexpr int X_STAGE = MN * BK * 2;
  static constexpr int STAGE = W_STAGE + X_STAGE;
  static constexpr int STAGES = (108 * 1024) / STAGE;  // 6 for MN = 16, 5 for MN = 32
  static constexpr int RING = STAGES * STAGE;
  // NACC interleaved accumulators per segment: consecutive K=16 MMAs go to different
  // accumulators, so the chain of dependent accumulates is NACC times shorter; the
  // epilogue adds them in a fixed order.
  static constexpr int NACC = 4;
  static constexpr int SET = NACC * MN;           // TMEM columns of one accumulator set
  static constexpr int TMEM = 2 * SET;            // double-buffered sets: 128 or 256 columns
  static_assert(STAGE % 1024 == 0, "stage bases stay 1024-byte aligned");
  static_assert(TMEM <= 512, "TMEM has 512 columns");
};

template <int STAGES_>
struct __align__(8) SkBars {
  uint64_t full[STAGES_];
  uint64_t empty[STAGES_];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int last;
};

template <int MN>
constexpr int sk_smem_bytes() {
  return 1024 + Sk<MN>::RING + int(sizeof(SkBars<Sk<MN>::STAGES>));
}

__device__ __forceinline__ int64_t sk_unit_start(int cta, int64_t units, int grid) {
  return static_cast<int64_t>(cta) * units / grid;
}
// CTA whose range contains unit u: the largest c with floor(c*U/G) <= u.
__device__ __forceinline__ int sk_cta_of(int64_t u, int64_t units, int grid) {
  return static_cast<int>(((u + 1) * grid - 1) / units);
}

template <typename T, int MN>
__global__ void __launch_bounds__(THREADS, 2)
    gemv_tc_sk_kernel(const __grid_constant__ CUtensorMap tmap_w,
                      const __grid_constant__ CUtensorMap tmap_x, T* __restrict__ out, int M, int N,
                      int K, float* __restrict__ part, int* __restrict__ ticket, KernelCtl ctl) {
  using C = Sk<MN>;
  constexpr int STAGES_ = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  auto* bars = reinterpret_cast<SkBars<STAGES_>*>(ring + C::RING);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grid = gridDim.x, cta = blockIdx.x;
  const int num_kb = (K + BK - 1) / BK;
  const int tiles = (N + BM - 1) / BM;
  const int64_t units = static_cast<int64_t>(tiles) * num_kb;
  const int64_t u0 = sk_unit_start(cta, units, grid);
  const int64_t u1 = sk_unit_start(cta + 1, units, grid);
  volatile int* abort_flag = &bars->abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES_; ++s) {
      mbar_init(smem_u32(&bars->full[s]), 1);
      mbar_init(smem_u32(&bars->empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&bars->tmem_full[a]), 1);
      mbar_init(smem_u32(&bars->tmem_empty[a]), 4);  // one arrival per epilogue warp
    }
    mbar_init(smem_u32(&bars->drain), 1);
    bars->abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_x);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&bars->tmem_base), C::TMEM);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;
  pdl_begin();  // global memory is touched only after this

  if (warp == 0) {
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, issued = 0, issued_parity = 0;
      bool ok = true;
      int tile = static_cast<int>(u0 / num_kb), kb = static_cast<int>(u0 % num_kb);
      for (int64_t u = u0; u < u1; ++u, kb = (kb + 1 == num_kb) ? 0 : kb + 1, tile += (kb == 0)) {
        if (!mbar_wait_bounded(smem_u32(&bars->empty[stage]), phase ^ 1, ctl.timeout_ns,
                               abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t full = smem_u32(&bars->full[stage]);
        uint8_t* base = ring + stage * C::STAGE;
        mbar_arrive_expect_tx(full, C::STAGE);
        tma_load_2d(smem_u32(base), &tmap_w, full, kb * BK, tile * BM);
        tma_load_2d(smem_u32(base + W_STAGE), &tmap_x, full, kb * BK, 0);
        issued |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == STAGES_) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_PRODUCER);
      }
      int never = 0;
      for (int s = 0; s < STAGES_; ++s)
        if ((issued >> s) & 1u)
          if (!mbar_wait_bounded(smem_u32(&bars->full[s]), (issued_parity >> s) & 1u,
                                 ctl.timeout_ns, &never))
            atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_DRAIN);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc =
          umma_idesc_f16(std::is_same<T, __nv_bfloat16>::value, BM, MN, false, false);
      uint32_t stage = 0, phase = 0, seg = 0, acc = 0, kk = 0;
      bool ok = true;
      int kb = static_cast<int>(u0 % num_kb);
      for (int64_t u = u0; u < u1 && ok; ++u, kb = (kb + 1 == num_kb) ? 0 : kb + 1) {
        const bool first = (u == u0) || kb == 0;
        if (first) kk = 0;
        const bool last = (u + 1 == u1) || kb + 1 == num_kb;
        if (first) {
          acc = seg & 1;
          if (!mbar_wait_bounded(smem_u32(&bars->tmem_empty[acc]), ((seg >> 1) & 1) ^ 1,
                                 ctl.timeout_ns, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        if (!mbar_wait_bounded(smem_u32(&bars->full[stage]), phase, ctl.timeout_ns, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t w0 = smem_u32(ring + stage * C::STAGE);
        const uint32_t x0 = w0 + W_STAGE;
#pragma unroll
        for (int k = 0; k < BK / UMMA_K; ++k, ++kk) {
          const uint64_t adesc = umma_desc_sw128(w0 + k * UMMA_K * 2, 16, 1024);
          const uint64_t bdesc = umma_desc_sw128(x0 + k * UMMA_K * 2, 16, 1024);
          const uint32_t j = kk % C::NACC;  // the first NACC MMAs of a segment initialise
          tc_mma_f16(tmem_base + acc * C::SET + j * MN, adesc, bdesc, idesc, kk >= C::NACC ? 1u : 0u);
        }
        tc_commit(smem_u32(&bars->empty[stage]));
        if (++stage == STAGES_) {
          stage = 0;
          phase ^= 1;
        }
        if (last) {
          tc_commit(smem_u32(&bars->tmem_full[acc]));
          ++seg;
        }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_MMA);
      }
      tc_commit(smem_u32(&bars->drain));
      int never = 0;
      if (!mbar_wait_bounded(smem_u32(&bars->drain), 0, ctl.timeout_ns, &never))
        atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_DRAIN);
    }
  } else {
    const int quarter = warp & 3;
    const int row_local = quarter * 32 + lane;
    uint32_t seg = 0;
    for (int64_t u = u0; u < u1; ++seg) {
      const int tile = static_cast<int>(u / num_kb);
      const int64_t seg_end = min(u1, static_cast<int64_t>(tile + 1) * num_kb);
      const uint32_t acc = seg & 1;
      const bool got = mbar_wait_bounded(smem_u32(&bars->tmem_full[acc]), (seg >> 1) & 1,
                                         ctl.timeout_ns, abort_flag);
      if (!__all_sync(0xffffffffu, got)) {
        *abort_flag = 1;
        if (lane == 0) atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_EPILOGUE);
        break;
      }
      tc_fence_after();
      float a[MN];
#pragma unroll
      for (int j = 0; j < MN; ++j) a[j] = 0.f;
      // Accumulators written in this segment: min(NACC, MMAs issued) -- the rest hold stale data.
      const int64_t mmas = (seg_end - u) * (BK / UMMA_K);
      const int used = mmas < C::NACC ? static_cast<int>(mmas) : C::NACC;
      for (int q = 0; q < used; ++q) {
        uint32_t r[MN];
        tmem_ld_cols<MN>(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * C::SET + q * MN, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < MN; ++j) a[j] += __uint_as_float(r[j]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars->tmem_empty[acc]));

      const int c_first = sk_cta_of(static_cast<int64_t>(tile) * num_kb, units, grid);
      const int c_last = sk_cta_of(static_cast<int64_t>(tile + 1) * num_kb - 1, units, grid);
      bool store = true;
      if (c_first != c_last) {
        float* mine = part + (static_cast<size_t>(cta) * 2 + (u == u0 ? 0 : 1)) * BM * MN +
                      static_cast<size_t>(row_local) * MN;
#pragma unroll
        for (int j = 0; j < MN; j += 4)
          *reinterpret_cast<float4*>(mine + j) = make_float4(a[j], a[j + 1], a[j + 2], a[j + 3]);
        __threadfence();
        epilogue_bar_sync();
        if (warp == 2 && lane == 0) bars->last = atomicAdd(ticket + tile, 1) == c_last - c_first;
        epilogue_bar_sync();
        store = bars->last != 0;
        if (store) {
          __threadfence();
#pragma unroll
          for (int j = 0; j < MN; ++j) a[j] = 0.f;
          // Partials are loaded PF CTAs at a time (all loads in flight before the adds,
          // so a tile shared by many CTAs costs a few L2 round trips, not one per CTA)
          // and added in CTA order, which keeps the result deterministic.
          constexpr int PF = MN <= 16 ? 4 : 2;
          for (int c0 = c_first; c0 <= c_last; c0 += PF) {
            float4 v[PF][MN / 4];
#pragma unroll
            for (int q = 0; q < PF; ++q) {
              const int c = c0 + q;
              if (c <= c_last) {
                // Slot 0 holds a CTA's first segment; its tile is the one containing its first unit.
                const bool first_seg = sk_unit_start(c, units, grid) >= static_cast<int64_t>(tile) * num_kb;
                const float* src = part + (static_cast<size_t>(c) * 2 + (first_seg ? 0 : 1)) * BM * MN +
                                   static_cast<size_t>(row_local) * MN;
#pragma unroll
                for (int j = 0; j < MN / 4; ++j) v[q][j] = __ldcg(reinterpret_cast<const float4*>(src) + j);
              }
            }
#pragma unroll
            for (int q = 0; q < PF; ++q) {
              if (c0 + q <= c_last) {
#pragma unroll
                for (int j = 0; j < MN / 4; ++j) {
                  a[4 * j] += v[q][j].x;
                  a[4 * j + 1] += v[q][j].y;
                  a[4 * j + 2] += v[q][j].z;
                  a[4 * j + 3] += v[q][j].w;
                }
              }
            }
          }
          if (warp == 2 && lane == 0) ticket[tile] = 0;
        }
      }
      const int row = tile * BM + row_local;
      if (store && row < N) {
#pragma unroll
        for (int m = 0; m < MN; ++m)
          if (m < M) out[static_cast<size_t>(m) * N + row] = from_f32<T>(a[m]);
      }
      u = seg_end;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM);
  }
}

}  // namespace gtc

namespace {

// Stream-K grid: two CTAs per SM, at most one per work unit.
int sk_grid(int64_t M, int64_t N, int64_t K) {
  (void)M;
  const int64_t units = ((N + gtc::BM - 1) / gtc::BM) * ((K + gtc::BK - 1) / gtc::BK);
  int64_t g = 2ll * device_sm_count();
  if (g > 480) g = 480;
  if (g > units) g = units;
  return g < 1 ? 1 : static_cast<int>(g);
}

// Bytes of partial sums one stream-K CTA owns (two slots of a BM x MN fp32 tile).
size_t sk_cta_bytes(int64_t M) {
  const int mn = M <= 16 ? 16 : 32;
  return static_cast<size_t>(2) * gtc::BM * mn * sizeof(float);
}

// Tickets live in the workspace's fixed ticket prefix (kept zero by every strategy).
size_t sk_ticket_bytes(int64_t N) {
  (void)N;
  return RK_GEMV_WORKSPACE_TICKET_BYTES;
}

bool sk_fits(int64_t N) {
  return (N + gtc::BM - 1) / gtc::BM <= static_cast<int64_t>(RK_GEMV_WORKSPACE_TICKET_BYTES / sizeof(int));
}

// Stream-K workspace bytes (ticket counters + two partial slots per CTA).
size_t sk_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  return sk_ticket_bytes(N) + static_cast<size_t>(sk_grid(M, N, K)) * sk_cta_bytes(M);
}

// Stream-K CTAs a workspace of `bytes` holds partial slots for (0: not even one), capped
// at the full grid.  A caller's workspace sized by rk_gemv_workspace_size gets the full
// grid; the fixed array of rk_gemv_fixed_scratch gets as many CTAs as it has room for.
int sk_grid_within(int64_t M, int64_t N, int64_t K, size_t bytes) {
  const size_t tickets = sk_ticket_bytes(N);
  if (bytes <= tickets) return 0;
  const int64_t room = static_cast<int64_t>((bytes - tickets) / sk_cta_bytes(M));
  const int full = sk_grid(M, N, K);
  return room < full ? static_cast<int>(room) : full;
}

// Workspace the automatic strategy can use.  Measured on B200, cluster split-K beats
// stream-K at every weight size (stream-K's workspace fix-up and its per-CTA TMA rate
// cost more than its perfect balance gains), so the automatic strategy uses no
// workspace; stream-K runs when selected explicitly (tuning value -1) or through
// rk_gemv_fixed_scratch.
size_t workspace_bytes_for(int64_t M, int64_t N, int64_t K) {
  return g_gemv_tc_cluster.load() == -1 && sk_fits(N) ? sk_workspace_bytes(M, N, K) : 0;
}

// Clusters of `csize` CTAs of the pushed-exchange kernel that can be resident at once
// (cudaOccupancyMaxActiveClusters; one CTA per SM, clusters confined to a GPC), per device.
// The kernel's shared-memory attribute must be set before the first query.
template <typename T, int MN>
int push_capacity(int dev, int csize) {
  static std::once_flag once[64][2];
  static int capacity[64][2];
  const int slot = csize == 2 ? 0 : 1;
  std::call_once(once[dev & 63][slot], [&] {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(csize) * 64u);
    cfg.blockDim = dim3(gtc::THREADS);
    cfg.dynamicSmemBytes = gtc::smem_bytes<MN, true>();
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = static_cast<unsigned>(csize);
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gtc::gemv_tc_kernel<T, MN, true>, &cfg) != cudaSuccess) {
      (void)cudaGetLastError();
      n = 0;
    }
    capacity[dev & 63][slot] = n;
  });
  return capacity[dev & 63][slot];
}

template <typename T, int MN>
rk_status launch_gemv_tc(const void* x, const void* W, void* out, int64_t M, int64_t N, int64_t K,
                         rk_dtype dt, cudaStream_t s, int csize_override, void* workspace,
                         size_t workspace_bytes, bool stream_k) {
  CUtensorMap tw, tx;
  rk_status st = make_tmap_2d(&tx, x, dt, K, M, 64, MN);
  if (st != RK_OK) return st;
  LaunchCtl lc;
  if ((st = launch_ctl(&lc)) != RK_OK) return st;
  KernelCtl ctl{lc.status, lc.timeout_ns, 0};

  constexpr int smem = gtc::smem_bytes<MN, false>();
  constexpr int smem_push = gtc::smem_bytes<MN, true>();
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [&] {
    cudaError_t e = cudaFuncSetAttribute(gtc::gemv_tc_kernel<T, MN, false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gtc::gemv_tc_kernel<T, MN, true>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, smem_push);
    // All of the SM's unified memory as shared memory: two pulled CTAs per SM.
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gtc::gemv_tc_kernel<T, MN, false>,
                               cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gtc::gemv_tc_kernel<T, MN, true>,
                               cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    attr_err[dev & 63] = e;
  });
  if (attr_err[dev & 63] != cudaSuccess) return cuda_status(attr_err[dev & 63]);

  const int64_t tiles = (N + gtc::BM - 1) / gtc::BM;
  const int64_t num_kb = (K + gtc::BK - 1) / gtc::BK;
  const int sk_ctas = workspace != nullptr ? sk_grid_within(M, N, K, workspace_bytes) : 0;
  // A caller's workspace must hold the full grid's slots (rk_gemv_workspace_size); the fixed
  // array (stream_k) runs with the CTAs it has room for.
  if ((stream_k || csize_override == -1) && sk_fits(N) && sk_ctas >= 1 &&
      (stream_k || sk_ctas == sk_grid(M, N, K))) {
    // Stream-K over all SMs, shared tiles meet in the caller's workspace.
    constexpr int sk_smem = gtc::sk_smem_bytes<MN>();
    static std::once_flag sk_once[64];
    static cudaError_t sk_err[64];
    std::call_once(sk_once[dev & 63], [&] {
      sk_err[dev & 63] = cudaFuncSetAttribute(gtc::gemv_tc_sk_kernel<T, MN>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, sk_smem);
    });
    if (sk_err[dev & 63] != cudaSuccess) return cuda_status(sk_err[dev & 63]);
    if ((st = make_tmap_2d(&tw, W, dt, K, N, 64, gtc::BM)) != RK_OK) return st;
    int* ticket = static_cast<int*>(workspace);
    float* part = reinterpret_cast<float*>(static_cast<char*>(workspace) + sk_ticket_bytes(N));
    const cudaError_t e = launch_kernel(gtc::gemv_tc_sk_kernel<T, MN>, dim3(sk_ctas),
                                        dim3(gtc::THREADS), sk_smem, s, 0, tw, tx,
                                        static_cast<T*>(out), static_cast<int>(M),
                                        static_cast<int>(N), static_cast<int>(K), part, ticket, ctl);
    note_launch("gemv_tc_sk_kernel");
    return cuda_status(e);
  }
  // Split K over a thread-block cluster, reduced through DSMEM.
  int csize = csize_override;
  if (csize <= 0) {
    // Measured on B200: 8-CTA clusters only pay off for very short weights (<= 12 row
    // tiles); otherwise the largest of 1/2/4 keeping the grid within one wave of the pulled
    // CTAs that fit an SM -- two with 16-wide accumulators (109 KiB of shared memory each),
    // one with 32-wide ones (124 KiB): at M = 17..32, N = 8192 clusters of 4 would launch
    // a second wave (36.5 us) where clusters of 2 take 28.5 us.
    static std::once_flag occ_once[64];
    static int occ[64];
    std::call_once(occ_once[dev & 63], [&] {
      // Shared memory is what binds: the SM's over the CTA's plus its reservation.
      int per_sm = 0, reserved = 0;
      cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
      cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev);
      const int n = per_sm / (smem + reserved);
      occ[dev & 63] = n < 1 ? 1 : (n > 2 ? 2 : n);
    });
    const int64_t target = static_cast<int64_t>(occ[dev & 63]) * device_sm_count();
    const int cap = tiles <= 12 ? 8 : 4;
    csize = 1;
    while (csize < cap && tiles * csize * 2 <= target && csize * 2 <= num_kb) csize *= 2;
  }
  if (csize > gtc::MAX_CLUSTER) csize = gtc::MAX_CLUSTER;
  while (csize > 1 && csize > num_kb) csize /= 2;

  // Pushed exchange where every cluster of the grid is resident at once at one CTA per SM
  // and the grid is no narrower than the pulled one: clusters of 2 or 4 (of the largest
  // size that fits, when the size is automatic).  Measured on B200: [4096 x 14336] at
  // M = 4 takes 23.3 us pushed against 24.4 us pulled (clusters of 4 either way), and
  // shortening the row tiles to spread the weight over all 37 resident clusters instead
  // of 32 gains nothing (DRAM, not the SM count, bounds the stream).
  const int mode = g_gemv_tc_exchange.load();
  bool push = false;
  if (mode != 1 && csize > 1) {
    const bool automatic = csize_override <= 0;
    for (int c = automatic ? gtc::PUSH_MAX_CLUSTER : csize; c >= 2 && c >= csize; c /= 2) {
      if (c > gtc::PUSH_MAX_CLUSTER || c > num_kb) continue;
      const int resident = push_capacity<T, MN>(dev, c);
      if (mode == 2 || tiles <= resident) {
        csize = c;
        push = true;
        break;
      }
    }
  }
  if ((st = make_tmap_2d(&tw, W, dt, K, N, 64, gtc::BM)) != RK_OK) return st;
  const unsigned grid = static_cast<unsigned>(tiles * csize);
  cudaError_t e;
  if (push) {
    e = launch_kernel(gtc::gemv_tc_kernel<T, MN, true>, dim3(grid), dim3(gtc::THREADS), smem_push, s,
                      csize, tw, tx, static_cast<T*>(out), static_cast<int>(M), static_cast<int>(N),
                      static_cast<int>(K), csize, ctl);
    note_launch("gemv_tc_kernel<push>");
  } else {
    e = launch_kernel(gtc::gemv_tc_kernel<T, MN, false>, dim3(grid), dim3(gtc::THREADS), smem, s,
                      csize, tw, tx, static_cast<T*>(out), static_cast<int>(M), static_cast<int>(N),
                      static_cast<int>(K), csize, ctl);
    note_launch("gemv_tc_kernel");
  }
  return cuda_status(e);
}

}  // namespace

size_t gemv_tc_workspace_bytes(int64_t M, int64_t N, int64_t K) { return workspace_bytes_for(M, N, K); }
size_t gemv_tc_stream_k_bytes(int64_t M, int64_t N, int64_t K) { return sk_workspace_bytes(M, N, K); }

void gemv_tc_set_cluster(int c) { g_gemv_tc_cluster.store(c); }
void gemv_tc_set_exchange(int mode) { g_gemv_tc_exchange.store(mode == 1 || mode == 2 ? mode : 0); }

bool gemv_tc_supported(const void* x, const void* W, const void* out, int64_t M, int64_t N,
                       int64_t K) {
  (void)out;
  if (device_cc_major() != 10) return false;
  if (M < 1 || M > 32 || N < 1 || K < 8 || K % 8 != 0) return false;
  if (!aligned16(x) || !aligned16(W)) return false;
  if (N > (1ll << 31) - 256 || K > (1ll << 31) - 64) return false;
  return true;
}

rk_status gemv_tc_launch(const void* x, const void* W, void* out, int64_t M, int64_t N, int64_t K,
                         rk_dtype dt, cudaStream_t s, void* workspace, size_t workspace_bytes,
                         bool stream_k) {
  if (!gemv_tc_supported(x, W, out, M, N, K)) return RK_ERR_UNSUPPORTED;
  const int c = g_gemv_tc_cluster.load();
  if (M <= 16) {
    if (dt == RK_DTYPE_BF16)
      return launch_gemv_tc<__nv_bfloat16, 16>(x, W, out, M, N, K, dt, s, c, workspace, workspace_bytes, stream_k);
    return launch_gemv_tc<__half, 16>(x, W, out, M, N, K, dt, s, c, workspace, workspace_bytes, stream_k);
  }
  if (dt == RK_DTYPE_BF16)
    return launch_gemv_tc<__nv_bfloat16, 32>(x, W, out, M, N, K, dt, s, c, workspace, workspace_bytes, stream_k);
  return launch_gemv_tc<__half, 32>(x, W, out, M, N, K, dt, s, c, workspace, workspace_bytes, stream_k);
}

}  // namespace rk

// ---------------------------------------------------------------------------
// rk_gemv_fixed_scratch: the stream-K tensor-core GEMV (the variant that needs split-K
// scratch) with that scratch taken from a fixed array compiled into this library
// instead of from the caller.
//
// Some callers cannot hand the library device memory for scratch: plugins hosted
// by an engine that owns every device allocation and passes a custom op only its
// input and output buffers, and latency-critical serving loops that must not call
// cudaMalloc on the hot path (it can synchronise the device and can fail under
// memory pressure).  For them this entry point uses RK_GEMV_FIXED_SCRATCH_BYTES of
// device memory that every GPU loading the library holds until the process exits.
//
// Host code must not pass `g_gemv_fixed_scratch` itself to a kernel: in host code
// that name is a host-side stand-in, not a device address.  The device address is
// looked up once per device with cudaGetSymbolAddress while that device is current
// (the first call on a device does this), and that address is what the kernel gets.
namespace {

static __device__ __align__(256) unsigned char g_gemv_fixed_scratch[RK_GEMV_FIXED_SCRATCH_BYTES];

// Device address of the array, per device; looked up under the lock until a lookup
// succeeds (a failed lookup -- say inside a stream capture -- is retried next call).
std::mutex g_fixed_scratch_mu;
void* g_fixed_scratch_ptr[64] = {};

rk_status fixed_scratch_address(int dev, void** ptr) {
  std::lock_guard<std::mutex> lock(g_fixed_scratch_mu);
  if (g_fixed_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_gemv_fixed_scratch);
    if (e != cudaSuccess) return rk::cuda_status(e);
    if (p == nullptr) {
      rk::note_error("cudaGetSymbolAddress returned no address for the fixed GEMV scratch");
      return RK_ERR_CUDA;
    }
    g_fixed_scratch_ptr[dev] = p;
  }
  *ptr = g_fixed_scratch_ptr[dev];
  return RK_OK;
}

}  // namespace

extern "C" rk_status rk_gemv_fixed_scratch(const void* x, const void* weight, void* out,
                                           int64_t M, int64_t N, int64_t K, rk_dtype dt,
                                           rk_stream_t stream) {
  using namespace rk;
  if (M < 1 || M > 32 || N < 1 || K < 1 || (dt != RK_DTYPE_FP16 && dt != RK_DTYPE_BF16))
    return RK_ERR_INVALID_ARGUMENT;
  if (x == nullptr || weight == nullptr || out == nullptr) return RK_ERR_INVALID_ARGUMENT;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return RK_ERR_NO_DEVICE;
  if (!gemv_tc_supported(x, weight, out, M, N, K)) return RK_ERR_UNSUPPORTED;
  // One ticket per 128-row tile of the weight lives in the array's ticket prefix.
  if (!sk_fits(N)) return RK_ERR_TOO_LARGE;
  void* scratch = nullptr;
  const rk_status found = fixed_scratch_address(dev, &scratch);
  if (found != RK_OK) return found;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // The array keeps whatever the previous call left; the split-K tickets at its start
  // must be zero when the kernel begins (the partial slots are written before read).
  const size_t used_tickets = ((N + gtc::BM - 1) / gtc::BM * sizeof(int) + 255) / 256 * 256;
  const rk_status st = cuda_status(cudaMemsetAsync(scratch, 0, used_tickets, s));
  if (st != RK_OK) return st;
  return gemv_tc_launch(x, weight, out, M, N, K, dt, s, scratch, RK_GEMV_FIXED_SCRATCH_BYTES, true);
}

// Test hook: fills the whole fixed array of the current device with `byte`, as a
// previous call stopped midway could leave it (non-zero tickets, stale partial sums).
extern "C" rk_status rk_debug_fill_fixed_scratch(int byte, rk_stream_t stream) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return RK_ERR_NO_DEVICE;
  void* scratch = nullptr;
  const rk_status found = fixed_scratch_address(dev, &scratch);
  if (found != RK_OK) return found;
  return rk::cuda_status(cudaMemsetAsync(scratch, byte & 0xff, RK_GEMV_FIXED_SCRATCH_BYTES,
                                         reinterpret_cast<cudaStream_t>(stream)));
}
