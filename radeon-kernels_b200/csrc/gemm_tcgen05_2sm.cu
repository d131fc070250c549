// gemm_tcgen05_2sm.cu -- tcgen05 GEMM on SM pairs (cta_group::2), 256 x 256 tiles.
//
//   C[M,N] = A[M,K] @ B[K,N], fp16/bf16 in, fp32 accumulation, RN output.
//
// A cluster of 2 CTAs on one TPC computes a 256 x 256 output tile with single
// tcgen05.mma.cta_group::2 instructions (M = 256, N = 256, K = 16) issued by the even
// CTA.  Each CTA stages only its half of the operands -- A rows [128*rank, +128) and
// B columns [128*rank, +128) -- so per SM the shared-memory operand traffic per FLOP is
// 2/3 of the 1-SM 128 x 256 tile (32 KiB instead of 48 KiB per 64-deep K block), and
// each CTA's TMEM receives its 128 rows of the 256-column accumulator.
//   * warp 0 (both CTAs): TMA producer, 6-stage ring of {A 128x64, B 64x128};
//     both CTAs' bulk copies complete on the even CTA's full barrier, which the even
//     CTA arms with the bytes of both halves (no multicast anywhere);
//   * warp 1: TMEM allocation for the pair (512 columns each: two accumulators);
//     on the even CTA one thread issues the MMAs and commits with CTA mask 0b11 so
//     ring slots and accumulators are released/published in both CTAs;
//   * warps 2..5 (both CTAs): epilogue from each CTA's own TMEM; each warp reports
//     "accumulator drained" to the even CTA's barrier (remote arrive for the odd CTA).
// Persistent: clusters walk 256x256 tiles in the grouped order; edges handled by TMA
// zero fill + predicated stores, as in the 1-SM kernel.  Operand layouts as in the 1-SM
// kernel: A_MN = A stored [K, M] (each CTA stages its 128 rows as two M-major 64 x 64
// boxes), B_K = B stored [N, K] (each CTA stages its 128 columns as one K-major box).  Every wait is bounded; the
// two cluster barriers (after initialisation and before exit) are reached by every
// thread unconditionally.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>
#include <type_traits>

#include "rk_device.cuh"
#include "rk_internal.h"
#include "rk_peer.cuh"
#include "rk_tma.h"

namespace rk {
namespace tc2 {

constexpr int BM = 256;       // tile rows per pair (128 per CTA)
constexpr int BN = 256;       // tile columns per pair (128 of B per CTA)
constexpr int HALF = 128;
constexpr int BK = 64;
constexpr int UMMA_K = 16;
constexpr int A_STAGE = HALF * BK * 2;  // 16 KiB
constexpr int B_BOX = 64 * BK * 2;      // 8 KiB
constexpr int B_STAGE = BK * HALF * 2;  // 16 KiB
constexpr int STAGE_BYTES = A_STAGE + B_STAGE;
constexpr int STAGES = 6;
constexpr int THREADS = 192;
constexpr int TMEM_COLS = 2 * BN;
constexpr int GROUP_M = 8;  // in 256-row blocks

struct __align__(8) Bars {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + int(sizeof(Bars));
// PEERS form: a 32-row x 64-column staging tile per epilogue warp after the barriers.
constexpr int PEER_STAGE_OFFSET = STAGES * STAGE_BYTES + 1024;
constexpr int PEER_STAGE_WARP = 32 * 128;
constexpr int SMEM_BYTES_PEERS = 1024 + PEER_STAGE_OFFSET + 4 * PEER_STAGE_WARP;
static_assert(int(sizeof(Bars)) <= 1024, "barriers fit before the staging tiles");
static_assert(SMEM_BYTES_PEERS <= 227 * 1024, "shared memory per CTA");

__device__ __forceinline__ void st_shared_v4(uint32_t addr, const uint4& v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// First tile that is split into two 128-column halves: the last partial wave, when it
// occupies at most half of the pairs (then its 2x as many half units still fit one wave, which
// takes half as long -- 896 tiles on 74 pairs: 12 waves + 8 tiles, the 13th wave 24 -> 12 us).
inline int64_t tail_split_from(int64_t tiles, int64_t pairs) {
  const int64_t left = pairs > 0 ? tiles % pairs : 0;
  return (tiles > pairs && left > 0 && 2 * left <= pairs) ? tiles - left : tiles;
}

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& mb, int& nb) {
  const int per_group = GROUP_M * num_n;
  const int group = t / per_group;
  const int first_m = group * GROUP_M;
  const int gsize = min(num_m - first_m, GROUP_M);
  const int in_group = t - group * per_group;
  mb = first_m + in_group % gsize;
  nb = in_group / gsize;
}

// Work units of a launch: tiles [0, split_from) whole, every later tile as two 256 x 128
// halves (half = 0, 1; -1 for a whole tile).  The host splits the last partial wave this way
// when it fills at most half the SM pairs, so that wave takes half as long.
__device__ __forceinline__ void unit_coords(int u, int split_from, int num_m, int num_n, int& mb,
                                            int& nb, int& half) {
  int t = u;
  half = -1;
  if (u >= split_from) {
    t = split_from + ((u - split_from) >> 1);
    half = (u - split_from) & 1;
  }
  tile_coords(t, num_m, num_n, mb, nb);
}

// SWIGLU: B is [K, 2N] = [gate | up]; a tile has 128 output columns, the even CTA
// stages the tile's 128 gate columns and the odd CTA the matching 128 up columns, so
// accumulator columns 0-127 hold gate and 128-255 up for the CTA's rows, and the
// epilogue stores silu(gate) * up (N is the output width).
//
// PEERS: the fused all-gather form (rk_gemm_allgather).  B is this rank's column block
// [K, N] and C is unused: each epilogue warp converts 64 accumulator columns of its 32 rows
// into a swizzled staging tile in shared memory, releases the accumulator after the last
// TMEM read of the tile, and then writes the staged rows -- 8 lanes per 128-byte row
// segment -- into every rank's full output (peer.out[j], row stride peer.ldo) with plain
// 16-byte stores, so each tile crosses NVLink while the next one accumulates.  The first
// peer store waits until every rank has started this call; the exchange then completes as
// rk_peer.cuh describes.
template <typename T, bool SWIGLU = false, bool A_MN = false, bool B_K = false, bool PEERS = false>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmap_a,
                    const __grid_constant__ CUtensorMap tmap_b, T* __restrict__ C, int M, int N,
                    int K, int split_from, KernelCtl ctl, const __grid_constant__ PeerOut<T> peer) {
  static_assert(!(PEERS && (SWIGLU || A_MN || B_K)), "the fused all-gather GEMM takes the nn layout");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + STAGES * A_STAGE;
  Bars* bars = reinterpret_cast<Bars*>(smem + STAGES * STAGE_BYTES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = even CTA (issues the MMAs), 1 = odd
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;
  const int num_m = (M + BM - 1) / BM;
  const int num_n = SWIGLU ? (N + HALF - 1) / HALF : (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  // Half units exist only in the nn, non-SwiGLU forms (their B tile is two 64-column boxes).
  const int split = (SWIGLU || A_MN || B_K) ? num_tiles : min(split_from, num_tiles);
  const int num_units = split + 2 * (num_tiles - split);
  const int num_kb = (K + BK - 1) / BK;
  volatile int* abort_flag = &bars->abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&bars->full[s]), 1);
      mbar_init(smem_u32(&bars->empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&bars->tmem_full[a]), 1);
      mbar_init(smem_u32(&bars->tmem_empty[a]), 2 * 4);  // 4 epilogue warps x 2 CTAs
    }
    mbar_init(smem_u32(&bars->drain), 1);
    bars->abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(&bars->tmem_base), TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  cluster_sync_all();  // both CTAs' barriers exist before either signals the other
  const uint32_t tmem_base = bars->tmem_base;
  pdl_begin();  // global memory is touched only after this
  uint32_t epoch = 0;
  if constexpr (PEERS) {
    epoch = peer_call_epoch(peer);
    if (blockIdx.x == 0 && threadIdx.x == 64) peer_announce(peer, epoch);
  }

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------- producer
      uint32_t stage = 0, phase = 0, issued = 0, issued_parity = 0;
      bool ok = true;
      for (int u = pair; u < num_units && ok; u += num_pairs) {
        int mb, nb, half;
        unit_coords(u, split, num_m, num_n, mb, nb, half);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&bars->empty[stage]), phase ^ 1, ctl.timeout_ns,
                                 abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t full_local = smem_u32(&bars->full[stage]);
          const uint32_t full_even = map_to_rank(full_local, 0);
          if (rank == 0) mbar_arrive_expect_tx(full_local, half < 0 ? 2 * STAGE_BYTES : 2 * (A_STAGE + B_BOX));
          const int arow = mb * BM + static_cast<int>(rank) * HALF;
          if constexpr (A_MN) {
#pragma unroll
            for (int j = 0; j < HALF / 64; ++j)
              tma_load_2d_pair(smem_u32(smem_a + stage * A_STAGE + j * B_BOX), &tmap_a,
                               full_even, arow + j * 64, kb * BK);
          } else {
            tma_load_2d_pair(smem_u32(smem_a + stage * A_STAGE), &tmap_a, full_even, kb * BK,
                             arow);
          }
          const int bcol = SWIGLU ? (rank == 0 ? nb * HALF : N + nb * HALF)
                           : half < 0 ? nb * BN + static_cast<int>(rank) * HALF
                                      : nb * BN + half * HALF + static_cast<int>(rank) * 64;
          if constexpr (B_K) {
            tma_load_2d_pair(smem_u32(smem_b + stage * B_STAGE), &tmap_b, full_even, kb * BK,
                             bcol);
          } else {
            const int boxes = half < 0 ? HALF / 64 : 1;  // a half unit's CTA stages 64 columns
            for (int j = 0; j < boxes; ++j)
              tma_load_2d_pair(smem_u32(smem_b + stage * B_STAGE + j * B_BOX), &tmap_b,
                               full_even, bcol + j * 64, kb * BK);
          }
          issued |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_PRODUCER);
      }
      if (rank == 0) {
        // The even CTA's full barriers count both CTAs' copies: wait for the last phase
        // armed on each stage so no copy into either CTA is left in flight.
        int never = 0;
        for (int s = 0; s < STAGES; ++s)
          if ((issued >> s) & 1u)
            if (!mbar_wait_bounded(smem_u32(&bars->full[s]), (issued_parity >> s) & 1u,
                                   ctl.timeout_ns, &never))
              atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_DRAIN);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ------------------------------------------------ MMA issuer (even CTA only)
      const uint32_t idesc_whole =
          umma_idesc_f16(std::is_same<T, __nv_bfloat16>::value, BM, BN, A_MN, !B_K);
      const uint32_t idesc_half =
          umma_idesc_f16(std::is_same<T, __nv_bfloat16>::value, BM, HALF, A_MN, !B_K);
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      int i = 0;
      for (int u = pair; u < num_units && ok; u += num_pairs, ++i) {
        const uint32_t idesc = u < split ? idesc_whole : idesc_half;
        const uint32_t acc = i & 1, acc_phase = (i >> 1) & 1;
        if (!mbar_wait_cluster_bounded(smem_u32(&bars->tmem_empty[acc]), acc_phase ^ 1,
                                       ctl.timeout_ns, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&bars->full[stage]), phase, ctl.timeout_ns, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem_a + stage * A_STAGE);
          const uint32_t b0 = smem_u32(smem_b + stage * B_STAGE);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            const uint64_t adesc = A_MN ? umma_desc_sw128(a0 + k * UMMA_K * 128, B_BOX, 1024)
                                        : umma_desc_sw128(a0 + k * UMMA_K * 2, 16, 1024);
            const uint64_t bdesc = B_K ? umma_desc_sw128(b0 + k * UMMA_K * 2, 16, 1024)
                                       : umma_desc_sw128(b0 + k * UMMA_K * 128, B_BOX, 1024);
            tc_mma_f16_pair(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          tc_commit_pair(smem_u32(&bars->empty[stage]), 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit_pair(smem_u32(&bars->tmem_full[acc]), 0x3);
      }
      if (!ok) {
        *abort_flag = 1;
        atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_MMA);
      }
      tc_commit_pair(smem_u32(&bars->drain), 0x1);
      int never = 0;
      if (!mbar_wait_bounded(smem_u32(&bars->drain), 0, ctl.timeout_ns, &never))
        atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_DRAIN);
    }
  } else {
    // --------------------------------------------------------------- epilogue
    const int quarter = warp & 3;
    int i = 0;
    bool peers_checked = false;
    for (int u = pair; u < num_units; u += num_pairs, ++i) {
      int mb, nb, half;
      unit_coords(u, split, num_m, num_n, mb, nb, half);
      const int cols = half < 0 ? BN : HALF;           // accumulator columns of this unit
      const int col0 = nb * BN + (half < 0 ? 0 : half * HALF);
      const uint32_t acc = i & 1, acc_phase = (i >> 1) & 1;
      const bool got = mbar_wait_bounded(smem_u32(&bars->tmem_full[acc]), acc_phase,
                                         ctl.timeout_ns, abort_flag);
      if (!__all_sync(0xffffffffu, got)) {
        *abort_flag = 1;
        if (lane == 0) atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_EPILOGUE);
        break;
      }
      tc_fence_after();
      if constexpr (PEERS) {
        if (!peers_checked) {
          int ok = 1;
          if (lane == 0) ok = peer_wait_ready(peer, epoch) ? 1 : 0;
          peers_checked = true;
          if (__shfl_sync(0xffffffffu, ok, 0) == 0) {
            *abort_flag = 1;  // a rank never started: stop every role, store nothing
            break;
          }
        }
        const int row0 = mb * BM + static_cast<int>(rank) * HALF + quarter * 32;
        const uint32_t stage = smem_u32(smem + PEER_STAGE_OFFSET + quarter * PEER_STAGE_WARP);
        const uint32_t tbase =
            tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
        const int unit = lane & 7;
#pragma unroll 1
        for (int c2 = 0; c2 < cols / 64; ++c2) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tbase + (2 * c2 + h) * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 v;
              v.x = Pack2<T>::from_floats(__uint_as_float(r[8 * q + 0]), __uint_as_float(r[8 * q + 1]));
              v.y = Pack2<T>::from_floats(__uint_as_float(r[8 * q + 2]), __uint_as_float(r[8 * q + 3]));
              v.z = Pack2<T>::from_floats(__uint_as_float(r[8 * q + 4]), __uint_as_float(r[8 * q + 5]));
              v.w = Pack2<T>::from_floats(__uint_as_float(r[8 * q + 6]), __uint_as_float(r[8 * q + 7]));
              // Row `lane`, 16-byte unit h*4+q; the unit index is XORed with the row so the
              // eight lanes of each store phase hit eight different bank groups.
              st_shared_v4(stage + lane * 128 + (((h * 4 + q) ^ (lane & 7)) << 4), v);
            }
          }
          if (c2 == cols / 64 - 1) {
            // Last TMEM read of this accumulator: hand it back before the stores.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(map_to_rank(smem_u32(&bars->tmem_empty[acc]), 0));
          } else {
            __syncwarp();
          }
          const int gcol = col0 + c2 * 64 + unit * 8;
#pragma unroll 4
          for (int it = 0; it < 8; ++it) {
            const int rr = (lane >> 3) + 4 * it;  // lanes 8k..8k+7 cover one row's 128 bytes
            const uint4 v = ld_shared_v4(stage + rr * 128 + ((unit ^ (rr & 7)) << 4));
            const int grow = row0 + rr;
            if (grow < M && gcol + 8 <= N) {
              const size_t at = static_cast<size_t>(grow) * peer.ldo + gcol;
              for (int j = 0; j < peer.world; ++j) *reinterpret_cast<uint4*>(peer.out[j] + at) = v;
            }
          }
          __syncwarp();  // the staging tile is rewritten by the next column group
        }
        continue;
      }
      const int row = mb * BM + static_cast<int>(rank) * HALF + quarter * 32 + lane;
      T* crow = C + static_cast<size_t>(row) * N;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < (SWIGLU ? HALF : cols) / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tbase + c * 32, r);
        if (SWIGLU) {
          uint32_t u[32];
          tmem_ld_32x32b_x32(tbase + HALF + c * 32, u);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j)
            r[j] = __float_as_uint(swiglu_f32(__uint_as_float(r[j]), __uint_as_float(u[j])));
        } else {
          tmem_ld_wait();
        }
        const int n0 = (SWIGLU ? nb * HALF : col0) + c * 32;
        if (row < M) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if (n0 + 8 * q + 8 <= N) {
              uint4 v;
              v.x = Pack2<T>::from_floats(__uint_as_float(r[8 * q + 0]), __uint_as_float(r[8 * q + 1]));
              v.y = Pack2<T>::from_floats(__uint_as_float(r[8 * q + 2]), __uint_as_float(r[8 * q + 3]));
              v.z = Pack2<T>::from_floats(__uint_as_float(r[8 * q + 4]), __uint_as_float(r[8 * q + 5]));
              v.w = Pack2<T>::from_floats(__uint_as_float(r[8 * q + 6]), __uint_as_float(r[8 * q + 7]));
              *reinterpret_cast<uint4*>(crow + n0 + 8 * q) = v;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(map_to_rank(smem_u32(&bars->tmem_empty[acc]), 0));
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the even CTA's MMAs read the odd CTA's shared memory until here
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
  if constexpr (PEERS) {
    // The CTA barrier above orders the epilogue warps' peer stores before thread 0's
    // system-scope fence in peer_finish (the grid-synchronisation pattern).
    if (threadIdx.x == 0) peer_finish(peer, epoch, gridDim.x);
  }
}

}  // namespace tc2

namespace {
template <typename T, bool SWIGLU = false, bool A_MN = false, bool B_K = false>
rk_status launch_tc2(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                     rk_dtype dt, cudaStream_t s) {
  static_assert(!(SWIGLU && (A_MN || B_K)), "the fused SwiGLU GEMM takes the nn layout");
  CUtensorMap ta, tb;
  rk_status st = A_MN ? make_tmap_2d(&ta, A, dt, M, K, 64, tc2::BK)
                      : make_tmap_2d(&ta, A, dt, K, M, 64, tc2::HALF);
  if (st != RK_OK) return st;
  st = B_K ? make_tmap_2d(&tb, B, dt, K, N, 64, tc2::HALF)
           : make_tmap_2d(&tb, B, dt, SWIGLU ? 2 * N : N, K, 64, tc2::BK);
  if (st != RK_OK) return st;
  LaunchCtl lc;
  if ((st = launch_ctl(&lc)) != RK_OK) return st;
  KernelCtl ctl{lc.status, lc.timeout_ns, 0};

  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [&] {
    attr_err[dev & 63] = cudaFuncSetAttribute(tc2::gemm_tc2_kernel<T, SWIGLU, A_MN, B_K>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              tc2::SMEM_BYTES);
  });
  if (attr_err[dev & 63] != cudaSuccess) return cuda_status(attr_err[dev & 63]);

  const int64_t tile_n = SWIGLU ? tc2::HALF : tc2::BN;
  const int64_t tiles = ((M + tc2::BM - 1) / tc2::BM) * ((N + tile_n - 1) / tile_n);
  const int64_t pairs_max = device_sm_count() / 2;
  const int64_t pairs = tiles < pairs_max ? tiles : pairs_max;
  const int64_t split_from = (SWIGLU || A_MN || B_K) ? tiles : tc2::tail_split_from(tiles, pairs);

  const cudaError_t e = launch_kernel(tc2::gemm_tc2_kernel<T, SWIGLU, A_MN, B_K>,
                                      dim3(static_cast<unsigned>(2 * pairs)),
                                      dim3(tc2::THREADS), tc2::SMEM_BYTES, s, 2, ta, tb,
                                      reinterpret_cast<T*>(C), static_cast<int>(M),
                                      static_cast<int>(N), static_cast<int>(K),
                                      static_cast<int>(split_from), ctl, PeerOut<T>{});
  note_launch("gemm_tc2_kernel");
  return cuda_status(e);
}

template <typename T>
rk_status launch_tc2_peers(const void* A, const void* B, int64_t M, int64_t N, int64_t K,
                           rk_dtype dt, const PeerTargets& t, cudaStream_t s) {
  CUtensorMap ta, tb;
  rk_status st = make_tmap_2d(&ta, A, dt, K, M, 64, tc2::HALF);
  if (st != RK_OK) return st;
  st = make_tmap_2d(&tb, B, dt, N, K, 64, tc2::BK);
  if (st != RK_OK) return st;
  LaunchCtl lc;
  if ((st = launch_ctl(&lc)) != RK_OK) return st;
  // The roles' waits may include another rank's late start: give them the group's limit.
  KernelCtl ctl{lc.status, lc.timeout_ns > t.timeout_ns ? lc.timeout_ns : t.timeout_ns, 0};
  PeerOut<T> peer{};
  for (int j = 0; j < t.world; ++j) {
    peer.out[j] = static_cast<T*>(t.out[j]);
    peer.ctl[j] = static_cast<PeerCtl*>(t.ctl[j]);
  }
  peer.ldo = t.ldo;
  peer.rank = t.rank;
  peer.world = t.world;
  peer.timeout_ns = t.timeout_ns;
  peer.status = lc.status;

  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [&] {
    attr_err[dev & 63] = cudaFuncSetAttribute(tc2::gemm_tc2_kernel<T, false, false, false, true>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              tc2::SMEM_BYTES_PEERS);
  });
  if (attr_err[dev & 63] != cudaSuccess) return cuda_status(attr_err[dev & 63]);

  const int64_t tiles = ((M + tc2::BM - 1) / tc2::BM) * ((N + tc2::BN - 1) / tc2::BN);
  const int64_t pairs_max = device_sm_count() / 2;
  const int64_t pairs = tiles < pairs_max ? tiles : pairs_max;
  const cudaError_t e = launch_kernel(tc2::gemm_tc2_kernel<T, false, false, false, true>,
                                      dim3(static_cast<unsigned>(2 * pairs)), dim3(tc2::THREADS),
                                      tc2::SMEM_BYTES_PEERS, s, 2, ta, tb, static_cast<T*>(nullptr),
                                      static_cast<int>(M), static_cast<int>(N),
                                      static_cast<int>(K),
                                      static_cast<int>(tc2::tail_split_from(tiles, pairs)), ctl, peer);
  note_launch("gemm_tc2_kernel<PEERS>");
  return cuda_status(e);
}
}  // namespace

rk_status gemm_tc2_allgather_launch(const void* A, const void* B, int64_t M, int64_t N_block,
                                    int64_t K, rk_dtype dt, const PeerTargets& t, cudaStream_t s) {
  if (!gemm_tc_supported(A, B, t.out[t.rank], M, N_block, K, RK_LAYOUT_NN)) return RK_ERR_UNSUPPORTED;
  if (device_sm_count() < 2) return RK_ERR_UNSUPPORTED;
  if (dt == RK_DTYPE_BF16) return launch_tc2_peers<__nv_bfloat16>(A, B, M, N_block, K, dt, t, s);
  return launch_tc2_peers<__half>(A, B, M, N_block, K, dt, t, s);
}

template <typename T>
rk_status launch_tc2_layout(const void* A, const void* B, void* C, int64_t M, int64_t N,
                            int64_t K, rk_layout layout, rk_dtype dt, cudaStream_t s) {
  switch (layout) {
    case RK_LAYOUT_NN: return launch_tc2<T, false, false, false>(A, B, C, M, N, K, dt, s);
    case RK_LAYOUT_NT: return launch_tc2<T, false, false, true>(A, B, C, M, N, K, dt, s);
    case RK_LAYOUT_TN: return launch_tc2<T, false, true, false>(A, B, C, M, N, K, dt, s);
    case RK_LAYOUT_TT: return launch_tc2<T, false, true, true>(A, B, C, M, N, K, dt, s);
  }
  return RK_ERR_INVALID_ARGUMENT;
}

rk_status gemm_tc_2sm_launch(const void* A, const void* B, void* C, int64_t M, int64_t N,
                             int64_t K, rk_layout layout, rk_dtype dt, cudaStream_t s) {
  if (!gemm_tc_supported(A, B, C, M, N, K, layout)) return RK_ERR_UNSUPPORTED;
  if (device_sm_count() < 2) return RK_ERR_UNSUPPORTED;
  if (dt == RK_DTYPE_BF16) return launch_tc2_layout<__nv_bfloat16>(A, B, C, M, N, K, layout, dt, s);
  return launch_tc2_layout<__half>(A, B, C, M, N, K, layout, dt, s);
}

rk_status gemm_swiglu_2sm_launch(const void* A, const void* B, void* C, int64_t M, int64_t N,
                                 int64_t K, rk_dtype dt, cudaStream_t s) {
  if (!gemm_swiglu_supported(A, B, C, M, N, K)) return RK_ERR_UNSUPPORTED;
  if (device_sm_count() < 2) return RK_ERR_UNSUPPORTED;
  if (dt == RK_DTYPE_BF16) return launch_tc2<__nv_bfloat16, true>(A, B, C, M, N, K, dt, s);
  return launch_tc2<__half, true>(A, B, C, M, N, K, dt, s);
}

}  // namespace rk
