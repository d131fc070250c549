// gemm_tcgen05.cu -- persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   C[M,N] = A[M,K] @ B[K,N], fp16/bf16 in, fp32 accumulate in TMEM, output
//   rounded to nearest-even in the operand dtype.
//
// One CTA per SM walks output tiles of 128 x 256 (grouped raster for L2 reuse):
//   warp 0      TMA producer: A tile 128x64 (K-major, 128B swizzle) and the
//               B tile 64x256 as four 64x64 boxes (N-major, 128B swizzle)
//               into a 4-stage shared-memory ring, completion on mbarriers;
//   warp 1      allocates 512 TMEM columns (two 128x256 fp32 accumulators)
//               and one elected thread issues tcgen05.mma (M=128, N=256, K=16)
//               with A K-major and B MN-major straight from the swizzled
//               tiles (no transpose pass), tcgen05.commit frees ring slots and
//               publishes finished accumulators;
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns, fp32 -> 16-bit
//               cast, 16-byte stores; runs on accumulator i while the MMA
//               warp fills accumulator i^1.
// Edges need no special code: TMA zero-fills out-of-range rows/columns and
// the epilogue predicates stores on M and on 8-column groups of N.
// Requirements: N % 8 == 0, K % 8 == 0, 16-byte aligned A, B, C (TMA row
// strides are multiples of 16 bytes).
//
// Operand layouts (the reference's Layout enum, src/radeon_kernels/ops/gemm/spec.py:12-15):
// A_MN = A stored transposed, [K, M] row-major ("tn"); B_K = B stored transposed,
// [N, K] row-major ("nt").  Neither needs a transpose pass: an M-major A tile is two
// 64 x 64 boxes laid out like the N-major B chunks (the UMMA descriptor's MN-major
// form), and a K-major B tile is one 64 x BN box laid out like the K-major A tile;
// the instruction descriptor's major bits tell the tensor core which is which.
// A stored [K, M] adds M % 8 == 0 (its row stride is M elements).
//
// Role of the reference: replaces wmma_gemm_kernel
// (src/radeon_kernels/ops/gemm/native/wmma_gemm.hip:20-193), which stages
// A and a transposed B panel in LDS and runs rocWMMA 16x16x16 fragments.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>
#include <type_traits>

#include "rk_device.cuh"
#include "rk_internal.h"
#include "rk_tma.h"

namespace rk {
namespace tc1 {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 x 16-bit = 128 bytes = one swizzle row
constexpr int UMMA_K = 16;
constexpr int A_STAGE = BM * BK * 2;  // 16 KiB
constexpr int B_BOX = 64 * BK * 2;    // 8 KiB: 64 N-columns x 64 K-rows
constexpr int THREADS = 192;
constexpr int GROUP_M = 8;
constexpr int RING_BYTES = 192 * 1024;  // shared-memory ring shared by all tile widths

// Per tile width BN (64, 128 or 256): ring depth and TMEM footprint.
template <int BN>
struct Tile {
  static constexpr int B_STAGE = BK * BN * 2;
  static constexpr int STAGE_BYTES = A_STAGE + B_STAGE;
  static constexpr int STAGES = RING_BYTES / STAGE_BYTES;  // 4, 6 or 8
  static constexpr int TMEM_COLS = 2 * BN;                 // two fp32 accumulators
  static_assert(BN == 64 || BN == 128 || BN == 256, "tile width");
};

template <int STAGES>
struct __align__(8) Barriers {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint64_t stall;  // test hook: nothing ever arrives here
  uint32_t tmem_base;
  int abort;
};

template <int BN>
constexpr int smem_bytes() {
  return 1024 /*alignment slack*/ + Tile<BN>::STAGES * Tile<BN>::STAGE_BYTES +
         int(sizeof(Barriers<Tile<BN>::STAGES>));
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

// SWIGLU (BN = 256 only): B is [K, 2N] = [gate | up]; a tile has 128 output columns,
// B chunks 0-1 come from the gate columns and 2-3 from the matching up columns, and the
// epilogue stores silu(gate) * up (N is the output width).
template <typename T, int BN, bool SWIGLU = false, bool A_MN = false, bool B_K = false>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc1_kernel(const __grid_constant__ CUtensorMap tmap_a,
                    const __grid_constant__ CUtensorMap tmap_b, T* __restrict__ C, int M, int N,
                    int K, KernelCtl ctl) {
  constexpr int STAGES = Tile<BN>::STAGES;
  constexpr int B_STAGE = Tile<BN>::B_STAGE;
  constexpr int STAGE_BYTES = Tile<BN>::STAGE_BYTES;
  constexpr int TMEM_COLS = Tile<BN>::TMEM_COLS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + STAGES * A_STAGE;
  auto* bars = reinterpret_cast<Barriers<STAGES>*>(smem + STAGES * STAGE_BYTES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM;
  static_assert(!SWIGLU || BN == 256, "the fused SwiGLU epilogue pairs 128 gate and 128 up columns");
  const int num_n = SWIGLU ? (N + 127) / 128 : (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + BK - 1) / BK;
  volatile int* abort_flag = &bars->abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&bars->full[s]), 1);
      mbar_init(smem_u32(&bars->empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&bars->tmem_full[a]), 1);
      mbar_init(smem_u32(&bars->tmem_empty[a]), 4 * 32);
    }
    mbar_init(smem_u32(&bars->drain), 1);
    mbar_init(smem_u32(&bars->stall), 1);
    bars->abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&bars->tmem_base), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;
  pdl_begin();  // global memory is touched only after this

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      uint32_t stage = 0, phase = 0;
      uint32_t issued = 0, issued_parity = 0;  // per-stage bits, for the drain below
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, num_m, num_n, mb, nb);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&bars->empty[stage]), phase ^ 1, ctl.timeout_ns,
                                 abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t full = smem_u32(&bars->full[stage]);
          mbar_arrive_expect_tx(full, STAGE_BYTES);
          if constexpr (A_MN) {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j)
              tma_load_2d(smem_u32(smem_a + stage * A_STAGE + j * B_BOX), &tmap_a, full,
                          mb * BM + j * 64, kb * BK);
          } else {
            tma_load_2d(smem_u32(smem_a + stage * A_STAGE), &tmap_a, full, kb * BK, mb * BM);
          }
          if constexpr (B_K) {
            tma_load_2d(smem_u32(smem_b + stage * B_STAGE), &tmap_b, full, kb * BK, nb * BN);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) {
              const int bcol = SWIGLU ? (j < 2 ? nb * 128 + j * 64 : N + nb * 128 + (j - 2) * 64)
                                      : nb * BN + j * 64;
              tma_load_2d(smem_u32(smem_b + stage * B_STAGE + j * B_BOX), &tmap_b, full, bcol,
                          kb * BK);
            }
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
      // Never leave while a bulk copy into this CTA's shared memory is in flight.
      int never = 0;
      for (int s = 0; s < STAGES; ++s)
        if ((issued >> s) & 1u)
          if (!mbar_wait_bounded(smem_u32(&bars->full[s]), (issued_parity >> s) & 1u,
                                 ctl.timeout_ns, &never))
            atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_DRAIN);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc_bf16 = umma_idesc_f16(true, BM, BN, A_MN, !B_K);
      constexpr uint32_t idesc_f16 = umma_idesc_f16(false, BM, BN, A_MN, !B_K);
      const uint32_t idesc = std::is_same<T, __nv_bfloat16>::value ? idesc_bf16 : idesc_f16;
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      if (ctl.inject_stall) {
        ok = mbar_wait_bounded(smem_u32(&bars->stall), 0, ctl.timeout_ns, abort_flag);
      }
      int i = 0;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++i) {
        const uint32_t acc = i & 1, acc_phase = (i >> 1) & 1;
        if (!mbar_wait_bounded(smem_u32(&bars->tmem_empty[acc]), acc_phase ^ 1, ctl.timeout_ns,
                               abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&bars->full[stage]), phase, ctl.timeout_ns,
                                 abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem_a + stage * A_STAGE);
          const uint32_t b0 = smem_u32(smem_b + stage * B_STAGE);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            // K-major SW128 (A, or B stored [N, K]): 8-row core groups 1024 B apart;
            // K advances 32 B inside the swizzle row.  MN-major SW128 (B, or A stored
            // [K, M]): 64-column chunks 8 KiB apart (LBO), 8-row K groups 1024 B
            // apart (SBO); K advances by two groups (16 rows) per MMA.
            const uint64_t adesc = A_MN ? umma_desc_sw128(a0 + k * UMMA_K * 128, B_BOX, 1024)
                                        : umma_desc_sw128(a0 + k * UMMA_K * 2, 16, 1024);
            const uint64_t bdesc = B_K ? umma_desc_sw128(b0 + k * UMMA_K * 2, 16, 1024)
                                       : umma_desc_sw128(b0 + k * UMMA_K * 128, B_BOX, 1024);
            tc_mma_f16(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          tc_commit(smem_u32(&bars->empty[stage]));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(smem_u32(&bars->tmem_full[acc]));
      }
      if (!ok) {
        *abort_flag = 1;
        atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_MMA);
      }
      // Every MMA this thread issued must finish before TMEM is released.
      tc_commit(smem_u32(&bars->drain));
      int never = 0;
      if (!mbar_wait_bounded(smem_u32(&bars->drain), 0, ctl.timeout_ns, &never))
        atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_DRAIN);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter+32)
    int i = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++i) {
      int mb, nb;
      tile_coords(t, num_m, num_n, mb, nb);
      const uint32_t acc = i & 1, acc_phase = (i >> 1) & 1;
      const bool got = mbar_wait_bounded(smem_u32(&bars->tmem_full[acc]), acc_phase,
                                         ctl.timeout_ns, abort_flag);
      // tcgen05.ld is warp-collective: the whole warp leaves together or not at all.
      if (!__all_sync(0xffffffffu, got)) {
        *abort_flag = 1;
        if (lane == 0) atomicOr(ctl.status, RK_DEV_ERR_TIMEOUT_EPILOGUE);
        break;
      }
      tc_fence_after();
      const int row = mb * BM + quarter * 32 + lane;
      T* crow = C + static_cast<size_t>(row) * N;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < (SWIGLU ? 128 : BN) / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tbase + c * 32, r);
        if (SWIGLU) {
          uint32_t u[32];
          tmem_ld_32x32b_x32(tbase + 128 + c * 32, u);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j)
            r[j] = __float_as_uint(swiglu_f32(__uint_as_float(r[j]), __uint_as_float(u[j])));
        } else {
          tmem_ld_wait();
        }
        const int n0 = (SWIGLU ? nb * 128 : nb * BN) + c * 32;
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
      mbar_arrive(smem_u32(&bars->tmem_empty[acc]));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace tc1

namespace {
template <typename T, int BN, bool SWIGLU = false, bool A_MN = false, bool B_K = false>
rk_status launch_tc1(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                     rk_dtype dt, cudaStream_t s) {
  static_assert(!(SWIGLU && (A_MN || B_K)), "the fused SwiGLU GEMM takes the nn layout");
  CUtensorMap ta, tb;
  rk_status st = A_MN ? make_tmap_2d(&ta, A, dt, /*inner*/ M, /*outer*/ K, 64, tc1::BK)
                      : make_tmap_2d(&ta, A, dt, /*inner*/ K, /*outer*/ M, /*box_inner*/ 64,
                                     /*box_outer*/ tc1::BM);
  if (st != RK_OK) return st;
  st = B_K ? make_tmap_2d(&tb, B, dt, K, N, 64, BN)
           : make_tmap_2d(&tb, B, dt, SWIGLU ? 2 * N : N, K, 64, tc1::BK);
  if (st != RK_OK) return st;
  LaunchCtl lc;
  if ((st = launch_ctl(&lc)) != RK_OK) return st;
  KernelCtl ctl{lc.status, lc.timeout_ns, lc.inject_stall};

  constexpr int smem = tc1::smem_bytes<BN>();
  static std::once_flag attr_once[64];
  static cudaError_t attr_err[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(attr_once[dev & 63], [&] {
    attr_err[dev & 63] = cudaFuncSetAttribute(
        tc1::gemm_tc1_kernel<T, BN, SWIGLU, A_MN, B_K>, cudaFuncAttributeMaxDynamicSharedMemorySize,
        smem);
  });
  if (attr_err[dev & 63] != cudaSuccess) return cuda_status(attr_err[dev & 63]);

  const int64_t tile_n = SWIGLU ? 128 : BN;
  const int64_t num_tiles = ((M + tc1::BM - 1) / tc1::BM) * ((N + tile_n - 1) / tile_n);
  const int grid = static_cast<int>(num_tiles < device_sm_count() ? num_tiles : device_sm_count());
  const cudaError_t e = launch_kernel(tc1::gemm_tc1_kernel<T, BN, SWIGLU, A_MN, B_K>, dim3(grid),
                                      dim3(tc1::THREADS),
                                      smem, s, 0, ta, tb, reinterpret_cast<T*>(C),
                                      static_cast<int>(M), static_cast<int>(N),
                                      static_cast<int>(K), ctl);
  note_launch("gemm_tc1_kernel");
  return cuda_status(e);
}

// Tile width for a problem: fewest "waves" of persistent tiles weighted by the
// per-tile cost (narrower tiles re-read A more often per flop).
int pick_tile_n(int64_t M, int64_t N) {
  const int64_t sms = device_sm_count();
  const int widths[3] = {256, 128, 64};
  const double cost[3] = {256.0, 128.0 * 1.05, 64.0 * 1.25};
  int best = 256;
  double best_cost = 1e300;
  for (int i = 0; i < 3; ++i) {
    const int64_t tiles = ((M + tc1::BM - 1) / tc1::BM) * ((N + widths[i] - 1) / widths[i]);
    const int64_t waves = (tiles + sms - 1) / sms;
    const double c = static_cast<double>(waves) * cost[i];
    if (c < best_cost * 0.999) {
      best_cost = c;
      best = widths[i];
    }
  }
  return best;
}

template <typename T, bool A_MN, bool B_K>
rk_status launch_tc1_auto(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                          rk_dtype dt, cudaStream_t s, int bn) {
  if (bn <= 0) bn = pick_tile_n(M, N);
  switch (bn) {
    case 64: return launch_tc1<T, 64, false, A_MN, B_K>(A, B, C, M, N, K, dt, s);
    case 128: return launch_tc1<T, 128, false, A_MN, B_K>(A, B, C, M, N, K, dt, s);
    default: return launch_tc1<T, 256, false, A_MN, B_K>(A, B, C, M, N, K, dt, s);
  }
}

template <typename T>
rk_status launch_tc1_layout(const void* A, const void* B, void* C, int64_t M, int64_t N,
                            int64_t K, rk_layout layout, rk_dtype dt, cudaStream_t s, int bn) {
  switch (layout) {
    case RK_LAYOUT_NN: return launch_tc1_auto<T, false, false>(A, B, C, M, N, K, dt, s, bn);
    case RK_LAYOUT_NT: return launch_tc1_auto<T, false, true>(A, B, C, M, N, K, dt, s, bn);
    case RK_LAYOUT_TN: return launch_tc1_auto<T, true, false>(A, B, C, M, N, K, dt, s, bn);
    case RK_LAYOUT_TT: return launch_tc1_auto<T, true, true>(A, B, C, M, N, K, dt, s, bn);
  }
  return RK_ERR_INVALID_ARGUMENT;
}
}  // namespace

static std::atomic<int> g_tile_n_override{0};

void gemm_set_tile_n(int bn) { g_tile_n_override.store(bn); }

bool gemm_swiglu_supported(const void* A, const void* B, const void* C, int64_t M, int64_t N,
                           int64_t K) {
  // B is [K, 2N]: the same rules as the plain GEMM with 2N columns, plus an output width
  // that is a multiple of 8 (16-byte stores).
  return N <= (1ll << 30) - 256 && gemm_tc_supported(A, B, C, M, 2 * N, K, RK_LAYOUT_NN) &&
         N % 8 == 0;
}

bool gemm_tc_supported(const void* A, const void* B, const void* C, int64_t M, int64_t N,
                       int64_t K, rk_layout layout) {
  if (device_cc_major() != 10) return false;
  if (M <= 0 || N <= 0 || K <= 0) return false;
  if (N % 8 != 0 || K % 8 != 0) return false;
  // A stored [K, M] has a row stride of M elements; TMA strides are multiples of 16 bytes.
  if ((layout == RK_LAYOUT_TN || layout == RK_LAYOUT_TT) && M % 8 != 0) return false;
  if (!aligned16(A) || !aligned16(B) || !aligned16(C)) return false;
  // TMA coordinates and the kernel's tile arithmetic are 32-bit.
  if (M > (1ll << 31) - 256 || N > (1ll << 31) - 256 || K > (1ll << 31) - 64) return false;
  if (M * N > (1ll << 62)) return false;
  return true;
}

rk_status gemm_swiglu_1sm_launch(const void* A, const void* B, void* C, int64_t M, int64_t N,
                                 int64_t K, rk_dtype dt, cudaStream_t s) {
  if (!gemm_swiglu_supported(A, B, C, M, N, K)) return RK_ERR_UNSUPPORTED;
  if (dt == RK_DTYPE_BF16) return launch_tc1<__nv_bfloat16, 256, true>(A, B, C, M, N, K, dt, s);
  return launch_tc1<__half, 256, true>(A, B, C, M, N, K, dt, s);
}

rk_status gemm_tc_1sm_launch(const void* A, const void* B, void* C, int64_t M, int64_t N,
                             int64_t K, rk_layout layout, rk_dtype dt, cudaStream_t s) {
  if (!gemm_tc_supported(A, B, C, M, N, K, layout)) return RK_ERR_UNSUPPORTED;
  const int bn = g_tile_n_override.load();
  if (dt == RK_DTYPE_BF16)
    return launch_tc1_layout<__nv_bfloat16>(A, B, C, M, N, K, layout, dt, s, bn);
  return launch_tc1_layout<__half>(A, B, C, M, N, K, layout, dt, s, bn);
}

}  // namespace rk
