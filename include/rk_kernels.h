/*
 * rk_kernels.h -- C ABI of the B200 (sm_100a) dense-contraction kernels.
 *
 * This is the drop-in boundary for the hot path of radeon-kernels:
 *   rk.gemm(a, b)      C[M,N] = A[M,K] @ B[K,N]        (row-major "nn")
 *   rk.gemv(x, weight) out[M,N] = x[M,K] @ weight[N,K]^T (weight layout "nk")
 * fp16 or bf16 operands, fp32 accumulation, output in the operand dtype,
 * rounded to nearest-even.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream,
 * never throws and never allocates device memory.  All launches are
 * asynchronous on the given stream (NULL = legacy default stream); the
 * caller owns every buffer.  Nothing here depends on PyTorch.
 *
 * Errors are reported in two places:
 *   - host-side argument and launch errors as the returned rk_status;
 *   - device-side failures (a bounded wait inside a kernel that ran out)
 *     in a per-device status word that rk_device_status() reads and clears.
 *     No kernel traps or spins forever: every wait has a time limit.
 */
#ifndef RK_KERNELS_H_
#define RK_KERNELS_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RK_ABI_VERSION 1

#if defined(__GNUC__)
#define RK_API __attribute__((visibility("default")))
#else
#define RK_API
#endif

/* CUDA stream handle; identical to cudaStream_t / CUstream. */
typedef struct CUstream_st* rk_stream_t;

typedef enum rk_status {
  RK_OK = 0,
  RK_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, K mismatch, M>32 for GEMV */
  RK_ERR_UNSUPPORTED = 2,      /* variant cannot run this shape / alignment / device */
  RK_ERR_CUDA = 3,             /* a CUDA runtime or driver call failed */
  RK_ERR_TIMEOUT = 4,          /* a device-side bounded wait expired (kernel gave up) */
  RK_ERR_NO_DEVICE = 5,        /* no usable sm_100 device is current */
  RK_ERR_TOO_LARGE = 6         /* request exceeds a fixed capacity of the entry point */
} rk_status;

typedef enum rk_dtype {
  RK_DTYPE_FP16 = 0,
  RK_DTYPE_BF16 = 1
} rk_dtype;

/* GEMM variants (the `variant` launch parameter of the dispatch manifest). */
enum {
  RK_GEMM_AUTO = 0,        /* pick from shape, alignment and device */
  RK_GEMM_SIMT = 1,        /* generic predicated CUDA-core kernel: any shape, any alignment */
  RK_GEMM_TC_1SM = 2,      /* tcgen05 + TMA, 128x256 tile per SM, persistent */
  RK_GEMM_TC_2SM = 3,      /* tcgen05 cta_group::2, 256x256 tile per SM pair, persistent */
  RK_GEMM_VARIANT_COUNT = 4
};

/* Operand storage for rk_gemm_layout, named as in the reference's Layout enum
 * (src/radeon_kernels/ops/gemm/spec.py:12-15): the first letter describes A, the second
 * B; "n" = stored as the operand ([M,K] for A, [K,N] for B), "t" = stored transposed
 * ([K,M] for A, [N,K] for B), each row-major and dense.  TT is an extension. */
typedef enum rk_layout {
  RK_LAYOUT_NN = 0,
  RK_LAYOUT_NT = 1,
  RK_LAYOUT_TN = 2,
  RK_LAYOUT_TT = 3
} rk_layout;

/* GEMV variants. */
enum {
  RK_GEMV_AUTO = 0,        /* pick from M, N, K and alignment */
  RK_GEMV_SCALAR = 1,      /* generic kernel: any K, any alignment */
  RK_GEMV_STREAM = 2,      /* 128-bit weight streaming, in-CTA split-K, needs K%8==0 + 16B alignment */
  RK_GEMV_TC = 3,          /* tcgen05 skinny GEMM (W as the 128-row operand, x as N=16/32), TMA ring,
                              cluster split-K reduced through distributed shared memory */
  RK_GEMV_VARIANT_COUNT = 4
};

/*
 * C = A @ B.  A: [M,K] row-major (lda = K), B: [K,N] row-major (ldb = N),
 * C: [M,N] row-major (ldc = N), all of dtype `dt`.  M, N, K >= 0; when K == 0
 * C is zero-filled.  Replaces the reference's pybind entry `gemm_out(a, b,
 * out, variant)` (src/radeon_kernels/ops/gemm/native/wmma_gemm.hip:294-316)
 * and its variant switch `launch<T>` (wmma_gemm.hip:234-277).  Unlike the
 * reference kernel it has no divisibility requirement: RK_GEMM_AUTO runs a
 * tensor-core variant when N%8==0, K%8==0 and the pointers are 16-byte
 * aligned, and the generic kernel otherwise.
 */
RK_API rk_status rk_gemm(const void* A, const void* B, void* C, int64_t M, int64_t N,
                  int64_t K, rk_dtype dt, int variant, rk_stream_t stream);

/*
 * C = op(A) @ op(B) with either operand read in its stored orientation (rk_layout):
 * RK_LAYOUT_NT takes B as [N,K] row-major (C = A @ B^T, the activation gradient
 * dA = dC @ B^T of C = A @ B), RK_LAYOUT_TN takes A as [K,M] row-major (C = A^T @ B,
 * the weight gradient dB = A^T @ dC).  No transpose copy is made: the tensor-core
 * variants load the stored tiles with TMA in the matching major order.  These are the
 * layouts the reference declares (src/radeon_kernels/ops/gemm/spec.py:12-15) but never
 * runs natively -- its rk.gemm signs every call "nn" (ops/gemm/api.py:93) and transposed
 * views reach torch.mm through the fallback.  Same variants and K == 0 rule as rk_gemm;
 * RK_GEMM_AUTO uses tensor cores when N%8 == 0, K%8 == 0, pointers are 16-byte aligned
 * and, for a transposed A, M%8 == 0.  rk_gemm(...) equals rk_gemm_layout(...,
 * RK_LAYOUT_NN, ...).
 */
RK_API rk_status rk_gemm_layout(const void* A, const void* B, void* C, int64_t M, int64_t N,
                  int64_t K, rk_layout layout, rk_dtype dt, int variant,
                  rk_stream_t stream);

/*
 * out = x @ weight^T.  x: [M,K] row-major, weight: [N,K] row-major ("nk"),
 * out: [M,N] row-major.  1 <= M <= 32 (the reference contract's maximum_m,
 * contracts/gemv-1.0.json:11), N, K >= 1.  Replaces the reference's
 * `gemv_impl<OutputsPerWave>` behind the `gemv_wave1/2/4` pybind entries
 * (benchmarks/gemv/native_gemv.hip:277-297, :343-377); unlike those, the
 * output buffer is the caller's.  Deterministic: the K reduction order is
 * fixed by (M, N, K, variant).
 */
RK_API rk_status rk_gemv(const void* x, const void* weight, void* out, int64_t M,
                  int64_t N, int64_t K, rk_dtype dt, int variant,
                  rk_stream_t stream);

/*
 * rk_gemv with a caller-owned workspace for strategies that need split-K scratch.
 * rk_gemv_workspace_size() tells how much the selected strategy uses (0: none).
 * Strategies that use it split K over independent CTAs that meet in the workspace:
 * fp32 partial tiles plus one ticket counter per shared tile; the last CTA of a tile
 * adds the partials in a fixed order.  The first RK_GEMV_WORKSPACE_TICKET_BYTES of the
 * workspace hold the ticket counters: they must be zero before the first use and every
 * call leaves them zero; the rest is scratch.  A workspace can therefore be reused
 * across problem sizes and strategies.  Calls that share a workspace must be ordered
 * (same stream).  NULL / too small: same as rk_gemv.  No counterpart in the reference.
 */
#define RK_GEMV_WORKSPACE_TICKET_BYTES (64u << 10)
RK_API rk_status rk_gemv_ex(const void* x, const void* weight, void* out, int64_t M,
                            int64_t N, int64_t K, rk_dtype dt, int variant,
                            void* workspace, size_t workspace_bytes, rk_stream_t stream);

/* Workspace bytes rk_gemv_ex can use for this problem (0: none needed). */
RK_API rk_status rk_gemv_workspace_size(int64_t M, int64_t N, int64_t K, rk_dtype dt,
                                        int variant, size_t* bytes);

/* Capacity of the scratch array behind rk_gemv_fixed_scratch (8 MiB per device). */
#define RK_GEMV_FIXED_SCRATCH_BYTES (8u << 20)

/*
 * The stream-K tensor-core GEMV -- the variant that needs split-K scratch -- for
 * callers that cannot allocate device memory: it allocates nothing and takes no
 * workspace.  No counterpart in the reference.
 *
 * Who needs it: plugins hosted by an engine that owns all device allocations and
 * gives a custom op only its input and output buffers, and latency-critical serving
 * loops that must not call cudaMalloc on the hot path (it can synchronise the device
 * and fail under memory pressure).  The caller still passes x, weight and out.
 *
 * The split-K scratch is a fixed array of RK_GEMV_FIXED_SCRATCH_BYTES compiled into
 * the library; every GPU that loads the library holds it until the process exits.
 * The first call on a device looks up its device address (cudaGetSymbolAddress) with
 * that device current; make that first call before any stream capture.  All calls
 * on a device share the one array and each call re-zeroes the part that must start
 * at zero, so calls that may overlap on the GPU (different streams without ordering)
 * race and must not be issued.  The array holds one split-K ticket per 128-row tile of
 * the weight (RK_GEMV_WORKSPACE_TICKET_BYTES of them: N <= 2,097,152) and the fp32
 * partial tiles of as many stream-K CTAs as fit in the rest (up to the full grid of two
 * per SM); taller weights are rejected with RK_ERR_TOO_LARGE, shapes the tensor-core
 * GEMV cannot run (K % 8 != 0, unaligned pointers, non-sm_100 device) with
 * RK_ERR_UNSUPPORTED.
 */
RK_API rk_status rk_gemv_fixed_scratch(const void* x, const void* weight, void* out,
                                       int64_t M, int64_t N, int64_t K, rk_dtype dt,
                                       rk_stream_t stream);

/*
 * Column-block gather for N-sharded GEMM/GEMV results.  `blocks` holds G
 * contiguous blocks [G][M][N/G] (the layout an NCCL all-gather of per-rank
 * C blocks produces); `out` receives the row-major [M, N] matrix.  N % G == 0.
 * No counterpart in the reference (it has no multi-GPU path).
 */
RK_API rk_status rk_gather_column_blocks(const void* blocks, void* out, int64_t G,
                                  int64_t M, int64_t N, rk_dtype dt,
                                  rk_stream_t stream);

/*
 * Multi-GPU: N-column sharding with the all-gather fused into the kernel.  No
 * counterpart in the reference (it has no multi-GPU path).
 *
 * One process per GPU.  A group of `world` ranks shares, per rank, a full output
 * buffer [M, world * N_block] and a control block of RK_PEER_CTL_BYTES (zeroed before
 * the first call, 512-byte aligned), each mapped into every other rank's process with
 * rk_ipc_export / rk_ipc_open (rk_gemv_allgather needs a larger control area, sized by
 * rk_gemv_allgather_ctl_bytes).  Rank r owns the column block [r*N_block, (r+1)*N_block)
 * of the result.  Its kernel computes that block and sends it over NVLink with plain peer
 * stores while the rest of the block is still being computed.  The GEMM stores finished
 * tiles straight into every rank's output.  The GEMV sends 8-byte packets that carry the
 * call number into each rank's staging area, and each rank copies them into its own
 * output.  When the call completes on a rank's stream, that rank's full output holds every
 * rank's block.
 *
 * Rules: every rank of the group makes the same sequence of calls on one group, each
 * rank on one stream; a rank's output may be read until that rank's next call on the
 * group (the next call lets the other ranks overwrite it only after it has started on
 * this rank, i.e. after everything queued before it on the stream completed).  Cross-GPU
 * waits are bounded by `timeout_ns` (0: 10 s); a wait that runs out is reported by
 * rk_device_status() as RK_ERR_TIMEOUT and the group must be rebuilt.
 */
#define RK_PEER_MAX 8
#define RK_PEER_CTL_BYTES 512

typedef struct rk_ipc_handle {
  unsigned char bytes[64]; /* cudaIpcMemHandle_t of the allocation holding the pointer */
  uint64_t offset;         /* pointer - allocation base */
} rk_ipc_handle;

typedef struct rk_peer_group {
  int32_t rank;              /* this process's rank, 0 <= rank < world */
  int32_t world;             /* ranks in the group, 1..RK_PEER_MAX */
  void* out[RK_PEER_MAX];    /* out[j]: rank j's full output as mapped in this process */
  void* ctl[RK_PEER_MAX];    /* ctl[j]: rank j's control block as mapped in this process */
  uint64_t timeout_ns;       /* limit of each cross-GPU wait (0: 10 s) */
} rk_peer_group;

/* Handle to the device allocation holding `ptr` (any pointer into it, e.g. a PyTorch
 * tensor's data_ptr()), for another process to map with rk_ipc_open. */
RK_API rk_status rk_ipc_export(const void* ptr, rk_ipc_handle* handle);
/* Maps another process's exported pointer into this process (current device); opening
 * the same allocation again shares the mapping. */
RK_API rk_status rk_ipc_open(const rk_ipc_handle* handle, void** ptr);
/* Releases one rk_ipc_open of `handle`; the last release unmaps the allocation. */
RK_API rk_status rk_ipc_close(const rk_ipc_handle* handle);

/*
 * out = x @ weight^T with the weight split by rows: weight_block holds rows
 * [rank*N_block, (rank+1)*N_block) of the [world*N_block, K] weight; x [M, K] is the same
 * on every rank.  The 128-bit streaming kernel of RK_GEMV_STREAM (identical results to
 * rk_gemv with that variant on the unsplit weight) computes the rank's block, and every
 * rank's out[j] [M, world*N_block] receives it.  The block crosses NVLink as 8-byte packets
 * that carry the call number, written into a staging area that follows each rank's control
 * block, so no fence or flag round trip is paid per call: ctl[j] must span
 * rk_gemv_allgather_ctl_bytes(M, N_block, world) bytes, zeroed before the first call.
 * 1 <= M <= 32; K % 8 == 0 and 16-byte-aligned x and weight (RK_ERR_UNSUPPORTED otherwise).
 */
RK_API rk_status rk_gemv_allgather(const void* x, const void* weight_block, int64_t M,
                                   int64_t N_block, int64_t K, rk_dtype dt,
                                   const rk_peer_group* group, rk_stream_t stream);

/* Bytes of the control area each rank needs for rk_gemv_allgather with these sizes: the
 * RK_PEER_CTL_BYTES control block followed by the packet staging area (2 x world x M x
 * N_block packets of 8 bytes).  No counterpart in the reference. */
RK_API rk_status rk_gemv_allgather_ctl_bytes(int64_t M, int64_t N_block, int32_t world, size_t* bytes);

/*
 * C = A @ B with B split by columns: B_block is [K, N_block] (columns [rank*N_block,
 * (rank+1)*N_block) of the [K, world*N_block] B, row-major), A [M, K] is the same on every
 * rank.  The 2-SM tcgen05 kernel of RK_GEMM_TC_2SM (identical results to rk_gemm with that
 * variant on the unsplit B) stages each finished 256 x 256 tile in shared memory and stores
 * it, 128 contiguous bytes per row segment, into every rank's out[j] [M, world*N_block]
 * while the next tile accumulates.  N_block % 8 == 0, K % 8 == 0, 16-byte-aligned operands
 * and outputs (RK_ERR_UNSUPPORTED otherwise).
 */
RK_API rk_status rk_gemm_allgather(const void* A, const void* B_block, int64_t M,
                                   int64_t N_block, int64_t K, rk_dtype dt,
                                   const rk_peer_group* group, rk_stream_t stream);

/*
 * Fused FFN-up projection with SwiGLU: C = silu(A @ B[:, :N]) * (A @ B[:, N:]).
 * A: [M,K] row-major; B: [K, 2N] row-major, the gate projection in columns [0, N) and the
 * up projection in columns [N, 2N) (torch.cat([w_gate, w_up], dim=1)); C: [M,N].  Both
 * products accumulate in fp32 in TMEM and the epilogue applies silu(g) * u to the fp32
 * sums before the one rounding to `dt`, so neither the [M, 2N] intermediate nor a second
 * kernel touches HBM.  variant: RK_GEMM_AUTO, RK_GEMM_TC_1SM or RK_GEMM_TC_2SM; needs
 * N % 8 == 0, K % 8 == 0 and 16-byte-aligned pointers (RK_ERR_UNSUPPORTED otherwise --
 * callers then run rk_gemm into a [M, 2N] buffer followed by rk_silu_mul).  No
 * counterpart in the reference, whose FFN runs rk.gemm and rk.silu_mul
 * (src/radeon_kernels/ops/swiglu/api.py) as separate operators.
 */
RK_API rk_status rk_gemm_swiglu(const void* A, const void* B, void* C, int64_t M, int64_t N,
                                int64_t K, rk_dtype dt, int variant, rk_stream_t stream);

/*
 * Decode attention over a paged K/V cache, one query token per sequence:
 *   out[b,h,:] = softmax_t(scale * query[b,h,:] . K[b,t,:]) @ V[b,t,:],  t < context_lengths[b]
 * query, out: [batch, query_heads, head_dim]; key_cache, value_cache: [num_blocks,
 * block_size, kv_heads, head_dim] ("block_slot_head_dim"); block_tables: [batch,
 * max_blocks_per_sequence] and context_lengths: [batch], both int32 (index_bits 32) or
 * int64 (index_bits 64) on the device.  Query head h reads KV head h / (query_heads /
 * kv_heads).  head_dim 64, 128 or 256; query and caches 16-byte aligned.  fp32 scores,
 * softmax and sum, one rounding of the output; a sequence with context length 0 gives NaN
 * (as the reference's softmax of an all -inf row).  Context lengths above
 * max_blocks_per_sequence * block_size are clamped to it.  Block-table entries outside
 * [0, num_blocks) are not dereferenced: those positions are skipped and
 * rk_device_status() reports RK_ERR_INVALID_ARGUMENT.  Long contexts are split over
 * several CTAs per sequence whose partial results meet in `workspace`
 * (rk_paged_attention_workspace_size(); no initialisation needed); NULL or too small when
 * one is needed -> RK_ERR_INVALID_ARGUMENT.  Replaces the reference's pybind entries
 * attention_wave1/4/8 (benchmarks/paged_attention/native_paged_attention.hip:192-283)
 * behind rk.paged_attention_decode (src/radeon_kernels/ops/paged_attention/api.py:38-157).
 */
RK_API rk_status rk_paged_attention_decode(const void* query, const void* key_cache,
                                           const void* value_cache, const void* block_tables,
                                           const void* context_lengths, void* out,
                                           int64_t batch, int64_t query_heads,
                                           int64_t kv_heads, int64_t head_dim,
                                           int64_t num_blocks, int64_t block_size,
                                           int64_t max_blocks_per_sequence, float scale,
                                           rk_dtype dt, int index_bits, void* workspace,
                                           size_t workspace_bytes, rk_stream_t stream);

/* Workspace bytes rk_paged_attention_decode needs for this shape (0: none). */
RK_API rk_status rk_paged_attention_workspace_size(int64_t batch, int64_t query_heads,
                                                   int64_t kv_heads, int64_t head_dim,
                                                   int64_t block_size,
                                                   int64_t max_blocks_per_sequence,
                                                   size_t* bytes);

/*
 * out = silu(gate) * up elementwise, silu(g) = g / (1 + exp(-g)) evaluated as
 * g * (1 / (1 + exp(-g))) in fp32, one rounding to `dt` per element.  gate, up,
 * out: [tokens, hidden] row-major, same dtype; tokens, hidden >= 0.  Replaces the
 * reference's pybind entry `silu_mul(gate, up)` (benchmarks/llm_ops/
 * native_llm_ops.hip:397-416, kernel :125-133) behind rk.silu_mul (operator
 * "swiglu", src/radeon_kernels/ops/swiglu/api.py:22-62); the output buffer is the
 * caller's.
 */
RK_API rk_status rk_silu_mul(const void* gate, const void* up, void* out, int64_t tokens,
                             int64_t hidden, rk_dtype dt, rk_stream_t stream);

/*
 * out = x * (1 / sqrt(mean(x^2) + eps)) * weight per row, fp32 arithmetic, one
 * rounding per element.  x, out: [tokens, hidden]; weight: [hidden]; eps > 0.
 * Replaces the reference's pybind entry `rms_norm(input, weight, eps)`
 * (native_llm_ops.hip:306-325, kernel :51-67) behind rk.rms_norm
 * (src/radeon_kernels/ops/rms_norm/api.py:22-61).
 */
RK_API rk_status rk_rms_norm(const void* x, const void* weight, void* out, int64_t tokens,
                             int64_t hidden, float eps, rk_dtype dt, rk_stream_t stream);

/*
 * residual_out = x + residual (rounded to `dt`), out = rms_norm(residual_out, weight,
 * eps).  x, residual, out, residual_out: [tokens, hidden]; weight: [hidden].
 * Replaces the reference's pybind entry `add_rms_norm(input, residual, weight, eps)`
 * (native_llm_ops.hip:327-353, kernel :69-94) behind rk.add_rms_norm
 * (src/radeon_kernels/ops/add_rms_norm/api.py:22-79).
 */
RK_API rk_status rk_add_rms_norm(const void* x, const void* residual, const void* weight,
                                 void* out, void* residual_out, int64_t tokens,
                                 int64_t hidden, float eps, rk_dtype dt,
                                 rk_stream_t stream);

/*
 * Backward passes of the three neighbours.  The reference runs inputs that require
 * gradients through its torch fallbacks (ops/swiglu/api.py:49, ops/rms_norm/api.py:53,
 * ops/add_rms_norm/api.py:57), so its gradients are the autograd of those fp32 graphs
 * (swiglu/reference.py:6-9, rms_norm/reference.py:6-10, add_rms_norm/reference.py:8-12);
 * these kernels evaluate the same chain-rule terms in fp32 and round once to the dtype.
 * All tensors are contiguous [tokens, hidden] (weight and its gradient [hidden]) of
 * dtype `dt`.
 *
 * rk_silu_mul_backward: grad_gate = dy * u * s * (1 + g * (1 - s)) (evaluated as
 * t*s + ((t*g)*(1-s))*s with t = dy*u), grad_up = dy * (g * s), s = sigmoid(gate).
 */
RK_API rk_status rk_silu_mul_backward(const void* grad_out, const void* gate, const void* up,
                                      void* grad_gate, void* grad_up, int64_t tokens,
                                      int64_t hidden, rk_dtype dt, rk_stream_t stream);

/*
 * Workspace bytes rk_rms_norm_backward / rk_add_rms_norm_backward need on the current
 * device when a weight gradient is requested (fp32 partial column sums, one row per CTA;
 * 0 for tokens == 0).  Without a weight gradient no workspace is used.
 */
RK_API rk_status rk_rms_norm_backward_workspace_size(int64_t tokens, int64_t hidden,
                                                     size_t* bytes);

/*
 * rms_norm backward: grad_input = (dy*w)*r + (((-0.5*c)*r^3)/H)*(2*x) with
 * r = rsqrt(mean(x^2) + eps) and c = sum_j (dy_j*w_j)*x_j per row; grad_weight (nullable:
 * not computed) = sum over rows of dy*(x*r), added in a fixed order (deterministic).
 * hidden <= 49152 when grad_weight is requested (RK_ERR_UNSUPPORTED otherwise).
 */
RK_API rk_status rk_rms_norm_backward(const void* grad_out, const void* input,
                                      const void* weight, void* grad_input, void* grad_weight,
                                      int64_t tokens, int64_t hidden, float eps, rk_dtype dt,
                                      void* workspace, size_t workspace_bytes,
                                      rk_stream_t stream);

/*
 * add_rms_norm backward, from the saved residual_out s = x + residual: the rms_norm
 * input gradient at s, rounded, plus grad_residual_out (nullable: no gradient flows into
 * residual_out), rounded again, is stored to grad_input and (nullable) grad_residual --
 * both inputs of the add receive it; grad_weight as in rk_rms_norm_backward.
 */
RK_API rk_status rk_add_rms_norm_backward(const void* grad_out, const void* grad_residual_out,
                                          const void* residual_out, const void* weight,
                                          void* grad_input, void* grad_residual,
                                          void* grad_weight, int64_t tokens, int64_t hidden,
                                          float eps, rk_dtype dt, void* workspace,
                                          size_t workspace_bytes, rk_stream_t stream);

/*
 * Scaled dot-product self-attention (prefill), inference only: for every batch b, query
 * head h and query position q,
 *   out[b,h,q,:] = sum_k softmax_k(scale * Q[b,h,q,:] . K[b,g,k,:]) V[b,g,k,:],
 * g = h / (query_heads / kv_heads), keys k < sequence (and k <= q when is_causal), fp32
 * softmax and accumulation, output rounded once.  query/out: [batch, query_heads,
 * sequence, head_dim], key/value: [batch, kv_heads, sequence, head_dim], contiguous, 16-byte
 * aligned, of dtype `dt`; head_dim 64, 128 or 256; query_heads % kv_heads == 0; scale > 0
 * and finite.  Replaces the reference's rk.sdpa (src/radeon_kernels/ops/sdpa/api.py:102-118),
 * which runs torch's scaled_dot_product_attention (ops/sdpa/reference.py:39-57; its manifest,
 * dispatch/sdpa-1.0.json, has no native entry).  tcgen05 flash attention: one CTA per
 * 128-row query tile and head, S = Q K^T and O += P V on the tensor cores, P rounded to the
 * dtype between them.
 */
RK_API rk_status rk_sdpa(const void* query, const void* key, const void* value, void* out,
                         int64_t batch, int64_t query_heads, int64_t kv_heads,
                         int64_t sequence, int64_t head_dim, int is_causal, float scale,
                         rk_dtype dt, rk_stream_t stream);

/* Static description of a status code; never NULL. */
RK_API const char* rk_status_string(rk_status status);

/* Message of the last CUDA error seen by this thread's calls ("" if none). */
RK_API const char* rk_last_error(void);

/*
 * Reads and clears the device-side status word of the current device after
 * synchronising `stream`.  Returns RK_OK, RK_ERR_TIMEOUT when a kernel launched
 * since the previous call gave up on a bounded wait, or RK_ERR_INVALID_ARGUMENT
 * when one met an out-of-range index in device memory (a paged-attention block
 * table entry) and skipped it.
 */
RK_API rk_status rk_device_status(rk_stream_t stream);

/* Programmatic dependent launch (on by default; no counterpart in the reference,
 * whose kernels launch one after another).  When enabled every kernel of this
 * library is launched with programmatic stream serialisation: it may be scheduled
 * while the previous kernel in the stream is still finishing, runs its set-up
 * (barrier initialisation, tensor-memory allocation, descriptor prefetch), then waits
 * in griddepcontrol.wait until every earlier kernel of the stream has completed and
 * its writes are visible, before it reads or writes global memory.  Results are
 * identical either way; 0 disables it (kernels then start only after the previous
 * kernel completes).  Returns the previous setting.  Process-wide. */
RK_API int rk_set_programmatic_launch(int enable);

/*
 * ---------------------------------------------------------------------------------
 * Tuning and debugging hooks.  Process-wide settings read when a kernel is launched:
 * they change the choices of every caller in the process, so they are for tests,
 * benchmarks and tuning sweeps, not for concurrent production use.  None of them
 * changes results beyond the documented reduction order of the variant it selects.
 * No counterpart in the reference.
 * ---------------------------------------------------------------------------------
 */
/* Tuning hook for RK_GEMV_STREAM: weight rows per warp (1, 2, 4) and in-CTA
 * K split (1, 2, 4, 8); 0 restores the built-in heuristic.  Process-wide. */
RK_API void rk_gemv_set_tuning(int rows_per_warp, int ksplit);

/* Tuning hook for the tensor-core GEMM variants: output tile width (64, 128,
 * 256); 0 restores the built-in choice (fewest weighted waves).  Process-wide. */
RK_API void rk_gemm_set_tile_n(int tile_n);

/* Tuning hook for rk_rms_norm / rk_add_rms_norm: threads per row (64, 128, 256); 0
 * restores the built-in choice (256 for few rows, 128 from two rows per SM).
 * Process-wide. */
RK_API void rk_norm_set_threads(int threads_per_row);

/* Kernel choice of rk_paged_attention_decode: 0 automatic (the tcgen05 kernel for head_dim
 * 64/128, up to 16 query heads per KV head and block sizes 8-128 in powers of two, except
 * head_dim-64 MHA; the CUDA-core kernel otherwise), 1 always the CUDA-core kernel, 2 the
 * tcgen05 kernel (RK_ERR_UNSUPPORTED where it does not apply).  Process-wide; for tests and
 * tuning. */
RK_API void rk_paged_attention_set_path(int path);

/* Tuning hook for the rms_norm backward row kernel: CTAs per SM (1..32); 0 restores the
 * built-in choice (1024 threads per SM with a weight gradient, 2048 without).
 * Process-wide.  Changes the workspace size. */
RK_API void rk_norm_backward_set_ctas_per_sm(int ctas_per_sm);

/* Tuning hook for RK_GEMV_TC: thread-block cluster size (K split), 1..8; -1 selects
 * stream-K through the rk_gemv_ex workspace (without one it falls back to cluster
 * split-K); 0 restores the built-in choice.  Process-wide. */
RK_API void rk_gemv_tc_set_cluster(int cluster_size);

/* Tuning hook for RK_GEMV_TC's cluster split-K: how the cluster's partial sums reach its
 * leader CTA -- 1 pulled (parked in each CTA's own ring, read by the leader through
 * distributed shared memory; two CTAs per SM), 2 pushed (stored straight into a receive
 * area of the leader's shared memory; one CTA per SM, an 8-stage ring, clusters of at most
 * 4); 0 restores the built-in choice (pushed when every cluster of the grid is resident at
 * once and the grid is no narrower).  For a given cluster size both forms add the same
 * partial sums in the same order.  Process-wide. */
RK_API void rk_gemv_tc_set_exchange(int mode);

/* Sets the per-wait time limit (nanoseconds, default 1e9) used by kernels
 * launched after the call.  0 restores the default. */
RK_API void rk_set_wait_timeout_ns(uint64_t ns);

/* Test hook: when nonzero, the next tensor-core GEMM launch makes its MMA
 * role wait on a barrier that nothing arrives on, so the bounded wait runs
 * out and the kernel reports RK_ERR_TIMEOUT.  Resets itself after one launch. */
RK_API void rk_debug_inject_stall(int enable);

/* Name of the last kernel this thread launched through the library ("gemv_tc_sk_kernel",
 * "gemm_tc2_kernel", ...; "" before the first launch, "other" for unnamed ones). */
RK_API const char* rk_debug_last_kernel(void);

/* Test hook: fills the whole array behind rk_gemv_fixed_scratch on the current device
 * with `byte` (stream-ordered), as an interrupted call could leave it. */
RK_API rk_status rk_debug_fill_fixed_scratch(int byte, rk_stream_t stream);

/* Human-readable name of a variant ("gemm:tc_1sm", "gemv:stream", ...). */
RK_API const char* rk_variant_name(int op /* 0 = gemm, 1 = gemv */, int variant);

/* The variant RK_GEMM_AUTO / RK_GEMV_AUTO would pick for this problem. */
RK_API int rk_gemm_select_variant(const void* A, const void* B, const void* C,
                           int64_t M, int64_t N, int64_t K, rk_dtype dt);
RK_API int rk_gemv_select_variant(const void* x, const void* weight, const void* out,
                           int64_t M, int64_t N, int64_t K, rk_dtype dt);

/* Number of kernel launches this library issued on any stream since load
 * (host-side counter, for launch accounting in benchmarks). */
RK_API uint64_t rk_launch_count(void);

RK_API int rk_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* RK_KERNELS_H_ */
