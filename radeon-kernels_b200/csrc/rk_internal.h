// rk_internal.h -- host-side declarations shared by the translation units of
// librk_kernels.so.  Not part of the public ABI (see include/rk_kernels.h).
#pragma once

#include <cuda_runtime.h>

#include <string>
#include <cstdint>
#include <utility>

#include "rk_kernels.h"

namespace rk {

struct LaunchCtl {
  uint32_t* status;     // device address of this device's status word
  uint64_t timeout_ns;  // per-wait limit handed to the kernels
  int inject_stall;     // test hook, see rk_debug_inject_stall()
};

// Fills `ctl` for the current device (status word address, limits).
rk_status launch_ctl(LaunchCtl* ctl);
// Cached per-device properties.
int device_sm_count();
int device_cc_major();
// Counts one kernel launch (rk_launch_count()) and records the kernel's name for this
// thread (rk_debug_last_kernel(); null: "other").
void note_launch(const char* kernel = nullptr);
// Programmatic dependent launch switch (rk_set_programmatic_launch()).
bool programmatic_launch();
bool set_programmatic_launch(bool enable);

// Launches `kernel` with programmatic stream serialisation when it is enabled (the
// kernel must call pdl_begin() before touching global memory) and, for cluster > 0,
// with that thread-block cluster size along x.
template <typename... Params, typename... Args>
cudaError_t launch_kernel(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t s, int cluster, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (programmatic_launch()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster > 0) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = static_cast<unsigned>(cluster);
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
// Maps a CUDA error to a status code (and remembers the message).
rk_status cuda_status(cudaError_t e);
// Records a message for rk_last_error() (this thread) without changing any status.
void note_error(const std::string& message);

// Kernel families.  All validate what they need and return RK_ERR_UNSUPPORTED
// when the variant cannot run the request.
rk_status gemm_simt_launch(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                           rk_layout layout, rk_dtype dt, cudaStream_t s);
rk_status gemm_tc_1sm_launch(const void* A, const void* B, void* C, int64_t M, int64_t N,
                             int64_t K, rk_layout layout, rk_dtype dt, cudaStream_t s);
rk_status gemm_tc_2sm_launch(const void* A, const void* B, void* C, int64_t M, int64_t N,
                             int64_t K, rk_layout layout, rk_dtype dt, cudaStream_t s);
bool gemm_tc_supported(const void* A, const void* B, const void* C, int64_t M, int64_t N,
                       int64_t K, rk_layout layout);
// Fused FFN-up + SwiGLU: C[M,N] = silu(A @ B[:, :N]) * (A @ B[:, N:]), B [K, 2N].
bool gemm_swiglu_supported(const void* A, const void* B, const void* C, int64_t M, int64_t N,
                           int64_t K);
rk_status gemm_swiglu_1sm_launch(const void* A, const void* B, void* C, int64_t M, int64_t N,
                                 int64_t K, rk_dtype dt, cudaStream_t s);
rk_status gemm_swiglu_2sm_launch(const void* A, const void* B, void* C, int64_t M, int64_t N,
                                 int64_t K, rk_dtype dt, cudaStream_t s);

rk_status gemv_scalar_launch(const void* x, const void* W, void* out, int64_t M, int64_t N,
                             int64_t K, rk_dtype dt, cudaStream_t s);
rk_status gemv_stream_launch(const void* x, const void* W, void* out, int64_t M, int64_t N,
                             int64_t K, rk_dtype dt, cudaStream_t s);
rk_status gemv_tc_launch(const void* x, const void* W, void* out, int64_t M, int64_t N, int64_t K,
                         rk_dtype dt, cudaStream_t s, void* workspace, size_t workspace_bytes,
                         bool stream_k = false);
size_t gemv_tc_workspace_bytes(int64_t M, int64_t N, int64_t K);
size_t gemv_tc_stream_k_bytes(int64_t M, int64_t N, int64_t K);
bool gemv_tc_supported(const void* x, const void* W, const void* out, int64_t M, int64_t N,
                       int64_t K);
bool gemv_stream_supported(const void* x, const void* W, const void* out, int64_t M, int64_t N,
                           int64_t K);

// Paged decode attention (paged_attention.cu).
size_t paged_attention_workspace_bytes(int64_t batch, int64_t hq, int64_t hkv, int64_t head_dim,
                                       int64_t max_blocks, int64_t block_size);
rk_status paged_attention_launch(const void* query, const void* key_cache, const void* value_cache,
                                 const void* block_tables, const void* context_lengths, void* out,
                                 int64_t batch, int64_t hq, int64_t hkv, int64_t head_dim,
                                 int64_t num_blocks, int64_t block_size, int64_t max_blocks,
                                 float scale, rk_dtype dt, int index_bits, void* workspace,
                                 size_t workspace_bytes, cudaStream_t s);

// Decode neighbours (llm_ops.cu).  rms_norm_launch: residual == nullptr -> rms_norm,
// else add_rms_norm (residual_out receives x + residual).
rk_status silu_mul_launch(const void* gate, const void* up, void* out, int64_t tokens,
                          int64_t hidden, rk_dtype dt, cudaStream_t s);
rk_status rms_norm_launch(const void* x, const void* residual, const void* weight, void* out,
                          void* residual_out, int64_t tokens, int64_t hidden, float eps,
                          rk_dtype dt, cudaStream_t s);
void norm_set_threads(int threads);
// Backward passes (llm_ops_backward.cu).  rms_norm_backward_launch: add == false ->
// rms_norm (x = input, dres/dres_out unused); add == true -> add_rms_norm (x =
// residual_out, dres nullable = no residual_out gradient, dres_out nullable).  dw
// nullable: no weight gradient (no workspace needed).
rk_status silu_mul_backward_launch(const void* dy, const void* gate, const void* up, void* dgate,
                                   void* dup, int64_t tokens, int64_t hidden, rk_dtype dt,
                                   cudaStream_t s);
rk_status rms_norm_backward_launch(const void* dy, const void* x, const void* w, bool add,
                                   const void* dres, void* dx, void* dres_out, void* dw,
                                   int64_t tokens, int64_t hidden, float eps, rk_dtype dt,
                                   void* workspace, size_t workspace_bytes, cudaStream_t s);
size_t rms_norm_backward_workspace_bytes(int64_t tokens, int64_t hidden);
void norm_backward_set_ctas_per_sm(int ctas);
// Paged decode attention on the tensor cores (paged_attention_tc.cu).
struct PagedTcArgs {
  const void *q, *k, *v, *tables, *lens;
  void* out;
  float *part_acc, *part_ml;
  int64_t batch, hq, hkv, head_dim, num_blocks, block_size, max_blocks;
  int partitions, part_tokens, index_bits;
  float scale;
  rk_dtype dt;
};
bool paged_attention_tc_supported(const void* query, const void* key_cache, const void* value_cache,
                                  int64_t hq, int64_t hkv, int64_t head_dim, int64_t block_size);
void paged_attention_tc_plan(int64_t batch, int64_t hkv, int64_t max_ctx, int sms, int* partitions,
                             int* part_tokens);
rk_status paged_attention_tc_launch(const PagedTcArgs& a, cudaStream_t s);
void paged_attention_set_path(int path);  // 0 automatic, 1 CUDA cores, 2 tensor cores

// Prefill attention (sdpa_tcgen05.cu).
rk_status sdpa_launch(const void* q, const void* k, const void* v, void* out, int64_t B,
                      int64_t Hq, int64_t Hkv, int64_t S, int64_t D, bool causal, float scale,
                      rk_dtype dt, cudaStream_t s);

rk_status gather_column_blocks_launch(const void* blocks, void* out, int64_t G, int64_t M,
                                      int64_t N, rk_dtype dt, cudaStream_t s);

// Host view of an rk_peer_group for one fused call: out[j] is rank j's full output
// advanced to this rank's column block, ctl[j] rank j's control block.
struct PeerTargets {
  void* out[RK_PEER_MAX];
  void* ctl[RK_PEER_MAX];
  int64_t ldo;
  int rank;
  int world;
  uint64_t timeout_ns;
};
// RK_OK when a usable device is current on this thread (binds its primary context).
rk_status device_ready();
// Fused compute + all-gather launchers (peer.cu validates; protocol in rk_peer.cuh).
rk_status gemv_stream_allgather_launch(const void* x, const void* W, int64_t M, int64_t N_block,
                                       int64_t K, rk_dtype dt, const PeerTargets& t,
                                       cudaStream_t s);
rk_status gemm_tc2_allgather_launch(const void* A, const void* B, int64_t M, int64_t N_block,
                                    int64_t K, rk_dtype dt, const PeerTargets& t, cudaStream_t s);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace rk
