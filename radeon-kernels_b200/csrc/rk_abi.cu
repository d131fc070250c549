// rk_abi.cu -- the extern "C" boundary of librk_kernels.so (include/rk_kernels.h):
// argument validation, variant selection, per-device state (status word,
// SM count), error mapping.  No entry point allocates device memory.
#include <cuda_runtime.h>

#include <atomic>
#include <cstring>
#include <mutex>
#include <string>

#include "rk_device.cuh"
#include "rk_internal.h"

namespace rk {
void gemv_set_tuning(int rows, int ks);
void gemm_set_tile_n(int bn);
void gemv_tc_set_cluster(int c);
void gemv_tc_set_exchange(int mode);
}

// One status word per device: kernels atomicOr RK_DEV_ERR_* bits into it when
// a bounded wait runs out; rk_device_status() reads and clears it.
__device__ uint32_t rk_device_status_word;

namespace rk {
namespace {

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  std::once_flag once;
  cudaError_t err = cudaSuccess;
  uint32_t* status = nullptr;
  int sm_count = 0;
  int cc_major = 0;
  int cc_minor = 0;
};

DeviceInfo g_devices[kMaxDevices];
std::atomic<uint64_t> g_timeout_ns{1000000000ull};
std::atomic<int> g_inject_stall{0};
std::atomic<uint64_t> g_launches{0};
thread_local std::string g_last_error;

DeviceInfo* current_device_info() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  // Make the device's primary context current on this thread.  A thread whose device was
  // never set explicitly (PyTorch's autograd worker threads, for instance: device 0 is
  // already "current", so no cudaSetDevice happens) has no current driver context until
  // its first runtime launch, and the driver calls made here before any launch --
  // cuTensorMapEncodeTiled -- then fail with CUDA_ERROR_INVALID_CONTEXT.
  thread_local int bound_device = -1;
  if (bound_device != dev) {
    if (cudaSetDevice(dev) != cudaSuccess) return nullptr;
    bound_device = dev;
  }
  DeviceInfo* d = &g_devices[dev];
  std::call_once(d->once, [d, dev] {
    cudaDeviceProp prop;
    cudaError_t e = cudaGetDeviceProperties(&prop, dev);
    if (e == cudaSuccess) {
      d->sm_count = prop.multiProcessorCount;
      d->cc_major = prop.major;
      d->cc_minor = prop.minor;
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, rk_device_status_word);
      d->status = static_cast<uint32_t*>(p);
    }
    d->err = e;
  });
  return d->err == cudaSuccess ? d : nullptr;
}

bool valid_dtype(rk_dtype dt) { return dt == RK_DTYPE_FP16 || dt == RK_DTYPE_BF16; }

}  // namespace

rk_status cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return RK_OK;
  g_last_error = cudaGetErrorString(e);
  return RK_ERR_CUDA;
}

void note_error(const std::string& message) { g_last_error = message; }

namespace {
thread_local const char* g_last_kernel = "";
}  // namespace

void note_launch(const char* kernel) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  g_last_kernel = kernel != nullptr ? kernel : "other";
}

namespace {
std::atomic<bool> g_pdl{true};
}  // namespace

bool programmatic_launch() { return g_pdl.load(std::memory_order_relaxed); }
bool set_programmatic_launch(bool enable) { return g_pdl.exchange(enable); }

int device_sm_count() {
  DeviceInfo* d = current_device_info();
  return d ? d->sm_count : 1;
}

int device_cc_major() {
  DeviceInfo* d = current_device_info();
  return d ? d->cc_major : 0;
}

rk_status device_ready() { return current_device_info() != nullptr ? RK_OK : RK_ERR_NO_DEVICE; }

rk_status launch_ctl(LaunchCtl* ctl) {
  DeviceInfo* d = current_device_info();
  if (d == nullptr) return RK_ERR_NO_DEVICE;
  ctl->status = d->status;
  ctl->timeout_ns = g_timeout_ns.load();
  ctl->inject_stall = g_inject_stall.exchange(0);
  return RK_OK;
}

}  // namespace rk

using namespace rk;

namespace {
int select_gemm_variant(const void* A, const void* B, const void* C, int64_t M, int64_t N,
                        int64_t K, rk_layout layout) {
  if (!gemm_tc_supported(A, B, C, M, N, K, layout)) return RK_GEMM_SIMT;
  // SM pairs with 256x256 tiles once there is at least one tile per pair (they halve the
  // per-SM operand traffic); smaller problems keep more, narrower 1-SM tiles in flight.
  const int64_t pair_tiles = ((M + 255) / 256) * ((N + 255) / 256);
  if (pair_tiles >= device_sm_count() / 2) return RK_GEMM_TC_2SM;
  return RK_GEMM_TC_1SM;
}

bool valid_layout(rk_layout layout) {
  return layout == RK_LAYOUT_NN || layout == RK_LAYOUT_NT || layout == RK_LAYOUT_TN ||
         layout == RK_LAYOUT_TT;
}
}  // namespace

extern "C" {

const char* rk_status_string(rk_status status) {
  switch (status) {
    case RK_OK: return "ok";
    case RK_ERR_INVALID_ARGUMENT: return "invalid argument";
    case RK_ERR_UNSUPPORTED: return "variant does not support this problem";
    case RK_ERR_CUDA: return "CUDA error";
    case RK_ERR_TIMEOUT: return "device-side wait timed out";
    case RK_ERR_NO_DEVICE: return "no usable CUDA device";
    case RK_ERR_TOO_LARGE: return "request exceeds the entry point's fixed capacity";
  }
  return "unknown status";
}

const char* rk_last_error(void) { return g_last_error.c_str(); }

int rk_abi_version(void) { return RK_ABI_VERSION; }

uint64_t rk_launch_count(void) { return g_launches.load(); }

const char* rk_debug_last_kernel(void) { return g_last_kernel; }

void rk_set_wait_timeout_ns(uint64_t ns) { g_timeout_ns.store(ns ? ns : 1000000000ull); }

void rk_debug_inject_stall(int enable) { g_inject_stall.store(enable ? 1 : 0); }

void rk_gemv_set_tuning(int rows, int ksplit) { rk::gemv_set_tuning(rows, ksplit); }

void rk_gemm_set_tile_n(int tile_n) { rk::gemm_set_tile_n(tile_n); }

void rk_gemv_tc_set_cluster(int cluster_size) { rk::gemv_tc_set_cluster(cluster_size); }
void rk_gemv_tc_set_exchange(int mode) { rk::gemv_tc_set_exchange(mode); }

void rk_norm_set_threads(int threads_per_row) { rk::norm_set_threads(threads_per_row); }

int rk_set_programmatic_launch(int enable) { return rk::set_programmatic_launch(enable != 0) ? 1 : 0; }

const char* rk_variant_name(int op, int variant) {
  if (op == 0) {
    switch (variant) {
      case RK_GEMM_AUTO: return "gemm:auto";
      case RK_GEMM_SIMT: return "gemm:simt";
      case RK_GEMM_TC_1SM: return "gemm:tc_1sm";
      case RK_GEMM_TC_2SM: return "gemm:tc_2sm";
    }
  } else if (op == 1) {
    switch (variant) {
      case RK_GEMV_AUTO: return "gemv:auto";
      case RK_GEMV_SCALAR: return "gemv:scalar";
      case RK_GEMV_STREAM: return "gemv:stream";
      case RK_GEMV_TC: return "gemv:tc";
    }
  }
  return "unknown";
}

int rk_gemm_select_variant(const void* A, const void* B, const void* C, int64_t M, int64_t N,
                           int64_t K, rk_dtype dt) {
  (void)dt;
  return select_gemm_variant(A, B, C, M, N, K, RK_LAYOUT_NN);
}

int rk_gemv_select_variant(const void* x, const void* W, const void* out, int64_t M, int64_t N,
                           int64_t K, rk_dtype dt) {
  (void)dt;
  // M <= 2 streams on CUDA cores; from M = 3 the tensor-core kernel keeps the weight
  // stream at HBM speed where CUDA cores become FMA/L1 bound.
  if (M >= 3 && gemv_tc_supported(x, W, out, M, N, K)) return RK_GEMV_TC;
  return gemv_stream_supported(x, W, out, M, N, K) ? RK_GEMV_STREAM : RK_GEMV_SCALAR;
}

rk_status rk_gemm(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                  rk_dtype dt, int variant, rk_stream_t stream) {
  return rk_gemm_layout(A, B, C, M, N, K, RK_LAYOUT_NN, dt, variant, stream);
}

rk_status rk_gemm_layout(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                         rk_layout layout, rk_dtype dt, int variant, rk_stream_t stream) {
  if (M < 0 || N < 0 || K < 0 || !valid_dtype(dt) || !valid_layout(layout))
    return RK_ERR_INVALID_ARGUMENT;
  if (variant < 0 || variant >= RK_GEMM_VARIANT_COUNT) return RK_ERR_UNSUPPORTED;
  if (M == 0 || N == 0) return RK_OK;
  if (C == nullptr || (K > 0 && (A == nullptr || B == nullptr))) return RK_ERR_INVALID_ARGUMENT;
  if (current_device_info() == nullptr) return RK_ERR_NO_DEVICE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (K == 0) {
    // Empty inner dimension: C is the zero matrix (torch.mm semantics).
    return cuda_status(cudaMemsetAsync(C, 0, static_cast<size_t>(M) * N * 2, s));
  }
  if (variant == RK_GEMM_AUTO) variant = select_gemm_variant(A, B, C, M, N, K, layout);
  switch (variant) {
    case RK_GEMM_SIMT: return gemm_simt_launch(A, B, C, M, N, K, layout, dt, s);
    case RK_GEMM_TC_1SM: return gemm_tc_1sm_launch(A, B, C, M, N, K, layout, dt, s);
    case RK_GEMM_TC_2SM: return gemm_tc_2sm_launch(A, B, C, M, N, K, layout, dt, s);
  }
  return RK_ERR_UNSUPPORTED;
}

rk_status rk_gemv_ex(const void* x, const void* W, void* out, int64_t M, int64_t N, int64_t K,
                     rk_dtype dt, int variant, void* workspace, size_t workspace_bytes,
                     rk_stream_t stream) {
  if (M < 1 || M > 32 || N < 1 || K < 1 || !valid_dtype(dt)) return RK_ERR_INVALID_ARGUMENT;
  if (x == nullptr || W == nullptr || out == nullptr) return RK_ERR_INVALID_ARGUMENT;
  if (variant < 0 || variant >= RK_GEMV_VARIANT_COUNT) return RK_ERR_UNSUPPORTED;
  if (current_device_info() == nullptr) return RK_ERR_NO_DEVICE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (variant == RK_GEMV_AUTO) variant = rk_gemv_select_variant(x, W, out, M, N, K, dt);
  switch (variant) {
    case RK_GEMV_SCALAR: return gemv_scalar_launch(x, W, out, M, N, K, dt, s);
    case RK_GEMV_STREAM: return gemv_stream_launch(x, W, out, M, N, K, dt, s);
    case RK_GEMV_TC: return gemv_tc_launch(x, W, out, M, N, K, dt, s, workspace, workspace_bytes);
  }
  return RK_ERR_UNSUPPORTED;
}

rk_status rk_paged_attention_workspace_size(int64_t batch, int64_t query_heads,
                                           int64_t kv_heads, int64_t head_dim,
                                           int64_t block_size, int64_t max_blocks,
                                           size_t* bytes) {
  if (bytes == nullptr) return RK_ERR_INVALID_ARGUMENT;
  *bytes = 0;
  if (batch < 1 || query_heads < 1 || kv_heads < 1 || query_heads % kv_heads != 0 ||
      block_size < 1 || max_blocks < 1 || (head_dim != 64 && head_dim != 128 && head_dim != 256))
    return RK_ERR_INVALID_ARGUMENT;
  if (current_device_info() == nullptr) return RK_ERR_NO_DEVICE;
  *bytes = paged_attention_workspace_bytes(batch, query_heads, kv_heads, head_dim, max_blocks,
                                           block_size);
  return RK_OK;
}

rk_status rk_paged_attention_decode(const void* query, const void* key_cache,
                                    const void* value_cache, const void* block_tables,
                                    const void* context_lengths, void* out, int64_t batch,
                                    int64_t query_heads, int64_t kv_heads, int64_t head_dim,
                                    int64_t num_blocks, int64_t block_size, int64_t max_blocks,
                                    float scale, rk_dtype dt, int index_bits, void* workspace,
                                    size_t workspace_bytes, rk_stream_t stream) {
  if (batch < 1 || query_heads < 1 || kv_heads < 1 || query_heads % kv_heads != 0 ||
      num_blocks < 1 || block_size < 1 || max_blocks < 1 || !valid_dtype(dt) ||
      (index_bits != 32 && index_bits != 64) || !(scale > 0.0f && scale <= 3.4e38f))
    return RK_ERR_INVALID_ARGUMENT;
  if (head_dim != 64 && head_dim != 128 && head_dim != 256) return RK_ERR_INVALID_ARGUMENT;
  if (query == nullptr || key_cache == nullptr || value_cache == nullptr ||
      block_tables == nullptr || context_lengths == nullptr || out == nullptr)
    return RK_ERR_INVALID_ARGUMENT;
  if (!aligned16(query) || !aligned16(key_cache) || !aligned16(value_cache)) return RK_ERR_UNSUPPORTED;
  if (num_blocks > INT32_MAX || block_size > INT32_MAX || max_blocks > INT32_MAX ||
      max_blocks * block_size > INT32_MAX || batch * query_heads > INT32_MAX)
    return RK_ERR_UNSUPPORTED;
  if (current_device_info() == nullptr) return RK_ERR_NO_DEVICE;
  return paged_attention_launch(query, key_cache, value_cache, block_tables, context_lengths, out,
                                batch, query_heads, kv_heads, head_dim, num_blocks, block_size,
                                max_blocks, scale, dt, index_bits, workspace, workspace_bytes,
                                reinterpret_cast<cudaStream_t>(stream));
}

rk_status rk_gemm_swiglu(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                         rk_dtype dt, int variant, rk_stream_t stream) {
  if (M < 0 || N < 0 || K < 0 || !valid_dtype(dt)) return RK_ERR_INVALID_ARGUMENT;
  if (M > 0 && N > 0 && (A == nullptr || B == nullptr || C == nullptr)) return RK_ERR_INVALID_ARGUMENT;
  if (variant < 0 || variant >= RK_GEMM_VARIANT_COUNT) return RK_ERR_UNSUPPORTED;
  if (current_device_info() == nullptr) return RK_ERR_NO_DEVICE;
  if (M == 0 || N == 0) return RK_OK;
  if (!gemm_swiglu_supported(A, B, C, M, N, K)) return RK_ERR_UNSUPPORTED;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (variant == RK_GEMM_AUTO) {
    // SM pairs once there is a 256 x 128 output tile per pair (the plain GEMM's rule with
    // the fused tile's 128 output columns).
    const int64_t pair_tiles = ((M + 255) / 256) * ((N + 127) / 128);
    variant = pair_tiles >= device_sm_count() / 2 ? RK_GEMM_TC_2SM : RK_GEMM_TC_1SM;
  }
  switch (variant) {
    case RK_GEMM_TC_1SM: return gemm_swiglu_1sm_launch(A, B, C, M, N, K, dt, s);
    case RK_GEMM_TC_2SM: return gemm_swiglu_2sm_launch(A, B, C, M, N, K, dt, s);
  }
  return RK_ERR_UNSUPPORTED;
}

rk_status rk_silu_mul(const void* gate, const void* up, void* out, int64_t tokens,
                      int64_t hidden, rk_dtype dt, rk_stream_t stream) {
  if (tokens < 0 || hidden < 0 || !valid_dtype(dt)) return RK_ERR_INVALID_ARGUMENT;
  if (tokens > 0 && hidden > 0 && (gate == nullptr || up == nullptr || out == nullptr))
    return RK_ERR_INVALID_ARGUMENT;
  if (hidden > 0 && tokens > INT64_MAX / hidden) return RK_ERR_INVALID_ARGUMENT;
  if (current_device_info() == nullptr) return RK_ERR_NO_DEVICE;
  return silu_mul_launch(gate, up, out, tokens, hidden, dt, reinterpret_cast<cudaStream_t>(stream));
}

static bool valid_eps(float eps) { return eps > 0.0f && eps <= 3.4e38f; }  // positive, finite

rk_status rk_rms_norm(const void* x, const void* weight, void* out, int64_t tokens,
                      int64_t hidden, float eps, rk_dtype dt, rk_stream_t stream) {
  if (tokens < 0 || hidden < 1 || !valid_dtype(dt) || !valid_eps(eps)) return RK_ERR_INVALID_ARGUMENT;
  if (x == nullptr || weight == nullptr || out == nullptr) return RK_ERR_INVALID_ARGUMENT;
  if (current_device_info() == nullptr) return RK_ERR_NO_DEVICE;
  return rms_norm_launch(x, nullptr, weight, out, nullptr, tokens, hidden, eps, dt,
                         reinterpret_cast<cudaStream_t>(stream));
}

rk_status rk_add_rms_norm(const void* x, const void* residual, const void* weight, void* out,
                          void* residual_out, int64_t tokens, int64_t hidden, float eps,
                          rk_dtype dt, rk_stream_t stream) {
  if (tokens < 0 || hidden < 1 || !valid_dtype(dt) || !valid_eps(eps)) return RK_ERR_INVALID_ARGUMENT;
  if (x == nullptr || residual == nullptr || weight == nullptr || out == nullptr ||
      residual_out == nullptr)
    return RK_ERR_INVALID_ARGUMENT;
  if (current_device_info() == nullptr) return RK_ERR_NO_DEVICE;
  return rms_norm_launch(x, residual, weight, out, residual_out, tokens, hidden, eps, dt,
                         reinterpret_cast<cudaStream_t>(stream));
}

rk_status rk_silu_mul_backward(const void* grad_out, const void* gate, const void* up,
                               void* grad_gate, void* grad_up, int64_t tokens, int64_t hidden,
                               rk_dtype dt, rk_stream_t stream) {
  if (tokens < 0 || hidden < 0 || !valid_dtype(dt)) return RK_ERR_INVALID_ARGUMENT;
  if (tokens > 0 && hidden > 0 &&
      (grad_out == nullptr || gate == nullptr || up == nullptr || grad_gate == nullptr ||
       grad_up == nullptr))
    return RK_ERR_INVALID_ARGUMENT;
  if (hidden > 0 && tokens > INT64_MAX / hidden) return RK_ERR_INVALID_ARGUMENT;
  if (current_device_info() == nullptr) return RK_ERR_NO_DEVICE;
  return silu_mul_backward_launch(grad_out, gate, up, grad_gate, grad_up, tokens, hidden, dt,
                                  reinterpret_cast<cudaStream_t>(stream));
}

rk_status rk_rms_norm_backward_workspace_size(int64_t tokens, int64_t hidden, size_t* bytes) {
  if (bytes == nullptr) return RK_ERR_INVALID_ARGUMENT;
  *bytes = 0;
  if (tokens < 0 || hidden < 1) return RK_ERR_INVALID_ARGUMENT;
  if (current_device_info() == nullptr) return RK_ERR_NO_DEVICE;
  *bytes = rms_norm_backward_workspace_bytes(tokens, hidden);
  return RK_OK;
}

rk_status rk_rms_norm_backward(const void* grad_out, const void* input, const void* weight,
                               void* grad_input, void* grad_weight, int64_t tokens,
                               int64_t hidden, float eps, rk_dtype dt, void* workspace,
                               size_t workspace_bytes, rk_stream_t stream) {
  if (tokens < 0 || hidden < 1 || !valid_dtype(dt) || !valid_eps(eps)) return RK_ERR_INVALID_ARGUMENT;
  if (tokens > 0 && (grad_out == nullptr || input == nullptr || grad_input == nullptr))
    return RK_ERR_INVALID_ARGUMENT;
  if (weight == nullptr) return RK_ERR_INVALID_ARGUMENT;
  if (current_device_info() == nullptr) return RK_ERR_NO_DEVICE;
  return rms_norm_backward_launch(grad_out, input, weight, false, nullptr, grad_input, nullptr,
                                  grad_weight, tokens, hidden, eps, dt, workspace,
                                  workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

rk_status rk_add_rms_norm_backward(const void* grad_out, const void* grad_residual_out,
                                   const void* residual_out, const void* weight, void* grad_input,
                                   void* grad_residual, void* grad_weight, int64_t tokens,
                                   int64_t hidden, float eps, rk_dtype dt, void* workspace,
                                   size_t workspace_bytes, rk_stream_t stream) {
  if (tokens < 0 || hidden < 1 || !valid_dtype(dt) || !valid_eps(eps)) return RK_ERR_INVALID_ARGUMENT;
  if (tokens > 0 && (grad_out == nullptr || residual_out == nullptr || grad_input == nullptr))
    return RK_ERR_INVALID_ARGUMENT;
  if (weight == nullptr) return RK_ERR_INVALID_ARGUMENT;
  if (current_device_info() == nullptr) return RK_ERR_NO_DEVICE;
  return rms_norm_backward_launch(grad_out, residual_out, weight, true, grad_residual_out,
                                  grad_input, grad_residual, grad_weight, tokens, hidden, eps, dt,
                                  workspace, workspace_bytes,
                                  reinterpret_cast<cudaStream_t>(stream));
}

rk_status rk_sdpa(const void* query, const void* key, const void* value, void* out, int64_t batch,
                  int64_t query_heads, int64_t kv_heads, int64_t sequence, int64_t head_dim,
                  int is_causal, float scale, rk_dtype dt, rk_stream_t stream) {
  if (!valid_dtype(dt) || batch < 1 || query_heads < 1 || kv_heads < 1 || sequence < 1 ||
      query_heads % kv_heads != 0 || (head_dim != 64 && head_dim != 128 && head_dim != 256) ||
      !(scale > 0.0f && scale <= 3.4e38f))
    return RK_ERR_INVALID_ARGUMENT;
  if (query == nullptr || key == nullptr || value == nullptr || out == nullptr)
    return RK_ERR_INVALID_ARGUMENT;
  if (current_device_info() == nullptr) return RK_ERR_NO_DEVICE;
  return sdpa_launch(query, key, value, out, batch, query_heads, kv_heads, sequence, head_dim,
                     is_causal != 0, scale, dt, reinterpret_cast<cudaStream_t>(stream));
}

void rk_paged_attention_set_path(int path) { paged_attention_set_path(path); }

void rk_norm_backward_set_ctas_per_sm(int ctas_per_sm) {
  norm_backward_set_ctas_per_sm(ctas_per_sm >= 1 && ctas_per_sm <= 32 ? ctas_per_sm : 0);
}

rk_status rk_gemv(const void* x, const void* W, void* out, int64_t M, int64_t N, int64_t K,
                  rk_dtype dt, int variant, rk_stream_t stream) {
  return rk_gemv_ex(x, W, out, M, N, K, dt, variant, nullptr, 0, stream);
}

rk_status rk_gemv_workspace_size(int64_t M, int64_t N, int64_t K, rk_dtype dt, int variant,
                                 size_t* bytes) {
  if (bytes == nullptr) return RK_ERR_INVALID_ARGUMENT;
  *bytes = 0;
  if (M < 1 || M > 32 || N < 1 || K < 1 || !valid_dtype(dt)) return RK_ERR_INVALID_ARGUMENT;
  if (variant < 0 || variant >= RK_GEMV_VARIANT_COUNT) return RK_ERR_UNSUPPORTED;
  if (current_device_info() == nullptr) return RK_ERR_NO_DEVICE;
  // Only the tensor-core variant splits K through a workspace; AUTO picks it for M >= 3.
  if (variant == RK_GEMV_TC || (variant == RK_GEMV_AUTO && M >= 3 && device_cc_major() == 10 &&
                                K % 8 == 0))
    *bytes = gemv_tc_workspace_bytes(M, N, K);
  return RK_OK;
}

rk_status rk_gather_column_blocks(const void* blocks, void* out, int64_t G, int64_t M, int64_t N,
                                  rk_dtype dt, rk_stream_t stream) {
  if (G < 1 || M < 0 || N < 0 || N % G != 0 || !valid_dtype(dt)) return RK_ERR_INVALID_ARGUMENT;
  if (M == 0 || N == 0) return RK_OK;
  if (blocks == nullptr || out == nullptr) return RK_ERR_INVALID_ARGUMENT;
  if (current_device_info() == nullptr) return RK_ERR_NO_DEVICE;
  return gather_column_blocks_launch(blocks, out, G, M, N, dt,
                                     reinterpret_cast<cudaStream_t>(stream));
}

rk_status rk_device_status(rk_stream_t stream) {
  DeviceInfo* d = current_device_info();
  if (d == nullptr) return RK_ERR_NO_DEVICE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint32_t word = 0;
  cudaError_t e = cudaMemcpyAsync(&word, d->status, sizeof(word), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_status(e);
  if (word != 0) {
    e = cudaMemsetAsync(d->status, 0, sizeof(uint32_t), s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_status(e);
    return (word & ~static_cast<uint32_t>(RK_DEV_ERR_BAD_INDEX)) != 0 ? RK_ERR_TIMEOUT
                                                                      : RK_ERR_INVALID_ARGUMENT;
  }
  return RK_OK;
}

}  // extern "C"
