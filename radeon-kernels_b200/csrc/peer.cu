// peer.cu -- the multi-GPU part of the C ABI: CUDA IPC export / open of device buffers,
// and the fused compute + all-gather entry points rk_gemv_allgather / rk_gemm_allgather
// (validation, the peer table handed to the kernels; protocol in rk_peer.cuh).
//
// No counterpart in the reference, which is single-GPU.  The sharding is the one the
// N-column split implies: rank r owns the column block [r*N_block, (r+1)*N_block) of the
// output (GEMM: the same columns of B; GEMV: the same rows of the weight), computes it and
// stores it into every rank's full [M, world*N_block] output.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>
#include <map>
#include <mutex>
#include <string>

#include "rk_internal.h"
#include "rk_peer.cuh"

namespace rk {
namespace {

using GetAddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

GetAddressRangeFn address_range_fn() {
  static GetAddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetAddressRangeFn>(p);
  });
  return fn;
}

// Opened IPC allocations of this process, keyed by the handle bytes: the runtime maps an
// allocation once per process, so repeated opens share the mapping (reference counted).
struct Mapping {
  void* base = nullptr;
  int refs = 0;
};
std::mutex g_ipc_mu;
std::map<std::string, Mapping> g_ipc;

std::string handle_key(const rk_ipc_handle* h) {
  return std::string(reinterpret_cast<const char*>(h->bytes), sizeof(h->bytes));
}

constexpr uint64_t kDefaultPeerTimeoutNs = 10ull * 1000 * 1000 * 1000;

rk_status peer_targets(const rk_peer_group* g, int64_t M, int64_t N_block, PeerTargets* t) {
  if (g == nullptr || g->world < 1 || g->world > RK_PEER_MAX || g->rank < 0 ||
      g->rank >= g->world)
    return RK_ERR_INVALID_ARGUMENT;
  if (M < 1 || N_block < 1 || N_block > INT32_MAX / g->world) return RK_ERR_INVALID_ARGUMENT;
  std::memset(t, 0, sizeof(*t));
  t->rank = g->rank;
  t->world = g->world;
  t->ldo = N_block * g->world;
  t->timeout_ns = g->timeout_ns ? g->timeout_ns : kDefaultPeerTimeoutNs;
  for (int j = 0; j < g->world; ++j) {
    if (g->out[j] == nullptr || g->ctl[j] == nullptr) return RK_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(g->ctl[j]) & (alignof(PeerCtl) - 1)) != 0)
      return RK_ERR_INVALID_ARGUMENT;
    // This rank's column block inside rank j's full output (16-bit elements).
    t->out[j] = static_cast<char*>(g->out[j]) + static_cast<size_t>(g->rank) * N_block * 2;
    t->ctl[j] = g->ctl[j];
  }
  return RK_OK;
}

}  // namespace
}  // namespace rk

using namespace rk;

extern "C" {

rk_status rk_ipc_export(const void* ptr, rk_ipc_handle* handle) {
  if (ptr == nullptr || handle == nullptr) return RK_ERR_INVALID_ARGUMENT;
  if (device_ready() != RK_OK) return RK_ERR_NO_DEVICE;
  GetAddressRangeFn range = address_range_fn();
  if (range == nullptr) return RK_ERR_CUDA;
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) {
    note_error("cuMemGetAddressRange failed (CUresult " + std::to_string(static_cast<int>(r)) + ")");
    return RK_ERR_CUDA;
  }
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_status(e);
  static_assert(sizeof(h) <= sizeof(handle->bytes), "IPC handle size");
  std::memset(handle, 0, sizeof(*handle));
  std::memcpy(handle->bytes, &h, sizeof(h));
  handle->offset = static_cast<uint64_t>(reinterpret_cast<uintptr_t>(ptr) - base);
  return RK_OK;
}

rk_status rk_ipc_open(const rk_ipc_handle* handle, void** ptr) {
  if (handle == nullptr || ptr == nullptr) return RK_ERR_INVALID_ARGUMENT;
  *ptr = nullptr;
  if (device_ready() != RK_OK) return RK_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(g_ipc_mu);
  Mapping& m = g_ipc[handle_key(handle)];
  if (m.refs == 0) {
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle->bytes, sizeof(h));
    void* base = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      g_ipc.erase(handle_key(handle));
      return cuda_status(e);
    }
    m.base = base;
  }
  ++m.refs;
  *ptr = static_cast<char*>(m.base) + handle->offset;
  return RK_OK;
}

rk_status rk_ipc_close(const rk_ipc_handle* handle) {
  if (handle == nullptr) return RK_ERR_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(g_ipc_mu);
  auto it = g_ipc.find(handle_key(handle));
  if (it == g_ipc.end() || it->second.refs < 1) return RK_ERR_INVALID_ARGUMENT;
  if (--it->second.refs == 0) {
    const cudaError_t e = cudaIpcCloseMemHandle(it->second.base);
    g_ipc.erase(it);
    return cuda_status(e);
  }
  return RK_OK;
}

rk_status rk_gemv_allgather_ctl_bytes(int64_t M, int64_t N_block, int32_t world, size_t* bytes) {
  if (bytes == nullptr) return RK_ERR_INVALID_ARGUMENT;
  *bytes = 0;
  if (M < 1 || M > 32 || N_block < 1 || world < 1 || world > RK_PEER_MAX) return RK_ERR_INVALID_ARGUMENT;
  // Control block, then 8-byte packets [call parity 2][source rank][M][N_block] (rk_peer.cuh).
  const uint64_t packets = 2ull * static_cast<uint64_t>(world) * static_cast<uint64_t>(M) * static_cast<uint64_t>(N_block);
  *bytes = static_cast<size_t>(RK_PEER_CTL_BYTES + packets * 8ull);
  return RK_OK;
}

rk_status rk_gemv_allgather(const void* x, const void* weight_block, int64_t M, int64_t N_block,
                            int64_t K, rk_dtype dt, const rk_peer_group* group,
                            rk_stream_t stream) {
  if (M < 1 || M > 32 || N_block < 1 || K < 1 || (dt != RK_DTYPE_FP16 && dt != RK_DTYPE_BF16))
    return RK_ERR_INVALID_ARGUMENT;
  if (x == nullptr || weight_block == nullptr) return RK_ERR_INVALID_ARGUMENT;
  PeerTargets t;
  rk_status st = peer_targets(group, M, N_block, &t);
  if (st != RK_OK) return st;
  if (device_ready() != RK_OK) return RK_ERR_NO_DEVICE;
  if (!gemv_stream_supported(x, weight_block, nullptr, M, N_block, K)) return RK_ERR_UNSUPPORTED;
  return gemv_stream_allgather_launch(x, weight_block, M, N_block, K, dt, t,
                                      reinterpret_cast<cudaStream_t>(stream));
}

rk_status rk_gemm_allgather(const void* A, const void* B_block, int64_t M, int64_t N_block,
                            int64_t K, rk_dtype dt, const rk_peer_group* group,
                            rk_stream_t stream) {
  if (M < 1 || N_block < 1 || K < 1 || (dt != RK_DTYPE_FP16 && dt != RK_DTYPE_BF16))
    return RK_ERR_INVALID_ARGUMENT;
  if (A == nullptr || B_block == nullptr) return RK_ERR_INVALID_ARGUMENT;
  PeerTargets t;
  rk_status st = peer_targets(group, M, N_block, &t);
  if (st != RK_OK) return st;
  if (device_ready() != RK_OK) return RK_ERR_NO_DEVICE;
  // 16-byte stores into every rank's output: block columns and base addresses aligned.
  if (N_block % 8 != 0) return RK_ERR_UNSUPPORTED;
  for (int j = 0; j < t.world; ++j)
    if (!aligned16(t.out[j])) return RK_ERR_UNSUPPORTED;
  return gemm_tc2_allgather_launch(A, B_block, M, N_block, K, dt, t,
                                   reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
