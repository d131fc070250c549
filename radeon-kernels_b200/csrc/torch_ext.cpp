// torch_ext.cpp -- thin PyTorch binding over the C ABI (include/rk_kernels.h).
//
// Built twice from this one source:
//   _rk_ext    the built-in "cuda" provider of radeon_kernels (links
//              librk_kernels.so);
//   rk_sm100a  the python_extension artifact of the sm_100a kernel pack
//              (kernels linked in statically, so the SHA-256 in the pack
//              manifest covers them).
// It unwraps tensors into pointers and sizes, launches on the caller's
// current CUDA stream, and turns a non-OK rk_status into RuntimeError.
//
// Entry points mirror the reference's pybind modules:
//   gemm_out(a, b, out, variant) -> out   (wmma_gemm.hip:294-316, :326-329)
//   gemm(a, b, variant) -> new tensor
//   gemm_views(a, b, out=None, variant) -> C   (transposed views in place: rk_gemm_layout)
//   gemv_*(input, weight) -> new tensor   (native_gemv.hip:343-391)
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/extension.h>
#include <pybind11/stl.h>

#include <map>
#include <vector>
#include <mutex>
#include <utility>

#include "rk_kernels.h"

namespace {

// Split-K workspaces for rk_gemv_ex, one per (device, stream): calls on one stream are
// ordered, so they can share it; the kernels leave it zeroed after every call.  Grown
// (never shrunk) through the PyTorch caching allocator and zero-filled when created.
void* gemv_workspace(const at::Tensor& like, size_t bytes, rk_stream_t stream) {
  if (bytes == 0) return nullptr;
  static std::mutex mu;
  static std::map<std::pair<int, rk_stream_t>, at::Tensor> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto key = std::make_pair(static_cast<int>(like.get_device()), stream);
  auto it = cache.find(key);
  if (it == cache.end() || static_cast<size_t>(it->second.numel()) < bytes) {
    at::Tensor ws = at::zeros({static_cast<int64_t>(bytes)}, like.options().dtype(at::kByte));
    cache[key] = ws;
    return ws.data_ptr();
  }
  return it->second.data_ptr();
}

rk_dtype dtype_of(const at::Tensor& t, const char* name) {
  if (t.scalar_type() == at::kHalf) return RK_DTYPE_FP16;
  if (t.scalar_type() == at::kBFloat16) return RK_DTYPE_BF16;
  TORCH_CHECK(false, name, " must use torch.float16 or torch.bfloat16");
}

void check_matrix(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.dim() == 2, name, " must be rank 2");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
  dtype_of(t, name);
}

void check_rows(const at::Tensor& t, const char* name, int64_t rank) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.dim() == rank, name, " must be rank ", rank);
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
  dtype_of(t, name);
}

void check_status(rk_status st, const char* what) {
  if (st == RK_OK) return;
  const std::string detail = rk_last_error();
  TORCH_CHECK(false, what, " failed: ", rk_status_string(st),
              (st == RK_ERR_CUDA || (st == RK_ERR_UNSUPPORTED && !detail.empty())
                   ? std::string(" (") + detail + ")"
                   : std::string()));
}

rk_stream_t current_stream(const at::Tensor& t) {
  return reinterpret_cast<rk_stream_t>(c10::cuda::getCurrentCUDAStream(t.get_device()).stream());
}

at::Tensor gemm_out(const at::Tensor& a, const at::Tensor& b, at::Tensor out, int64_t variant) {
  check_matrix(a, "a");
  check_matrix(b, "b");
  check_matrix(out, "out");
  TORCH_CHECK(a.device() == b.device() && out.device() == a.device(),
              "a, b and out must be on the same device");
  TORCH_CHECK(a.scalar_type() == b.scalar_type() && out.scalar_type() == a.scalar_type(),
              "a, b and out must have the same dtype");
  TORCH_CHECK(a.size(1) == b.size(0), "incompatible GEMM dimensions");
  TORCH_CHECK(out.size(0) == a.size(0) && out.size(1) == b.size(1), "out has the wrong shape");
  c10::cuda::CUDAGuard guard(a.device());
  check_status(rk_gemm(a.data_ptr(), b.data_ptr(), out.data_ptr(), a.size(0), b.size(1),
                       a.size(1), dtype_of(a, "a"), static_cast<int>(variant), current_stream(a)),
               "rk_gemm");
  return out;
}

at::Tensor gemm(const at::Tensor& a, const at::Tensor& b, int64_t variant) {
  check_matrix(a, "a");
  check_matrix(b, "b");
  TORCH_CHECK(a.size(1) == b.size(0), "incompatible GEMM dimensions");
  auto out = at::empty({a.size(0), b.size(1)}, a.options());
  return gemm_out(a, b, out, variant);
}

// Orientation of a 2-D view: 'n' when it is row-major dense, 't' when it is the transpose
// of a row-major dense matrix (x.t() of a contiguous x), 0 otherwise.
char orientation(const at::Tensor& t) {
  if (t.is_contiguous()) return 'n';
  if (t.t().is_contiguous()) return 't';
  return 0;
}

// C = a @ b where a and b may be transposed views (rk_gemm_layout): a.t() or b.t() of a
// contiguous matrix is read in place, with no transpose copy.  out (optional) must be
// contiguous [M, N].
at::Tensor gemm_views(const at::Tensor& a, const at::Tensor& b, c10::optional<at::Tensor> out_opt,
                      int64_t variant) {
  for (const auto* t : {&a, &b}) {
    TORCH_CHECK(t->is_cuda(), "gemm operands must be CUDA tensors");
    TORCH_CHECK(t->dim() == 2, "gemm operands must be rank 2");
  }
  const rk_dtype dt = dtype_of(a, "a");
  TORCH_CHECK(a.scalar_type() == b.scalar_type(), "a and b must have the same dtype");
  TORCH_CHECK(a.device() == b.device(), "a and b must be on the same device");
  TORCH_CHECK(a.size(1) == b.size(0), "incompatible GEMM dimensions");
  const char oa = orientation(a), ob = orientation(b);
  TORCH_CHECK(oa != 0 && ob != 0, "gemm operands must be dense matrices or their transposes");
  const rk_layout layout = oa == 'n' ? (ob == 'n' ? RK_LAYOUT_NN : RK_LAYOUT_NT)
                                     : (ob == 'n' ? RK_LAYOUT_TN : RK_LAYOUT_TT);
  at::Tensor out = out_opt.has_value() ? *out_opt : at::empty({a.size(0), b.size(1)}, a.options());
  check_matrix(out, "out");
  TORCH_CHECK(out.device() == a.device() && out.scalar_type() == a.scalar_type(),
              "out must match the operands' device and dtype");
  TORCH_CHECK(out.size(0) == a.size(0) && out.size(1) == b.size(1), "out has the wrong shape");
  c10::cuda::CUDAGuard guard(a.device());
  const std::string what = "rk_gemm_layout(layout " + std::to_string(static_cast<int>(layout)) +
                           ", M " + std::to_string(a.size(0)) + ", N " + std::to_string(b.size(1)) +
                           ", K " + std::to_string(a.size(1)) + ")";
  check_status(rk_gemm_layout(a.data_ptr(), b.data_ptr(), out.data_ptr(), a.size(0), b.size(1),
                              a.size(1), layout, dt, static_cast<int>(variant), current_stream(a)),
               what.c_str());
  return out;
}

at::Tensor gemv_out(const at::Tensor& x, const at::Tensor& weight, at::Tensor out,
                    int64_t variant) {
  check_matrix(x, "input");
  check_matrix(weight, "weight");
  check_matrix(out, "out");
  TORCH_CHECK(x.device() == weight.device() && out.device() == x.device(),
              "input, weight and out must use the same device");
  TORCH_CHECK(x.scalar_type() == weight.scalar_type() && out.scalar_type() == x.scalar_type(),
              "input, weight and out must use the same dtype");
  TORCH_CHECK(x.size(0) > 0 && x.size(0) <= 32, "input M must be in [1, 32]");
  TORCH_CHECK(x.size(1) > 0 && weight.size(0) > 0, "N and K must be positive");
  TORCH_CHECK(x.size(1) == weight.size(1), "input and weight must share K");
  TORCH_CHECK(out.size(0) == x.size(0) && out.size(1) == weight.size(0), "out has the wrong shape");
  c10::cuda::CUDAGuard guard(x.device());
  const rk_dtype dt = dtype_of(x, "input");
  const rk_stream_t stream = current_stream(x);
  size_t ws_bytes = 0;
  check_status(rk_gemv_workspace_size(x.size(0), weight.size(0), x.size(1), dt,
                                      static_cast<int>(variant), &ws_bytes),
               "rk_gemv_workspace_size");
  void* ws = gemv_workspace(x, ws_bytes, stream);
  check_status(rk_gemv_ex(x.data_ptr(), weight.data_ptr(), out.data_ptr(), x.size(0),
                          weight.size(0), x.size(1), dt, static_cast<int>(variant), ws, ws_bytes,
                          stream),
               "rk_gemv");
  return out;
}

at::Tensor gemv(const at::Tensor& x, const at::Tensor& weight, int64_t variant) {
  check_matrix(x, "input");
  check_matrix(weight, "weight");
  auto out = at::empty({x.size(0), weight.size(0)}, x.options());
  return gemv_out(x, weight, out, variant);
}

at::Tensor gemv_stream(const at::Tensor& x, const at::Tensor& weight) {
  return gemv(x, weight, RK_GEMV_STREAM);
}

at::Tensor gemv_scalar(const at::Tensor& x, const at::Tensor& weight) {
  return gemv(x, weight, RK_GEMV_SCALAR);
}

at::Tensor gather_column_blocks(const at::Tensor& blocks, at::Tensor out) {
  TORCH_CHECK(blocks.is_cuda() && blocks.dim() == 3 && blocks.is_contiguous(),
              "blocks must be a contiguous CUDA tensor [G, M, N/G]");
  check_matrix(out, "out");
  TORCH_CHECK(blocks.device() == out.device(), "blocks and out must use the same device");
  TORCH_CHECK(out.scalar_type() == blocks.scalar_type(), "dtype mismatch");
  TORCH_CHECK(out.size(0) == blocks.size(1) && out.size(1) == blocks.size(0) * blocks.size(2),
              "out must be [M, G * N/G]");
  c10::cuda::CUDAGuard guard(out.device());
  check_status(rk_gather_column_blocks(blocks.data_ptr(), out.data_ptr(), blocks.size(0),
                                       out.size(0), out.size(1), dtype_of(out, "out"),
                                       current_stream(out)),
               "rk_gather_column_blocks");
  return out;
}

// Fused compute + all-gather (rk_gemv_allgather / rk_gemm_allgather).  `out` is this rank's
// full output (a view into its exchange buffer, entry `rank` of out_ptrs); out_ptrs and
// ctl_ptrs list every rank's output and control block as mapped in this process.
rk_peer_group peer_group(const at::Tensor& out, const std::vector<int64_t>& out_ptrs,
                         const std::vector<int64_t>& ctl_ptrs, int64_t rank, int64_t timeout_ns) {
  const int64_t world = static_cast<int64_t>(out_ptrs.size());
  TORCH_CHECK(world >= 1 && world <= RK_PEER_MAX, "the group must have 1 to ", RK_PEER_MAX, " ranks");
  TORCH_CHECK(static_cast<int64_t>(ctl_ptrs.size()) == world, "one control block per rank");
  TORCH_CHECK(rank >= 0 && rank < world, "rank out of range");
  TORCH_CHECK(out_ptrs[rank] == reinterpret_cast<int64_t>(out.data_ptr()),
              "out must be this rank's entry of out_ptrs");
  rk_peer_group g{};
  g.rank = static_cast<int32_t>(rank);
  g.world = static_cast<int32_t>(world);
  for (int64_t j = 0; j < world; ++j) {
    g.out[j] = reinterpret_cast<void*>(out_ptrs[j]);
    g.ctl[j] = reinterpret_cast<void*>(ctl_ptrs[j]);
  }
  g.timeout_ns = static_cast<uint64_t>(timeout_ns);
  return g;
}

at::Tensor gemv_allgather(const at::Tensor& x, const at::Tensor& weight_block, at::Tensor out,
                          const std::vector<int64_t>& out_ptrs, const std::vector<int64_t>& ctl_ptrs,
                          int64_t rank, int64_t timeout_ns) {
  check_matrix(x, "input");
  check_matrix(weight_block, "weight");
  check_matrix(out, "out");
  TORCH_CHECK(x.device() == weight_block.device() && out.device() == x.device(),
              "input, weight and out must use the same device");
  TORCH_CHECK(x.scalar_type() == weight_block.scalar_type() && out.scalar_type() == x.scalar_type(),
              "input, weight and out must use the same dtype");
  TORCH_CHECK(x.size(0) > 0 && x.size(0) <= 32, "input M must be in [1, 32]");
  TORCH_CHECK(x.size(1) == weight_block.size(1), "input and weight must share K");
  const rk_peer_group g = peer_group(out, out_ptrs, ctl_ptrs, rank, timeout_ns);
  TORCH_CHECK(out.size(0) == x.size(0) && out.size(1) == weight_block.size(0) * g.world,
              "out must be [M, world * N_block]");
  c10::cuda::CUDAGuard guard(x.device());
  check_status(rk_gemv_allgather(x.data_ptr(), weight_block.data_ptr(), x.size(0),
                                 weight_block.size(0), x.size(1), dtype_of(x, "input"), &g,
                                 current_stream(x)),
               "rk_gemv_allgather");
  return out;
}

at::Tensor gemm_allgather(const at::Tensor& a, const at::Tensor& b_block, at::Tensor out,
                          const std::vector<int64_t>& out_ptrs, const std::vector<int64_t>& ctl_ptrs,
                          int64_t rank, int64_t timeout_ns) {
  check_matrix(a, "a");
  check_matrix(b_block, "b");
  check_matrix(out, "out");
  TORCH_CHECK(a.device() == b_block.device() && out.device() == a.device(),
              "a, b and out must use the same device");
  TORCH_CHECK(a.scalar_type() == b_block.scalar_type() && out.scalar_type() == a.scalar_type(),
              "a, b and out must use the same dtype");
  TORCH_CHECK(a.size(1) == b_block.size(0), "a and b must share K");
  const rk_peer_group g = peer_group(out, out_ptrs, ctl_ptrs, rank, timeout_ns);
  TORCH_CHECK(out.size(0) == a.size(0) && out.size(1) == b_block.size(1) * g.world,
              "out must be [M, world * N_block]");
  c10::cuda::CUDAGuard guard(a.device());
  check_status(rk_gemm_allgather(a.data_ptr(), b_block.data_ptr(), a.size(0), b_block.size(1),
                                 a.size(1), dtype_of(a, "a"), &g, current_stream(a)),
               "rk_gemm_allgather");
  return out;
}

// Paged decode attention: the reference's argument order
// (query, key_cache, value_cache, block_tables, context_lengths, scale) -> new output.
at::Tensor paged_attention_decode(const at::Tensor& query, const at::Tensor& key_cache,
                                  const at::Tensor& value_cache, const at::Tensor& block_tables,
                                  const at::Tensor& context_lengths, double scale) {
  check_rows(query, "query", 3);
  check_rows(key_cache, "key_cache", 4);
  check_rows(value_cache, "value_cache", 4);
  TORCH_CHECK(block_tables.is_cuda() && block_tables.dim() == 2 && block_tables.is_contiguous(),
              "block_tables must be a contiguous CUDA tensor [batch, max_blocks]");
  TORCH_CHECK(context_lengths.is_cuda() && context_lengths.dim() == 1 && context_lengths.is_contiguous(),
              "context_lengths must be a contiguous CUDA tensor [batch]");
  TORCH_CHECK(block_tables.scalar_type() == context_lengths.scalar_type() &&
                  (block_tables.scalar_type() == at::kInt || block_tables.scalar_type() == at::kLong),
              "index tensors must share int32 or int64");
  TORCH_CHECK(query.scalar_type() == key_cache.scalar_type() &&
                  key_cache.scalar_type() == value_cache.scalar_type(),
              "query and caches must share a dtype");
  TORCH_CHECK(key_cache.sizes() == value_cache.sizes(), "K/V cache shapes must match");
  TORCH_CHECK(query.device() == key_cache.device() && query.device() == value_cache.device() &&
                  query.device() == block_tables.device() && query.device() == context_lengths.device(),
              "all inputs must use the query's device");
  const int64_t batch = query.size(0), hq = query.size(1), d = query.size(2);
  TORCH_CHECK(block_tables.size(0) == batch && context_lengths.size(0) == batch,
              "index tensors must have one row per sequence");
  TORCH_CHECK(key_cache.size(3) == d, "query and cache head dimensions must match");
  c10::cuda::CUDAGuard guard(query.device());
  auto out = at::empty_like(query);
  size_t ws_bytes = 0;
  check_status(rk_paged_attention_workspace_size(batch, hq, key_cache.size(2), d, key_cache.size(1),
                                                 block_tables.size(1), &ws_bytes),
               "rk_paged_attention_workspace_size");
  at::Tensor ws;
  if (ws_bytes > 0) ws = at::empty({static_cast<int64_t>(ws_bytes)}, query.options().dtype(at::kByte));
  check_status(rk_paged_attention_decode(
                   query.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(),
                   block_tables.data_ptr(), context_lengths.data_ptr(), out.data_ptr(), batch, hq,
                   key_cache.size(2), d, key_cache.size(0), key_cache.size(1), block_tables.size(1),
                   static_cast<float>(scale), dtype_of(query, "query"),
                   block_tables.scalar_type() == at::kInt ? 32 : 64,
                   ws_bytes > 0 ? ws.data_ptr() : nullptr, ws_bytes, current_stream(query)),
               "rk_paged_attention_decode");
  return out;
}

// Fused FFN-up + SwiGLU (rk_gemm_swiglu): b is [K, 2N] = [gate | up], returns [M, N].
at::Tensor gemm_swiglu(const at::Tensor& a, const at::Tensor& b, int64_t variant) {
  check_matrix(a, "a");
  check_matrix(b, "b");
  TORCH_CHECK(a.device() == b.device() && a.scalar_type() == b.scalar_type(),
              "a and b must share device and dtype");
  TORCH_CHECK(a.size(1) == b.size(0), "incompatible GEMM dimensions");
  TORCH_CHECK(b.size(1) % 2 == 0, "b must hold the gate and up projections side by side");
  c10::cuda::CUDAGuard guard(a.device());
  const int64_t n = b.size(1) / 2;
  auto out = at::empty({a.size(0), n}, a.options());
  check_status(rk_gemm_swiglu(a.data_ptr(), b.data_ptr(), out.data_ptr(), a.size(0), n,
                              a.size(1), dtype_of(a, "a"), static_cast<int>(variant),
                              current_stream(a)),
               "rk_gemm_swiglu");
  return out;
}

// Decode neighbours: the reference's pybind names and signatures
// (benchmarks/llm_ops/native_llm_ops.hip:306-353, :397-416), outputs allocated here.
at::Tensor silu_mul(const at::Tensor& gate, const at::Tensor& up) {
  check_rows(gate, "gate", 2);
  check_rows(up, "up", 2);
  TORCH_CHECK(gate.device() == up.device() && gate.scalar_type() == up.scalar_type(),
              "gate and up must share device and dtype");
  TORCH_CHECK(gate.sizes() == up.sizes(), "up shape must match gate");
  c10::cuda::CUDAGuard guard(gate.device());
  auto out = at::empty_like(gate);
  check_status(rk_silu_mul(gate.data_ptr(), up.data_ptr(), out.data_ptr(), gate.size(0),
                           gate.size(1), dtype_of(gate, "gate"), current_stream(gate)),
               "rk_silu_mul");
  return out;
}

at::Tensor rms_norm(const at::Tensor& input, const at::Tensor& weight, double eps) {
  check_rows(input, "input", 2);
  check_rows(weight, "weight", 1);
  TORCH_CHECK(input.device() == weight.device() && input.scalar_type() == weight.scalar_type(),
              "input and weight must share device and dtype");
  TORCH_CHECK(weight.numel() == input.size(1), "weight must match hidden size");
  c10::cuda::CUDAGuard guard(input.device());
  auto out = at::empty_like(input);
  check_status(rk_rms_norm(input.data_ptr(), weight.data_ptr(), out.data_ptr(), input.size(0),
                           input.size(1), static_cast<float>(eps), dtype_of(input, "input"),
                           current_stream(input)),
               "rk_rms_norm");
  return out;
}

std::vector<at::Tensor> add_rms_norm(const at::Tensor& input, const at::Tensor& residual,
                                     const at::Tensor& weight, double eps) {
  check_rows(input, "input", 2);
  check_rows(residual, "residual", 2);
  check_rows(weight, "weight", 1);
  TORCH_CHECK(input.device() == residual.device() && input.device() == weight.device(),
              "input, residual and weight must share a device");
  TORCH_CHECK(input.scalar_type() == residual.scalar_type() &&
                  input.scalar_type() == weight.scalar_type(),
              "input, residual and weight must share a dtype");
  TORCH_CHECK(input.sizes() == residual.sizes(), "residual shape must match input");
  TORCH_CHECK(weight.numel() == input.size(1), "weight must match hidden size");
  c10::cuda::CUDAGuard guard(input.device());
  auto out = at::empty_like(input);
  auto residual_out = at::empty_like(input);
  check_status(rk_add_rms_norm(input.data_ptr(), residual.data_ptr(), weight.data_ptr(),
                               out.data_ptr(), residual_out.data_ptr(), input.size(0),
                               input.size(1), static_cast<float>(eps), dtype_of(input, "input"),
                               current_stream(input)),
               "rk_add_rms_norm");
  return {out, residual_out};
}

// Prefill attention (rk_sdpa): query [B, Hq, S, D], key/value [B, Hkv, S, D].
at::Tensor sdpa(const at::Tensor& query, const at::Tensor& key, const at::Tensor& value,
                bool is_causal, double scale) {
  check_rows(query, "query", 4);
  check_rows(key, "key", 4);
  check_rows(value, "value", 4);
  TORCH_CHECK(query.device() == key.device() && key.device() == value.device(),
              "query, key and value must share a device");
  TORCH_CHECK(query.scalar_type() == key.scalar_type() && key.scalar_type() == value.scalar_type(),
              "query, key and value must share a dtype");
  TORCH_CHECK(key.sizes() == value.sizes(), "key and value must have the same shape");
  TORCH_CHECK(query.size(0) == key.size(0) && query.size(2) == key.size(2) &&
                  query.size(3) == key.size(3),
              "query and key must share batch, sequence and head_dim");
  c10::cuda::CUDAGuard guard(query.device());
  auto out = at::empty_like(query);
  check_status(rk_sdpa(query.data_ptr(), key.data_ptr(), value.data_ptr(), out.data_ptr(),
                       query.size(0), query.size(1), key.size(1), query.size(2), query.size(3),
                       is_causal ? 1 : 0, static_cast<float>(scale), dtype_of(query, "query"),
                       current_stream(query)),
               "rk_sdpa");
  return out;
}

// ------------------------------------------------------------------ backward passes
std::vector<at::Tensor> silu_mul_backward(const at::Tensor& grad, const at::Tensor& gate,
                                          const at::Tensor& up) {
  for (const auto& [t, name] : {std::pair<const at::Tensor*, const char*>{&grad, "grad"},
                                {&gate, "gate"}, {&up, "up"}}) {
    check_rows(*t, name, 2);
    TORCH_CHECK(t->device() == gate.device() && t->scalar_type() == gate.scalar_type(),
                "grad, gate and up must share device and dtype");
    TORCH_CHECK(t->sizes() == gate.sizes(), "grad, gate and up must have one shape");
  }
  c10::cuda::CUDAGuard guard(gate.device());
  auto grad_gate = at::empty_like(gate);
  auto grad_up = at::empty_like(gate);
  check_status(rk_silu_mul_backward(grad.data_ptr(), gate.data_ptr(), up.data_ptr(),
                                    grad_gate.data_ptr(), grad_up.data_ptr(), gate.size(0),
                                    gate.size(1), dtype_of(gate, "gate"), current_stream(gate)),
               "rk_silu_mul_backward");
  return {grad_gate, grad_up};
}

// Shared by rms_norm_backward / add_rms_norm_backward: the weight gradient (when wanted)
// and its workspace.
struct WeightGrad {
  at::Tensor grad, workspace;
};

WeightGrad weight_grad_buffers(const at::Tensor& x, const at::Tensor& weight, bool want) {
  WeightGrad w;
  if (!want) return w;
  w.grad = at::empty_like(weight);
  size_t bytes = 0;
  check_status(rk_rms_norm_backward_workspace_size(x.size(0), x.size(1), &bytes),
               "rk_rms_norm_backward_workspace_size");
  if (bytes > 0) w.workspace = at::empty({static_cast<int64_t>(bytes)}, x.options().dtype(at::kByte));
  return w;
}

// Returns [grad_input, grad_weight]; grad_weight is undefined (None) when not wanted.
std::vector<at::Tensor> rms_norm_backward(const at::Tensor& grad, const at::Tensor& input,
                                          const at::Tensor& weight, double eps,
                                          bool weight_grad) {
  check_rows(grad, "grad", 2);
  check_rows(input, "input", 2);
  check_rows(weight, "weight", 1);
  TORCH_CHECK(grad.sizes() == input.sizes(), "grad shape must match input");
  TORCH_CHECK(grad.device() == input.device() && weight.device() == input.device() &&
                  grad.scalar_type() == input.scalar_type() &&
                  weight.scalar_type() == input.scalar_type(),
              "grad, input and weight must share device and dtype");
  TORCH_CHECK(weight.numel() == input.size(1), "weight must match hidden size");
  c10::cuda::CUDAGuard guard(input.device());
  auto grad_input = at::empty_like(input);
  WeightGrad w = weight_grad_buffers(input, weight, weight_grad);
  check_status(rk_rms_norm_backward(grad.data_ptr(), input.data_ptr(), weight.data_ptr(),
                                    grad_input.data_ptr(),
                                    w.grad.defined() ? w.grad.data_ptr() : nullptr, input.size(0),
                                    input.size(1), static_cast<float>(eps),
                                    dtype_of(input, "input"),
                                    w.workspace.defined() ? w.workspace.data_ptr() : nullptr,
                                    w.workspace.defined() ? w.workspace.numel() : 0,
                                    current_stream(input)),
               "rk_rms_norm_backward");
  return {grad_input, w.grad};
}

// Returns [grad_input, grad_residual, grad_weight] (grad_weight undefined when not wanted);
// grad_residual_out may be None (no gradient flows into residual_out).
std::vector<at::Tensor> add_rms_norm_backward(const at::Tensor& grad,
                                              c10::optional<at::Tensor> grad_residual_out,
                                              const at::Tensor& residual_out,
                                              const at::Tensor& weight, double eps,
                                              bool weight_grad) {
  check_rows(grad, "grad", 2);
  check_rows(residual_out, "residual_out", 2);
  check_rows(weight, "weight", 1);
  TORCH_CHECK(grad.sizes() == residual_out.sizes(), "grad shape must match residual_out");
  TORCH_CHECK(grad.device() == residual_out.device() && weight.device() == residual_out.device() &&
                  grad.scalar_type() == residual_out.scalar_type() &&
                  weight.scalar_type() == residual_out.scalar_type(),
              "grad, residual_out and weight must share device and dtype");
  TORCH_CHECK(weight.numel() == residual_out.size(1), "weight must match hidden size");
  const void* dres = nullptr;
  if (grad_residual_out.has_value() && grad_residual_out->defined()) {
    check_rows(*grad_residual_out, "grad_residual_out", 2);
    TORCH_CHECK(grad_residual_out->sizes() == residual_out.sizes() &&
                    grad_residual_out->device() == residual_out.device() &&
                    grad_residual_out->scalar_type() == residual_out.scalar_type(),
                "grad_residual_out must match residual_out");
    dres = grad_residual_out->data_ptr();
  }
  c10::cuda::CUDAGuard guard(residual_out.device());
  auto grad_input = at::empty_like(residual_out);
  auto grad_residual = at::empty_like(residual_out);
  WeightGrad w = weight_grad_buffers(residual_out, weight, weight_grad);
  check_status(rk_add_rms_norm_backward(
                   grad.data_ptr(), dres, residual_out.data_ptr(), weight.data_ptr(),
                   grad_input.data_ptr(), grad_residual.data_ptr(),
                   w.grad.defined() ? w.grad.data_ptr() : nullptr, residual_out.size(0),
                   residual_out.size(1), static_cast<float>(eps),
                   dtype_of(residual_out, "residual_out"),
                   w.workspace.defined() ? w.workspace.data_ptr() : nullptr,
                   w.workspace.defined() ? w.workspace.numel() : 0, current_stream(residual_out)),
               "rk_add_rms_norm_backward");
  return {grad_input, grad_residual, w.grad};
}

int64_t device_status() {
  return static_cast<int64_t>(rk_device_status(
      reinterpret_cast<rk_stream_t>(c10::cuda::getCurrentCUDAStream().stream())));
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "B200 (sm_100a) GEMM/GEMV kernels behind the rk_kernels C ABI";
  m.def("gemm_out", &gemm_out, "C = A @ B into the caller's output", py::arg("a"), py::arg("b"),
        py::arg("out"), py::arg("variant") = 0);
  m.def("gemm", &gemm, "C = A @ B", py::arg("a"), py::arg("b"), py::arg("variant") = 0);
  m.def("gemm_views", &gemm_views, "C = A @ B with A and/or B transposed views read in place",
        py::arg("a"), py::arg("b"), py::arg("out") = py::none(), py::arg("variant") = 0);
  m.def("gemv", &gemv, "out = x @ weight.T", py::arg("input"), py::arg("weight"),
        py::arg("variant") = 0);
  m.def("gemv_out", &gemv_out, "out = x @ weight.T into the caller's output", py::arg("input"),
        py::arg("weight"), py::arg("out"), py::arg("variant") = 0);
  m.def("gemv_stream", &gemv_stream, "128-bit weight-streaming GEMV (K % 8 == 0, 16B aligned)");
  // The reference pack's GEMV entrypoint names (benchmarks/gemv/native_gemv.hip:381-391):
  // its dispatch entries launch gemv_wave1 / gemv_wave2 (one or two outputs per wavefront)
  // with no arguments beyond (input, weight).  Here the outputs-per-wave choice has no
  // counterpart -- the automatic kernel choice runs -- so a manifest naming either resolves.
  m.def("gemv_wave1", [](const at::Tensor& x, const at::Tensor& w) { return gemv(x, w, RK_GEMV_AUTO); },
        "out = x @ weight.T (reference entrypoint name)", py::arg("input"), py::arg("weight"));
  m.def("gemv_wave2", [](const at::Tensor& x, const at::Tensor& w) { return gemv(x, w, RK_GEMV_AUTO); },
        "out = x @ weight.T (reference entrypoint name)", py::arg("input"), py::arg("weight"));
  m.def("gemv_scalar", &gemv_scalar, "generic GEMV (any K, any alignment)");
  m.def("gather_column_blocks", &gather_column_blocks, "[G,M,N/G] blocks -> row-major [M,N]");
  m.def("gemv_allgather", &gemv_allgather,
        "row-sharded x @ W.T with the output all-gather fused into the kernel (peer stores)",
        py::arg("input"), py::arg("weight_block"), py::arg("out"), py::arg("out_ptrs"),
        py::arg("ctl_ptrs"), py::arg("rank"), py::arg("timeout_ns") = 0);
  m.def("gemm_allgather", &gemm_allgather,
        "column-sharded A @ B with the output all-gather fused into the kernel (peer stores)",
        py::arg("a"), py::arg("b_block"), py::arg("out"), py::arg("out_ptrs"),
        py::arg("ctl_ptrs"), py::arg("rank"), py::arg("timeout_ns") = 0);
  m.def("paged_attention_decode", &paged_attention_decode, "decode attention over a paged K/V cache",
        py::arg("query"), py::arg("key_cache"), py::arg("value_cache"), py::arg("block_tables"),
        py::arg("context_lengths"), py::arg("scale"));
  m.def("gemm_swiglu", &gemm_swiglu, "silu(a @ b[:, :N]) * (a @ b[:, N:])", py::arg("a"),
        py::arg("b"), py::arg("variant") = 0);
  m.def("silu_mul", &silu_mul, "silu(gate) * up", py::arg("gate"), py::arg("up"));
  m.def("rms_norm", &rms_norm, "row RMS normalisation", py::arg("input"), py::arg("weight"),
        py::arg("eps"));
  m.def("add_rms_norm", &add_rms_norm, "residual add + row RMS normalisation -> [out, residual_out]",
        py::arg("input"), py::arg("residual"), py::arg("weight"), py::arg("eps"));
  m.def("sdpa", &sdpa, "scaled dot-product self-attention (prefill)", py::arg("query"),
        py::arg("key"), py::arg("value"), py::arg("is_causal"), py::arg("scale"));
  m.def("silu_mul_backward", &silu_mul_backward, "gradients of silu(gate) * up -> [grad_gate, grad_up]",
        py::arg("grad"), py::arg("gate"), py::arg("up"));
  m.def("rms_norm_backward", &rms_norm_backward, "rms_norm gradients -> [grad_input, grad_weight]",
        py::arg("grad"), py::arg("input"), py::arg("weight"), py::arg("eps"),
        py::arg("weight_grad") = true);
  m.def("add_rms_norm_backward", &add_rms_norm_backward,
        "add_rms_norm gradients -> [grad_input, grad_residual, grad_weight]", py::arg("grad"),
        py::arg("grad_residual_out"), py::arg("residual_out"), py::arg("weight"), py::arg("eps"),
        py::arg("weight_grad") = true);
  m.def("paged_attention_set_path", [](int path) { rk_paged_attention_set_path(path); });
  m.def("norm_backward_set_ctas_per_sm", [](int c) { rk_norm_backward_set_ctas_per_sm(c); });
  m.def("device_status", &device_status, "read and clear the device status word");
  m.def("set_wait_timeout_ns", [](uint64_t ns) { rk_set_wait_timeout_ns(ns); });
  m.def("debug_inject_stall", [](bool on) { rk_debug_inject_stall(on ? 1 : 0); });
  m.def("gemv_set_tuning", [](int rows, int ks) { rk_gemv_set_tuning(rows, ks); });
  m.def("gemm_set_tile_n", [](int bn) { rk_gemm_set_tile_n(bn); });
  m.def("launch_count", []() { return rk_launch_count(); });
  m.def("variant_name", [](int op, int v) { return std::string(rk_variant_name(op, v)); });
  m.def("abi_version", []() { return rk_abi_version(); });
}
