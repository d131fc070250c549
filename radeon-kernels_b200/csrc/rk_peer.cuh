// rk_peer.cuh -- the exchange protocol of the fused compute + all-gather kernels
// (rk_gemv_allgather, rk_gemm_allgather): every rank's kernel stores its column block of
// the result straight into every rank's full output through peer pointers (CUDA IPC
// mappings over NVLink / NVSwitch, plain st.global -- no TMA and no multicast touches
// peer memory), and two flag rounds in each rank's control block order the calls:
//
//   ready[j]   written by rank j when its call e starts (after griddepcontrol.wait, so every
//              earlier kernel of its stream -- the consumers of call e-1's output -- has
//              completed): from then on the other ranks may overwrite rank j's output.
//   arrive[j]  written by rank j once every store of its call e into this rank's output has
//              been made visible (per CTA: a barrier, then one thread's system-scope fence
//              and a grid-wide count -- the grid-synchronisation pattern; the last CTA of
//              the grid sends it).
//   epoch      calls completed by this rank on this control block; written only by this
//              rank, read at the start of the next call (which begins after it in stream
//              order), so all ranks agree on the call number without host involvement and
//              a captured CUDA graph replays correctly.
//   done_ctas  CTAs of the running call that have finished storing; the last resets it.
//
// Two ways to move the data.  The GEMM (large blocks) stores every finished tile into every
// rank's output from the CTA that made it, while the next tile accumulates, and ends with
// peer_finish: the last CTA of each rank waits until every rank's arrive[] reaches the call's
// epoch.  The GEMV (a block of at most 32 x N elements, a few microseconds of work) cannot
// afford that fence and flag round trip: every CTA sends its rows to the peers as 8-byte
// packets that carry the call number (peer_stage), and polls its rows of every peer's block
// from its own staging area, so data and "arrived" travel in one store and no fence is
// needed.  Its slots alternate by call parity: a peer's slot of parity e & 1 was last read
// in that peer's call e - 2, so a rank may send once every peer has started call e - 1
// (ready[]), which in steady state holds already.  Either way, when the kernel completes the
// local full output is complete.  Every wait is bounded (time and iteration count); a wait
// that runs out sets RK_DEV_ERR_TIMEOUT_PEER in the status word and the kernel finishes
// without the missing data (the group must then be rebuilt).
#pragma once

#include <cstdint>

#include "rk_device.cuh"

namespace rk {

constexpr int kPeerMax = 8;
constexpr uint32_t RK_DEV_ERR_TIMEOUT_PEER = 1u << 5;

// One per rank, at the start of that rank's control allocation (RK_PEER_CTL_BYTES).
struct __align__(256) PeerCtl {
  uint32_t ready[kPeerMax];
  uint32_t pad0[24];
  uint32_t arrive[kPeerMax];
  uint32_t pad1[24];
  uint32_t epoch;
  uint32_t done_ctas;
  uint32_t pad2[62];
};
static_assert(sizeof(PeerCtl) == 512, "PeerCtl layout");

// Kernel-side view of a group: out[j] is rank j's full output as mapped in this process,
// already advanced to this rank's column block; ctl[j] rank j's control block.
template <typename T>
struct PeerOut {
  T* out[kPeerMax];
  PeerCtl* ctl[kPeerMax];
  int64_t ldo;  // row stride of the full output (elements)
  int rank;
  int world;
  uint64_t timeout_ns;
  uint32_t* status;
};

// Relaxed system-scope store: after a fence it forms the release pattern (fence, then a
// morally strong store), so the ranks' flags go out back to back instead of each waiting
// for the previous remote store to be acknowledged, as a release store per flag would.
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_acq_rel_sys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// 8-byte packets of the GEMV exchange: a single naturally aligned 64-bit access, so a reader
// sees either the old packet or the new one whole.
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// rk_gemv_allgather's staging area, right after a rank's control block: 8-byte packets
// [call parity 2][source rank world][M][N_block], each {value bits (low 32), call number
// (high 32)}.
__device__ __forceinline__ uint64_t* peer_stage(PeerCtl* ctl) {
  return reinterpret_cast<uint64_t*>(reinterpret_cast<char*>(ctl) + sizeof(PeerCtl));
}

__device__ __forceinline__ uint32_t ld_relaxed_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Epoch number of the call this kernel runs (1 for the first call on a control block).
template <typename T>
__device__ __forceinline__ uint32_t peer_call_epoch(const PeerOut<T>& p) {
  return ld_relaxed_gpu(&p.ctl[p.rank]->epoch) + 1u;
}

// Tells every rank that this rank's call `e` has started (one thread): one fence, then the
// flags.  Nothing of this call precedes it that the others read; what the flag stands for --
// every earlier reader of this rank's output has finished -- holds before the kernel passed
// its dependency wait.
template <typename T>
__device__ __forceinline__ void peer_announce(const PeerOut<T>& p, uint32_t e) {
  fence_acq_rel_sys();
  for (int j = 0; j < p.world; ++j) st_relaxed_sys(&p.ctl[j]->ready[p.rank], e);
}

// Publishes this rank's arrival for call `e` to every rank (one thread, after a system-scope
// fence that follows every store of the call into the peers' outputs).
template <typename T>
__device__ __forceinline__ void peer_publish_arrival(const PeerOut<T>& p, uint32_t e) {
  for (int j = 0; j < p.world; ++j) st_relaxed_sys(&p.ctl[j]->arrive[p.rank], e);
}

// Bounded wait until flags[j] has reached `e` for every rank j < world (one thread).
__device__ __forceinline__ bool peer_wait_all(const uint32_t* flags, int world, uint32_t e,
                                              uint64_t timeout_ns) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 0; it < (1u << 30); ++it) {
    bool all = true;
    for (int j = 0; j < world; ++j)
      all &= static_cast<int32_t>(ld_acquire_sys(&flags[j]) - e) >= 0;
    if (all) return true;
    if ((it & 15u) == 15u && globaltimer_ns() - t0 > timeout_ns) return false;
  }
  return false;
}

// Bounded wait until every rank has started call `e` (one thread); afterwards this rank may
// store into every rank's output.
template <typename T>
__device__ __forceinline__ bool peer_wait_ready(const PeerOut<T>& p, uint32_t e) {
  const bool ok = peer_wait_all(p.ctl[p.rank]->ready, p.world, e, p.timeout_ns);
  if (!ok) atomicOr(p.status, RK_DEV_ERR_TIMEOUT_PEER);
  return ok;
}

// End of a CTA's part of call `e`: called by one thread after a CTA-wide barrier that follows
// every peer store of the CTA; its system-scope fence makes those stores visible before the
// count.  The last CTA of the grid publishes this rank's arrival to every rank, waits for
// every rank's, and advances the epoch.
template <typename T>
__device__ __forceinline__ void peer_finish(const PeerOut<T>& p, uint32_t e, uint32_t grid_ctas) {
  PeerCtl* mine = p.ctl[p.rank];
  __threadfence_system();
  const uint32_t before = atomicAdd(&mine->done_ctas, 1u);
  if (before != grid_ctas - 1u) return;
  __threadfence_system();  // acquire side of the count: every CTA's stores precede the flags
  mine->done_ctas = 0u;    // the next call starts after this kernel completes
  peer_publish_arrival(p, e);
  if (!peer_wait_all(mine->arrive, p.world, e, p.timeout_ns)) atomicOr(p.status, RK_DEV_ERR_TIMEOUT_PEER);
  *reinterpret_cast<volatile uint32_t*>(&mine->epoch) = e;
}

}  // namespace rk
