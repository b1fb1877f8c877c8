// peer_protocol.cuh — the cross-GPU K-split protocol's mailbox layout and
// flag primitives, shared by the stand-alone push / reduce kernels
// (b2g_peer.cu) and the GEMM engine's fused exchange (gemm_engine.cuh).
//
// A mailbox (one per rank, device memory, opened by the others through CUDA
// IPC) for partials of `elems` floats and `world` ranks holds:
//   ready[nchunk][world] u64     chunk c of rank r landed for epoch e (root's mailbox)
//   consumed[nchunk] u64         the root has read chunk c of epoch e (each rank's own)
//   count u64                    the fused exchange's grid-wide arrival count (own)
//   landing[2][world][elems]     the non-root partials, slot = epoch % 2 (root's)
// Chunks are kPeerChunk floats.  Flags only grow (epochs), so nothing is reset.
#pragma once
#include <cstdint>

#include "ptx_sm100.cuh"

namespace b2g {

constexpr int kPeerChunk = 1024;      // floats per chunk
constexpr int kPeerMaxRanks = 16;
enum : int { kErrPeerCredit = 0x201, kErrPeerReady = 0x202, kErrPeerGrid = 0x203 };

struct PeerLayout {
  int64_t nchunk, ready_off, consumed_off, count_off, flag_bytes, landing_off, slot_stride, total;
};

__host__ __device__ inline PeerLayout peer_layout(int64_t elems, int world) {
  PeerLayout l;
  l.nchunk = (elems + kPeerChunk - 1) / kPeerChunk;
  l.ready_off = 0;
  l.consumed_off = l.nchunk * world * 8;
  l.count_off = l.consumed_off + l.nchunk * 8;
  l.flag_bytes = ((l.count_off + 8 + 255) / 256) * 256;
  l.landing_off = l.flag_bytes;
  l.slot_stride = ((elems * 4 + 255) / 256) * 256;   // bytes per (slot, rank) region
  l.total = l.landing_off + 2 * world * l.slot_stride;
  return l;
}

#ifdef __CUDACC__
__device__ __forceinline__ uint64_t peer_ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void peer_st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Spin (with a short sleep) until *flag >= want; false after limit_ns.
__device__ __forceinline__ bool peer_wait_at_least(const uint64_t* flag, uint64_t want,
                                                   long long limit_ns) {
  if (peer_ld_acquire_sys(flag) >= want) return true;
  const uint64_t t0 = ptx::globaltimer_ns();
  for (unsigned spin = 0; peer_ld_acquire_sys(flag) < want; ++spin) {
    if (ptx::globaltimer_ns() - t0 > static_cast<uint64_t>(limit_ns)) return false;
    if (spin > 64) __nanosleep(32);   // poll tight first: the flag usually lands within ~1 us
  }
  return true;
}
#endif

}  // namespace b2g
