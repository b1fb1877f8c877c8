// peer_protocol.cuh — the cross-GPU K-split protocol's mailbox layout and
// flag primitives, shared by the stand-alone push / reduce kernels
// (b2g_peer.cu) and the GEMM engine's fused exchange (gemm_engine.cuh).
//
// A mailbox (one per rank, device memory, opened by the others through CUDA
// IPC) for partials of `elems` floats and `world` ranks holds:
//   consumed[nchunk] u64         the root has read its landing slots up to epoch e (each rank's own)
//   count u64                    the fused exchange's grid-wide arrival count (own)
//   landing[2][world][elems] u64 the non-root partials, slot = epoch % 2 (root's)
// Each landed value is one 8-byte word {fp32 bits, low 32 bits of the epoch}
// written by a 16-byte store of two such words, so the root knows a value
// has arrived by its flag half and no separate ready flag (and no release
// fence on the sender's critical path) is needed.  Chunks are kPeerChunk
// floats.  The whole mailbox starts at zero; flags only grow, so nothing is
// reset.
#pragma once
#include <cstdint>

#include "ptx_sm100.cuh"

namespace b2g {

constexpr int kPeerChunk = 1024;      // floats per chunk
constexpr int kPeerMaxRanks = 16;
enum : int { kErrPeerCredit = 0x201, kErrPeerReady = 0x202, kErrPeerGrid = 0x203 };

struct PeerLayout {
  int64_t nchunk, consumed_off, count_off, flag_bytes, landing_off, slot_stride, total;
};

__host__ __device__ inline PeerLayout peer_layout(int64_t elems, int world) {
  PeerLayout l;
  l.nchunk = (elems + kPeerChunk - 1) / kPeerChunk;
  l.consumed_off = 0;
  l.count_off = l.nchunk * 8;
  l.flag_bytes = ((l.count_off + 8 + 255) / 256) * 256;
  l.landing_off = l.flag_bytes;
  l.slot_stride = ((elems * 8 + 255) / 256) * 256;   // bytes per (slot, rank) region
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

// Land values i .. i+3 (a 16-byte aligned group) as four {bits, flag} words.
__device__ __forceinline__ void peer_ll_put4(uint64_t* words, float4 v, uint32_t flag) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(words),
               "r"(__float_as_uint(v.x)), "r"(flag), "r"(__float_as_uint(v.y)), "r"(flag)
               : "memory");
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(words + 2),
               "r"(__float_as_uint(v.z)), "r"(flag), "r"(__float_as_uint(v.w)), "r"(flag)
               : "memory");
}
__device__ __forceinline__ void peer_ll_put1(uint64_t* word, float v, uint32_t flag) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(word), "r"(__float_as_uint(v)),
               "r"(flag)
               : "memory");
}
// Read values i .. i+3 once both flag halves of each 16-byte pair show
// `flag`; false when that takes longer than limit_ns.
__device__ __forceinline__ bool peer_ll_get4(const uint64_t* words, uint32_t flag,
                                             long long limit_ns, float4* out) {
  uint32_t a0, f0, a1, f1, b0, g0, b1, g1;
  uint64_t t0 = 0;
  for (unsigned spin = 0;; ++spin) {
    asm volatile("ld.relaxed.gpu.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(a0), "=r"(f0), "=r"(a1), "=r"(f1) : "l"(words) : "memory");
    asm volatile("ld.relaxed.gpu.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(b0), "=r"(g0), "=r"(b1), "=r"(g1) : "l"(words + 2) : "memory");
    if (f0 == flag && f1 == flag && g0 == flag && g1 == flag) break;
    if (spin == 0) t0 = ptx::globaltimer_ns();
    else if (ptx::globaltimer_ns() - t0 > static_cast<uint64_t>(limit_ns)) return false;
    if (spin > 64) __nanosleep(32);
  }
  *out = make_float4(__uint_as_float(a0), __uint_as_float(a1), __uint_as_float(b0),
                     __uint_as_float(b1));
  return true;
}
__device__ __forceinline__ bool peer_ll_get1(const uint64_t* word, uint32_t flag,
                                             long long limit_ns, float* out) {
  uint32_t a, f;
  uint64_t t0 = 0;
  for (unsigned spin = 0;; ++spin) {
    asm volatile("ld.relaxed.gpu.global.v2.u32 {%0, %1}, [%2];" : "=r"(a), "=r"(f) : "l"(word)
                 : "memory");
    if (f == flag) break;
    if (spin == 0) t0 = ptx::globaltimer_ns();
    else if (ptx::globaltimer_ns() - t0 > static_cast<uint64_t>(limit_ns)) return false;
    if (spin > 64) __nanosleep(32);
  }
  *out = __uint_as_float(a);
  return true;
}
// The landed values i .. i+3 of every rank but `root`, summed in rank order
// (the root then adds the sum to its own partial: out + (p_a + p_b + ...)).
__device__ __forceinline__ bool peer_ll_sum4(const uint64_t* slot, long long stride, int world,
                                             int root, long long i, uint32_t flag,
                                             long long limit_ns, float4* sum) {
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int r = 0; r < world; ++r) {
    if (r == root) continue;
    float4 v;
    if (!peer_ll_get4(slot + r * stride + i, flag, limit_ns, &v)) return false;
    acc.x += v.x;
    acc.y += v.y;
    acc.z += v.z;
    acc.w += v.w;
  }
  *sum = acc;
  return true;
}
#endif

}  // namespace b2g
