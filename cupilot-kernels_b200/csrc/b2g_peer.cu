// b2g_peer.cu — the cross-GPU step of a K split over the GPUs of one node.
//
// The reference's large-K kernel splits K over 8 CUDA streams on one GPU
// and sums the partial products with 7 `C.add_` calls
// (kernels/6_Matmul_with_large_K_dimension_best_kernel.cu:147-200).  Here K
// is split over ranks, one process per GPU; each rank computes its partial
// product with the GEMM engine, and the partials are summed on the root
// over NVLink by the two kernels below, through peer memory:
//
//   non-root rank r: peer_push_kernel copies its partial, chunk by chunk,
//     into landing slot [epoch % 2][r] of the root's mailbox through the
//     peer mapping, each value as an 8-byte word {value, epoch} written by
//     16-byte stores (no ready flag, no release fence).  Before writing a
//     chunk it waits until the root has consumed the same slot two epochs
//     ago (consumed[c] in its own mailbox).
//   root: peer_reduce_kernel waits until every landed word of its chunk
//     carries this epoch (polled while its own GEMM may still run), sums
//     them in rank order and adds the sum to its own partial (already in C;
//     deterministic), and, once the previous epoch's kernels have finished,
//     stamps consumed[c] = epoch - 1 in every other rank's mailbox.
//
// Every wait is bounded (B2G_WAIT_LIMIT_MS): a wait that gives up records a
// code in the device error word and the CTA returns; nothing traps.  Only
// plain loads and stores touch peer memory (no TMA, no bulk copies, no
// multicast), and only the mailboxes do.  b2g_gemm_splitk_peer runs the same
// protocol inside the GEMM engine's epilogue (gemm_engine.cuh, xgpu_exchange).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>

#include "../../include/b2g_gemm.h"
#include "b2g_internal.h"
#include "peer_protocol.cuh"
#include "ptx_sm100.cuh"

namespace {

using b2g::kErrPeerCredit;
using b2g::kErrPeerReady;
using b2g::peer_layout;
using Layout = b2g::PeerLayout;
constexpr int kThreads = 256;
constexpr int64_t kChunk = kThreads * 4;   // floats per chunk: one float4 per thread
static_assert(kChunk == b2g::kPeerChunk, "push / reduce kernels move one protocol chunk per CTA");
constexpr int kMaxRanks = B2G_PEER_MAX_RANKS;
static_assert(kMaxRanks == b2g::kPeerMaxRanks, "rank limit");

Layout layout(int64_t elems, int world) { return peer_layout(elems, world); }

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  b2g::peer_st_release_sys(p, v);
}
__device__ __forceinline__ bool wait_at_least(const uint64_t* flag, uint64_t want,
                                              long long limit_ns) {
  return b2g::peer_wait_at_least(flag, want, limit_ns);
}

struct PeerArgs {
  unsigned char* mbox[kMaxRanks];   // every rank's mailbox as mapped in this process
};

// One CTA per chunk.  partial: this rank's partial product (elems floats).
__global__ void __launch_bounds__(kThreads) peer_push_kernel(const float* __restrict__ partial,
                                                             int64_t elems, PeerArgs args,
                                                             Layout lay, int world, int rank,
                                                             int root, long long epoch,
                                                             long long limit_ns, int* err) {
  // Let the stream's next kernel (the next GEMM) launch and do its set-up
  // now; it waits for this grid to finish before it touches memory.
  b2g::ptx::griddep_launch_dependents();
  __shared__ int abort_flag;
  const int64_t c = blockIdx.x;
  unsigned char* mine = args.mbox[rank];
  unsigned char* rootb = args.mbox[root];
  if (threadIdx.x == 0) {
    // The slot this epoch writes was last read by the root two epochs ago.
    // (Waited for before the GEMM has finished: launched programmatically,
    // this CTA polls while the GEMM's last units run.)
    const uint64_t* consumed = reinterpret_cast<const uint64_t*>(mine + lay.consumed_off) + c;
    const long long need = epoch - 2;
    abort_flag = (need > 0 && !wait_at_least(consumed, static_cast<uint64_t>(need), limit_ns));
  }
  // The partial was written by the preceding GEMM.
  b2g::ptx::griddep_wait();
  __syncthreads();
  if (abort_flag) {
    if (threadIdx.x == 0 && err) atomicCAS(err, 0, kErrPeerCredit);
    return;
  }
  // Each value lands with the epoch in its flag half: no ready flag, no fence.
  uint64_t* dst = reinterpret_cast<uint64_t*>(rootb + lay.landing_off +
                                              ((epoch & 1) * world + rank) * lay.slot_stride);
  const uint32_t flag = static_cast<uint32_t>(epoch);
  const int64_t i = c * kChunk + static_cast<int64_t>(threadIdx.x) * 4;
  if (i + 4 <= elems) {
    b2g::peer_ll_put4(dst + i, __ldcg(reinterpret_cast<const float4*>(partial + i)), flag);
  } else {
    for (int64_t j = i; j < elems; ++j) b2g::peer_ll_put1(dst + j, __ldcg(partial + j), flag);
  }
}

// Root, one CTA per chunk: out += sum over the other ranks of their landed
// partials, in rank order.
__global__ void __launch_bounds__(kThreads) peer_reduce_kernel(float* __restrict__ out,
                                                               int64_t elems, PeerArgs args,
                                                               Layout lay, int world, int root,
                                                               long long epoch, long long limit_ns,
                                                               int* err) {
  b2g::ptx::griddep_launch_dependents();   // as in peer_push_kernel
  __shared__ int abort_flag;
  const int64_t c = blockIdx.x;
  unsigned char* mine = args.mbox[root];
  if (threadIdx.x == 0) abort_flag = 0;
  __syncthreads();
  const int t = threadIdx.x;
  const uint32_t flag = static_cast<uint32_t>(epoch);
  const uint64_t* slot = reinterpret_cast<const uint64_t*>(mine + lay.landing_off +
                                                           (epoch & 1) * world * lay.slot_stride);
  const int64_t stride = lay.slot_stride / 8;
  const int64_t i = c * kChunk + static_cast<int64_t>(t) * 4;
  // The other ranks' values do not depend on this rank's GEMM: they are
  // awaited, read and summed (rank order) while the GEMM may still run.
  float4 lsum = make_float4(0.f, 0.f, 0.f, 0.f);
  bool ok = true;
  if (i + 4 <= elems) ok = b2g::peer_ll_sum4(slot, stride, world, root, i, flag, limit_ns, &lsum);
  if (!ok) {
    atomicExch(&abort_flag, 1);
    if (err) atomicCAS(err, 0, kErrPeerReady);
  }
  // out holds this rank's own partial, written by the preceding GEMM; the
  // previous epoch's reduce has finished, so its slots are free again.
  b2g::ptx::griddep_wait();
  if (t < world && t != root && epoch > 1) {
    uint64_t* consumed = reinterpret_cast<uint64_t*>(args.mbox[t] + lay.consumed_off) + c;
    st_release_sys(consumed, static_cast<uint64_t>(epoch - 1));
  }
  __syncthreads();
  if (abort_flag) return;
  // out + (sum of the other ranks' partials): the same order as the fused
  // kernel's, so the two paths give identical sums.
  if (i + 4 <= elems) {
    float4 acc = *reinterpret_cast<const float4*>(out + i);
    acc.x += lsum.x;
    acc.y += lsum.y;
    acc.z += lsum.z;
    acc.w += lsum.w;
    *reinterpret_cast<float4*>(out + i) = acc;
  } else {
    for (int64_t j = i; j < elems; ++j) {
      float s = 0.f;
      for (int r = 0; r < world; ++r) {
        float x = 0.f;
        if (r != root && !b2g::peer_ll_get1(slot + r * stride + j, flag, limit_ns, &x)) {
          if (err) atomicCAS(err, 0, kErrPeerReady);
          return;
        }
        s += x;
      }
      out[j] += s;
    }
  }
}

}  // namespace

extern "C" int64_t b2g_peer_mailbox_bytes(int64_t elems, int world) {
  if (elems <= 0 || world < 1 || world > kMaxRanks) return -1;
  return layout(elems, world).total;
}

extern "C" int b2g_peer_mailbox_create(int64_t elems, int world, void** mailbox,
                                       b2g_ipc_handle* handle) {
  if (!mailbox || !handle || elems <= 0 || world < 1 || world > kMaxRanks)
    return B2G_ERR_INVALID_ARG;
  *mailbox = nullptr;
  const Layout l = layout(elems, world);
  void* p = nullptr;
  if (cudaMalloc(&p, l.total) != cudaSuccess) return B2G_ERR_LAUNCH;
  // Everything starts at 0: flags have no epoch yet, and no landing word
  // carries an epoch's flag before a rank writes it.
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, l.total) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return B2G_ERR_LAUNCH;
  }
  static_assert(sizeof(h) <= sizeof(handle->bytes), "IPC handle does not fit");
  std::memset(handle->bytes, 0, sizeof(handle->bytes));
  std::memcpy(handle->bytes, &h, sizeof(h));
  *mailbox = p;
  return B2G_OK;
}

extern "C" int b2g_peer_mailbox_open(const b2g_ipc_handle* handle, void** mailbox) {
  if (!handle || !mailbox) return B2G_ERR_INVALID_ARG;
  *mailbox = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle->bytes, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return B2G_ERR_LAUNCH;
  *mailbox = p;
  return B2G_OK;
}

extern "C" int b2g_peer_mailbox_close(void* mailbox) {
  if (!mailbox) return B2G_ERR_INVALID_ARG;
  return cudaIpcCloseMemHandle(mailbox) == cudaSuccess ? B2G_OK : B2G_ERR_LAUNCH;
}

extern "C" int b2g_peer_mailbox_destroy(void* mailbox) {
  if (!mailbox) return B2G_ERR_INVALID_ARG;
  return cudaFree(mailbox) == cudaSuccess ? B2G_OK : B2G_ERR_LAUNCH;
}

extern "C" int b2g_splitk_peer_reduce(const float* partial, float* out, int64_t elems,
                                      void* const* mailboxes, int world, int rank, int root,
                                      int64_t epoch, b2g_stream_t stream_handle) {
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world || root < 0 || root >= world)
    return B2G_ERR_INVALID_ARG;
  if (elems < 0 || epoch < 1 || !mailboxes) return B2G_ERR_INVALID_ARG;
  if (elems == 0 || world == 1) return B2G_OK;
  const bool is_root = rank == root;
  if (is_root ? !out : !partial) return B2G_ERR_INVALID_ARG;
  const void* mine = is_root ? static_cast<const void*>(out) : static_cast<const void*>(partial);
  if (reinterpret_cast<uintptr_t>(mine) % 16) return B2G_ERR_UNSUPPORTED;
  PeerArgs args;
  std::memset(&args, 0, sizeof(args));
  for (int r = 0; r < world; ++r) {
    if (!mailboxes[r]) return B2G_ERR_INVALID_ARG;
    args.mbox[r] = static_cast<unsigned char*>(mailboxes[r]);
  }
  int* err = b2g::current_error_word();
  if (!err) return B2G_ERR_NO_DEVICE;
  const Layout lay = layout(elems, world);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_handle);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(lay.nchunk), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.stream = stream;
  // Programmatic launch after the GEMM that produced the partial: the set-up
  // overlaps the GEMM's tail; the kernels wait for it before reading.
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = b2g::pdl_enabled() ? 1 : 0;
  const long long limit = b2g::current_wait_limit_ns();
  cudaError_t e;
  if (is_root)
    e = cudaLaunchKernelEx(&cfg, peer_reduce_kernel, out, elems, args, lay, world, root,
                           static_cast<long long>(epoch), limit, err);
  else
    e = cudaLaunchKernelEx(&cfg, peer_push_kernel, partial, elems, args, lay, world, rank, root,
                           static_cast<long long>(epoch), limit, err);
  if (e != cudaSuccess) return B2G_ERR_LAUNCH;
  return cudaGetLastError() == cudaSuccess ? B2G_OK : B2G_ERR_LAUNCH;
}
