// sdpa_engine.cuh — fused scaled-dot-product attention on tcgen05 (sm_100a).
//
// out[b,h] = softmax(Q[b,h] K[b,h]^T * scale) V[b,h] for fp16 Q, K, V of
// shape (batch, heads, seq, dim), fp32 accumulation and softmax, fp16 out.
// Replaces fused_attention_cuda (kernels/97_ScaledDotProductAttention_best_kernel.cu:256),
// which computes the same with CUDA-core fp32 dot products, a full-row
// softmax of seq <= 512 scores and scale = 1/sqrt(dim) (:266-274).
//
// One work unit = 256 query rows of one (batch, head), computed by a CTA
// pair (cluster of 2, tcgen05 cta_group::2): each CTA holds 128 of the rows
// in its TMEM lanes and loads half of every K / V tile, so K and V cross
// L2 once per 256 query rows.  A persistent pair runs units round-robin
// through three roles (per CTA):
//   warp 0   TMA producer: phase 1 streams (Q rows, K keys) slices along
//            dim, 64 wide; phase 2 streams V in 128-key slices, this CTA's
//            half of each output chunk of up to 256 columns.
//   warp 1   MMA issuer (the pair leader's lane 0): phase 1 accumulates
//            S = Q K^T for all keys (<= 512) into TMEM columns [0, 512) from a
//            7-slot ring (3 slots plus the P buffer, idle until the softmax);
//            phase 2 accumulates O = P V chunk by chunk into two 256-column
//            TMEM buffers.
//   warps 2-9 two warps per TMEM lane quadrant, each one thread per query
//            row over half of the key columns: the row max and the
//            exponentials of S (max and sum exchanged through shared memory),
//            P = exp(S - max) written as fp16 into shared memory in the
//            K-major operand layout, then each O chunk (half of its columns
//            per warp) scaled by 1 / rowsum, converted to fp16 and stored.
// The whole score row stays on chip (S in TMEM, P in shared memory); only O
// is written.
#pragma once

#include <cuda_fp16.h>

#include "gemm_engine.cuh"

namespace b2g {
namespace sdpa {

constexpr int kBM = 128;           // query rows per CTA (one per TMEM lane)
constexpr int kUnitM = 2 * kBM;    // query rows per pair unit
constexpr int kBD = 64;            // dim slice per phase-1 stage (128 bytes of fp16)
constexpr int kKeysMax = 512;      // S uses all 512 TMEM columns
constexpr int kKBox = 256;         // keys per phase-1 MMA (N); 128 of them per CTA
constexpr int kVKeys = 128;        // keys per phase-2 stage
constexpr int kOChunk = 256;       // output columns per TMEM buffer; 128 loaded per CTA
constexpr int kStages = 3;          // stage slots outside the P buffer (phase 2 uses these)
constexpr int kSlots1 = 7;          // phase 1 also borrows the idle P buffer: 3 + 4 slots
constexpr int kQBytes = kBM * kBD * 2;             // 16 KB
constexpr int kKBytes = (kKBox / 2) * kBD * 2;     // 16 KB: this CTA's 128 keys
constexpr int kVBoxBytes = kVKeys * 64 * 2;        // 16 KB: 128 keys x 64 columns
constexpr int kStageBytes = kQBytes + kKBytes;     // 32 KB (a V stage: 2 boxes of 16 KB)
constexpr int kPBlockBytes = kBM * 64 * 2;         // 16 KB: 128 rows x 64 keys
constexpr int kOffP = kStages * kStageBytes;
constexpr int kOffBar = kOffP + (kKeysMax / 64) * kPBlockBytes;
constexpr int kNumBars = 2 * kSlots1 + 8;
constexpr int kOffRed = kOffBar + kNumBars * 8;    // row partials of the two halves: 2 x 128 floats
constexpr int kOffMisc = kOffRed + 2 * kBM * 4;
constexpr int kSmemBytes = kOffMisc + 16 + 1024;
constexpr int kRowWarps = 8;                       // softmax / epilogue warps per CTA
constexpr int kThreads = (2 + kRowWarps) * 32;
static_assert(kSmemBytes <= 232448, "shared memory budget");

enum : int { kErrSdpaFull = 0x201, kErrSdpaEmpty = 0x202, kErrSdpaS = 0x203,
             kErrSdpaP = 0x204, kErrSdpaO = 0x205, kErrSdpaOEmpty = 0x206 };

struct Params {
  int S, D, BH;
  int qblocks;               // pair units per (batch, head)
  long long units;
  float scale_log2;          // scale * log2(e): exp(x*scale) = exp2(x*scale_log2)
  __half* out;
  long long wait_limit_ns;
  int* err;
};

// 2^x with the hardware approximation (relative error ~2^-22, flushes
// denormal results to zero), as the softmax needs only fp16-accurate values.
__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// The two row warps of TMEM lane quadrant `quad` meet here (64 threads).
__device__ __forceinline__ void quad_sync(int quad) {
  asm volatile("bar.sync %0, 64;" ::"r"(quad + 1) : "memory");
}

__device__ __forceinline__ void sdpa_error(int* err, volatile int* abort, int code) {
  atomicCAS(err, 0, code);
  *abort = 1;
}

__device__ __forceinline__ void mma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Byte offset of (row, key) in the P buffer: 64-key blocks of 16 KB, rows of
// 128 bytes, 16-byte chunks XOR-swizzled by row % 8 (the 128-byte swizzle
// the MMA's K-major descriptor expects).
__device__ __forceinline__ uint32_t p_offset(int row, int key) {
  const int blk = key >> 6;
  const int chunk = (key & 63) >> 3;
  return static_cast<uint32_t>(blk * kPBlockBytes + row * 128 + ((chunk ^ (row & 7)) << 4));
}

// Output columns an O chunk covers (cw) and computes (a multiple of 128, so
// each CTA loads whole 64-column V boxes; columns past dim are zero-filled).
__device__ __forceinline__ int chunk_width(int D, int c) {
  return min(kOChunk, D - c * kOChunk);
}
__device__ __forceinline__ int chunk_width_padded(int D, int c) {
  return (chunk_width(D, c) + 127) & ~127;
}

__global__ void __launch_bounds__(kThreads, 1)
    sdpa_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                const __grid_constant__ CUtensorMap map_v, const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + kSlots1;
  uint64_t* s_full = bars + 2 * kSlots1;
  uint64_t* p_ready = s_full + 1;
  uint64_t* o_full = s_full + 2;
  uint64_t* o_empty = s_full + 4;
  uint64_t* mma_drain = s_full + 6;
  uint64_t* p_free = s_full + 7;     // the last P . V MMA of a unit has read P
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = ptx::cluster_ctarank();
  const bool leader = rank == 0;
  const long long unit0 = blockIdx.x >> 1, unit_step = gridDim.x >> 1;
  const int nk = (p.S + kKBox - 1) / kKBox;          // phase-1 key boxes (1 or 2)
  const int nd = p.D / kBD;                          // phase-1 dim slices
  const int nkb = (p.S + kVKeys - 1) / kVKeys;       // phase-2 key slices
  const int nchunks = (p.D + kOChunk - 1) / kOChunk;
  const int n1 = nd * nk;                            // phase-1 stages per unit
  // Stage i of a unit lives in slot i % 7 in phase 1 (slots 3-6 are the P
  // buffer, free until the softmax writes P), in slot (i - n1) % 3 in phase 2.
  auto slot_of = [&](int i) -> int { return i < n1 ? i % kSlots1 : (i - n1) % kStages; };
  auto slot_ptr = [&](int slot) -> uint8_t* {
    return slot < kStages ? smem + slot * kStageBytes : smem + kOffP + (slot - kStages) * kStageBytes;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots1; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    ptx::mbar_init(p_free, 1);
    ptx::mbar_init(s_full, 1);
    ptx::mbar_init(p_ready, 2 * kRowWarps);          // both CTAs' row warps (leader's)
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(&o_full[b], 1);
      ptx::mbar_init(&o_empty[b], 2 * kRowWarps);
    }
    ptx::mbar_init(mma_drain, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&map_q);
    ptx::prefetch_tmap(&map_k);
    ptx::prefetch_tmap(&map_v);
  }
  if (warp == 1) {
    ptx::tmem_alloc_pair(tmem_slot, 512);
    ptx::tmem_relinquish_pair();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::cluster_sync();   // peer barriers initialised before any remote arrive
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Launched with programmatic stream serialization: the set-up above may
  // overlap the previous kernel's tail; every global-memory access (operand
  // loads, unit tables, counters, output) comes after this wait.
  ptx::griddep_launch_dependents();
  ptx::griddep_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint32_t full_leader = ptx::mapa_shared(ptx::smem_addr(full), 0);
      // A unit's stages: nd*nk (Q slice, K keys) pairs, then nchunks*nkb V slices.
      const int n_items = n1 + nchunks * nkb;
      // Issue the boxes of stage `i` of unit `w` into stage memory `st`.
      auto stage_boxes = [&](long long w, int i, uint8_t* st, uint32_t bar) {
        const int bh = static_cast<int>(w / p.qblocks);
        const int q0 = static_cast<int>(w % p.qblocks) * kUnitM + static_cast<int>(rank) * kBM;
        if (i < n1) {
          const int d = i / nk, h = i % nk;
          const int k0 = h * kKBox + static_cast<int>(rank) * (kKBox / 2);
          ptx::tma_load_3d_pair(st, &map_q, bar, d * kBD, q0, bh);
          ptx::tma_load_3d_pair(st + kQBytes, &map_k, bar, d * kBD, k0, bh);
          return;
        }
        const int c = (i - n1) / nkb, kb = (i - n1) % nkb;
        const int half_w = chunk_width_padded(p.D, c) / 2;   // this CTA's columns
        const int col0 = c * kOChunk + static_cast<int>(rank) * half_w;
        for (int g = 0; g < half_w / 64; ++g)
          ptx::tma_load_3d_pair(st + g * kVBoxBytes, &map_v, bar, col0 + g * 64, kb * kVKeys, bh);
      };
      auto stage_bytes = [&](int i) -> uint32_t {
        if (i < n1) return kQBytes + kKBytes;
        const int c = (i - n1) / nkb;
        return static_cast<uint32_t>(chunk_width_padded(p.D, c) / 128) * kVBoxBytes;
      };
      uint32_t uses[kSlots1] = {0, 0, 0, 0, 0, 0, 0};
      uint32_t unit_i = 0;
      bool ok = true;
      for (long long w = unit0; w < p.units && ok; w += unit_step, ++unit_i) {
        for (int i = 0; i < n_items; ++i) {
          const int s = slot_of(i);
          // First P-buffer slot of this unit: the previous unit's P . V is done.
          if (i == kStages && unit_i > 0 &&
              !ptx::mbar_wait(p_free, (unit_i - 1) & 1, abort_flag, p.wait_limit_ns)) {
            sdpa_error(p.err, abort_flag, kErrSdpaEmpty);
            ok = false;
            break;
          }
          const uint32_t ph = uses[s]++ & 1;
          if (!ptx::mbar_wait(&empty[s], ph ^ 1, abort_flag, p.wait_limit_ns)) {
            sdpa_error(p.err, abort_flag, kErrSdpaEmpty);
            ok = false;
            break;
          }
          // The leader's barrier counts both CTAs' bytes.
          if (leader) ptx::mbar_arrive_expect_tx(&full[s], 2 * stage_bytes(i));
          stage_boxes(w, i, slot_ptr(s), full_leader + s * 8);
        }
      }
      // Drain: every issued load lands before the CTA may exit (bounded).
      // The leader's barriers count the peer's loads too.
      if (leader) {
        volatile int never = 0;
        for (int s = 0; s < kSlots1; ++s)
          if (uses[s] > 0) ptx::mbar_wait(&full[s], (uses[s] - 1) & 1, &never, kDrainLimitNs);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {
      constexpr uint32_t idesc_s = ptx::idesc_f16(kUnitM, kKBox, false, false);
      uint32_t uses[kSlots1] = {0, 0, 0, 0, 0, 0, 0};
      uint32_t unit_i = 0, qc = 0;
      bool ok = true;
      auto wait_full = [&](int i, int* s_out) -> bool {
        const int s = slot_of(i);
        const uint32_t ph = uses[s]++ & 1;
        if (!ptx::mbar_wait(&full[s], ph, abort_flag, p.wait_limit_ns)) {
          sdpa_error(p.err, abort_flag, kErrSdpaFull);
          return false;
        }
        ptx::tc_fence_after();
        *s_out = s;
        return true;
      };
      // Chunk q is the (q >> 1)-th use of O buffer q & 1: before it, the
      // epilogue of both CTAs must have drained the previous use.
      auto wait_o_empty = [&](uint32_t q) -> bool {
        const uint32_t b = q & 1, n = q >> 1;
        if (n == 0) return true;
        if (!ptx::mbar_wait(&o_empty[b], (n - 1) & 1, abort_flag, p.wait_limit_ns)) {
          sdpa_error(p.err, abort_flag, kErrSdpaOEmpty);
          return false;
        }
        return true;
      };
      for (long long w = unit0; w < p.units && ok; w += unit_step, ++unit_i) {
        // S overwrites both O buffers: wait for the previous unit's last two chunks.
        if (qc >= 1 && !wait_o_empty(qc + 1)) break;
        if (qc >= 2 && !wait_o_empty(qc)) break;
        ptx::tc_fence_after();
        for (int d = 0; d < nd && ok; ++d)
          for (int h = 0; h < nk && ok; ++h) {
            int s;
            if (!wait_full(d * nk + h, &s)) { ok = false; break; }
            const uint32_t sq = ptx::smem_addr(slot_ptr(s));
            const uint32_t sk = sq + kQBytes;
#pragma unroll
            for (int k16 = 0; k16 < kBD / 16; ++k16) {
              const uint64_t da = ptx::smem_desc(sq + k16 * 32, 16, 1024, ptx::kLayoutSw128);
              const uint64_t db = ptx::smem_desc(sk + k16 * 32, 16, 1024, ptx::kLayoutSw128);
              mma_f16_pair(tmem_base + h * kKBox, da, db, idesc_s, (d > 0 || k16 > 0) ? 1u : 0u);
            }
            ptx::mma_commit_pair(&empty[s], 0x3);
          }
        if (!ok) break;
        ptx::mma_commit_pair(s_full, 0x3);
        // Phase 2: P (written by both CTAs' row warps) times V, chunk by chunk.
        if (!ptx::mbar_wait(p_ready, unit_i & 1, abort_flag, p.wait_limit_ns)) {
          sdpa_error(p.err, abort_flag, kErrSdpaP);
          break;
        }
        ptx::tc_fence_after();
        const uint32_t sp = ptx::smem_addr(smem + kOffP);
        for (int c = 0; c < nchunks && ok; ++c, ++qc) {
          if (!wait_o_empty(qc)) { ok = false; break; }
          ptx::tc_fence_after();
          const uint32_t idesc_o = ptx::idesc_f16(kUnitM, chunk_width_padded(p.D, c), false, true);
          const uint32_t d_tmem = tmem_base + (qc & 1) * kOChunk;
          for (int kb = 0; kb < nkb && ok; ++kb) {
            int s;
            if (!wait_full(n1 + c * nkb + kb, &s)) { ok = false; break; }
            const uint32_t sv = ptx::smem_addr(slot_ptr(s));
#pragma unroll
            for (int k16 = 0; k16 < kVKeys / 16; ++k16) {
              // P: 64-key blocks of 16 KB; a 16-key step is 32 B inside a row.
              const uint64_t da = ptx::smem_desc(
                  sp + (kb * (kVKeys / 64) + k16 / 4) * kPBlockBytes + (k16 % 4) * 32, 16, 1024,
                  ptx::kLayoutSw128);
              // V slice (MN-major): 64-column boxes of 128 keys (128-byte
              // rows, one per key) 16 KB apart (LBO); 8-key groups 1024 B
              // apart (SBO); a 16-key step is 16 rows.
              const uint64_t db =
                  ptx::smem_desc(sv + k16 * 16 * 128, kVBoxBytes, 1024, ptx::kLayoutSw128);
              mma_f16_pair(d_tmem, da, db, idesc_o, (kb > 0 || k16 > 0) ? 1u : 0u);
            }
            ptx::mma_commit_pair(&empty[s], 0x3);
          }
          if (ok) ptx::mma_commit_pair(&o_full[qc & 1], 0x3);
        }
        if (ok) ptx::mma_commit_pair(p_free, 0x3);
      }
      // Drain: no MMA may still write TMEM when it is freed, also after an
      // early exit (bounded; immediate on the normal path).
      ptx::mma_commit_pair(mma_drain, 0x1);
      volatile int never = 0;
      ptx::mbar_wait(mma_drain, 0, &never, kDrainLimitNs);
    }
  } else {
    // ------------------------------------------------------ softmax + epilogue
    const int quad = warp & 3;                 // TMEM lane quadrant of this warp
    const int half = (warp - 2) >> 2;          // which half of the columns
    const int row = quad * 32 + lane;          // query row within this CTA's 128
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t p_ready_leader = ptx::mapa_shared(ptx::smem_addr(p_ready), 0);
    const uint32_t o_empty_leader = ptx::mapa_shared(ptx::smem_addr(o_empty), 0);
    float* red = reinterpret_cast<float*>(smem + kOffRed);   // [half][row]: max, then sum
    uint32_t unit_i = 0, qc = 0;
    for (long long w = unit0; w < p.units; w += unit_step, ++unit_i) {
      const int bh = static_cast<int>(w / p.qblocks);
      const int q = static_cast<int>(w % p.qblocks) * kUnitM + static_cast<int>(rank) * kBM + row;
      if (!ptx::mbar_wait_sleepy(s_full, unit_i & 1, abort_flag, p.wait_limit_ns)) {
        if (lane == 0) sdpa_error(p.err, abort_flag, kErrSdpaS);
        break;
      }
      ptx::tc_fence_after();
      // This warp's key columns: [c_lo, c_hi) of the computed nk * 256.
      const int ncols = nk * kKBox;
      const int c_lo = half * (ncols / 2), c_hi = c_lo + ncols / 2;
      float m = -INFINITY;
      for (int c0 = c_lo; c0 < c_hi; c0 += 32) {
        uint32_t r[32];
        ptx::tmem_ld_32x32b_x32(lane_base + c0, r);
        tmem_ld_wait_regs(r);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c0 + j < p.S) m = fmaxf(m, __uint_as_float(r[j]));
      }
      quad_sync(quad);                   // the partner has read the previous unit's sums
      red[half * kBM + row] = m;
      quad_sync(quad);
      m = fmaxf(red[row], red[kBM + row]);
      // P = exp(scale * (s - max)) as fp16 into the operand layout; row sum in fp32.
      const float mb = m * p.scale_log2;
      float l = 0.f;
      for (int c0 = c_lo; c0 < c_hi; c0 += 32) {
        uint32_t r[32];
        ptx::tmem_ld_32x32b_x32(lane_base + c0, r);
        tmem_ld_wait_regs(r);
        uint32_t h2[16];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float e0 =
              (c0 + j < p.S) ? exp2_approx(__uint_as_float(r[j]) * p.scale_log2 - mb) : 0.f;
          const float e1 =
              (c0 + j + 1 < p.S) ? exp2_approx(__uint_as_float(r[j + 1]) * p.scale_log2 - mb) : 0.f;
          l += e0 + e1;
          const __half2 hv = __floats2half2_rn(e0, e1);
          h2[j / 2] = *reinterpret_cast<const uint32_t*>(&hv);
        }
        if (c0 < nkb * kVKeys) {
#pragma unroll
          for (int g = 0; g < 4; ++g)
            *reinterpret_cast<uint4*>(smem + kOffP + p_offset(row, c0 + g * 8)) =
                make_uint4(h2[4 * g], h2[4 * g + 1], h2[4 * g + 2], h2[4 * g + 3]);
        }
      }
      // P visible to the tensor core (the leader's MMAs read this CTA's P).
      asm volatile("fence.proxy.async;" ::: "memory");
      ptx::tc_fence_before();            // every read of S done before O overwrites it
      quad_sync(quad);                   // both halves have read the maxima
      red[half * kBM + row] = l;
      quad_sync(quad);
      const float inv_l = 1.f / (red[row] + red[kBM + row]);
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive_cluster(p_ready_leader);
      // Output chunks: this warp stores columns [half*128, half*128+128) of each.
      bool ok = true;
      for (int c = 0; c < nchunks; ++c, ++qc) {
        const int cw = chunk_width(p.D, c);
        if (!ptx::mbar_wait_sleepy(&o_full[qc & 1], (qc >> 1) & 1, abort_flag, p.wait_limit_ns)) {
          if (lane == 0) sdpa_error(p.err, abort_flag, kErrSdpaO);
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t obuf = lane_base + (qc & 1) * kOChunk;
        __half* orow = p.out + (static_cast<long long>(bh) * p.S + q) * p.D + c * kOChunk;
        const int o_lo = half * (kOChunk / 2), o_hi = min(cw, o_lo + kOChunk / 2);
        for (int c0 = o_lo; c0 < o_hi; c0 += 32) {
          uint32_t r[32];
          ptx::tmem_ld_32x32b_x32(obuf + c0, r);
          tmem_ld_wait_regs(r);
          if (q < p.S) {
            uint32_t h2[16];
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              const __half2 hv = __floats2half2_rn(__uint_as_float(r[j]) * inv_l,
                                                   __uint_as_float(r[j + 1]) * inv_l);
              h2[j / 2] = *reinterpret_cast<const uint32_t*>(&hv);
            }
            uint4* dst = reinterpret_cast<uint4*>(orow + c0);
#pragma unroll
            for (int g = 0; g < 4; ++g)
              dst[g] = make_uint4(h2[4 * g], h2[4 * g + 1], h2[4 * g + 2], h2[4 * g + 3]);
          }
        }
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive_cluster(o_empty_leader + (qc & 1) * 8);
      }
      if (!ok) break;
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::cluster_sync();   // no CTA leaves while its peer may still signal it
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc_pair(tmem_base, 512);
  }
}

}  // namespace sdpa
}  // namespace b2g
