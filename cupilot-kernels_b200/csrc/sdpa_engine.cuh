// sdpa_engine.cuh — fused scaled-dot-product attention on tcgen05 (sm_100a).
//
// out[b,h] = softmax(Q[b,h] K[b,h]^T * scale) V[b,h] for fp16 Q, K, V of
// shape (batch, heads, seq, dim), fp32 accumulation and softmax, fp16 out.
// Replaces fused_attention_cuda (kernels/97_ScaledDotProductAttention_best_kernel.cu:256),
// which computes the same with CUDA-core fp32 dot products, a full-row
// softmax of seq <= 512 scores and scale = 1/sqrt(dim) (:266-274).
//
// One work unit = 128 query rows of one (batch, head).  A persistent CTA
// runs units round-robin through three roles:
//   warp 0   TMA producer: phase 1 streams (Q block, K block) pairs along
//            dim in 64-wide slices; phase 2 streams V in 64-key slices of
//            up to 256 output columns.
//   warp 1   MMA issuer (one thread): phase 1 accumulates S = Q K^T for all
//            keys (<= 512) into TMEM columns [0, 512); phase 2 accumulates
//            O = P V chunk by chunk into two 256-column TMEM buffers.
//   warps 2-5 one thread per query row (its TMEM lane): the row max and the
//            exponentials of S, P = exp(S - max) written as fp16 into shared
//            memory in the K-major operand layout, then each O chunk scaled
//            by 1 / rowsum, converted to fp16 and stored.
// The whole score row stays on chip (S in TMEM, P in shared memory), so Q,
// K and V are each read once per unit and nothing but O is written.
#pragma once

#include <cuda_fp16.h>

#include "gemm_engine.cuh"

namespace b2g {
namespace sdpa {

constexpr int kBM = 128;           // query rows per unit (one per TMEM lane)
constexpr int kBD = 64;            // dim slice per phase-1 stage (128 bytes of fp16)
constexpr int kKeysMax = 512;      // S uses all 512 TMEM columns
constexpr int kKBox = 256;         // keys per phase-1 MMA (N) and per K box
constexpr int kVKeys = 64;         // keys per phase-2 stage
constexpr int kOChunk = 256;       // output columns per TMEM buffer
constexpr int kStages = 2;
constexpr int kQBytes = kBM * kBD * 2;            // 16 KB
constexpr int kKBytes = kKBox * kBD * 2;          // 32 KB
constexpr int kVBoxBytes = kVKeys * 64 * 2;       // 8 KB: 64 keys x 64 columns
constexpr int kStageBytes = kQBytes + kKBytes;    // 48 KB (a V stage uses 32 KB of it)
constexpr int kPBlockBytes = kBM * 64 * 2;        // 16 KB: 128 rows x 64 keys
constexpr int kOffP = kStages * kStageBytes;
constexpr int kOffBar = kOffP + (kKeysMax / 64) * kPBlockBytes;
constexpr int kNumBars = 2 * kStages + 7;
constexpr int kOffMisc = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffMisc + 16 + 1024;
constexpr int kThreads = 6 * 32;
static_assert(kSmemBytes <= 232448, "shared memory budget");

enum : int { kErrSdpaFull = 0x201, kErrSdpaEmpty = 0x202, kErrSdpaS = 0x203,
             kErrSdpaP = 0x204, kErrSdpaO = 0x205, kErrSdpaOEmpty = 0x206 };

struct Params {
  int S, D, BH;
  int qblocks;
  long long units;
  float scale_log2;          // scale * log2(e): exp(x*scale) = exp2(x*scale_log2)
  __half* out;
  long long wait_limit_ns;
  int* err;
};

__device__ __forceinline__ void sdpa_error(int* err, volatile int* abort, int code) {
  atomicCAS(err, 0, code);
  *abort = 1;
}

// Byte offset of (row, key) in the P buffer: 64-key blocks of 16 KB, rows of
// 128 bytes, 16-byte chunks XOR-swizzled by row % 8 (the 128-byte swizzle
// the MMA's K-major descriptor expects).
__device__ __forceinline__ uint32_t p_offset(int row, int key) {
  const int blk = key >> 6;
  const int chunk = (key & 63) >> 3;
  return static_cast<uint32_t>(blk * kPBlockBytes + row * 128 + ((chunk ^ (row & 7)) << 4));
}

__global__ void __launch_bounds__(kThreads, 1)
    sdpa_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                const __grid_constant__ CUtensorMap map_v, const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + kStages;
  uint64_t* s_full = bars + 2 * kStages;
  uint64_t* p_ready = s_full + 1;
  uint64_t* o_full = s_full + 2;
  uint64_t* o_empty = s_full + 4;
  uint64_t* mma_drain = s_full + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nk = (p.S + kKBox - 1) / kKBox;          // phase-1 key boxes (1 or 2)
  const int nd = p.D / kBD;                          // phase-1 dim slices
  const int nkb = (p.S + kVKeys - 1) / kVKeys;       // phase-2 key slices
  const int nchunks = (p.D + kOChunk - 1) / kOChunk;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    ptx::mbar_init(s_full, 1);
    ptx::mbar_init(p_ready, 4);
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(&o_full[b], 1);
      ptx::mbar_init(&o_empty[b], 4);
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
    ptx::tmem_alloc(tmem_slot, 512);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (long long w = blockIdx.x; w < p.units && ok; w += gridDim.x) {
        const int bh = static_cast<int>(w / p.qblocks);
        const int q0 = static_cast<int>(w % p.qblocks) * kBM;
        auto next_stage = [&](uint32_t bytes) -> uint8_t* {
          const int s = it % kStages;
          const uint32_t ph = (it / kStages) & 1;
          if (!ptx::mbar_wait(&empty[s], ph ^ 1, abort_flag, p.wait_limit_ns)) {
            sdpa_error(p.err, abort_flag, kErrSdpaEmpty);
            ok = false;
            return nullptr;
          }
          ptx::mbar_arrive_expect_tx(&full[s], bytes);
          ++it;
          return smem + s * kStageBytes;
        };
        for (int d = 0; d < nd && ok; ++d)
          for (int h = 0; h < nk && ok; ++h) {
            uint8_t* st = next_stage(kQBytes + kKBytes);
            if (!st) break;
            const int s = (it - 1) % kStages;
            ptx::tma_load_3d(st, &map_q, &full[s], d * kBD, q0, bh);
            ptx::tma_load_3d(st + kQBytes, &map_k, &full[s], d * kBD, h * kKBox, bh);
          }
        for (int c = 0; c < nchunks && ok; ++c) {
          const int cw = min(kOChunk, p.D - c * kOChunk);
          for (int kb = 0; kb < nkb && ok; ++kb) {
            uint8_t* st = next_stage(static_cast<uint32_t>(cw / 64) * kVBoxBytes);
            if (!st) break;
            const int s = (it - 1) % kStages;
            for (int g = 0; g < cw / 64; ++g)
              ptx::tma_load_3d(st + g * kVBoxBytes, &map_v, &full[s], c * kOChunk + g * 64,
                               kb * kVKeys, bh);
          }
        }
      }
      // Drain: every issued load lands before the CTA may exit (bounded).
      volatile int never = 0;
      const uint32_t first = it > static_cast<uint32_t>(kStages) ? it - kStages : 0u;
      for (uint32_t j = first; j < it; ++j)
        ptx::mbar_wait(&full[j % kStages], (j / kStages) & 1, &never, kDrainLimitNs);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = ptx::idesc_f16(kBM, kKBox, false, false);
      uint32_t it = 0, unit_i = 0, qc = 0;
      bool ok = true;
      auto wait_full = [&](int* s_out) -> bool {
        const int s = it % kStages;
        const uint32_t ph = (it / kStages) & 1;
        if (!ptx::mbar_wait(&full[s], ph, abort_flag, p.wait_limit_ns)) {
          sdpa_error(p.err, abort_flag, kErrSdpaFull);
          return false;
        }
        ptx::tc_fence_after();
        *s_out = s;
        ++it;
        return true;
      };
      // An O buffer may be overwritten once the epilogue has drained its last use.
      auto wait_o_empty = [&](uint32_t q) -> bool {
        const uint32_t b = q & 1, n = q >> 1;   // n-th use of buffer b
        if (n == 0) return true;
        if (!ptx::mbar_wait(&o_empty[b], (n - 1) & 1, abort_flag, p.wait_limit_ns)) {
          sdpa_error(p.err, abort_flag, kErrSdpaOEmpty);
          return false;
        }
        return true;
      };
      for (long long w = blockIdx.x; w < p.units && ok; w += gridDim.x, ++unit_i) {
        // S overwrites both O buffers: wait for the previous unit's last two chunks.
        if (qc >= 1 && !wait_o_empty(qc + 1)) break;   // the use before qc+1 on its buffer
        if (qc >= 2 && !wait_o_empty(qc)) break;
        ptx::tc_fence_after();
        for (int d = 0; d < nd && ok; ++d)
          for (int h = 0; h < nk && ok; ++h) {
            int s;
            if (!wait_full(&s)) { ok = false; break; }
            const uint32_t sq = ptx::smem_addr(smem + s * kStageBytes);
            const uint32_t sk = sq + kQBytes;
#pragma unroll
            for (int k16 = 0; k16 < kBD / 16; ++k16) {
              const uint64_t da = ptx::smem_desc(sq + k16 * 32, 16, 1024, ptx::kLayoutSw128);
              const uint64_t db = ptx::smem_desc(sk + k16 * 32, 16, 1024, ptx::kLayoutSw128);
              ptx::mma_f16(tmem_base + h * kKBox, da, db, idesc_s, (d > 0 || k16 > 0) ? 1u : 0u);
            }
            ptx::mma_commit(&empty[s]);
          }
        if (!ok) break;
        ptx::mma_commit(s_full);
        // Phase 2: P (written by the softmax warps) times V, chunk by chunk.
        if (!ptx::mbar_wait(p_ready, unit_i & 1, abort_flag, p.wait_limit_ns)) {
          sdpa_error(p.err, abort_flag, kErrSdpaP);
          break;
        }
        ptx::tc_fence_after();
        for (int c = 0; c < nchunks && ok; ++c, ++qc) {
          const int cw = min(kOChunk, p.D - c * kOChunk);
          if (!wait_o_empty(qc)) { ok = false; break; }
          ptx::tc_fence_after();
          const uint32_t idesc_o = ptx::idesc_f16(kBM, cw, false, true);
          const uint32_t d_tmem = tmem_base + (qc & 1) * kOChunk;
          const uint32_t sp = ptx::smem_addr(smem + kOffP);
          for (int kb = 0; kb < nkb && ok; ++kb) {
            int s;
            if (!wait_full(&s)) { ok = false; break; }
            const uint32_t sv = ptx::smem_addr(smem + s * kStageBytes);
#pragma unroll
            for (int k16 = 0; k16 < kVKeys / 16; ++k16) {
              const uint64_t da =
                  ptx::smem_desc(sp + kb * kPBlockBytes + k16 * 32, 16, 1024, ptx::kLayoutSw128);
              // V slice: 64-column boxes of 64 keys (128-byte rows, one per
              // key) 8 KB apart (LBO); 8-key groups 1024 B apart (SBO).
              const uint64_t db =
                  ptx::smem_desc(sv + k16 * 16 * 128, kVBoxBytes, 1024, ptx::kLayoutSw128);
              ptx::mma_f16(d_tmem, da, db, idesc_o, (kb > 0 || k16 > 0) ? 1u : 0u);
            }
            ptx::mma_commit(&empty[s]);
          }
          if (ok) ptx::mma_commit(&o_full[qc & 1]);
        }
      }
      // Drain: no MMA may still write TMEM when it is freed, also after an
      // early exit (bounded; immediate on the normal path).
      ptx::mma_commit(mma_drain);
      volatile int never = 0;
      ptx::mbar_wait(mma_drain, 0, &never, kDrainLimitNs);
    }
  } else {
    // ------------------------------------------------------ softmax + epilogue
    const int quad = warp & 3;                 // TMEM lane quadrant of this warp
    const int row = quad * 32 + lane;          // query row within the unit
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    uint32_t unit_i = 0, qc = 0;
    for (long long w = blockIdx.x; w < p.units; w += gridDim.x, ++unit_i) {
      const int bh = static_cast<int>(w / p.qblocks);
      const int q = static_cast<int>(w % p.qblocks) * kBM + row;
      if (!ptx::mbar_wait_sleepy(s_full, unit_i & 1, abort_flag, p.wait_limit_ns)) {
        if (lane == 0) sdpa_error(p.err, abort_flag, kErrSdpaS);
        break;
      }
      ptx::tc_fence_after();
      const int ncols = nk * kKBox;
      // Row max over the valid keys.
      float m = -INFINITY;
      for (int c0 = 0; c0 < ncols; c0 += 32) {
        uint32_t r[32];
        ptx::tmem_ld_32x32b_x32(lane_base + c0, r);
        tmem_ld_wait_regs(r);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c0 + j < p.S) m = fmaxf(m, __uint_as_float(r[j]));
      }
      // P = exp(scale * (s - max)) as fp16 into the operand layout; row sum in fp32.
      const float mb = m * p.scale_log2;
      float l = 0.f;
      for (int c0 = 0; c0 < ncols; c0 += 32) {
        uint32_t r[32];
        ptx::tmem_ld_32x32b_x32(lane_base + c0, r);
        tmem_ld_wait_regs(r);
        uint32_t h2[16];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float e0 = (c0 + j < p.S) ? exp2f(__uint_as_float(r[j]) * p.scale_log2 - mb) : 0.f;
          const float e1 =
              (c0 + j + 1 < p.S) ? exp2f(__uint_as_float(r[j + 1]) * p.scale_log2 - mb) : 0.f;
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
      const float inv_l = 1.f / l;
      ptx::fence_proxy_async_smem();     // P visible to the tensor core
      ptx::tc_fence_before();            // every read of S done before O overwrites it
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(p_ready);
      // Output chunks.
      bool ok = true;
      for (int c = 0; c < nchunks; ++c, ++qc) {
        const int cw = min(kOChunk, p.D - c * kOChunk);
        if (!ptx::mbar_wait_sleepy(&o_full[qc & 1], (qc >> 1) & 1, abort_flag, p.wait_limit_ns)) {
          if (lane == 0) sdpa_error(p.err, abort_flag, kErrSdpaO);
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t obuf = lane_base + (qc & 1) * kOChunk;
        __half* orow = p.out + (static_cast<long long>(bh) * p.S + q) * p.D + c * kOChunk;
        for (int c0 = 0; c0 < cw; c0 += 32) {
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
        if (lane == 0) ptx::mbar_arrive(&o_empty[qc & 1]);
      }
      if (!ok) break;
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace sdpa
}  // namespace b2g
