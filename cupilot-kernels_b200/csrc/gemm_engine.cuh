// gemm_engine.cuh — the persistent, warp-specialised sm_100a fp32-input GEMM.
//
// One CTA per SM walks a list of work units (output tile x K-split).  Roles:
//   warp 0      TMA producer: 128B-swizzled A/B boxes into a STAGES-deep
//               mbarrier ring (full[s] / empty[s]).
//   warp 1      TMEM owner and MMA issuer: tcgen05.mma.kind::tf32 from the
//               shared-memory descriptors into a double-buffered fp32
//               accumulator in TMEM (tmem_full[b] / tmem_empty[b]).
//   warps 2..5  epilogue: tcgen05.ld TMEM -> registers -> a per-warp
//               swizzled shared-memory transpose -> coalesced 16-byte global
//               stores (or fp32 atomics for split-K), with the triangular
//               output mask applied on the way out.
//   warps 6..9  (XF variants only) operand transform between TMA and MMA:
//               triangular input masking (C = triu(triu(A) triu(B)) semantics
//               of kernels/14_Matmul_for_upper_triangular_matrices_best_kernel.cu:74-85)
//               and the 3xTF32 hi/lo split (ready[s]).
//
// Operand majorness lives in the descriptors, so A (M x K or K x M) and
// B (K x N or N x K) are consumed in place: no transpose pass.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "peer_protocol.cuh"
#include "ptx_sm100.cuh"

namespace b2g {

constexpr int kBlockM = 128;
constexpr int kBlockK = 32;              // fp32 elements in one 128-byte swizzle row
constexpr int kSwRowBytes = 128;
constexpr uint64_t kWaitLimitNs = 2000000000ull;   // default bound on a wait: 2 s
constexpr uint64_t kDrainLimitNs = 100000000ull;   // 0.1 s for in-flight loads at exit

enum : int { kTriNone = 0, kTriUpper = 1, kTriLower = 2 };

// Device error codes (written to the per-device error word, first one wins).
enum : int {
  kErrWaitEmpty = 0x101,
  kErrWaitFull = 0x102,
  kErrWaitReady = 0x103,
  kErrWaitTmemEmpty = 0x104,
  kErrWaitTmemFull = 0x105,
  kErrWaitXform = 0x106,
  kErrWaitUnit = 0x107,
  kErrWaitZero = 0x108,
};

struct EngineParams {
  int M, N, K, batch;
  int block_m;                 // output rows per work unit (128, or 256 for a CTA pair)
  int block_n;
  int tiles_m, tiles_n;
  int splits, kb_total, kb_per_split;
  int group_m;
  int tri;
  int a_batched, b_batched;
  long long work_units;
  float* C;
  long long ldc, stride_c;
  int atomic_out;              // split-K: accumulate into a cleared C
  int vec_ok;                  // C rows 16-byte aligned (direct-store path)
  int tma_store;               // write C with TMA tensor stores (reduce-add for split-K)
  int a_grouped, b_grouped;    // MN-major operand loaded as one 4-D box per stage
  long long wait_limit_ns;     // bound on every mbarrier wait
  int inject_stall;            // test hook: the MMA warp never signals tmem_full
  int tri_sorted;              // triangular op on square units: longest K range first
  int tri_diag;                // triangular inputs masked through diagonal-block copies
  const int4* unit_table;      // if set: unit w is {tm, tn, kb_lo, kb_hi | flags << 24}
  int diag_oob_row;            // a K row past every operand row (zero-filled by TMA)
  const float* row_bias;       // if set: C[b][i][j] += row_bias[i] (added by the K piece at 0)
  // If set: units are handed out dynamically.  sched[0] counts units drawn
  // past each CTA (pair)'s first, sched[1] the CTAs (pairs) done drawing; the
  // last one to finish resets both to 0 for the next launch.  Only for work
  // in which every unit has at least one K block.
  unsigned long long* sched;
  // Split-K without a host-side clear of C (TMA stores only): the K piece
  // that starts at 0 zeroes each of its epilogue warps' chunks of the tile
  // and then sets that warp's flag, tile_flags[tile * kFlagSlots + rank *
  // warps + warp], to `epoch`; the other pieces' matching warps wait for the
  // flag before their first reduce-add.  Null: C was cleared by the host.
  unsigned* tile_flags;
  unsigned epoch;
  int* err;
  // Tuning aid (null in normal use): per CTA, 64 words at trace[cta * 64]:
  // globaltimer stamps 0 entry, 1 after the grid-dependency wait, 2 first
  // operand stage landed (MMA warp), 3 last MMA issued, 4 first accumulator
  // ready (epilogue warp 0), 5 last store issued (epilogue warp 0), 6 exit,
  // 7 tile flag seen (split-K), 8.. epilogue warp 0's chunk groups of its
  // last unit: TMEM data in registers, store issued (pairs of stamps);
  // MMA warp totals 16 ns spent waiting for operand stages, 17 ns waiting
  // for a free accumulator buffer, 18 units; 20 + 2u / 21 + 2u: unit u's
  // first operand stage landed / last MMA issued (u < 20); 60-62 the fused
  // cross-GPU step: stores complete, grid arrival seen, exchange done.
  unsigned long long* trace;
  // Triangular unit tables with split tiles: their (tm, tn) in .x / .y of
  // n_split entries.  Every CTA (pair) first zeroes its share of them (tile
  // j by cluster j % clusters) and stamps tile_flags slot j, before it
  // takes any unit; the K pieces of a split tile then wait for that flag
  // and reduce-add.  No wait depends on the order in which units run.
  const int4* split_tiles;
  int n_split;
  // XF variants on triangular ops: 1 = only K blocks that the diagonal
  // crosses (partly masked operand boxes) go through the transform warps;
  // wholly masked boxes are loaded as TMA zero fill from outside the
  // operand, the rest go straight to the MMA.  0 = every stage is
  // transformed (3xTF32 split).
  int xf_gate;
  // Dynamic schedule: the pair leader's producer draws unit i + 1 from the
  // counter when it starts unit i, so the atomic's round trip overlaps
  // unit i's loads instead of delaying the next unit's first stage.
  int early_draw;
  // Fused cross-GPU K-split (xg.world > 1): this launch multiplies one
  // rank's K slice into C (its partial, M x N contiguous) and then sums the
  // ranks' partials on the root inside the same kernel, over the mailboxes
  // of peer_protocol.cuh: once every CTA's stores are complete (a grid-wide
  // count in this rank's mailbox), the epilogue warps of CTA i take protocol
  // chunks i, i + grid, ...: a non-root rank writes them into its landing
  // slot in the root's mailbox as {value, epoch} words; the root waits until
  // every landed word carries the epoch and adds them to its own in rank
  // order.  Same flags, slots and order of additions as the stand-alone
  // push / reduce kernels, so the two paths give identical sums.  Only plain
  // loads and stores touch peer memory.
  struct Xgpu {
    unsigned char* mbox[kPeerMaxRanks];   // every rank's mailbox as mapped here
    long long epoch, elems;
    long long nchunk, consumed_off, count_off, landing_off, slot_stride;
    int world, rank, root;
  } xg;
};

// Triangular masking of one operand box, for one CTA: 0 nothing masked,
// 1 partly masked (the diagonal crosses the box), 2 wholly masked.
// A: rows [m0, m0 + 128) x K block [k0, k0 + 32); upper zeroes k < i,
// lower k > i (kernels/14_...:74-75, kernels/15_... assumes the same).
__host__ __device__ inline int tri_mask_a(int tri, int m0, int k0) {
  if (tri == kTriUpper) {
    if (k0 + kBlockK - 1 < m0) return 2;
    return k0 >= m0 + kBlockM - 1 ? 0 : 1;
  }
  if (tri == kTriLower) {
    if (k0 > m0 + kBlockM - 1) return 2;
    return k0 + kBlockK - 1 <= m0 ? 0 : 1;
  }
  return 0;
}
// B: K block [k0, k0 + 32) x columns [n0, n0 + cols); upper zeroes k > j,
// lower k < j.
__host__ __device__ inline int tri_mask_b(int tri, int n0, int cols, int k0) {
  if (tri == kTriUpper) {
    if (k0 > n0 + cols - 1) return 2;
    return k0 + kBlockK - 1 <= n0 ? 0 : 1;
  }
  if (tri == kTriLower) {
    if (k0 + kBlockK - 1 < n0) return 2;
    return k0 >= n0 + cols - 1 ? 0 : 1;
  }
  return 0;
}

constexpr int kFlagSlots = 16;     // epilogue warps per tile (8 per CTA, a pair)

// Depth of the per-CTA ring through which the pair leader's producer hands
// dynamically drawn unit indices to every role of both CTAs.  A role can
// lag the producer by at most STAGES + 2 units (operand stages, then
// accumulator buffers, each unit holding >= 1 K block), far below it.
constexpr int kUnitQueue = 32;

// The sequence of units a CTA (pair) runs: unit0, unit0 + step, ... when
// static; the ring's entries, in order, when dynamic.  get() returns false
// when a bounded wait gave up.
struct UnitSource {
  uint64_t* bars;
  long long* slots;
  long long unit0, step;
  bool dyn;
  __device__ __forceinline__ bool get(uint32_t i, long long& w, volatile int* abort,
                                      uint64_t limit_ns) const {
    if (!dyn) {
      w = unit0 + static_cast<long long>(i) * step;
      return true;
    }
    const int q = static_cast<int>(i % kUnitQueue);
    if (!ptx::mbar_wait_cluster(&bars[q], (i / kUnitQueue) & 1, abort, limit_ns)) return false;
    w = *reinterpret_cast<volatile long long*>(&slots[q]);
    return true;
  }
};

struct WorkUnit {
  int b, tm, tn, kb_lo, kb_hi;
  int accumulate;   // reduce-add into C (a K piece of a split tile)
  int skip;         // padding entry of a unit table: no work, no output
  int flag;         // split tile: its slot in EngineParams::tile_flags, else -1
  int first;        // the K piece that clears the tile before any piece adds
};

// Unit-table entries: {tm | (flag slot + 1) << 16, tn, kb_lo, kb_hi | flags << 24}.
enum : int { kUnitAccumulate = 1, kUnitSkip = 2, kUnitFirst = 4 };

// Map a linear work-unit index to (batch, tile, K range).  Tiles are
// rasterised in groups of group_m tile-rows so CTAs that run together share
// B columns in L2; split-K pieces of one tile are adjacent.  Triangular ops
// clip the K range to the structurally non-zero band and give tiles that
// lie wholly in the masked triangle an empty range.
// Triangular ops on square units (block_m == block_n): enumerate the tiles
// by decreasing K-range length so a static round-robin schedule stays
// balanced.  Upper: tile (tm, tn) has K range [tm, tn] in units, length
// tn - tm + 1, for d = tn - tm >= 0; lower mirrors it.  Order: d = T-1 down
// to 0 (T - d tiles each), then the tiles wholly in the masked triangle.
__host__ __device__ inline void decode_tri_sorted(const EngineParams& p, long long t, int* tm,
                                                  int* tn) {
  const int T = p.tiles_n;
  long long rem = t;
  int d = T - 1;
  while (d >= 0 && rem >= T - d) {
    rem -= T - d;
    --d;
  }
  int lo, hi;            // lo: index along the diagonal, hi = lo + offset
  if (d >= 0) {
    lo = static_cast<int>(rem);
    hi = lo + d;
    if (p.tri == kTriUpper) { *tm = lo; *tn = hi; } else { *tm = hi; *tn = lo; }
    return;
  }
  // Masked tiles: offsets e = 1 .. T-1 with T - e tiles each.
  int e = 1;
  while (e < T && rem >= T - e) {
    rem -= T - e;
    ++e;
  }
  lo = static_cast<int>(rem);
  hi = lo + e;
  if (p.tri == kTriUpper) { *tm = hi; *tn = lo; } else { *tm = lo; *tn = hi; }
}

__host__ __device__ inline WorkUnit decode_unit(const EngineParams& p, long long w) {
  WorkUnit u;
  u.accumulate = 0;
  u.skip = 0;
  u.flag = -1;
  u.first = 0;
  if (p.unit_table != nullptr) {
#ifdef __CUDA_ARCH__
    const int4 e = __ldg(p.unit_table + w);
#else
    const int4 e = p.unit_table[w];
#endif
    u.b = 0;
    u.tm = e.x & 0xFFFF;
    u.flag = (e.x >> 16) - 1;
    u.tn = e.y;
    u.kb_lo = e.z;
    u.kb_hi = e.w & 0xFFFFFF;
    u.accumulate = (e.w >> 24) & kUnitAccumulate;
    u.skip = ((e.w >> 24) & kUnitSkip) ? 1 : 0;
    u.first = ((e.w >> 24) & kUnitFirst) ? 1 : 0;
    return u;
  }
  const int split = static_cast<int>(w % p.splits);
  const long long t = w / p.splits;
  const long long per_batch = static_cast<long long>(p.tiles_m) * p.tiles_n;
  u.b = static_cast<int>(t / per_batch);
  const long long r = t % per_batch;
  const long long span = static_cast<long long>(p.group_m) * p.tiles_n;
  const int grp = static_cast<int>(r / span);
  const int first_m = grp * p.group_m;
  const int rem_m = p.tiles_m - first_m;
  const int gsz = rem_m < p.group_m ? rem_m : p.group_m;
  const long long rr = r - static_cast<long long>(grp) * span;
  u.tm = first_m + static_cast<int>(rr % gsz);
  u.tn = static_cast<int>(rr / gsz);
  if (p.tri_sorted) decode_tri_sorted(p, r, &u.tm, &u.tn);
  int lo = split * p.kb_per_split;
  int hi = lo + p.kb_per_split;
  if (hi > p.kb_total) hi = p.kb_total;
  if (p.tri != kTriNone) {
    const long long m0 = static_cast<long long>(u.tm) * p.block_m;
    const long long n0 = static_cast<long long>(u.tn) * p.block_n;
    long long klo, khi;
    if (p.tri == kTriUpper) {  // k in [i, j]
      klo = m0;
      khi = n0 + p.block_n;
      if (n0 + p.block_n - 1 < m0) khi = klo;       // tile wholly below the diagonal
    } else {                   // k in [j, i]
      klo = n0;
      khi = m0 + p.block_m;
      if (n0 > m0 + p.block_m - 1) khi = klo;        // tile wholly above the diagonal
    }
    if (khi > p.K) khi = p.K;
    int tlo = static_cast<int>(klo / kBlockK);
    int thi = khi > klo ? static_cast<int>((khi + kBlockK - 1) / kBlockK) : tlo;
    if (tlo > lo) lo = tlo;
    if (thi < hi) hi = thi;
  }
  if (hi < lo) hi = lo;
  u.kb_lo = lo;
  u.kb_hi = hi;
  if (p.tile_flags != nullptr) {   // split-K: every piece of a tile shares its flags
    u.flag = static_cast<int>(t);
    u.first = split == 0;
  }
  return u;
}

// PAIR: a cluster of two CTAs computes one 256 x BN unit with
// tcgen05.mma.cta_group::2; each CTA holds 128 rows of A, its half of every
// N=256 B sub-tile and its 128 x BN part of the accumulator.  BN = 512 (pair
// only) issues two N=256 MMAs per K step over one shared A tile: more flops
// per operand byte streamed from L2, at the price of a single-buffered
// accumulator (512 TMEM columns), so its epilogue does not overlap the next
// unit's mainloop.
template <int BN, int STAGES, bool A_MN, bool B_MN, bool X3, bool XF, bool PAIR, int EPIG = 1,
          int EPIW = 8>
struct EngineCfg {
  static constexpr int kCtas = PAIR ? 2 : 1;
  static constexpr int kUnitM = kBlockM * kCtas;
  static constexpr int kMmaN = BN > 256 ? 256 : BN;           // N of one MMA instruction
  static constexpr int kNSub = BN / kMmaN;                    // MMAs per K=8 step
  static constexpr int kSubCols = kMmaN / kCtas;              // B columns per CTA per sub-tile
  static constexpr int kBnCta = BN / kCtas;                   // B columns loaded per CTA
  static constexpr int kABytes = kBlockM * kBlockK * 4;
  static constexpr int kBSubBytes = kSubCols * kBlockK * 4;
  static constexpr int kBBytes = kBnCta * kBlockK * 4;
  static constexpr bool kPreSplit = X3 && !XF;               // lo parts loaded by TMA
  static constexpr int kStageTx = (kABytes + kBBytes) * (kPreSplit ? 2 : 1);   // per CTA
  static constexpr int kOperandBufs = X3 ? 2 : 1;
  static constexpr int kOffA = 0;
  static constexpr int kOffB = STAGES * kABytes;
  static constexpr int kOffALo = STAGES * (kABytes + kBBytes);
  static constexpr int kOffBLo = kOffALo + STAGES * kABytes;
  static constexpr int kOffEpi = STAGES * (kABytes + kBBytes) * kOperandBufs;
  static constexpr int kEpiWarps = EPIW;                     // EPIW / 4 per TMEM lane quadrant
  static constexpr int kEpiParts = EPIW / 4;
  static_assert(EPIW % 4 == 0 && EPIW >= 4, "epilogue warps come in quadrant sets");
  static constexpr int kEpiBufBytes = 32 * 32 * 4;           // one 32 x 32 fp32 box
  // Staging boxes per epilogue warp.  One: each chunk waits for the previous
  // store to have read the box.  More: a ring, up to EPIG - 1 stores of the
  // warp still reading while the next box is written (output-bound shapes).
  static constexpr int kEpiBufs = EPIG;
  static constexpr int kEpiGroup = 1;                        // chunks staged per fence
  static constexpr int kEpiBytes = kEpiWarps * kEpiBufs * kEpiBufBytes;
  // A CTA's last unit stages its output in the idle operand stages instead:
  // a ring of this many boxes per epilogue warp, so its stores overlap.
  static constexpr int kTailBoxes = kOffEpi / (kEpiWarps * kEpiBufBytes);
  static constexpr int kOffBar = kOffEpi + kEpiBytes;
  static constexpr int kNumBars = 3 * STAGES + 5;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kOffQueue = kOffMisc + 16;            // unit ring: barriers, then slots
  static constexpr int kSmemBytes = kOffQueue + kUnitQueue * 16 + 1024;   // + alignment slack
  static constexpr int kAccBufs = BN > 256 ? 1 : 2;         // accumulator buffers in TMEM
  static constexpr int kTmemCols = kAccBufs * BN;
  static constexpr int kXformWarps = XF ? 4 : 0;
  static constexpr int kThreads = (2 + kEpiWarps + kXformWarps) * 32;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static_assert(kTmemCols == 256 || kTmemCols == 512, "TMEM allocation must be a power of two");
  static_assert(BN % 64 == 0 && BN <= (PAIR ? 512 : 256), "BN");
  static_assert(!(PAIR && XF) || kNSub == 1, "transform warps handle one B sub-tile");
};

__device__ __forceinline__ void record_error(int* err, volatile int* abort, int code) {
  atomicCAS(err, 0, code);
  *abort = 1;
}

// Zero (mask) and/or split one operand tile in shared memory.
// Tile layout as TMA wrote it:
//   !MN: 128-byte swizzle; rows are M (or N) indices, each row holds 32 K
//        values, 16-byte chunk c stored at c ^ (row % 8).
//   MN : 32-byte-atom swizzle; groups of 32 M (or N) values, within a group
//        rows are K indices, 32-byte chunk c stored at c ^ (row % 4).
// mn0 / k0 are the global coordinates of the tile's first element.
// rule: 0 none, 1 zero where k < mn, 2 zero where k > mn.
template <bool MN, int EXT, bool SPLIT>
__device__ __forceinline__ void transform_tile(float* tile, float* lo_tile, int mn0, int k0,
                                               int rule, int xt) {
  constexpr int kChunks = EXT * kBlockK / 4;   // 16-byte chunks in the tile
  if (rule == 0 && !SPLIT) return;
#pragma unroll 4
  for (int c = xt; c < kChunks; c += 128) {
    int mn_base, k_base, mn_step, k_step;
    if (!MN) {
      const int row = c >> 3;
      const int logc = (c & 7) ^ (row & 7);
      mn_base = mn0 + row;
      k_base = k0 + logc * 4;
      mn_step = 0;
      k_step = 1;
    } else {
      const int g = c / (kBlockK * 8);
      const int rem = c - g * (kBlockK * 8);
      const int krow = rem >> 3;
      const int phys = rem & 7;                              // 16-byte chunk in the row
      const int logc = ((((phys >> 1) ^ (krow & 3))) << 1) | (phys & 1);
      mn_base = mn0 + g * 32 + logc * 4;
      k_base = k0 + krow;
      mn_step = 1;
      k_step = 0;
    }
    if (!SPLIT) {
      // Masking only: classify the chunk's four elements first.  Wholly
      // masked chunks are overwritten with zeros without a read; chunks with
      // nothing masked are left alone; only chunks on the diagonal are read.
      const int kmin = k_base, kmax = k_base + 3 * k_step;
      const int mnmin = mn_base, mnmax = mn_base + 3 * mn_step;
      const bool all = (rule == 1) ? (kmax < mnmin) : (kmin > mnmax);
      const bool none = (rule == 1) ? (kmin >= mnmax) : (kmax <= mnmin);
      if (none) continue;
      if (all) {
        reinterpret_cast<float4*>(tile)[c] = make_float4(0.f, 0.f, 0.f, 0.f);
        continue;
      }
    }
    float4 v = reinterpret_cast<float4*>(tile)[c];
    float e[4] = {v.x, v.y, v.z, v.w};
    bool changed = false;
    if (rule != 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int mn = mn_base + q * mn_step;
        const int k = k_base + q * k_step;
        const bool zero = (rule == 1) ? (k < mn) : (k > mn);
        if (zero && e[q] != 0.0f) {
          e[q] = 0.0f;
          changed = true;
        }
      }
    }
    if (SPLIT) {
      float h[4], l[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        // hi keeps the 10 explicit mantissa bits a TF32 operand carries;
        // lo = x - hi is exact in fp32.
        h[q] = __uint_as_float(__float_as_uint(e[q]) & 0xFFFFE000u);
        l[q] = e[q] - h[q];
      }
      reinterpret_cast<float4*>(tile)[c] = make_float4(h[0], h[1], h[2], h[3]);
      reinterpret_cast<float4*>(lo_tile)[c] = make_float4(l[0], l[1], l[2], l[3]);
    } else if (changed) {
      reinterpret_cast<float4*>(tile)[c] = make_float4(e[0], e[1], e[2], e[3]);
    }
  }
}

__device__ __forceinline__ void store4(const EngineParams& p, float* crow, int grow, int gcol,
                                       float v0, float v1, float v2, float v3) {
  float e[4] = {v0, v1, v2, v3};
  if (p.tri == kTriUpper) {
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (gcol + q < grow) e[q] = 0.0f;
  } else if (p.tri == kTriLower) {
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (gcol + q > grow) e[q] = 0.0f;
  }
  if (p.vec_ok && gcol + 3 < p.N) {
    float4* dst = reinterpret_cast<float4*>(crow + gcol);
    if (p.atomic_out)
      atomicAdd(dst, make_float4(e[0], e[1], e[2], e[3]));
    else
      *dst = make_float4(e[0], e[1], e[2], e[3]);
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (gcol + q < p.N) {
        if (p.atomic_out)
          atomicAdd(crow + gcol + q, e[q]);
        else
          crow[gcol + q] = e[q];
      }
    }
  }
}

// Wait for the asynchronous tcgen05.ld results, and pin every register of
// `r` behind that wait so the compiler cannot read them earlier.
__device__ __forceinline__ void tmem_ld_wait_regs(uint32_t (&r)[32]) {
  ptx::tmem_ld_wait();
#pragma unroll
  for (int i = 0; i < 32; ++i) asm volatile("" : "+r"(r[i]));
}

// One 32-row x 32-column accumulator chunk held by a warp (row = lane) to
// global memory.  TMA path: swizzled 4 KB staging box -> tensor store (or
// fp32 add-reduction for split-K); otherwise a swizzled transpose and
// coalesced (or scalar, or atomic) stores.
template <int NBUF>
__device__ __forceinline__ void store_chunk(const EngineParams& p, const CUtensorMap* map_c,
                                            float* stg, uint32_t& seq, uint32_t (&r)[32], int b,
                                            int row0, int col0, int lane, int accumulate) {
  const int row = row0 + lane;
  if (p.tri == kTriUpper) {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col0 + j < row) r[j] = 0u;
  } else if (p.tri == kTriLower) {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col0 + j > row) r[j] = 0u;
  }
  if (p.tma_store) {
    // NBUF staging boxes per warp: wait until the store issued from this
    // box NBUF chunks ago has read it (up to NBUF - 1 stay in flight).
    float* buf = stg + (seq % NBUF) * (32 * 32);
    if (lane == 0) ptx::bulk_wait_read<NBUF - 1>();
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<float4*>(buf + lane * 32 + ((j ^ (lane & 7)) * 4)) =
          make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                      __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
    ptx::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      if (p.atomic_out || accumulate)
        ptx::tma_reduce_add_3d(map_c, buf, col0, row0, b);
      else
        ptx::tma_store_3d(map_c, buf, col0, row0, b);
      ptx::bulk_commit();
    }
    ++seq;
    return;
  }
  float* cb = p.C + static_cast<long long>(b) * p.stride_c;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    *reinterpret_cast<float4*>(stg + lane * 32 + ((j ^ (lane & 7)) * 4)) =
        make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                    __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
  __syncwarp();
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int r_local = it * 4 + (lane >> 3);
    const int jj = lane & 7;
    const float4 v =
        *reinterpret_cast<const float4*>(stg + r_local * 32 + ((jj ^ (r_local & 7)) * 4));
    const int grow = row0 + r_local;
    const int gcol = col0 + jj * 4;
    if (grow < p.M && gcol < p.N)
      store4(p, cb + static_cast<long long>(grow) * p.ldc, grow, gcol, v.x, v.y, v.z, v.w);
  }
  __syncwarp();
}

// G accumulator chunks of a warp (row = lane; chunk g at column col0[g]) to
// global memory through G swizzled staging boxes: one wait for the previous
// group's stores to have read the boxes, one proxy fence, G tensor stores
// (or fp32 add-reductions for split-K).
template <int G, int PENDING = 0>
__device__ __forceinline__ void store_group_tma(const EngineParams& p, const CUtensorMap* map_c,
                                                float* stg, uint32_t (&r)[G][32], int ng, int b,
                                                int row0, const int (&col0)[G], int lane,
                                                int accumulate) {
  const int row = row0 + lane;
  if (p.tri != kTriNone) {
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int col = col0[g] + j;
        if (p.tri == kTriUpper ? (col < row) : (col > row)) r[g][j] = 0u;
      }
  }
  // Staging boxes reused: wait until at most PENDING earlier store groups
  // of this warp may still be reading theirs (0: a single box).
  if (lane == 0) ptx::bulk_wait_read<PENDING>();
  __syncwarp();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (g < ng) {
      float* buf = stg + g * 32 * 32;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        *reinterpret_cast<float4*>(buf + lane * 32 + ((j ^ (lane & 7)) * 4)) =
            make_float4(__uint_as_float(r[g][4 * j]), __uint_as_float(r[g][4 * j + 1]),
                        __uint_as_float(r[g][4 * j + 2]), __uint_as_float(r[g][4 * j + 3]));
    }
  }
  ptx::fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      if (g < ng) {
        if (p.atomic_out || accumulate)
          ptx::tma_reduce_add_3d(map_c, stg + g * 32 * 32, col0[g], row0, b);
        else
          ptx::tma_store_3d(map_c, stg + g * 32 * 32, col0[g], row0, b);
      }
    }
    ptx::bulk_commit();
  }
}

// Barrier among the epilogue warps only (named barrier 1; the other roles
// never take part).
__device__ __forceinline__ void epi_bar_sync(int threads) {
  asm volatile("bar.sync 1, %0;" ::"r"(threads) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_gpu_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// The fused cross-GPU exchange (EngineParams::Xgpu), run by the `threads`
// epilogue threads of every CTA after their last store; t = thread index
// among them, flag = a shared-memory word for broadcasting.
// credit_ok: the non-root's slot credits, checked at the epilogue's start.
// trace (tuning aid, thread 0): words 60 stores complete, 58 first landed
// group read (root), 61 grid arrival seen, 63 landed values in registers,
// 62 exchange done.
// Not inlined, and given a copy of the exchange's parameters rather than the
// kernel's: the mainloop's register allocation and parameter accesses stay
// as they are without the exchange.
__device__ __noinline__ void xgpu_exchange(const EngineParams::Xgpu* xp, float* out_c,
                                           long long wait_limit_ns, int* err, int threads, int t,
                                           volatile int* abort_flag, volatile int* flag,
                                           int credit_ok, unsigned long long* trace) {
  const EngineParams::Xgpu& x = *xp;
  // 1. This thread's bulk stores (TMA stores / reduce-adds) are complete in
  //    global memory and visible to generic-proxy loads of any SM.
  if ((t & 31) == 0) {
    ptx::bulk_wait_all();
    ptx::fence_proxy_async_global();
  }
  epi_bar_sync(threads);
  if (trace && t == 0) trace[60] = ptx::globaltimer_ns();
  // 2. Grid-wide arrival in this rank's mailbox (the wait for the others
  //    comes below).  The count word carries the epoch in its upper bits:
  //    every CTA first raises it to at least this epoch's tag (a word left
  //    by an earlier epoch, or by a launch that gave up, drops to the tag),
  //    then adds one: two atomics per CTA and no retry loop (a
  //    compare-and-swap loop serialises the grid's arrivals).
  unsigned long long* cnt = reinterpret_cast<unsigned long long*>(x.mbox[x.rank] + x.count_off);
  const unsigned long long tag = static_cast<unsigned long long>(x.epoch) << 20;
  if (t == 0) {
    __threadfence();   // release: the CTA's stores (ordered by the barrier) before the count
    atomicMax(cnt, tag);
    atomicAdd(cnt, 1ull);
  }
  // Root: the other ranks' values do not depend on this rank's other CTAs,
  // so this thread's first group is awaited and read now, while the grid
  // completes (its first access to the landing slot is the slow one).
  const bool is_root = x.rank == x.root;
  const uint32_t lflag = static_cast<uint32_t>(x.epoch);
  const uint64_t* land_slot = reinterpret_cast<const uint64_t*>(
      x.mbox[x.root] + x.landing_off + (x.epoch & 1) * x.world * x.slot_stride);
  const long long stride = x.slot_stride / 8;   // words per (slot, rank) region
  const long long i_pre = static_cast<long long>(blockIdx.x) * kPeerChunk + 4ll * t;
  const bool have_pre = is_root && blockIdx.x < x.nchunk && 4ll * t < kPeerChunk &&
                        i_pre + 4 <= x.elems;
  float4 pre = make_float4(0.f, 0.f, 0.f, 0.f);   // landed values, summed in rank order
  bool pre_ok = true;
  if (have_pre) pre_ok = peer_ll_sum4(land_slot, stride, x.world, x.root, i_pre, lflag,
                                      wait_limit_ns, &pre);
  if (trace && t == 0) trace[58] = ptx::globaltimer_ns();
  // 3. Wait until every CTA of the grid has arrived.
  if (t == 0) {
    const unsigned long long want = tag + gridDim.x;
    const uint64_t t0 = ptx::globaltimer_ns();
    int ok = 1;
    while (ld_acquire_gpu_u64(cnt) != want) {
      if (*abort_flag || ptx::globaltimer_ns() - t0 > static_cast<uint64_t>(wait_limit_ns)) {
        ok = 0;
        break;
      }
      __nanosleep(64);
    }
    if (!ok && !*abort_flag) record_error(err, abort_flag, kErrPeerGrid);
    *flag = ok && !*abort_flag && (x.rank == x.root || credit_ok);
    if (trace) trace[61] = ptx::globaltimer_ns();
  }
  // Thread 0's acquire of the count and the barrier order every thread's
  // loads below after the other CTAs' stores.
  epi_bar_sync(threads);
  if (!*flag) return;
  float* out = out_c;
  for (long long c = blockIdx.x; c < x.nchunk; c += gridDim.x) {
    const long long i0 = c * kPeerChunk;
    const long long i1 = i0 + kPeerChunk < x.elems ? i0 + kPeerChunk : x.elems;
    if (!is_root) {
      // Each value lands with the epoch in its flag half: no ready flag and
      // no fence on this path.
      uint64_t* dst = const_cast<uint64_t*>(land_slot) + x.rank * stride;
      for (long long i = i0 + 4ll * t; i < i1; i += 4ll * threads) {
        if (i + 4 <= i1) {
          peer_ll_put4(dst + i, __ldcg(reinterpret_cast<const float4*>(out + i)), lflag);
        } else {
          for (long long j = i; j < i1; ++j) peer_ll_put1(dst + j, __ldcg(out + j), lflag);
        }
      }
    } else {
      for (long long i = i0 + 4ll * t; i < i1; i += 4ll * threads) {
        bool ok = true;
        if (i + 4 <= i1) {
          float4 lsum = pre;
          if (!(have_pre && i == i_pre))
            ok = peer_ll_sum4(land_slot, stride, x.world, x.root, i, lflag, wait_limit_ns, &lsum);
          else
            ok = pre_ok;
          if (trace && t == 0) trace[63] = ptx::globaltimer_ns();
          if (ok) {
            float4 acc = __ldcg(reinterpret_cast<const float4*>(out + i));
            acc.x += lsum.x;
            acc.y += lsum.y;
            acc.z += lsum.z;
            acc.w += lsum.w;
            *reinterpret_cast<float4*>(out + i) = acc;
          }
        } else {
          for (long long j = i; j < i1 && ok; ++j) {
            float lsum = 0.f;
            for (int r = 0; r < x.world && ok; ++r) {
              float v = 0.f;
              if (r != x.root) ok = peer_ll_get1(land_slot + r * stride + j, lflag,
                                                 wait_limit_ns, &v);
              lsum += v;
            }
            if (ok) out[j] = __ldcg(out + j) + lsum;
          }
        }
        if (!ok) {
          record_error(err, abort_flag, kErrPeerReady);
          break;
        }
      }
    }
  }
  if (trace && t == 0) trace[62] = ptx::globaltimer_ns();
}

template <int BN, int STAGES, bool A_MN, bool B_MN, bool X3, bool XF, bool PAIR, int EPIG,
          int EPIW>
__global__ void __launch_bounds__(
    EngineCfg<BN, STAGES, A_MN, B_MN, X3, XF, PAIR, EPIG, EPIW>::kThreads, 1)
    gemm_tf32_kernel(const __grid_constant__ CUtensorMap map_a,
                     const __grid_constant__ CUtensorMap map_b,
                     const __grid_constant__ CUtensorMap map_c,
                     const __grid_constant__ CUtensorMap map_ad,
                     const __grid_constant__ CUtensorMap map_bd, const EngineParams p) {
  using Cfg = EngineCfg<BN, STAGES, A_MN, B_MN, X3, XF, PAIR, EPIG, EPIW>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* ready = bars + 2 * STAGES;
  uint64_t* tmem_full = bars + 3 * STAGES;
  uint64_t* tmem_empty = tmem_full + 2;
  uint64_t* mma_drain = tmem_full + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Cfg::kOffMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? ptx::cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const long long unit0 = PAIR ? (blockIdx.x >> 1) : blockIdx.x;
  const long long unit_step = PAIR ? (gridDim.x >> 1) : gridDim.x;
  UnitSource units;
  units.bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffQueue);
  units.slots = reinterpret_cast<long long*>(smem + Cfg::kOffQueue + kUnitQueue * 8);
  units.unit0 = unit0;
  units.step = unit_step;
  units.dyn = p.sched != nullptr;
  // Does stage (u, kb) go through the transform warps?  Every stage of an XF
  // variant unless xf_gate; then only the K blocks that the diagonal crosses
  // for either CTA of the pair (both CTAs decide alike).
  auto gated = [&](const WorkUnit& u, int kb) -> bool {
    if (!XF) return false;
    if (X3 || !p.xf_gate) return true;
    const int k0 = kb * kBlockK;
#pragma unroll
    for (int r = 0; r < Cfg::kCtas; ++r) {
      if (tri_mask_a(p.tri, u.tm * Cfg::kUnitM + r * kBlockM, k0) == 1) return true;
      if (tri_mask_b(p.tri, u.tn * BN + r * Cfg::kSubCols, Cfg::kBnCta, k0) == 1) return true;
    }
    return false;
  };

  unsigned long long* trace = p.trace ? p.trace + static_cast<size_t>(blockIdx.x) * 64 : nullptr;
  if (trace && threadIdx.x == 0) trace[0] = ptx::globaltimer_ns();
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
      ptx::mbar_init(&ready[s], Cfg::kXformWarps > 0 ? Cfg::kXformWarps * Cfg::kCtas : 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(&tmem_full[b], 1);
      ptx::mbar_init(&tmem_empty[b], Cfg::kEpiWarps * Cfg::kCtas);
    }
    ptx::mbar_init(mma_drain, 1);
    for (int q = 0; q < kUnitQueue; ++q) ptx::mbar_init(&units.bars[q], 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&map_a);
    ptx::prefetch_tmap(&map_b);
    if (p.tma_store) ptx::prefetch_tmap(&map_c);
    if (p.tri_diag) {
      ptx::prefetch_tmap(&map_ad);
      ptx::prefetch_tmap(&map_bd);
    }
  }
  if (warp == 1) {
    if (PAIR) {
      ptx::tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
      ptx::tmem_relinquish_pair();
    } else {
      ptx::tmem_alloc(tmem_slot, Cfg::kTmemCols);
      ptx::tmem_relinquish();
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (PAIR) ptx::cluster_sync();   // peer barriers initialised before any remote arrive
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Launched with programmatic stream serialization: the set-up above may
  // overlap the previous kernel's tail; every global-memory access (operand
  // loads, unit tables, counters, output) comes after this wait.
  ptx::griddep_launch_dependents();
  ptx::griddep_wait();
  if (trace && threadIdx.x == 0) trace[1] = ptx::globaltimer_ns();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint32_t full_leader = PAIR ? ptx::mapa_shared(ptx::smem_addr(full), 0) : 0u;
      // The pair leader's producer draws the units (dynamic schedule) and
      // publishes each to both CTAs' rings; every other role reads a ring.
      const bool fetcher = units.dyn && leader;
      uint32_t it = 0;
      bool ok = true;
      unsigned long long drawn = 0;
      for (uint32_t ui = 0; ok; ++ui) {
        long long w;
        if (fetcher) {
          if (ui == 0)
            w = unit0;
          else if (p.early_draw)
            w = unit_step + static_cast<long long>(drawn);
          else
            w = unit_step + static_cast<long long>(atomicAdd(p.sched, 1ull));
          const int q = static_cast<int>(ui % kUnitQueue);
          *reinterpret_cast<volatile long long*>(&units.slots[q]) = w;
          ptx::mbar_arrive(&units.bars[q]);
          if (PAIR) {
            ptx::st_shared_cluster_u64(ptx::mapa_shared(ptx::smem_addr(&units.slots[q]), 1),
                                       static_cast<uint64_t>(w));
            ptx::mbar_arrive_cluster(ptx::mapa_shared(ptx::smem_addr(&units.bars[q]), 1));
          }
          // The next unit's index is only read at the top of the next
          // iteration, so the warp does not wait for the atomic here.
          if (p.early_draw && w < p.work_units) drawn = atomicAdd(p.sched, 1ull);
        } else if (!units.get(ui, w, abort_flag, p.wait_limit_ns)) {
          record_error(p.err, abort_flag, kErrWaitUnit);
          break;
        }
        if (w >= p.work_units) break;
        const WorkUnit u = decode_unit(p, w);
        const int m_cta = u.tm * Cfg::kUnitM + static_cast<int>(rank) * kBlockM;
        // B sub-tile j of this CTA: columns [n0 + j*kMmaN + rank*kSubCols, +kSubCols)
        const int n_cta = u.tn * BN + static_cast<int>(rank) * Cfg::kSubCols;
        const int ab = p.a_batched ? u.b : 0;
        const int bb = p.b_batched ? u.b : 0;
        for (int kb = u.kb_lo; kb < u.kb_hi; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!ptx::mbar_wait(&empty[s], ph ^ 1, abort_flag, p.wait_limit_ns)) {
            record_error(p.err, abort_flag, kErrWaitEmpty);
            ok = false;
            break;
          }
          // Each CTA's loads complete on its own barrier when transform warps
          // must see them; otherwise a pair's loads complete on the leader's
          // (and, in an XF pair, the other CTA arrives on its own barrier so
          // that its phases stay in step with the leader's).
          const bool xg = gated(u, kb);
          const bool pair_load = PAIR && !xg;
          if (!pair_load)
            ptx::mbar_arrive_expect_tx(&full[s], Cfg::kStageTx);
          else if (leader)
            ptx::mbar_arrive_expect_tx(&full[s], 2 * Cfg::kStageTx);
          else if (XF)
            ptx::mbar_arrive(&full[s]);
          uint8_t* sa = smem + Cfg::kOffA + s * Cfg::kABytes;
          uint8_t* sb = smem + Cfg::kOffB + s * Cfg::kBBytes;
          const int k0 = kb * kBlockK;
          // Gated triangular stages: a wholly masked box of this CTA is read
          // from a K coordinate before the operand (TMA writes zeros, no
          // memory traffic); a partly masked one is loaded and masked by the
          // transform warps.
          int ka = k0, kbb = k0;
          if (XF && !X3 && p.xf_gate) {
            if (tri_mask_a(p.tri, m_cta, k0) == 2) ka = -kBlockK;
            if (tri_mask_b(p.tri, n_cta, Cfg::kBnCta, k0) == 2) kbb = -kBlockK;
          }
          auto load = [&](void* dst, const CUtensorMap* map, int c0, int c1, int c2) {
            if (pair_load)
              ptx::tma_load_3d_pair(dst, map, full_leader + s * 8, c0, c1, c2);
            else
              ptx::tma_load_3d(dst, map, &full[s], c0, c1, c2);
          };
          // MN-major operand as {32, K, group, batch}: one box of all groups.
          auto load_grouped = [&](void* dst, const CUtensorMap* map, int kc, int g0, int c3) {
            if (pair_load)
              ptx::tma_load_4d_pair(dst, map, full_leader + s * 8, 0, kc, g0, c3);
            else
              ptx::tma_load_4d(dst, map, &full[s], 0, kc, g0, c3);
          };
          // Triangular operands through diagonal-block copies: a K block that
          // crosses this CTA's diagonal block comes from the masked copy, one
          // wholly in the masked triangle from outside every operand (TMA
          // fills zeros), any other from the operand itself.
          bool a_done = false, b_done = false;
          if (!A_MN && !XF && p.tri_diag) {
            const bool use_diag = p.tri == kTriUpper ? (k0 < m_cta + kBlockM)
                                                     : (k0 + kBlockK - 1 >= m_cta);
            if (use_diag) {
              load(sa, &map_ad, k0 - m_cta, m_cta, 0);   // x < 0 or >= 128: zero fill
              a_done = true;
            }
          }
          if (B_MN && !XF && p.tri_diag && Cfg::kNSub == 1) {
            const int c0 = n_cta;
            int y = -1;
            if (p.tri == kTriUpper) {
              if (k0 >= c0) y = k0 < c0 + Cfg::kSubCols ? k0 : p.diag_oob_row;
            } else {
              if (k0 < c0 + Cfg::kSubCols) y = k0 >= c0 ? k0 : -kBlockK;
            }
            if (y != -1) {
              if (pair_load)
                ptx::tma_load_4d_pair(sb, &map_bd, full_leader + s * 8, 0, y, 0, 0);
              else
                ptx::tma_load_4d(sb, &map_bd, &full[s], 0, y, 0, 0);
              b_done = true;
            }
          }
          if (X3 && !XF) {
            // 3xTF32 with pre-split operands: the lo parts come from their own
            // copies (map_ad / map_bd), at the same coordinates as A and B.
            uint8_t* sal = smem + Cfg::kOffALo + s * Cfg::kABytes;
            uint8_t* sbl = smem + Cfg::kOffBLo + s * Cfg::kBBytes;
            if (!A_MN) {
              load(sal, &map_ad, k0, m_cta, ab);
            } else if (p.a_grouped) {
              load_grouped(sal, &map_ad, k0, m_cta / 32, ab);
            } else {
#pragma unroll
              for (int j = 0; j < kBlockM / 32; ++j)
                load(sal + j * kBlockK * kSwRowBytes, &map_ad, m_cta + 32 * j, k0, ab);
            }
#pragma unroll
            for (int j = 0; j < Cfg::kNSub; ++j) {
              uint8_t* sblj = sbl + j * Cfg::kBSubBytes;
              const int nj = n_cta + j * Cfg::kMmaN;
              if (!B_MN) {
                load(sblj, &map_bd, k0, nj, bb);
              } else if (p.b_grouped) {
                load_grouped(sblj, &map_bd, k0, nj / 32, bb);
              } else {
#pragma unroll
                for (int g = 0; g < Cfg::kSubCols / 32; ++g)
                  load(sblj + g * kBlockK * kSwRowBytes, &map_bd, nj + 32 * g, k0, bb);
              }
            }
          }
          if (a_done) {
          } else if (!A_MN) {
            load(sa, &map_a, ka, m_cta, ab);
          } else if (p.a_grouped) {
            load_grouped(sa, &map_a, ka, m_cta / 32, ab);
          } else {
#pragma unroll
            for (int j = 0; j < kBlockM / 32; ++j)
              load(sa + j * kBlockK * kSwRowBytes, &map_a, m_cta + 32 * j, ka, ab);
          }
#pragma unroll
          for (int j = 0; j < Cfg::kNSub && !b_done; ++j) {
            uint8_t* sbj = sb + j * Cfg::kBSubBytes;
            const int nj = n_cta + j * Cfg::kMmaN;
            if (!B_MN) {
              load(sbj, &map_b, kbb, nj, bb);
            } else if (p.b_grouped) {
              load_grouped(sbj, &map_b, kbb, nj / 32, bb);
            } else {
#pragma unroll
              for (int g = 0; g < Cfg::kSubCols / 32; ++g)
                load(sbj + g * kBlockK * kSwRowBytes, &map_b, nj + 32 * g, kbb, bb);
            }
          }
        }
      }
      if (fetcher) {
        // Done drawing: the last CTA (pair) to get here resets the counters
        // for the next launch (every other one has drawn its last unit).
        __threadfence();
        if (atomicAdd(p.sched + 1, 1ull) == static_cast<unsigned long long>(unit_step - 1)) {
          atomicExch(p.sched, 0ull);
          atomicExch(p.sched + 1, 0ull);
        }
      }
      // Drain: the bytes of every stage issued must land before the CTA may
      // exit, also when another role gave up early (bounded; a no-op on the
      // normal path, where the MMA warp already waited for each of them).
      // The pair leader's barriers also count the peer's loads.
      if (!PAIR || XF || leader) {
        volatile int never = 0;
        const uint32_t first = it > static_cast<uint32_t>(STAGES) ? it - STAGES : 0u;
        for (uint32_t j = first; j < it; ++j)
          ptx::mbar_wait(&full[j % STAGES], (j / STAGES) & 1, &never, kDrainLimitNs);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = ptx::idesc_tf32(Cfg::kUnitM, Cfg::kMmaN, A_MN, B_MN);
      // Canonical layouts (byte offsets).  K-major (128-byte swizzle): rows
      // 128 B apart, 8-row atoms 1024 B apart (SBO), LBO unused; a K=8 step
      // advances 32 B inside the row.  MN-major (32-byte-atom swizzle):
      // groups of 32 M/N values kBlockK*128 B apart (LBO), 4-row K atoms
      // 512 B apart (SBO); a K=8 step advances 8 rows = 1024 B.
      constexpr uint32_t a_lbo = A_MN ? kBlockK * kSwRowBytes : 16;
      constexpr uint32_t b_lbo = B_MN ? kBlockK * kSwRowBytes : 16;
      constexpr uint32_t a_sbo = A_MN ? 512 : 1024;
      constexpr uint32_t b_sbo = B_MN ? 512 : 1024;
      constexpr uint32_t a_lay = A_MN ? ptx::kLayoutSw128Base32 : ptx::kLayoutSw128;
      constexpr uint32_t b_lay = B_MN ? ptx::kLayoutSw128Base32 : ptx::kLayoutSw128;
      constexpr uint32_t a_kstep = A_MN ? 8 * kSwRowBytes : 8 * 4;   // bytes per K=8 step
      constexpr uint32_t b_kstep = B_MN ? 8 * kSwRowBytes : 8 * 4;
      uint32_t it = 0, tl = 0;
      uint32_t ready_par = 0;   // bit s: phase parity of ready[s] (counts gated uses only)
      bool ok = true;
      for (uint32_t ui = 0; ok; ++ui) {
        long long w;
        if (!units.get(ui, w, abort_flag, p.wait_limit_ns)) {
          record_error(p.err, abort_flag, kErrWaitUnit);
          break;
        }
        if (w >= p.work_units) break;
        const WorkUnit u = decode_unit(p, w);
        if (u.kb_lo >= u.kb_hi) continue;
        const int buf = tl % Cfg::kAccBufs;
        const uint32_t uph = (tl / Cfg::kAccBufs) & 1;
        const uint64_t te0 = trace ? ptx::globaltimer_ns() : 0;
        if (!ptx::mbar_wait(&tmem_empty[buf], uph ^ 1, abort_flag, p.wait_limit_ns)) {
          record_error(p.err, abort_flag, kErrWaitTmemEmpty);
          break;
        }
        if (trace) trace[17] += ptx::globaltimer_ns() - te0;
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        uint32_t acc = 0;
        for (int kb = u.kb_lo; kb < u.kb_hi; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          const bool xg = gated(u, kb);
          uint64_t* gate = xg ? &ready[s] : &full[s];
          const uint32_t gph = xg ? ((ready_par >> s) & 1u) : ph;
          const uint64_t tf0 = trace ? ptx::globaltimer_ns() : 0;
          if (!ptx::mbar_wait(gate, gph, abort_flag, p.wait_limit_ns)) {
            record_error(p.err, abort_flag, xg ? kErrWaitReady : kErrWaitFull);
            ok = false;
            break;
          }
          if (xg) ready_par ^= 1u << s;
          if (trace) {
            const uint64_t tf1 = ptx::globaltimer_ns();
            trace[16] += tf1 - tf0;
            if (it == 0) trace[2] = tf1;
            if (kb == u.kb_lo && tl < 20) trace[20 + 2 * tl] = tf1;
          }
          ptx::tc_fence_after();
          const uint32_t sa = ptx::smem_addr(smem + Cfg::kOffA + s * Cfg::kABytes);
          const uint32_t sb = ptx::smem_addr(smem + Cfg::kOffB + s * Cfg::kBBytes);
          const uint32_t sal = ptx::smem_addr(smem + Cfg::kOffALo + s * Cfg::kABytes);
          const uint32_t sbl = ptx::smem_addr(smem + Cfg::kOffBLo + s * Cfg::kBBytes);
#pragma unroll
          for (int k8 = 0; k8 < kBlockK / 8; ++k8) {
            const uint64_t da = ptx::smem_desc(sa + k8 * a_kstep, a_lbo, a_sbo, a_lay);
            const uint64_t db = ptx::smem_desc(sb + k8 * b_kstep, b_lbo, b_sbo, b_lay);
#pragma unroll
            for (int j = 1; j < Cfg::kNSub; ++j) {
              const uint64_t dbj =
                  ptx::smem_desc(sb + j * Cfg::kBSubBytes + k8 * b_kstep, b_lbo, b_sbo, b_lay);
              if (PAIR)
                ptx::mma_tf32_pair(d_tmem + j * Cfg::kMmaN, da, dbj, idesc, acc);
              else
                ptx::mma_tf32(d_tmem + j * Cfg::kMmaN, da, dbj, idesc, acc);
            }
            if (PAIR)
              ptx::mma_tf32_pair(d_tmem, da, db, idesc, acc);
            else
              ptx::mma_tf32(d_tmem, da, db, idesc, acc);
            acc = 1;
            if (X3) {
              const uint64_t dal = ptx::smem_desc(sal + k8 * a_kstep, a_lbo, a_sbo, a_lay);
              const uint64_t dbl = ptx::smem_desc(sbl + k8 * b_kstep, b_lbo, b_sbo, b_lay);
              if (PAIR) {
                ptx::mma_tf32_pair(d_tmem, da, dbl, idesc, 1);
                ptx::mma_tf32_pair(d_tmem, dal, db, idesc, 1);
              } else {
                ptx::mma_tf32(d_tmem, da, dbl, idesc, 1);
                ptx::mma_tf32(d_tmem, dal, db, idesc, 1);
              }
            }
          }
          if (PAIR)
            ptx::mma_commit_pair(&empty[s], 0x3);
          else
            ptx::mma_commit(&empty[s]);
        }
        if (!ok) break;
        if (trace) {
          trace[3] = ptx::globaltimer_ns();
          if (tl < 20) trace[21 + 2 * tl] = trace[3];
          trace[18] += 1;
        }
        if (!p.inject_stall) {
          if (PAIR)
            ptx::mma_commit_pair(&tmem_full[buf], 0x3);
          else
            ptx::mma_commit(&tmem_full[buf]);
        }
        ++tl;
      }
      // Drain: no MMA may still write TMEM when the allocation is freed,
      // also after an early exit (bounded; immediate on the normal path).
      if (PAIR)
        ptx::mma_commit_pair(mma_drain, 0x1);
      else
        ptx::mma_commit(mma_drain);
      volatile int never = 0;
      ptx::mbar_wait(mma_drain, 0, &never, kDrainLimitNs);
    }
  } else if (warp < 2 + Cfg::kEpiWarps) {
    // ------------------------------------------------------------ epilogue
    // Epilogue warp e reads TMEM lane quadrant warp % 4 (the hardware rule)
    // and every kEpiParts-th 32-column chunk starting at e / 4.
    constexpr int kParts = Cfg::kEpiParts;
    const int quad = warp & 3;
    const int ew = warp - 2;
    const int half = ew >> 2;   // this warp's part: chunks half, half + kParts, ...
    float* stg = reinterpret_cast<float*>(smem + Cfg::kOffEpi) + ew * Cfg::kEpiBufs * 32 * 32;
    const uint32_t tmem_empty_leader =
        PAIR ? ptx::mapa_shared(ptx::smem_addr(tmem_empty), 0) : 0u;
    uint32_t tl = 0, seq = 0;
    if (p.xg.world > 1 && p.xg.rank == p.xg.root && ew == 0 && lane == 0 && p.xg.epoch > 1) {
      // Fused cross-GPU step, root: the previous epoch's kernels have
      // finished (this one is past its grid-dependency wait), so the other
      // ranks may reuse the landing slots of epoch - 1.
      const EngineParams::Xgpu& x = p.xg;
      for (long long c = blockIdx.x; c < x.nchunk; c += gridDim.x)
        for (int r = 0; r < x.world; ++r)
          if (r != x.root)
            peer_st_release_sys(reinterpret_cast<uint64_t*>(x.mbox[r] + x.consumed_off) + c,
                                static_cast<uint64_t>(x.epoch - 1));
    }
    if (p.xg.world > 1 && p.xg.rank != p.xg.root && ew == 0 && lane == 0) {
      // Fused cross-GPU step, non-root: the landing slots this epoch writes
      // were last read by the root two epochs ago; checked now, while the
      // mainloop runs, so that the exchange itself waits on nothing local.
      const EngineParams::Xgpu& x = p.xg;
      int ok = 1;
      for (long long c = blockIdx.x; ok && x.epoch > 2 && c < x.nchunk; c += gridDim.x) {
        const uint64_t* consumed =
            reinterpret_cast<const uint64_t*>(x.mbox[x.rank] + x.consumed_off) + c;
        ok = peer_wait_at_least(consumed, static_cast<uint64_t>(x.epoch - 2), p.wait_limit_ns);
      }
      if (!ok) record_error(p.err, abort_flag, kErrPeerCredit);
      *reinterpret_cast<volatile int*>(smem + Cfg::kOffMisc + 12) = ok;
    }
    // Zero this warp's chunks of a tile region (TMA zero boxes), wait until
    // the stores are complete, then stamp `flag` with the launch's epoch.
    auto zero_and_flag = [&](int row0, int n0, int b, unsigned* flag) {
      if (row0 < p.M) {
        if (lane == 0) ptx::bulk_wait_read<0>();
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; ++j)
          *reinterpret_cast<float4*>(stg + lane * 32 + j * 4) = make_float4(0.f, 0.f, 0.f, 0.f);
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          for (int ch = half; ch * 32 < BN && n0 + ch * 32 < p.N; ch += kParts)
            ptx::tma_store_3d(&map_c, stg, n0 + ch * 32, row0, b);
          ptx::bulk_commit();
          ptx::bulk_wait_all();
        }
      }
      __syncwarp();
      if (lane == 0) {
        ptx::fence_proxy_async_global();
        __threadfence();
        ptx::st_release_gpu(flag, p.epoch);
      }
    };
    if (p.split_tiles != nullptr && p.tile_flags != nullptr && p.tma_store) {
      const int cluster = static_cast<int>(unit0), clusters = static_cast<int>(unit_step);
      for (int j = cluster; j < p.n_split; j += clusters) {
        const int4 t = p.split_tiles[j];
        zero_and_flag(t.x * Cfg::kUnitM + static_cast<int>(rank) * kBlockM + quad * 32, t.y * BN,
                      0, p.tile_flags + j * kFlagSlots + static_cast<int>(rank) * Cfg::kEpiWarps + ew);
      }
    }
    for (uint32_t ui = 0;; ++ui) {
      long long w;
      if (!units.get(ui, w, abort_flag, p.wait_limit_ns)) {
        if (lane == 0) record_error(p.err, abort_flag, kErrWaitUnit);
        break;
      }
      if (w >= p.work_units) break;
      const WorkUnit u = decode_unit(p, w);
      const int row0 = u.tm * Cfg::kUnitM + static_cast<int>(rank) * kBlockM + quad * 32;
      const int n0 = u.tn * BN;
      if (u.skip) continue;
      if (u.kb_lo >= u.kb_hi && p.tma_store) {
        // Structurally zero tile (or K == 0): TMA-store a zeroed staging box
        // over this warp's chunks, unless the tile only accumulates.
        if (!p.atomic_out && !u.accumulate && row0 < p.M) {
          if (lane == 0) ptx::bulk_wait_read<0>();
          __syncwarp();
          const float z = (p.row_bias && row0 + lane < p.M) ? p.row_bias[row0 + lane] : 0.f;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4*>(stg + lane * 32 + j * 4) = make_float4(z, z, z, z);
          ptx::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            for (int ch = half; ch * 32 < BN && n0 + ch * 32 < p.N; ch += kParts)
              ptx::tma_store_3d(&map_c, stg, n0 + ch * 32, row0, u.b);
            ptx::bulk_commit();
          }
        }
        continue;
      }
      if (u.kb_lo >= u.kb_hi) {
        // Structurally zero tile (or K == 0): write zeros unless accumulating.
        if (!p.atomic_out && !u.accumulate && row0 < p.M) {
          float* cb = p.C + static_cast<long long>(u.b) * p.stride_c;
          for (int it = 0; it < 8 * (BN / 32); ++it) {
            const int cc = it >> 3;                      // 32-column chunk
            if (cc % kParts != half) continue;
            const int r_local = (it & 7) * 4 + (lane >> 3);
            const int gcol = n0 + cc * 32 + (lane & 7) * 4;
            const int grow = row0 + r_local;
            if (grow < p.M && gcol < p.N) {
              const float z = p.row_bias ? p.row_bias[grow] : 0.f;
              store4(p, cb + static_cast<long long>(grow) * p.ldc, grow, gcol, z, z, z, z);
            }
          }
        }
        continue;
      }
      unsigned* tile_flag = nullptr;
      if (p.tile_flags != nullptr && u.flag >= 0) {
        tile_flag = p.tile_flags + u.flag * kFlagSlots + static_cast<int>(rank) * Cfg::kEpiWarps + ew;
        // Split-K: the first K piece zeroes this warp's chunks of the tile
        // and publishes them (before waiting for the MMA).  Split tiles of a
        // unit table were zeroed before any unit (above).
        if (u.first && p.split_tiles == nullptr) zero_and_flag(row0, n0, u.b, tile_flag);
      }
      const int buf = tl % Cfg::kAccBufs;
      const uint32_t uph = (tl / Cfg::kAccBufs) & 1;
      if (!ptx::mbar_wait_sleepy(&tmem_full[buf], uph, abort_flag, p.wait_limit_ns)) {
        if (lane == 0) record_error(p.err, abort_flag, kErrWaitTmemFull);
        break;
      }
      if (trace && ew == 0 && lane == 0 && tl == 0) trace[4] = ptx::globaltimer_ns();
      ptx::tc_fence_after();
      if (tile_flag != nullptr && (!u.first || p.split_tiles != nullptr) && row0 < p.M) {
        // Later K piece: its reduce-adds land on chunks the first piece zeroes.
        int ok = 1;
        if (lane == 0) {
          const uint64_t t0 = ptx::globaltimer_ns();
          while (ptx::ld_acquire_gpu(tile_flag) != p.epoch) {
            if (*abort_flag || ptx::globaltimer_ns() - t0 > static_cast<uint64_t>(p.wait_limit_ns)) {
              ok = 0;
              break;
            }
            __nanosleep(64);
          }
          ptx::fence_proxy_async_global();
        }
        if (!__shfl_sync(0xffffffffu, ok, 0)) {
          if (lane == 0) record_error(p.err, abort_flag, kErrWaitZero);
          break;
        }
        if (trace && ew == 0 && lane == 0) trace[7] = ptx::globaltimer_ns();
      }
      auto release = [&]() {
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (PAIR)
            ptx::mbar_arrive_cluster(tmem_empty_leader + buf * 8);
          else
            ptx::mbar_arrive(&tmem_empty[buf]);
        }
      };
      int nch = (p.N - n0 + 31) / 32;
      if (nch > BN / 32) nch = BN / 32;
      // Row bias (this lane's output row), added once: by the K piece that starts at 0.
      const bool with_bias = p.row_bias != nullptr && u.kb_lo == 0;
      const float bias_v = (with_bias && row0 + lane < p.M) ? p.row_bias[row0 + lane] : 0.f;
      // Last unit of this CTA (pair): every MMA has read its operands and no
      // load will follow, so the operand stages are free for staging.
      bool tail = false;
      if (Cfg::kTailBoxes >= 2 && p.tma_store && Cfg::kEpiBufs == 1) {
        long long w_next;
        if (!units.get(ui + 1, w_next, abort_flag, p.wait_limit_ns)) {
          if (lane == 0) record_error(p.err, abort_flag, kErrWaitUnit);
          break;
        }
        tail = w_next >= p.work_units;
      }
      if (row0 < p.M && half < nch && p.tma_store && Cfg::kEpiBufs == 1) {
        // TMA path: groups of kEpiGroup chunks, one TMEM wait and one fence each.
        constexpr int G = Cfg::kEpiGroup;
        constexpr int kTail = Cfg::kTailBoxes >= 2 ? Cfg::kTailBoxes : 2;
        float* tail_stg = reinterpret_cast<float*>(smem) + ew * kTail * 32 * 32;
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + buf * BN;
        const int mine = (nch - half + kParts - 1) / kParts;   // chunks half, half+kParts, ...
#pragma unroll 1
        for (int g0 = 0; g0 < mine; g0 += G) {
          const int ng = mine - g0 < G ? mine - g0 : G;
          uint32_t r[G][32];
          int col0[G];
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const int ch = half + kParts * (g0 + (g < ng ? g : 0));
            col0[g] = n0 + ch * 32;
            if (g < ng) ptx::tmem_ld_32x32b_x32(taddr + ch * 32, r[g]);
          }
          ptx::tmem_ld_wait();
#pragma unroll
          for (int g = 0; g < G; ++g)
#pragma unroll
            for (int i = 0; i < 32; ++i) asm volatile("" : "+r"(r[g][i]));
          if (trace && ew == 0 && lane == 0 && g0 < 4) trace[8 + 2 * g0] = ptx::globaltimer_ns();
          if (with_bias) {
#pragma unroll
            for (int g = 0; g < G; ++g)
#pragma unroll
              for (int i = 0; i < 32; ++i) r[g][i] = __float_as_uint(__uint_as_float(r[g][i]) + bias_v);
          }
          if (g0 + G >= mine) release();                      // every TMEM read is done
          if (tail)
            store_group_tma<G, kTail - 1>(p, &map_c, tail_stg + ((g0 / G) % kTail) * G * 32 * 32,
                                          r, ng, u.b, row0, col0, lane, u.accumulate);
          else
            store_group_tma<G>(p, &map_c, stg, r, ng, u.b, row0, col0, lane, u.accumulate);
          if (trace && ew == 0 && lane == 0 && g0 < 4) trace[9 + 2 * g0] = ptx::globaltimer_ns();
        }
      } else if (row0 < p.M && half < nch) {
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + buf * BN;
        uint32_t ra[32], rb[32];
        ptx::tmem_ld_32x32b_x32(taddr + half * 32, ra);
        tmem_ld_wait_regs(ra);
#pragma unroll 1
        for (int ch = half; ch < nch; ch += kParts) {
          const bool more = ch + kParts < nch;
          if (more)
            ptx::tmem_ld_32x32b_x32(taddr + (ch + kParts) * 32, rb);   // in flight while ra drains
          else
            release();                                            // every TMEM read is done
          if (with_bias) {
#pragma unroll
            for (int i = 0; i < 32; ++i) ra[i] = __float_as_uint(__uint_as_float(ra[i]) + bias_v);
          }
          store_chunk<Cfg::kEpiBufs>(p, &map_c, stg, seq, ra, u.b, row0, n0 + ch * 32, lane,
                                     u.accumulate);
          if (more) {
            tmem_ld_wait_regs(rb);
#pragma unroll
            for (int i = 0; i < 32; ++i) ra[i] = rb[i];
          }
        }
      } else {
        release();
      }
      if (trace && ew == 0 && lane == 0) trace[5] = ptx::globaltimer_ns();
      ++tl;
    }
    if (p.xg.world > 1) {
      // Fused cross-GPU step (every CTA takes part, also one without units).
      const EngineParams::Xgpu xg_copy = p.xg;
      xgpu_exchange(&xg_copy, p.C, p.wait_limit_ns, p.err, Cfg::kEpiWarps * 32, ew * 32 + lane,
                    abort_flag,
                    reinterpret_cast<volatile int*>(smem + Cfg::kOffMisc + 8),
                    *reinterpret_cast<volatile int*>(smem + Cfg::kOffMisc + 12), trace);
    } else if (lane == 0) {
      ptx::bulk_wait_read<0>();   // staging boxes read before the CTA exits
    }
  } else if (XF) {
    // ------------------------------------------------------------ transform
    // Each CTA transforms its own slices (A rows m_cta.., B columns n_cta..)
    // and then signals the MMA issuer's ready[s] (the leader's in a pair).
    const int xt = threadIdx.x - (2 + Cfg::kEpiWarps) * 32;
    const uint32_t ready_leader = PAIR ? ptx::mapa_shared(ptx::smem_addr(ready), 0) : 0u;
    uint32_t it = 0;
    bool ok = true;
    for (uint32_t ui = 0; ok; ++ui) {
      long long w;
      if (!units.get(ui, w, abort_flag, p.wait_limit_ns)) {
        if (lane == 0) record_error(p.err, abort_flag, kErrWaitUnit);
        break;
      }
      if (w >= p.work_units) break;
      const WorkUnit u = decode_unit(p, w);
      const int m0 = u.tm * Cfg::kUnitM + static_cast<int>(rank) * kBlockM;
      const int n0 = u.tn * BN + static_cast<int>(rank) * Cfg::kSubCols;
      for (int kb = u.kb_lo; kb < u.kb_hi; ++kb, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        // Every phase of full[s] is waited for, also for stages that go
        // straight to the MMA: a parity wait that skipped a phase could
        // return on the skipped phase's parity before this stage landed.
        if (!ptx::mbar_wait(&full[s], ph, abort_flag, p.wait_limit_ns)) {
          if (lane == 0) record_error(p.err, abort_flag, kErrWaitXform);
          ok = false;
          break;
        }
        if (!gated(u, kb)) continue;       // straight to the MMA
        const int k0 = kb * kBlockK;
        int rule_a = 0, rule_b = 0;
        const int up = p.tri == kTriUpper;   // rule 1: zero k < mn; rule 2: zero k > mn
        if (p.xf_gate && !X3) {
          // Only partly masked boxes need work; wholly masked ones were
          // loaded as zeros.
          if (tri_mask_a(p.tri, m0, k0) == 1) rule_a = up ? 1 : 2;
          if (tri_mask_b(p.tri, n0, Cfg::kBnCta, k0) == 1) rule_b = up ? 2 : 1;
        } else if (p.tri != kTriNone) {
          if (tri_mask_a(p.tri, m0, k0) != 0) rule_a = up ? 1 : 2;
          if (tri_mask_b(p.tri, n0, Cfg::kBnCta, k0) != 0) rule_b = up ? 2 : 1;
        }
        float* ta = reinterpret_cast<float*>(smem + Cfg::kOffA + s * Cfg::kABytes);
        float* tb = reinterpret_cast<float*>(smem + Cfg::kOffB + s * Cfg::kBBytes);
        float* tal = reinterpret_cast<float*>(smem + Cfg::kOffALo + s * Cfg::kABytes);
        float* tbl = reinterpret_cast<float*>(smem + Cfg::kOffBLo + s * Cfg::kBBytes);
        transform_tile<A_MN, kBlockM, X3>(ta, tal, m0, k0, rule_a, xt);
        transform_tile<B_MN, Cfg::kBnCta, X3>(tb, tbl, n0, k0, rule_b, xt);
        if (PAIR)
          asm volatile("fence.proxy.async;" ::: "memory");   // visible to the pair's MMA
        else
          ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (PAIR)
            ptx::mbar_arrive_cluster(ready_leader + s * 8);
          else
            ptx::mbar_arrive(&ready[s]);
        }
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (PAIR) ptx::cluster_sync();   // no CTA leaves while its peer may still signal it
  if (trace && threadIdx.x == 0) trace[6] = ptx::globaltimer_ns();
  if (warp == 1) {
    ptx::tc_fence_after();
    if (PAIR)
      ptx::tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
    else
      ptx::tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace b2g
