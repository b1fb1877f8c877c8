// b2g_capi.cu — host dispatcher and C ABI (include/b2g_gemm.h).
//
// The dispatcher is pure host arithmetic (b2g_gemm_plan_for): tile width,
// pipeline depth, split-K and the persistent grid for a descriptor on a GPU
// with a given SM count.  b2g_gemm() turns the plan into tensor maps and one
// launch of the persistent tcgen05 engine; operands whose pitch or base
// breaks TMA's 16-byte rule are first copied to an aligned pitch in the
// caller's workspace.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <tuple>
#include <queue>
#include <vector>

#include "../../include/b2g_gemm.h"
#include "b2g_internal.h"
#include "gemm_engine.cuh"
#include "sdpa_engine.cuh"

#ifndef B2G_KERNEL_CLEAR
#define B2G_KERNEL_CLEAR 1     // split-K: the first K piece clears its tile in the kernel
#endif
#ifndef B2G_PDL
#define B2G_PDL 1              // launch engines with programmatic stream serialization
#endif
#ifndef B2G_DYNAMIC_UNITS
#define B2G_DYNAMIC_UNITS 1    // hand out work units dynamically (plain GEMMs)
#endif
#ifndef B2G_PAIR256_STAGES
#define B2G_PAIR256_STAGES 6   // pipeline depth of the CTA-pair 256-wide engine
#endif
#ifndef B2G_PAIR256_EPIG
#define B2G_PAIR256_EPIG 1     // accumulator chunks per epilogue store group
#endif
#ifndef B2G_PAIR256_EPIW
#define B2G_PAIR256_EPIW 8     // epilogue warps of the CTA-pair 256-wide engine
#endif
#ifndef B2G_PAIR256_LONGK_EPIW
#define B2G_PAIR256_LONGK_EPIW 4   // ... for units of >= 16 K blocks
#endif

namespace b2g {
namespace {

constexpr int kMaxDevices = 64;
constexpr int kTriDiagBlock = 128;   // diagonal-block width of the triangular masking copies

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int64_t round_up(int64_t a, int64_t b) { return cdiv(a, b) * b; }

// ---------------------------------------------------------------- per-device state
struct DeviceState {
  bool init = false;
  int num_sms = 0;
  int* err_word = nullptr;      // device error word (4 bytes)
};
std::mutex g_mu;
DeviceState g_dev[kMaxDevices];

// B2G_MAX_SMS=n (a test and tuning hook, read once per process) plans every
// launch as if the GPU had only n SMs: a small persistent grid then walks
// many more work units per CTA, which exercises the dynamic schedule's
// unit ring far past its wrap at small problem sizes.
int max_sms_override() {
  static const int v = [] {
    const char* e = std::getenv("B2G_MAX_SMS");
    const int n = (e && *e) ? std::atoi(e) : 0;
    return n >= 2 ? n : (1 << 30);
  }();
  return v;
}

int device_state(DeviceState** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return B2G_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceState& st = g_dev[dev];
  if (!st.init) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return B2G_ERR_NO_DEVICE;
    if (prop.major != 10) return B2G_ERR_NO_DEVICE;
    st.num_sms = std::min(prop.multiProcessorCount, max_sms_override());
    if (cudaMalloc(&st.err_word, sizeof(int)) != cudaSuccess) return B2G_ERR_LAUNCH;
    if (cudaMemset(st.err_word, 0, sizeof(int)) != cudaSuccess) return B2G_ERR_LAUNCH;
    st.init = true;
  }
  *out = &st;
  return B2G_OK;
}

// ---------------------------------------------------------------- fault-detection knobs
// B2G_WAIT_LIMIT_MS bounds every device-side wait (default 2000 ms).
// B2G_TEST_STALL_ONCE=1 is a test hook: the first GEMM launched in the
// process withholds its "accumulator ready" signal, so the epilogue's bounded
// wait runs out, the kernel records kErrWaitTmemFull in the device error
// word and unwinds; later launches are normal.  Nothing faults or traps.
long long wait_limit_ns() {
  static const long long ns = [] {
    const char* e = std::getenv("B2G_WAIT_LIMIT_MS");
    const long long ms = (e && *e) ? std::atoll(e) : 0;
    return ms > 0 ? ms * 1000000ll : static_cast<long long>(kWaitLimitNs);
  }();
  return ns;
}

// Tuning overrides of the dispatcher: B2G_TILE=pair512|pair256|pair128|
// single256|single128 pins the tile shape, B2G_SPLITS=n the split-K factor
// of plain GEMMs.  Read once per process, or at every call when the process
// started with B2G_TUNING=1 (sweeps that change them between calls).
bool tuning_mode() {
  static const bool on = [] {
    const char* e = std::getenv("B2G_TUNING");
    return e && *e == '1';
  }();
  return on;
}
const char* tile_override() {
  static const char* once = std::getenv("B2G_TILE");
  return tuning_mode() ? std::getenv("B2G_TILE") : once;
}
int splits_override() {
  auto read = [] {
    const char* e = std::getenv("B2G_SPLITS");
    return (e && *e) ? std::atoi(e) : 0;
  };
  static const int once = read();
  return tuning_mode() ? read() : once;
}

// Longest K piece of a triangular unit table, in percent of the mean load
// per cluster (B2G_TRI_SPLIT; a tuning knob, read like the overrides above).
int64_t tri_split_pct() {
  auto read = [] {
    const char* e = std::getenv("B2G_TRI_SPLIT");
    const int v = (e && *e) ? std::atoi(e) : 0;
    return v > 0 ? v : 100;
  };
  static const int once = read();
  return tuning_mode() ? read() : once;
}

// B2G_TRI_PATH=gate: untransposed triangular products through the gated
// transform warps instead of diagonal-block copies (tuning and comparison;
// read like the overrides above).
bool tri_path_gate() {
  auto read = [] {
    const char* e = std::getenv("B2G_TRI_PATH");
    return e && std::strcmp(e, "gate") == 0;
  };
  static const bool once = read();
  return tuning_mode() ? read() : once;
}

// Triangular units run 8 epilogue warps (B2G_TRI_EPIW=4 selects 4; a
// tuning knob, read like the overrides above).
bool tri_epiw8() {
  auto read = [] {
    const char* e = std::getenv("B2G_TRI_EPIW");
    return !(e && std::atoi(e) == 4);
  };
  static const bool once = read();
  return tuning_mode() ? read() : once;
}

// B2G_TRACE_PTR=<device address of 64 u64 per CTA> (tuning mode only): the
// engine writes its per-CTA phase stamps there (EngineParams::trace).
unsigned long long* trace_pointer() {
  if (!tuning_mode()) return nullptr;
  const char* e = std::getenv("B2G_TRACE_PTR");
  return (e && *e) ? reinterpret_cast<unsigned long long*>(std::strtoull(e, nullptr, 0)) : nullptr;
}

// B2G_EARLY_DRAW=0 turns off drawing the next dynamic unit one unit ahead
// (EngineParams::early_draw; a tuning knob, read once per process).
bool early_draw_on() {
  static const bool on = [] {
    const char* e = std::getenv("B2G_EARLY_DRAW");
    return !(e && *e == '0');
  }();
  return on;
}

int take_injected_stall() {
  static std::atomic<int> armed{-1};
  int v = armed.load();
  if (v < 0) {
    const char* e = std::getenv("B2G_TEST_STALL_ONCE");
    int want = (e && *e == '1') ? 1 : 0;
    armed.compare_exchange_strong(v, want);
  }
  int one = 1;
  return armed.compare_exchange_strong(one, 0) ? 1 : 0;
}

// ------------------------------------------------------- dynamic unit schedule
// Counter pairs of the dynamic schedule (EngineParams::sched), one per launch
// taken round-robin from a file-scope array: zero at module load, and each
// launch leaves its pair at zero when it ends.  Launches that share a slot
// are kSchedSlots launches apart, so never run at the same time.
constexpr int kSchedSlots = 4096;
static __device__ unsigned long long g_sched[kSchedSlots][2];

unsigned long long* sched_slot() {
  constexpr int kMaxDevices = 64;
  static std::atomic<unsigned long long*> base[kMaxDevices];
  static std::atomic<unsigned> next{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  unsigned long long* b = base[dev].load();
  if (!b) {
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_sched) != cudaSuccess) return nullptr;
    b = static_cast<unsigned long long*>(addr);
    base[dev].store(b);
  }
  return b + 2 * (next.fetch_add(1) % kSchedSlots);
}

// Flags of the in-kernel split-K clear (EngineParams::tile_flags): one
// region per launch from a ring, stamped with a per-process launch epoch, so
// stale flags never match and nothing is ever reset.  Launches sharing a
// region are kFlagRing launches apart.
constexpr int kFlagRing = 32;
constexpr int kFlagTiles = 128;
static __device__ unsigned g_tile_flags[kFlagRing][kFlagTiles * kFlagSlots];

bool tile_flag_region(unsigned** region, unsigned* epoch) {
  constexpr int kMaxDevices = 64;
  static std::atomic<unsigned*> base[kMaxDevices];
  static std::atomic<unsigned> next{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return false;
  unsigned* b = base[dev].load();
  if (!b) {
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_tile_flags) != cudaSuccess) return false;
    b = static_cast<unsigned*>(addr);
    base[dev].store(b);
  }
  unsigned e = next.fetch_add(1) + 1;
  if (e == 0) e = next.fetch_add(1) + 1;     // 0 is the flags' initial value
  *epoch = e;
  *region = b + static_cast<size_t>(e % kFlagRing) * kFlagTiles * kFlagSlots;
  return true;
}

// ---------------------------------------------------------------- tensor maps
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Rank-3 fp32 map {inner, outer, batch}.  K-major operands use the 128-byte
// swizzle (16-byte chunks); MN-major operands the 128-byte swizzle with
// 32-byte atoms, the shared-memory layout tcgen05 reads MN-major TF32 from.
bool make_map(CUtensorMap* map, const float* base, int64_t inner, int64_t outer, int64_t batch,
              int64_t ld, int64_t bstride, uint32_t box_inner, uint32_t box_outer, bool mn_major) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  if (batch <= 1) {
    batch = 1;
    bstride = round_up(ld * outer, 4);
  }
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer),
                        static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * 4, static_cast<cuuint64_t>(bstride) * 4};
  cuuint32_t box[3] = {box_inner, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// MN-major operand (element (k, mn) at base + k*ld + mn) as a rank-4 map
// {32, K, MN/32, batch}: one box {32, 32, groups, 1} lands all of a stage's
// 32-wide groups in the layout the MMA reads (groups kBlockK*128 B apart).
// Only for MN a multiple of 32, so the grouped view never reaches past the
// operand's last row.  Returns false if the driver rejects the layout.
bool make_map_grouped(CUtensorMap* map, const float* base, int64_t mn, int64_t k, int64_t batch,
                      int64_t ld, int64_t bstride, uint32_t groups) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || mn % 32 != 0) return false;
  if (batch <= 1) {
    batch = 1;
    bstride = round_up(ld * k, 4);
  }
  cuuint64_t dims[4] = {32, static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(mn / 32),
                        static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(ld) * 4, 128,
                           static_cast<cuuint64_t>(bstride) * 4};
  cuuint32_t box[4] = {32, static_cast<cuuint32_t>(kBlockK), groups, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// ---------------------------------------------------------------- staging copy
// dst[b][r][c] = src[b*sstride + r*sld + c] for c < cols, 0 for cols <= c
// < dld (the pitch, a multiple of 4; a multiple of 32 for MN-major
// operands, whose zero-padded columns let the loads use 32-wide groups).
__global__ void pitch_copy_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                  int64_t rows, int64_t cols, int64_t sld, int64_t sstride,
                                  int64_t dld, int64_t dstride, int64_t batch) {
  const int64_t total = batch * rows;
  for (int64_t rr = blockIdx.x; rr < total; rr += gridDim.x) {
    const int64_t b = rr / rows, r = rr - b * rows;
    const float* s = src + b * sstride + r * sld;
    float4* d = reinterpret_cast<float4*>(dst + b * dstride + r * dld);
    // The destination pitch is a multiple of 4 floats (16-byte rows): each
    // thread gathers float4s from unaligned source rows, two in flight.
    const int64_t n4 = dld / 4;
    auto gather = [&](int64_t q) {
      float e[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) e[j] = 4 * q + j < cols ? __ldg(s + 4 * q + j) : 0.f;
      return make_float4(e[0], e[1], e[2], e[3]);
    };
    for (int64_t q = threadIdx.x; q < n4; q += 2 * blockDim.x) {
      const int64_t q1 = q + blockDim.x;
      const float4 v0 = gather(q);
      const float4 v1 = q1 < n4 ? gather(q1) : make_float4(0.f, 0.f, 0.f, 0.f);
      d[q] = v0;
      if (q1 < n4) d[q1] = v1;
    }
  }
}

// ---------------------------------------------------------------- triangular diagonal blocks
// Masked copies of the 128 x 128 diagonal blocks of A and B (a row-major
// n x 128 array each: row r of block b holds src[b*128 + r][b*128 + c]).
// Upper: keep column >= row in both (A: k >= i, B: k <= j); lower: keep
// column <= row.  Columns past n are zero.  blockIdx.y selects A or B.
// Triangular pre-pass, one launch.  blockIdx.y 0 / 1: kTriDiagRows rows of
// one diagonal block of A / B into its masked copy.  blockIdx.y 2: one
// kTriDiagRows-row slice of a split tile's C region set to zero (the tile's
// K pieces then reduce-add into it).  Blocks past their y's work exit.
constexpr int kTriDiagRows = 8;
// The unit table and split-tile list travel as a kernel parameter (no host
// to device copy) when they fit: `words` 16-byte words, copied by the
// pre-pass into the workspace the engine then reads.
constexpr int kTableParamWords = 1900;
struct TableParam {
  int words;       // 0: the table was copied to the workspace by the host
  int split_off;   // word offset of the split-tile list (int2 pairs)
  int4 w[kTableParamWords];
};
// The pre-pass's work once the table is in place.  Split tile i is
// split4[i].{x,y} when split4 is set (the per-device table cache's image),
// else split2[i].
__device__ __forceinline__ void tri_prepare_body(
    const float* __restrict__ a, int64_t lda, const float* __restrict__ b, int64_t ldb, int64_t n,
    int upper, float* __restrict__ adiag, float* __restrict__ bdiag, float* __restrict__ c,
    int64_t ldc, const int2* __restrict__ split2, const int4* __restrict__ split4, int n_split,
    int block_m, int block_n) {
  constexpr int kSlices = kTriDiagBlock / kTriDiagRows;
  if (blockIdx.y == 2) {
    const int slices = (block_m + kTriDiagRows - 1) / kTriDiagRows;
    if (static_cast<int>(blockIdx.x) >= n_split * slices) return;
    const int si = blockIdx.x / slices;
    const int2 t = split4 ? make_int2(split4[si].x, split4[si].y) : split2[si];
    const int r0 = (blockIdx.x % slices) * kTriDiagRows;
    const int64_t col_base = static_cast<int64_t>(t.y) * block_n;
    if ((reinterpret_cast<uintptr_t>(c) % 16) == 0 && ldc % 4 == 0 && col_base + block_n <= n) {
      // Whole float4s: rows of the tile are 16-byte aligned and in range.
      for (int idx = threadIdx.x; idx < kTriDiagRows * block_n / 4; idx += blockDim.x) {
        const int r = r0 + idx / (block_n / 4);
        const int64_t row = static_cast<int64_t>(t.x) * block_m + r;
        if (r < block_m && row < n)
          *reinterpret_cast<float4*>(c + row * ldc + col_base + (idx % (block_n / 4)) * 4) =
              make_float4(0.f, 0.f, 0.f, 0.f);
      }
      return;
    }
    for (int idx = threadIdx.x; idx < kTriDiagRows * block_n; idx += blockDim.x) {
      const int r = r0 + idx / block_n;
      const int64_t row = static_cast<int64_t>(t.x) * block_m + r;
      const int64_t col = static_cast<int64_t>(t.y) * block_n + idx % block_n;
      if (r < block_m && row < n && col < n) c[row * ldc + col] = 0.f;
    }
    return;
  }
  if (static_cast<int64_t>(blockIdx.x) >= ((n + kTriDiagBlock - 1) / kTriDiagBlock) * kSlices)
    return;
  const float* src = blockIdx.y == 0 ? a : b;
  const int64_t ld = blockIdx.y == 0 ? lda : ldb;
  float* dst = blockIdx.y == 0 ? adiag : bdiag;
  const int64_t base = static_cast<int64_t>(blockIdx.x / kSlices) * kTriDiagBlock;
  const int r0 = (blockIdx.x % kSlices) * kTriDiagRows;
  if ((reinterpret_cast<uintptr_t>(src) % 16) == 0 && ld % 4 == 0 && base + kTriDiagBlock <= n) {
    // One float4 per thread (8 rows x 128 columns = 256 float4), masked per element.
    for (int q = threadIdx.x; q < kTriDiagRows * kTriDiagBlock / 4; q += blockDim.x) {
      const int r = r0 + q / (kTriDiagBlock / 4), c0 = (q % (kTriDiagBlock / 4)) * 4;
      const int64_t gi = base + r;
      if (gi >= n) break;
      float4 v = __ldg(reinterpret_cast<const float4*>(src + gi * ld + base + c0));
      float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (upper ? (c0 + j < r) : (c0 + j > r)) e[j] = 0.f;
      *reinterpret_cast<float4*>(dst + gi * kTriDiagBlock + c0) = make_float4(e[0], e[1], e[2], e[3]);
    }
    return;
  }
  for (int idx = threadIdx.x; idx < kTriDiagRows * kTriDiagBlock; idx += blockDim.x) {
    const int r = r0 + idx / kTriDiagBlock, cc = idx % kTriDiagBlock;
    const int64_t gi = base + r, gc = base + cc;
    if (gi >= n) break;
    const bool keep = upper ? (cc >= r) : (cc <= r);
    dst[gi * kTriDiagBlock + cc] = (keep && gc < n) ? __ldg(src + gi * ld + gc) : 0.0f;
  }
}

// Table in the kernel's parameters (calls whose table must live in the
// workspace, i.e. the allocation-free entry): the B blocks copy it there.
__global__ void __launch_bounds__(256) tri_prepare_kernel(
    const float* __restrict__ a, int64_t lda, const float* __restrict__ b, int64_t ldb, int64_t n,
    int upper, float* __restrict__ adiag, float* __restrict__ bdiag, float* __restrict__ c,
    int64_t ldc, const int2* __restrict__ split_tiles, int n_split, int block_m, int block_n,
    int4* __restrict__ table_dst, const __grid_constant__ TableParam tp) {
  // Launched with programmatic stream serialization: let the engine launch
  // (it waits for this grid before reading), and wait for the previous
  // kernel, which may still read the workspace this pass rewrites.
  ptx::griddep_launch_dependents();
  ptx::griddep_wait();
  if (tp.words > 0) {
    if (blockIdx.y == 1)   // B's blocks also copy the table (grid-stride over x)
      for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < tp.words; i += gridDim.x * blockDim.x)
        table_dst[i] = tp.w[i];
    split_tiles = reinterpret_cast<const int2*>(tp.w + tp.split_off);
  }
  tri_prepare_body(a, lda, b, ldb, n, upper, adiag, bdiag, c, ldc, split_tiles, nullptr, n_split,
                   block_m, block_n);
}

// Table already resident (the per-device cache): small parameters only, so
// the launch carries no 30 KB parameter block.
__global__ void __launch_bounds__(256) tri_prepare_cached_kernel(
    const float* __restrict__ a, int64_t lda, const float* __restrict__ b, int64_t ldb, int64_t n,
    int upper, float* __restrict__ adiag, float* __restrict__ bdiag, float* __restrict__ c,
    int64_t ldc, const int4* __restrict__ split4, int n_split, int block_m, int block_n) {
  ptx::griddep_launch_dependents();
  ptx::griddep_wait();
  tri_prepare_body(a, lda, b, ldb, n, upper, adiag, bdiag, c, ldc, nullptr, split4, n_split,
                   block_m, block_n);
}

// 3xTF32 pre-split of both operands in one launch (blockIdx.y: 0 = A,
// 1 = B): dst[b][r][c] = x - (x with its low 13 mantissa bits cleared),
// x = src[b*sstride + r*sld + c]; the tensor core truncates the original
// operand to its TF32 "hi" part itself.  Sources are 16-byte aligned rows
// (an operand with another pitch was staged first); each thread keeps four
// 16-byte loads in flight.  Launched programmatically: the engine behind it
// sets up meanwhile and waits for it before reading.
struct SplitJob {
  const float* src;
  float* dst;
  int64_t rows, cols, sld, sstride, dld, dstride, batch;
};
__global__ void __launch_bounds__(256) split_lo_kernel(const SplitJob ja, const SplitJob jb) {
  ptx::griddep_launch_dependents();
  ptx::griddep_wait();
  const SplitJob& j = blockIdx.y == 0 ? ja : jb;
  if (j.rows == 0) return;
  constexpr int kIlp = 4;
  auto lo = [](float x) { return x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); };
  const int64_t n4 = j.dld / 4;
  const int64_t total = j.batch * j.rows;
  for (int64_t rr = blockIdx.x; rr < total; rr += gridDim.x) {
    const int64_t b = rr / j.rows, r = rr - b * j.rows;
    const float* s = j.src + b * j.sstride + r * j.sld;
    float4* d = reinterpret_cast<float4*>(j.dst + b * j.dstride + r * j.dld);
    for (int64_t q0 = threadIdx.x; q0 < n4; q0 += kIlp * blockDim.x) {
      float4 v[kIlp];
#pragma unroll
      for (int u = 0; u < kIlp; ++u) {
        const int64_t q = q0 + static_cast<int64_t>(u) * blockDim.x;
        if (q < n4 && 4 * q + 3 < j.cols) {
          v[u] = __ldg(reinterpret_cast<const float4*>(s) + q);
        } else if (q < n4) {
          float e[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) e[t] = 4 * q + t < j.cols ? __ldg(s + 4 * q + t) : 0.f;
          v[u] = make_float4(e[0], e[1], e[2], e[3]);
        }
      }
#pragma unroll
      for (int u = 0; u < kIlp; ++u) {
        const int64_t q = q0 + static_cast<int64_t>(u) * blockDim.x;
        if (q < n4) d[q] = make_float4(lo(v[u].x), lo(v[u].y), lo(v[u].z), lo(v[u].w));
      }
    }
  }
}

// ---------------------------------------------------------------- row scale
// out[i][j] = d[i] * B[i][j]; 16-byte loads/stores when the layout allows.
__global__ void __launch_bounds__(256) rowscale_vec_kernel(const float* __restrict__ d,
                                                           const float4* __restrict__ b,
                                                           float4* __restrict__ out,
                                                           int64_t cols4, int64_t ldb4,
                                                           int64_t ldo4) {
  constexpr int kUnroll = 4;
  const int64_t row = blockIdx.y;
  const float s = __ldg(d + row);
  const float4* src = b + row * ldb4;
  float4* dst = out + row * ldo4;
  int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x * kUnroll + threadIdx.x;
  float4 v[kUnroll];
#pragma unroll
  for (int u = 0; u < kUnroll; ++u) {
    const int64_t cc = c + static_cast<int64_t>(u) * blockDim.x;
    if (cc < cols4) v[u] = __ldcs(src + cc);
  }
#pragma unroll
  for (int u = 0; u < kUnroll; ++u) {
    const int64_t cc = c + static_cast<int64_t>(u) * blockDim.x;
    if (cc < cols4) {
      float4 o;
      o.x = v[u].x * s;
      o.y = v[u].y * s;
      o.z = v[u].z * s;
      o.w = v[u].w * s;
      __stcs(dst + cc, o);
    }
  }
}

__global__ void rowscale_scalar_kernel(const float* __restrict__ d, const float* __restrict__ b,
                                       float* __restrict__ out, int64_t rows, int64_t cols,
                                       int64_t ldb, int64_t ldo) {
  const int64_t row = blockIdx.y;
  if (row >= rows) return;
  const float s = __ldg(d + row);
  for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < cols;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[row * ldo + c] = b[row * ldb + c] * s;
}

// ---------------------------------------------------------------- engine instantiations
template <int BN, int STAGES, bool A_MN, bool B_MN, bool X3, bool XF, bool PAIR, int EPIG,
          int EPIW>
int launch_engine(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc,
                  const CUtensorMap& mad, const CUtensorMap& mbd, const EngineParams& p, int grid,
                  cudaStream_t stream) {
  using Cfg = EngineCfg<BN, STAGES, A_MN, B_MN, X3, XF, PAIR, EPIG, EPIW>;
  auto kern = gemm_tf32_kernel<BN, STAGES, A_MN, B_MN, X3, XF, PAIR, EPIG, EPIW>;
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Cfg::kSmemBytes) != cudaSuccess)
      return B2G_ERR_LAUNCH;
    configured_dev = dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int nattr = 0;
  if (PAIR) {
    attr[nattr].id = cudaLaunchAttributeClusterDimension;
    attr[nattr].val.clusterDim.x = 2;
    attr[nattr].val.clusterDim.y = 1;
    attr[nattr].val.clusterDim.z = 1;
    ++nattr;
  }
  if (B2G_PDL) {
    // Back-to-back launches: this grid's CTAs may start (and set up) on SMs
    // the previous kernel has left; the kernel waits before touching memory.
    attr[nattr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[nattr].val.programmaticStreamSerializationAllowed = 1;
    ++nattr;
  }
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  if (cudaLaunchKernelEx(&cfg, kern, ma, mb, mc, mad, mbd, p) != cudaSuccess)
    return B2G_ERR_LAUNCH;
  return cudaGetLastError() == cudaSuccess ? B2G_OK : B2G_ERR_LAUNCH;
}

template <int BN, int STAGES, bool X3, bool XF, bool PAIR, int EPIG = 1, int EPIW = 8>
int launch_majors(bool a_mn, bool b_mn, const CUtensorMap (&m)[5], const EngineParams& p,
                  int grid, cudaStream_t st) {
  if (!a_mn && !b_mn)
    return launch_engine<BN, STAGES, false, false, X3, XF, PAIR, EPIG, EPIW>(m[0], m[1], m[2], m[3],
                                                                        m[4], p, grid, st);
  if (!a_mn && b_mn)
    return launch_engine<BN, STAGES, false, true, X3, XF, PAIR, EPIG, EPIW>(m[0], m[1], m[2], m[3],
                                                                       m[4], p, grid, st);
  if (a_mn && !b_mn)
    return launch_engine<BN, STAGES, true, false, X3, XF, PAIR, EPIG, EPIW>(m[0], m[1], m[2], m[3],
                                                                       m[4], p, grid, st);
  return launch_engine<BN, STAGES, true, true, X3, XF, PAIR, EPIG, EPIW>(m[0], m[1], m[2], m[3], m[4],
                                                                    p, grid, st);
}

// Unit table for triangular ops: every tile's K range (the engine's own
// clipping), tiles longer than the mean load per cluster cut into K pieces
// (which then reduce-add into a pre-zeroed C region), and a longest-first
// greedy assignment to the least-loaded cluster.  Entry r * clusters + c is
// cluster c's r-th unit (padding entries are skips), matching the kernel's
// static stride over units.
struct TriTable {
  std::vector<int4> units;
  std::vector<int2> split_tiles;
  // What the engine reads (unit-table path without a pre-pass): the units,
  // then one {tm, tn, 0, 0} entry per split tile.
  std::vector<int4> device_image() const {
    std::vector<int4> v(units);
    for (const int2& t : split_tiles) v.push_back(make_int4(t.x, t.y, 0, 0));
    return v;
  }
};

TriTable build_tri_table(const b2g_gemm_desc* d, int block_m, int block_n, int tiles_m,
                         int tiles_n, int clusters, bool allow_split) {
  EngineParams q;
  std::memset(&q, 0, sizeof(q));
  q.K = static_cast<int>(d->k);
  q.block_m = block_m;
  q.block_n = block_n;
  q.tiles_m = tiles_m;
  q.tiles_n = tiles_n;
  q.splits = 1;
  q.kb_total = static_cast<int>(cdiv(d->k, kBlockK));
  q.kb_per_split = std::max(q.kb_total, 1);
  q.group_m = 8;
  q.tri = d->op == B2G_OP_TRI_UPPER ? kTriUpper : kTriLower;
  struct Item { int tm, tn, lo, hi, flags, weight, slot; };
  std::vector<Item> items;
  const int64_t ntiles = static_cast<int64_t>(tiles_m) * tiles_n;
  int64_t total = 0;
  std::vector<WorkUnit> tiles(ntiles);
  for (int64_t t = 0; t < ntiles; ++t) {
    tiles[t] = decode_unit(q, t);
    total += tiles[t].kb_hi - tiles[t].kb_lo;
  }
  const int64_t lmax = allow_split
                           ? std::max<int64_t>(8, cdiv(total * tri_split_pct(), clusters * 100ll))
                           : (1ll << 40);
  TriTable out;
  for (const WorkUnit& u : tiles) {
    const int len = u.kb_hi - u.kb_lo;
    if (len == 0) {
      items.push_back({u.tm, u.tn, 0, 0, 0, 3, 0});   // zero tile: epilogue stores only
      continue;
    }
    // Split tiles get a flag slot (the engine's in-kernel clear of split
    // tiles has kFlagTiles of them); beyond that, tiles stay whole.
    int np = static_cast<int>(cdiv(len, lmax));
    if (np > 1 && static_cast<int>(out.split_tiles.size()) >= kFlagTiles) np = 1;
    const int slot = np > 1 ? static_cast<int>(out.split_tiles.size()) + 1 : 0;
    if (np > 1) out.split_tiles.push_back(make_int2(u.tm, u.tn));
    for (int j = 0; j < np; ++j) {
      const int lo = u.kb_lo + static_cast<int>(static_cast<int64_t>(len) * j / np);
      const int hi = u.kb_lo + static_cast<int>(static_cast<int64_t>(len) * (j + 1) / np);
      const int fl = np > 1 ? (kUnitAccumulate | (j == 0 ? kUnitFirst : 0)) : 0;
      items.push_back({u.tm, u.tn, lo, hi, fl, hi - lo + 2, slot});
    }
  }
  std::stable_sort(items.begin(), items.end(),
                   [](const Item& x, const Item& y) { return x.weight > y.weight; });
  using Load = std::pair<int64_t, int>;   // (load, cluster)
  std::priority_queue<Load, std::vector<Load>, std::greater<Load>> heap;
  for (int c = 0; c < clusters; ++c) heap.push({0, c});
  std::vector<std::vector<int>> per(clusters);
  for (int i = 0; i < static_cast<int>(items.size()); ++i) {
    Load l = heap.top();
    heap.pop();
    per[l.second].push_back(i);
    l.first += items[i].weight;
    heap.push(l);
  }
  // Within a cluster, wholly masked tiles (pure zero stores, no MMA) go
  // first: the epilogue writes them while the first real unit's mainloop
  // runs, instead of leaving them as a store-only tail.
  for (auto& v : per)
    std::stable_partition(v.begin(), v.end(),
                          [&](int i) { return items[i].lo == items[i].hi; });
  size_t rounds = 0;
  for (const auto& v : per) rounds = std::max(rounds, v.size());
  out.units.assign(rounds * clusters, make_int4(0, 0, 0, kUnitSkip << 24));
  for (int c = 0; c < clusters; ++c)
    for (size_t r = 0; r < per[c].size(); ++r) {
      const Item& it = items[per[c][r]];
      out.units[r * clusters + c] =
          make_int4(it.tm | (it.slot << 16), it.tn, it.lo, it.hi | (it.flags << 24));
    }
  return out;
}

// build_tri_table memoised on everything it depends on (shape, triangle,
// tiling, cluster count, whether K pieces may reduce-add): repeated calls of
// one shape reuse the table instead of re-sorting it on the host.  Entries
// are shared_ptrs: a caller keeps its table alive while another thread's
// call evicts it from the cache.
std::shared_ptr<const TriTable> cached_tri_table(const b2g_gemm_desc* d, int block_m,
                                                 int block_n, int tiles_m, int tiles_n,
                                                 int clusters, bool allow_split) {
  using Key = std::tuple<int64_t, int64_t, int, int, int, int, int, int, int, int>;
  static std::mutex mu;
  static std::map<Key, std::shared_ptr<const TriTable>> cache;
  const Key key{d->m,    d->k,    d->op,    block_m,     block_n,
                tiles_m, tiles_n, clusters, allow_split, tri_split_pct()};
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  auto t = std::make_shared<const TriTable>(
      build_tri_table(d, block_m, block_n, tiles_m, tiles_n, clusters, allow_split));
  std::lock_guard<std::mutex> lk(mu);
  if (cache.size() >= 64) cache.erase(cache.begin());
  return cache.emplace(key, std::move(t)).first->second;
}

bool valid_desc(const b2g_gemm_desc* d) {
  if (!d) return false;
  if (d->m < 0 || d->n < 0 || d->k < 0 || d->batch < 1) return false;
  if (d->op < B2G_OP_GEMM || d->op > B2G_OP_TRI_LOWER) return false;
  if (d->precision != B2G_PREC_TF32 && d->precision != B2G_PREC_3XTF32) return false;
  if (d->m > INT32_MAX / 2 || d->n > INT32_MAX / 2 || d->k > INT32_MAX / 2) return false;
  if (d->batch > 65535) return false;
  if (d->op != B2G_OP_GEMM && (d->m != d->n || d->n != d->k)) return false;
  const int64_t a_inner = d->trans_a ? d->m : d->k;
  const int64_t b_inner = d->trans_b ? d->k : d->n;
  if (d->m > 0 && d->n > 0 && d->k > 0) {
    if (!d->a || !d->b) return false;
    if (d->lda < std::max<int64_t>(1, a_inner) || d->ldb < std::max<int64_t>(1, b_inner))
      return false;
    if (d->stride_a < 0 || d->stride_b < 0) return false;
  }
  if (d->m > 0 && d->n > 0) {
    if (!d->c || d->ldc < std::max<int64_t>(1, d->n) || d->stride_c < 0) return false;
    if (d->batch > 1 && d->stride_c < d->m * d->ldc) return false;
  }
  return true;
}

bool tma_ok(const float* p, int64_t ld, int64_t stride, int64_t batch) {
  if (reinterpret_cast<uintptr_t>(p) % 16) return false;
  if (ld % 4) return false;
  if (batch > 1 && stride != 0 && stride % 4) return false;
  return true;
}

// Staged copy geometry of an operand (rows x cols per batch, aligned pitch).
struct Stage {
  int64_t rows, cols, pitch, bstride, nbatch, bytes;
};
Stage stage_geom(int64_t rows, int64_t cols, int64_t nbatch, int64_t align = 4) {
  Stage s;
  s.rows = rows;
  s.cols = cols;
  s.pitch = round_up(std::max<int64_t>(cols, 1), align);
  s.bstride = s.pitch * rows;
  s.nbatch = nbatch;
  s.bytes = round_up(s.bstride * nbatch * 4, 256);
  return s;
}

}  // namespace
}  // namespace b2g

namespace b2g {
int* current_error_word() {
  DeviceState* ds = nullptr;
  return device_state(&ds) == B2G_OK ? ds->err_word : nullptr;
}
long long current_wait_limit_ns() { return wait_limit_ns(); }
bool pdl_enabled() { return B2G_PDL != 0; }
}  // namespace b2g

using namespace b2g;

extern "C" int b2g_version(void) { return 100; }

extern "C" const char* b2g_status_string(int s) {
  switch (s) {
    case B2G_OK: return "ok";
    case B2G_ERR_INVALID_ARG: return "invalid argument";
    case B2G_ERR_UNSUPPORTED: return "unsupported layout or shape";
    case B2G_ERR_WORKSPACE: return "workspace missing or too small";
    case B2G_ERR_LAUNCH: return "CUDA launch or API failure";
    case B2G_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    case B2G_ERR_NO_DEVICE: return "no sm_100 device is current";
    case B2G_ERR_SCRATCH_LIMIT:
      return "operand staging needs more than the fixed no-allocation scratch (16 MiB)";
    default: return "unknown status";
  }
}

namespace {

// Split-K for a tile grid: split when the tiles alone leave more than a
// quarter of the SMs idle, keeping at least 8 K blocks per split (partial
// sums add into a cleared C).  Triangular ops never split.
void choose_splits(const b2g_gemm_desc* d, int64_t slots, int64_t kb_total, int num_sms,
                   int64_t* splits, int64_t* kbps) {
  int64_t s = 1;
  if (d->op == B2G_OP_GEMM && slots > 0 && slots * 4 < num_sms * 3 && kb_total >= 16)
    s = std::max<int64_t>(1, std::min<int64_t>(num_sms / slots, kb_total / 8));
  const int forced = splits_override();
  if (d->op == B2G_OP_GEMM && forced > 0) s = std::min<int64_t>(forced, std::max<int64_t>(kb_total, 1));
  *kbps = std::max<int64_t>(1, cdiv(kb_total, s));
  *splits = std::max<int64_t>(1, cdiv(kb_total, *kbps));
}

}  // namespace

extern "C" int b2g_gemm_plan_for(const b2g_gemm_desc* d, int num_sms, b2g_gemm_plan* pl) {
  if (!valid_desc(d) || !pl || num_sms <= 0) return B2G_ERR_INVALID_ARG;
  std::memset(pl, 0, sizeof(*pl));
  const bool x3 = d->precision == B2G_PREC_3XTF32;
  const int64_t kb_total = cdiv(d->k, kBlockK);
  const int64_t batch = d->batch;
  int bn = 256, ctas = 1;
  const char* forced = tile_override();
  // Triangular TF32 products on untransposed operands: a pre-pass writes
  // masked copies of the diagonal blocks that the engine's producer loads.
  // Other layouts (and B2G_TRI_PATH=gate, a tuning knob) mask inside the
  // engine: the K blocks that the diagonal crosses go through the transform
  // warps, wholly masked boxes are TMA zero fill.  At N = 4096 the copies
  // cost one 2-4 us pre-pass; gating costs a transform handshake on the
  // MMA's path at every crossing block (58 vs 103 us measured).
  const bool tri_diag = d->op != B2G_OP_GEMM && !x3 && !d->trans_a && !d->trans_b &&
                        !tri_path_gate();
  const bool tri_gate = d->op != B2G_OP_GEMM && !x3 && !tri_diag;
  // 3xTF32 on plain GEMMs: lo parts pre-split into workspace, loaded by TMA;
  // triangular 3xTF32 masks and splits in the (single-CTA) transform warps.
  const bool x3_split = x3 && d->op == B2G_OP_GEMM;
  if (x3 || d->op != B2G_OP_GEMM) {
    // CTA-pair 256 x 256 units once there are at least two 128-row blocks,
    // else one CTA with 128-wide tiles.  Triangular ops that still need the
    // transform warps stay on single-CTA units (measured at N = 4096: 106 us
    // vs 190 us for pairs, whose transform warps mask twice the tile).
    const bool force_single = forced && std::strncmp(forced, "single", 6) == 0;
    const bool force_pair = forced && std::strncmp(forced, "pair", 4) == 0;
    if (d->m > kBlockM && !force_single && (x3_split || tri_diag || tri_gate || force_pair)) {
      ctas = 2;
      bn = 256;
    } else {
      bn = 128;
    }
  } else {
    // Cost model: waves of CTAs over the SMs times the per-SM work of one
    // unit (tile width x K blocks of its split), divided by the per-SM
    // efficiency of the tile shape.  Efficiencies are measured throughputs
    // on B200 relative to the CTA-pair 256 x 256 unit (8192 x 8192 x 4096:
    // 712 / 590 / 474 / 452 TFLOP/s for pair256 / single256 / pair128 /
    // single128): wider units stream fewer operand bytes per flop through
    // L2 and shared memory, which costs power and so clock under the 1 kW
    // cap.  The 512-wide pair unit (no accumulator double buffering) pays
    // off only when a unit's K loop is long enough to hide its epilogue.
    // Units of at most two K blocks are output-bound: there single-CTA units
    // store faster than pairs (16384^2 x 32: 6.49 / 5.07 / 4.83 / 3.60 TB/s
    // for single256 / single128 / pair256 / pair128).
    struct Cand { int ctas, bn; double eff, eff_long_k, eff_short_k; };
    const Cand cands[] = {{2, 256, 1.0, 1.0, 1.0}, {2, 512, 0.85, 1.05, 0.85},
                          {1, 256, 0.83, 0.83, 1.34}, {2, 128, 0.66, 0.66, 0.75},
                          {1, 128, 0.63, 0.63, 1.05}};
    // B2G_TILE=pair512|pair256|pair128|single256|single128 pins the choice
    // (a tuning and test aid).
    double best = 0.0;
    for (const Cand& c : cands) {
      if (forced && *forced) {
        char name[16];
        std::snprintf(name, sizeof(name), "%s%d", c.ctas == 2 ? "pair" : "single", c.bn);
        if (std::strcmp(name, forced) != 0) continue;
      }
      const int64_t units = cdiv(d->m, kBlockM * c.ctas) * cdiv(d->n, c.bn) * batch;
      int64_t splits, kbps;
      choose_splits(d, units * c.ctas, kb_total, num_sms, &splits, &kbps);
      const double waves = static_cast<double>(cdiv(units * splits * c.ctas, num_sms));
      const double eff = kbps >= 64 ? c.eff_long_k : (kbps <= 2 ? c.eff_short_k : c.eff);
      const double cost = waves * c.bn * static_cast<double>(std::max<int64_t>(kbps, 1)) / eff;
      if (best == 0.0 || cost < best * 0.999) {
        best = cost;
        bn = c.bn;
        ctas = c.ctas;
      }
    }
  }
  pl->block_m = kBlockM * ctas;
  pl->block_n = bn;
  pl->block_k = kBlockK;
  pl->cluster_ctas = ctas;
  if (x3)
    pl->stages = 3;
  else if (d->op != B2G_OP_GEMM)
    pl->stages = 6;
  else if (ctas == 2)
    pl->stages = bn == 512 ? 4 : (bn == 256 ? 6 : 8);
  else
    pl->stages = bn == 256 ? 4 : 6;
  pl->tiles_m = static_cast<int32_t>(cdiv(d->m, pl->block_m));
  pl->tiles_n = static_cast<int32_t>(cdiv(d->n, bn));
  const int64_t tiles = static_cast<int64_t>(pl->tiles_m) * pl->tiles_n * batch;
  int64_t splits, kbps;
  choose_splits(d, tiles * ctas, kb_total, num_sms, &splits, &kbps);
  pl->splits = static_cast<int32_t>(splits);
  pl->kb_per_split = static_cast<int32_t>(kbps);
  pl->work_units = tiles * splits;
  pl->grid = static_cast<int32_t>(std::min<int64_t>(pl->work_units, num_sms / ctas) * ctas);
  pl->a_mn_major = d->trans_a ? 1 : 0;
  pl->b_mn_major = d->trans_b ? 0 : 1;
  pl->tma_store = (reinterpret_cast<uintptr_t>(d->c) % 16 == 0) && (d->ldc % 4 == 0) &&
                  (d->batch == 1 || d->stride_c % 4 == 0);
  pl->tri_diag = tri_diag ? 1 : 0;
  pl->x3_split = x3_split ? 1 : 0;
  const int64_t sa_batch = (d->stride_a == 0) ? 1 : batch;
  const int64_t sb_batch = (d->stride_b == 0) ? 1 : batch;
  pl->stage_a = tma_ok(d->a, d->lda, d->stride_a, sa_batch) ? 0 : 1;
  pl->stage_b = tma_ok(d->b, d->ldb, d->stride_b, sb_batch) ? 0 : 1;
  int64_t ws = 0;
  if (pl->stage_a)
    ws += stage_geom(d->trans_a ? d->k : d->m, d->trans_a ? d->m : d->k, sa_batch,
                     d->trans_a ? 32 : 4).bytes;
  if (pl->stage_b)
    ws += stage_geom(d->trans_b ? d->n : d->k, d->trans_b ? d->k : d->n, sb_batch,
                     d->trans_b ? 4 : 32).bytes;
  if (pl->x3_split) {
    ws += stage_geom(d->trans_a ? d->k : d->m, d->trans_a ? d->m : d->k, sa_batch,
                     d->trans_a ? 32 : 4).bytes;
    ws += stage_geom(d->trans_b ? d->n : d->k, d->trans_b ? d->k : d->n, sb_batch,
                     d->trans_b ? 4 : 32).bytes;
  }
  if (pl->tri_diag) {
    ws += 2 * round_up(d->m * kTriDiagBlock * 4, 256);
    const auto tt = cached_tri_table(d, pl->block_m, pl->block_n, pl->tiles_m, pl->tiles_n,
                                     pl->grid / ctas, pl->tma_store);
    ws += round_up(static_cast<int64_t>(tt->units.size()) * sizeof(int4), 256);
    ws += round_up(static_cast<int64_t>(tt->split_tiles.size()) * sizeof(int2), 256);
    pl->work_units = static_cast<int64_t>(tt->units.size());
  } else if (tri_gate) {
    // The unit table lives in a per-device cache (uploaded once per shape).
    const auto tt = cached_tri_table(d, pl->block_m, pl->block_n, pl->tiles_m, pl->tiles_n,
                                     pl->grid / ctas, pl->tma_store);
    pl->work_units = static_cast<int64_t>(tt->units.size());
  }
  pl->workspace_bytes = ws;
  return B2G_OK;
}

// SM count the launches on the current device are planned for (no
// allocation, no context state beyond the runtime's); 148 (a B200) when no
// device is usable, e.g. on a build host.
static int planning_sms() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      sms <= 0) {
    cudaGetLastError();   // clear the sticky-free error of a missing device
    return 148;
  }
  return std::min(sms, max_sms_override());
}

extern "C" int64_t b2g_gemm_workspace_bytes(const b2g_gemm_desc* d) {
  b2g_gemm_plan pl;
  if (b2g_gemm_plan_for(d, planning_sms(), &pl) != B2G_OK) return -1;
  return pl.workspace_bytes;
}

// Everything a GEMM call does once its plan is known and its workspace
// checked: staged copies of unaligned operands, tensor maps, split-K clear
// of C, and the engine launch.
// Device copies of triangular unit tables, per device, uploaded once per
// table (synchronously, at the first call of a shape: make that call before
// any stream capture) and kept with the host table that they copy.
const int4* device_tri_table(const std::shared_ptr<const TriTable>& t) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  struct Entry { std::shared_ptr<const TriTable> host; int4* dev; };
  static std::mutex mu;
  static std::map<const TriTable*, Entry> cache[kMaxDevices];
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache[dev].find(t.get());
  if (it != cache[dev].end()) return it->second.dev;
  const std::vector<int4> image = t->device_image();
  const size_t bytes = image.size() * sizeof(int4);
  void* ptr = nullptr;
  if (bytes == 0 || cudaMalloc(&ptr, bytes) != cudaSuccess) return nullptr;
  if (cudaMemcpy(ptr, image.data(), bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaFree(ptr);
    return nullptr;
  }
  cache[dev].emplace(t.get(), Entry{t, static_cast<int4*>(ptr)});
  return static_cast<int4*>(ptr);
}

// Bytes of caller workspace the triangular unit table takes when it must
// live there (allocation-free calls): 0 for other plans.
int64_t tri_gate_table_bytes(const b2g_gemm_desc* d, const b2g_gemm_plan& pl) {
  if (d->op == B2G_OP_GEMM || d->precision == B2G_PREC_3XTF32 || pl.tri_diag) return 0;
  const auto t = cached_tri_table(d, pl.block_m, pl.block_n, pl.tiles_m, pl.tiles_n,
                                  pl.grid / pl.cluster_ctas, pl.tma_store);
  return round_up(static_cast<int64_t>(t->units.size() + t->split_tiles.size()) * sizeof(int4),
                  256);
}

// table_in_workspace: the triangular unit table is copied into the
// workspace on every call (allocation-free callers) instead of the
// per-device cache.
static int run_planned(const b2g_gemm_desc* d, const b2g_gemm_plan& pl, void* workspace,
                       int* err_word, cudaStream_t stream, const float* row_bias = nullptr,
                       bool table_in_workspace = false,
                       const EngineParams::Xgpu* xgpu = nullptr) {
  const float* a = d->a;
  const float* b = d->b;
  int64_t lda = d->lda, ldb = d->ldb, sa = d->stride_a, sb = d->stride_b;
  const int64_t a_batch = (d->stride_a == 0) ? 1 : d->batch;
  const int64_t b_batch = (d->stride_b == 0) ? 1 : d->batch;
  char* ws = static_cast<char*>(workspace);
  // Extents of MN-major operands as the grouped loads see them (staged
  // copies are zero-padded to 32 columns).
  int64_t a_mn_ext = d->m, b_mn_ext = d->n;
  if (d->k > 0 && pl.stage_a) {
    Stage g = stage_geom(d->trans_a ? d->k : d->m, d->trans_a ? d->m : d->k, a_batch,
                         d->trans_a ? 32 : 4);
    if (d->trans_a) a_mn_ext = g.pitch;
    float* dst = reinterpret_cast<float*>(ws);
    const int64_t nrows = g.rows * g.nbatch;
    pitch_copy_kernel<<<static_cast<int>(std::min<int64_t>(nrows, 65535)), 256, 0, stream>>>(
        a, dst, g.rows, g.cols, lda, sa, g.pitch, g.bstride, g.nbatch);
    a = dst;
    lda = g.pitch;
    sa = (a_batch > 1) ? g.bstride : 0;
    ws += g.bytes;
  }
  if (d->k > 0 && pl.stage_b) {
    Stage g = stage_geom(d->trans_b ? d->n : d->k, d->trans_b ? d->k : d->n, b_batch,
                         d->trans_b ? 4 : 32);
    if (!d->trans_b) b_mn_ext = g.pitch;
    float* dst = reinterpret_cast<float*>(ws);
    const int64_t nrows = g.rows * g.nbatch;
    pitch_copy_kernel<<<static_cast<int>(std::min<int64_t>(nrows, 65535)), 256, 0, stream>>>(
        b, dst, g.rows, g.cols, ldb, sb, g.pitch, g.bstride, g.nbatch);
    b = dst;
    ldb = g.pitch;
    sb = (b_batch > 1) ? g.bstride : 0;
    ws += g.bytes;
  }

  // 3xTF32 pre-split: lo copies of A and B at a 16-byte pitch, one launch.
  const float* alo = nullptr;
  const float* blo = nullptr;
  int64_t ldalo = 0, ldblo = 0, salo = 0, sblo = 0;
  if (pl.x3_split && d->k > 0) {
    Stage ga = stage_geom(d->trans_a ? d->k : d->m, d->trans_a ? d->m : d->k, a_batch,
                          d->trans_a ? 32 : 4);
    float* da = reinterpret_cast<float*>(ws);
    ws += ga.bytes;
    Stage gb = stage_geom(d->trans_b ? d->n : d->k, d->trans_b ? d->k : d->n, b_batch,
                          d->trans_b ? 4 : 32);
    float* db = reinterpret_cast<float*>(ws);
    ws += gb.bytes;
    const SplitJob ja{a, da, ga.rows, ga.cols, lda, sa, ga.pitch, ga.bstride, ga.nbatch};
    const SplitJob jb{b, db, gb.rows, gb.cols, ldb, sb, gb.pitch, gb.bstride, gb.nbatch};
    const int64_t rows = std::max(ga.rows * ga.nbatch, gb.rows * gb.nbatch);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(std::min<int64_t>(rows, 65535)), 2, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = B2G_PDL ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, split_lo_kernel, ja, jb) != cudaSuccess) return B2G_ERR_LAUNCH;
    alo = da;
    blo = db;
    ldalo = ga.pitch;
    ldblo = gb.pitch;
    salo = a_batch > 1 ? ga.bstride : 0;
    sblo = b_batch > 1 ? gb.bstride : 0;
  }
  float* adiag = nullptr;
  float* bdiag = nullptr;
  int4* table = nullptr;
  if (pl.tri_diag) {
    const int64_t nbytes = round_up(d->m * kTriDiagBlock * 4, 256);
    adiag = reinterpret_cast<float*>(ws);
    bdiag = reinterpret_cast<float*>(ws + nbytes);
    ws += 2 * nbytes;
    // Unit table (longest-first, split long tiles) followed by the split
    // tiles' coordinates.  Normal calls read it from the per-device cache
    // (uploaded once per shape); allocation-free calls place it in their
    // workspace through the pre-pass's parameters (or a copy when larger).
    const auto tri_ptr = cached_tri_table(d, pl.block_m, pl.block_n, pl.tiles_m, pl.tiles_n,
                                          pl.grid / pl.cluster_ctas, pl.tma_store);
    const TriTable& tri = *tri_ptr;
    const int n_split = static_cast<int>(tri.split_tiles.size());
    const int64_t diag_blocks = cdiv(d->m, kTriDiagBlock) * (kTriDiagBlock / kTriDiagRows);
    const int64_t zero_blocks = static_cast<int64_t>(n_split) * cdiv(pl.block_m, kTriDiagRows);
    dim3 grid(static_cast<unsigned>(std::max(diag_blocks, zero_blocks)), n_split ? 3 : 2);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = B2G_PDL ? 1 : 0;
    const int upper = static_cast<int>(d->op == B2G_OP_TRI_UPPER);
    if (!table_in_workspace) {
      table = const_cast<int4*>(device_tri_table(tri_ptr));
      if (!table) return B2G_ERR_LAUNCH;
      const int4* split4 = table + tri.units.size();
      if (cudaLaunchKernelEx(&cfg, tri_prepare_cached_kernel, a, lda, b, ldb,
                             static_cast<int64_t>(d->m), upper, adiag, bdiag, d->c,
                             static_cast<int64_t>(d->ldc), split4, n_split,
                             static_cast<int>(pl.block_m),
                             static_cast<int>(pl.block_n)) != cudaSuccess)
        return B2G_ERR_LAUNCH;
    } else {
      const int64_t tbytes = static_cast<int64_t>(tri.units.size()) * sizeof(int4);
      const int64_t zbytes = static_cast<int64_t>(tri.split_tiles.size()) * sizeof(int2);
      std::vector<char> host(round_up(tbytes, 256) + zbytes);
      std::memcpy(host.data(), tri.units.data(), tbytes);
      if (zbytes) std::memcpy(host.data() + round_up(tbytes, 256), tri.split_tiles.data(), zbytes);
      table = reinterpret_cast<int4*>(ws);
      const int2* split_list = reinterpret_cast<const int2*>(ws + round_up(tbytes, 256));
      ws += round_up(tbytes, 256) + round_up(zbytes, 256);
      // Small tables ride in the pre-pass's parameters (no copy engine, no
      // staging of pageable memory); larger ones are copied.
      static thread_local TableParam tparam;
      const int64_t words = static_cast<int64_t>(host.size() + 15) / 16;
      if (words <= kTableParamWords) {
        host.resize(words * 16, 0);
        tparam.words = static_cast<int>(words);
        tparam.split_off = static_cast<int>(round_up(tbytes, 256) / 16);
        std::memcpy(tparam.w, host.data(), host.size());
      } else {
        tparam.words = 0;
        if (cudaMemcpyAsync(table, host.data(), host.size(), cudaMemcpyHostToDevice, stream) !=
            cudaSuccess)
          return B2G_ERR_LAUNCH;
      }
      if (cudaLaunchKernelEx(&cfg, tri_prepare_kernel, a, lda, b, ldb, static_cast<int64_t>(d->m),
                             upper, adiag, bdiag, d->c, static_cast<int64_t>(d->ldc), split_list,
                             n_split, static_cast<int>(pl.block_m), static_cast<int>(pl.block_n),
                             table, tparam) != cudaSuccess)
        return B2G_ERR_LAUNCH;
    }
  }

  // Triangular TF32 through the gated transform warps: the unit table from
  // the per-device cache (or copied into the workspace), split tiles
  // cleared in the kernel through tile flags.
  const bool tri_gate = d->op != B2G_OP_GEMM && d->precision != B2G_PREC_3XTF32 && !pl.tri_diag;
  std::shared_ptr<const TriTable> gate_table;
  if (tri_gate) {
    gate_table = cached_tri_table(d, pl.block_m, pl.block_n, pl.tiles_m, pl.tiles_n,
                                  pl.grid / pl.cluster_ctas, pl.tma_store);
    if (table_in_workspace) {
      // The image is staged by the runtime before the call returns (pageable
      // source), so the local vector may go out of scope.
      const std::vector<int4> image = gate_table->device_image();
      const int64_t tbytes = static_cast<int64_t>(image.size()) * sizeof(int4);
      table = reinterpret_cast<int4*>(ws);
      if (cudaMemcpyAsync(table, image.data(), tbytes, cudaMemcpyHostToDevice, stream) !=
          cudaSuccess)
        return B2G_ERR_LAUNCH;
      ws += round_up(tbytes, 256);
    } else {
      table = const_cast<int4*>(device_tri_table(gate_table));
      if (!table) return B2G_ERR_LAUNCH;
    }
  }

  EngineParams p;
  std::memset(&p, 0, sizeof(p));
  p.M = static_cast<int>(d->m);
  p.N = static_cast<int>(d->n);
  p.K = static_cast<int>(d->k);
  p.batch = static_cast<int>(d->batch);
  p.block_m = pl.block_m;
  p.block_n = pl.block_n;
  p.tiles_m = pl.tiles_m;
  p.tiles_n = pl.tiles_n;
  p.splits = pl.splits;
  p.kb_total = static_cast<int>(cdiv(d->k, kBlockK));
  p.kb_per_split = pl.kb_per_split;
  // Raster: groups of 8 tile-rows share B columns in L2; output-bound short-K
  // problems instead walk along N so concurrent units write whole row runs
  // (measured +3 % on 16384^2 x 32).
  p.group_m = p.kb_total <= 8 ? 1 : 8;
  p.tri = d->op == B2G_OP_TRI_UPPER ? kTriUpper : (d->op == B2G_OP_TRI_LOWER ? kTriLower : kTriNone);
  p.a_batched = a_batch > 1;
  p.b_batched = b_batch > 1;
  p.work_units = pl.work_units;
  p.C = d->c;
  p.ldc = d->ldc;
  p.stride_c = d->stride_c;
  p.atomic_out = pl.splits > 1;
  p.vec_ok = (reinterpret_cast<uintptr_t>(d->c) % 16 == 0) && (d->ldc % 4 == 0) &&
             (d->batch == 1 || d->stride_c % 4 == 0);
  p.tma_store = pl.tma_store;
  p.wait_limit_ns = wait_limit_ns();
  p.inject_stall = take_injected_stall();
  p.tri_sorted = (p.tri != kTriNone && pl.block_m == pl.block_n) ? 1 : 0;
  p.tri_diag = pl.tri_diag;
  p.unit_table = table;
  p.xf_gate = tri_gate ? 1 : 0;
  if (tri_gate && !gate_table->split_tiles.empty()) {
    if (!tile_flag_region(&p.tile_flags, &p.epoch)) return B2G_ERR_LAUNCH;
    p.split_tiles = table + gate_table->units.size();
    p.n_split = static_cast<int>(gate_table->split_tiles.size());
  }
  p.diag_oob_row = static_cast<int>(d->m);
  p.row_bias = row_bias;
  p.err = err_word;
  if (xgpu) p.xg = *xgpu;
  p.trace = trace_pointer();
  // Dynamic schedule: plain GEMMs with more units than CTAs (pairs), every
  // unit holding at least one K block (no structurally empty units).
  const int64_t slots = pl.grid / pl.cluster_ctas;
  if (B2G_DYNAMIC_UNITS && d->op == B2G_OP_GEMM && d->k > 0 && pl.work_units > slots &&
      static_cast<int64_t>(pl.splits - 1) * pl.kb_per_split < p.kb_total) {
    p.sched = sched_slot();
    p.early_draw = early_draw_on() ? 1 : 0;
  }

  // Split-K accumulates into C, which must start at zero: the first K piece
  // of each tile clears it in the kernel (TMA stores, at most kFlagTiles
  // tiles), else the host clears C first.
  const int64_t n_tiles = static_cast<int64_t>(pl.tiles_m) * pl.tiles_n * d->batch;
  if (B2G_KERNEL_CLEAR && p.atomic_out && pl.tma_store && p.tri == kTriNone &&
      p.unit_table == nullptr && n_tiles <= kFlagTiles &&
      tile_flag_region(&p.tile_flags, &p.epoch)) {
  } else if (p.atomic_out) {
    for (int64_t bi = 0; bi < d->batch; ++bi) {
      cudaError_t e = cudaMemset2DAsync(d->c + bi * d->stride_c, d->ldc * 4, 0, d->n * 4, d->m,
                                        stream);
      if (e != cudaSuccess) return B2G_ERR_LAUNCH;
    }
  }

  CUtensorMap ma, mb, mc;
  // B box: one N=256 MMA sub-tile's share per CTA (the whole tile for one CTA).
  const int bn_cta = std::min(pl.block_n, 256) / pl.cluster_ctas;
  const int64_t k_ext = std::max<int64_t>(d->k, 1);
  bool ok;
  if (!pl.a_mn_major) {
    ok = make_map(&ma, a, k_ext, d->m, a_batch, lda, sa, kBlockK, kBlockM, false);
  } else {
    p.a_grouped = make_map_grouped(&ma, a, a_mn_ext, k_ext, a_batch, lda, sa, kBlockM / 32);
    ok = p.a_grouped || make_map(&ma, a, d->m, k_ext, a_batch, lda, sa, 32, kBlockK, true);
  }
  if (!ok) return B2G_ERR_UNSUPPORTED;
  if (!pl.b_mn_major) {
    ok = make_map(&mb, b, k_ext, d->n, b_batch, ldb, sb, kBlockK, bn_cta, false);
  } else {
    p.b_grouped = make_map_grouped(&mb, b, b_mn_ext, k_ext, b_batch, ldb, sb, bn_cta / 32);
    ok = p.b_grouped || make_map(&mb, b, d->n, k_ext, b_batch, ldb, sb, 32, kBlockK, true);
  }
  if (!ok) return B2G_ERR_UNSUPPORTED;
  if (pl.tma_store) {
    // C boxes of 32 x 32 fp32, 128-byte swizzled like the epilogue's staging.
    if (!make_map(&mc, d->c, d->n, d->m, d->batch, d->ldc, d->stride_c, 32, 32, false))
      return B2G_ERR_UNSUPPORTED;
  } else {
    mc = ma;   // unused by the kernel
  }
  CUtensorMap mad = ma, mbd = ma;   // diagonal-block copies (triangular) or lo parts (3xTF32)
  if (pl.x3_split && alo) {
    // The lo copies are laid out like the operands (same majorness and box),
    // so they take the same map geometry; a grouped A/B implies a grouped copy.
    if (!pl.a_mn_major)
      ok = make_map(&mad, alo, k_ext, d->m, a_batch, ldalo, salo, kBlockK, kBlockM, false);
    else if (p.a_grouped)
      ok = make_map_grouped(&mad, alo, a_mn_ext, k_ext, a_batch, ldalo, salo, kBlockM / 32);
    else
      ok = make_map(&mad, alo, d->m, k_ext, a_batch, ldalo, salo, 32, kBlockK, true);
    if (!ok) return B2G_ERR_UNSUPPORTED;
    if (!pl.b_mn_major)
      ok = make_map(&mbd, blo, k_ext, d->n, b_batch, ldblo, sblo, kBlockK, bn_cta, false);
    else if (p.b_grouped)
      ok = make_map_grouped(&mbd, blo, b_mn_ext, k_ext, b_batch, ldblo, sblo, bn_cta / 32);
    else
      ok = make_map(&mbd, blo, d->n, k_ext, b_batch, ldblo, sblo, 32, kBlockK, true);
    if (!ok) return B2G_ERR_UNSUPPORTED;
  }
  if (pl.tri_diag) {
    const int bcols = std::min(pl.block_n, 256) / pl.cluster_ctas;
    if (bcols != kTriDiagBlock ||
        !make_map(&mad, adiag, kTriDiagBlock, d->m, 1, kTriDiagBlock, 0, kBlockK, kBlockM, false) ||
        !make_map_grouped(&mbd, bdiag, kTriDiagBlock, d->m, 1, kTriDiagBlock, 0,
                          kTriDiagBlock / 32))
      return B2G_ERR_UNSUPPORTED;
  }

  const bool a_mn = pl.a_mn_major, b_mn = pl.b_mn_major;
  const bool x3 = d->precision == B2G_PREC_3XTF32;
  const bool tri_xf = p.tri != kTriNone && !pl.tri_diag;   // triangular via transform warps
  const int grid = pl.grid;
  const CUtensorMap maps[5] = {ma, mb, mc, mad, mbd};
  if (x3 && pl.x3_split && pl.cluster_ctas == 2)
    return launch_majors<256, 3, true, false, true>(a_mn, b_mn, maps, p, grid, stream);
  if (x3 && pl.x3_split)
    return launch_majors<128, 3, true, false, false>(a_mn, b_mn, maps, p, grid, stream);
  if (x3)   // triangular 3xTF32: masking and split in the transform warps
    return launch_majors<128, 3, true, true, false>(a_mn, b_mn, maps, p, grid, stream);
  if (tri_xf && pl.cluster_ctas == 2)
    return launch_majors<256, 6, false, true, true>(a_mn, b_mn, maps, p, grid, stream);
  if (tri_xf)
    return launch_majors<128, 6, false, true, false>(a_mn, b_mn, maps, p, grid, stream);
  if (pl.cluster_ctas == 2) {
    if (pl.block_n == 512)
      return launch_majors<512, 4, false, false, true>(a_mn, b_mn, maps, p, grid, stream);
    if (pl.block_n == 256 && p.kb_per_split >= 16 && !(p.tri != kTriNone && tri_epiw8()))
      // Long K loops: 4 epilogue warps drain a unit well inside the next
      // unit's mainloop and compete less with it (bmm 128 x 512x2048x1024:
      // +7 % in bursts, +2 % sustained under the power cap).
      return launch_majors<256, B2G_PAIR256_STAGES, false, false, true, B2G_PAIR256_EPIG,
                           B2G_PAIR256_LONGK_EPIW>(
          a_mn, b_mn, maps, p, grid, stream);
    if (pl.block_n == 256)
      return launch_majors<256, B2G_PAIR256_STAGES, false, false, true, B2G_PAIR256_EPIG,
                           B2G_PAIR256_EPIW>(a_mn, b_mn, maps, p, grid, stream);
    return launch_majors<128, 8, false, false, true>(a_mn, b_mn, maps, p, grid, stream);
  }
  if (pl.block_n == 256)
    return launch_majors<256, 4, false, false, false>(a_mn, b_mn, maps, p, grid, stream);
  return launch_majors<128, 6, false, false, false>(a_mn, b_mn, maps, p, grid, stream);
}

extern "C" int b2g_gemm(const b2g_gemm_desc* d, b2g_stream_t stream_handle) {
  if (!valid_desc(d)) return B2G_ERR_INVALID_ARG;
  if (d->m == 0 || d->n == 0) return B2G_OK;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_handle);
  DeviceState* ds = nullptr;
  int rc = device_state(&ds);
  if (rc != B2G_OK) return rc;
  b2g_gemm_plan pl;
  rc = b2g_gemm_plan_for(d, ds->num_sms, &pl);
  if (rc != B2G_OK) return rc;
  if (pl.workspace_bytes > 0 && (!d->workspace || d->workspace_bytes < pl.workspace_bytes))
    return B2G_ERR_WORKSPACE;
  return run_planned(d, pl, d->workspace, ds->err_word, stream);
}

extern "C" int b2g_gemm_splitk_peer(const b2g_gemm_desc* d, void* const* mailboxes, int world,
                                    int rank, int root, int64_t epoch,
                                    b2g_stream_t stream_handle) {
  if (!valid_desc(d)) return B2G_ERR_INVALID_ARG;
  if (world < 1 || world > kPeerMaxRanks || rank < 0 || rank >= world || root < 0 ||
      root >= world || epoch < 1 || !mailboxes)
    return B2G_ERR_INVALID_ARG;
  if (world == 1) return b2g_gemm(d, stream_handle);
  // One contiguous M x N output (the protocol moves it as a flat array).
  if (d->op != B2G_OP_GEMM || d->batch != 1 || d->ldc != d->n || d->m == 0 || d->n == 0)
    return B2G_ERR_UNSUPPORTED;
  if (reinterpret_cast<uintptr_t>(d->c) % 16) return B2G_ERR_UNSUPPORTED;
  for (int r = 0; r < world; ++r)
    if (!mailboxes[r]) return B2G_ERR_INVALID_ARG;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_handle);
  DeviceState* ds = nullptr;
  int rc = device_state(&ds);
  if (rc != B2G_OK) return rc;
  b2g_gemm_plan pl;
  rc = b2g_gemm_plan_for(d, ds->num_sms, &pl);
  if (rc != B2G_OK) return rc;
  if (pl.workspace_bytes > 0 && (!d->workspace || d->workspace_bytes < pl.workspace_bytes))
    return B2G_ERR_WORKSPACE;
  const int64_t elems = d->m * d->n;
  const PeerLayout lay = peer_layout(elems, world);
  EngineParams::Xgpu x;
  std::memset(&x, 0, sizeof(x));
  for (int r = 0; r < world; ++r) x.mbox[r] = static_cast<unsigned char*>(mailboxes[r]);
  x.epoch = epoch;
  x.elems = elems;
  x.nchunk = lay.nchunk;
  x.consumed_off = lay.consumed_off;
  x.count_off = lay.count_off;
  x.landing_off = lay.landing_off;
  x.slot_stride = lay.slot_stride;
  x.world = world;
  x.rank = rank;
  x.root = root;
  return run_planned(d, pl, d->workspace, ds->err_word, stream, nullptr, false, &x);
}

namespace b2g {
namespace {
// in_channels == 0: every output of channel o is bias[o] (or 0).
__global__ void conv_bias_fill_kernel(const float* __restrict__ bias, float* __restrict__ out,
                                      int64_t planes, int64_t cout, int64_t spatial) {
  for (int64_t pl = blockIdx.x; pl < planes; pl += gridDim.x) {
    const float v = bias ? bias[pl % cout] : 0.f;
    float* o = out + pl * spatial;
    for (int64_t i = threadIdx.x; i < spatial; i += blockDim.x) o[i] = v;
  }
}

// The batched GEMM a pointwise convolution runs as: out[n] = W . in[n].
bool conv_desc(int64_t batch, int64_t cin, int64_t cout, int64_t spatial, int precision,
               b2g_gemm_desc* d) {
  if (batch < 0 || cin < 0 || cout < 0 || spatial < 0) return false;
  std::memset(d, 0, sizeof(*d));
  d->op = B2G_OP_GEMM;
  d->precision = precision;
  d->m = cout;
  d->n = spatial;
  d->k = cin;
  d->batch = std::max<int64_t>(batch, 1);
  d->lda = std::max<int64_t>(cin, 1);
  d->stride_a = 0;   // one weight for every image
  d->ldb = std::max<int64_t>(spatial, 1);
  d->stride_b = cin * spatial;
  d->ldc = std::max<int64_t>(spatial, 1);
  d->stride_c = cout * spatial;
  return true;
}
}  // namespace
}  // namespace b2g

extern "C" int64_t b2g_pointwise_conv_workspace_bytes(const float* in, const float* weight,
                                                      const float* out, int64_t batch,
                                                      int64_t cin, int64_t cout, int64_t spatial,
                                                      int precision) {
  b2g_gemm_desc d;
  if (!conv_desc(batch, cin, cout, spatial, precision, &d)) return -1;
  if (batch == 0 || cout == 0 || spatial == 0) return 0;
  d.a = weight;
  d.b = in;
  d.c = const_cast<float*>(out);
  return b2g_gemm_workspace_bytes(&d);
}

extern "C" int b2g_pointwise_conv(const float* in, const float* weight, const float* bias,
                                  float* out, int64_t batch, int64_t cin, int64_t cout,
                                  int64_t spatial, int precision, void* workspace,
                                  int64_t workspace_bytes, b2g_stream_t stream_handle) {
  b2g_gemm_desc d;
  if (!conv_desc(batch, cin, cout, spatial, precision, &d)) return B2G_ERR_INVALID_ARG;
  if (batch == 0 || cout == 0 || spatial == 0) return B2G_OK;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_handle);
  if (!out) return B2G_ERR_INVALID_ARG;
  if (cin == 0) {
    const int64_t planes = batch * cout;
    conv_bias_fill_kernel<<<static_cast<unsigned>(std::min<int64_t>(planes, 65535)), 256, 0,
                            stream>>>(bias, out, planes, cout, spatial);
    return cudaGetLastError() == cudaSuccess ? B2G_OK : B2G_ERR_LAUNCH;
  }
  d.a = weight;
  d.b = in;
  d.c = out;
  d.workspace = workspace;
  d.workspace_bytes = workspace_bytes;
  if (!valid_desc(&d)) return B2G_ERR_INVALID_ARG;
  DeviceState* ds = nullptr;
  int rc = device_state(&ds);
  if (rc != B2G_OK) return rc;
  b2g_gemm_plan pl;
  rc = b2g_gemm_plan_for(&d, ds->num_sms, &pl);
  if (rc != B2G_OK) return rc;
  if (pl.workspace_bytes > 0 && (!workspace || workspace_bytes < pl.workspace_bytes))
    return B2G_ERR_WORKSPACE;
  return run_planned(&d, pl, workspace, ds->err_word, stream, bias);
}

extern "C" int b2g_rowscale(const float* d, const float* b, float* out, int64_t rows, int64_t cols,
                            int64_t ldb, int64_t ldo, b2g_stream_t stream_handle) {
  if (rows < 0 || cols < 0) return B2G_ERR_INVALID_ARG;
  if (rows == 0 || cols == 0) return B2G_OK;
  if (!d || !b || !out || ldb < cols || ldo < cols) return B2G_ERR_INVALID_ARG;
  if (rows > 65535 * 64) return B2G_ERR_UNSUPPORTED;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_handle);
  const bool vec = (reinterpret_cast<uintptr_t>(b) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(out) % 16 == 0) && cols % 4 == 0 &&
                   ldb % 4 == 0 && ldo % 4 == 0;
  // Rows go on grid.y (limit 65535); larger row counts are issued in slabs.
  for (int64_t r0 = 0; r0 < rows; r0 += 65535) {
    const int64_t nr = std::min<int64_t>(65535, rows - r0);
    if (vec) {
      const int64_t cols4 = cols / 4;
      dim3 grid(static_cast<unsigned>(cdiv(cols4, 256 * 4)), static_cast<unsigned>(nr));
      rowscale_vec_kernel<<<grid, 256, 0, stream>>>(
          d + r0, reinterpret_cast<const float4*>(b + r0 * ldb),
          reinterpret_cast<float4*>(out + r0 * ldo), cols4, ldb / 4, ldo / 4);
    } else {
      dim3 grid(static_cast<unsigned>(std::min<int64_t>(cdiv(cols, 256), 64)),
                static_cast<unsigned>(nr));
      rowscale_scalar_kernel<<<grid, 256, 0, stream>>>(d + r0, b + r0 * ldb, out + r0 * ldo, nr,
                                                       cols, ldb, ldo);
    }
    if (cudaGetLastError() != cudaSuccess) return B2G_ERR_LAUNCH;
  }
  return B2G_OK;
}

// ---------------------------------------------------------------- attention
namespace b2g {
namespace {
// fp16 (rows x inner) matrices, nbatch of them rows*inner apart, boxes of
// 64 (128 bytes, 128-byte swizzle) x box_rows.
bool make_map_f16(CUtensorMap* map, const void* base, int64_t inner, int64_t rows, int64_t nbatch,
                  uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(nbatch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(inner) * 2,
                           static_cast<cuuint64_t>(inner * rows) * 2};
  cuuint32_t box[3] = {64, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace
}  // namespace b2g

extern "C" int b2g_sdpa(const void* q, const void* k, const void* v, void* out, int64_t batch,
                        int64_t heads, int64_t seq, int64_t dim, float scale,
                        b2g_stream_t stream_handle) {
  if (batch < 0 || heads < 0 || seq < 0 || dim < 0) return B2G_ERR_INVALID_ARG;
  const int64_t bh = batch * heads;
  if (bh == 0 || seq == 0 || dim == 0) return B2G_OK;
  if (!q || !k || !v || !out) return B2G_ERR_INVALID_ARG;
  if (seq > sdpa::kKeysMax || dim % 64 != 0 || bh > (1ll << 30) || dim * seq > (1ll << 30))
    return B2G_ERR_UNSUPPORTED;
  for (const void* ptr : {q, k, v, static_cast<const void*>(out)})
    if (reinterpret_cast<uintptr_t>(ptr) % 16) return B2G_ERR_UNSUPPORTED;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_handle);
  DeviceState* ds = nullptr;
  int rc = device_state(&ds);
  if (rc != B2G_OK) return rc;
  CUtensorMap mq, mk, mv;
  if (!make_map_f16(&mq, q, dim, seq, bh, sdpa::kBM) ||
      !make_map_f16(&mk, k, dim, seq, bh, sdpa::kKBox / 2) ||
      !make_map_f16(&mv, v, dim, seq, bh, sdpa::kVKeys))
    return B2G_ERR_UNSUPPORTED;
  sdpa::Params p;
  p.S = static_cast<int>(seq);
  p.D = static_cast<int>(dim);
  p.BH = static_cast<int>(bh);
  p.qblocks = static_cast<int>(cdiv(seq, sdpa::kUnitM));
  p.units = bh * p.qblocks;
  const float sc = scale > 0.f ? scale : 1.0f / std::sqrt(static_cast<float>(dim));
  p.scale_log2 = sc * 1.4426950408889634f;
  p.out = static_cast<__half*>(out);
  p.wait_limit_ns = wait_limit_ns();
  p.err = ds->err_word;
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    if (cudaFuncSetAttribute(sdpa::sdpa_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             sdpa::kSmemBytes) != cudaSuccess)
      return B2G_ERR_LAUNCH;
    configured_dev = dev;
  }
  // CTA pairs (clusters of 2), persistent: one pair per two SMs at most.
  const int pairs = static_cast<int>(std::min<int64_t>(p.units, ds->num_sms / 2));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(sdpa::kThreads, 1, 1);
  cfg.dynamicSmemBytes = sdpa::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = B2G_PDL ? 2 : 1;
  if (cudaLaunchKernelEx(&cfg, sdpa::sdpa_kernel, mq, mk, mv, p) != cudaSuccess)
    return B2G_ERR_LAUNCH;
  return cudaGetLastError() == cudaSuccess ? B2G_OK : B2G_ERR_LAUNCH;
}

extern "C" int b2g_read_device_error(int device, int32_t* code) {
  if (!code || device < 0 || device >= kMaxDevices) return B2G_ERR_INVALID_ARG;
  int prev = 0;
  cudaGetDevice(&prev);
  if (cudaSetDevice(device) != cudaSuccess) return B2G_ERR_NO_DEVICE;
  DeviceState* ds = nullptr;
  int rc = device_state(&ds);
  if (rc == B2G_OK) {
    int v = 0;
    if (cudaDeviceSynchronize() != cudaSuccess ||
        cudaMemcpy(&v, ds->err_word, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemset(ds->err_word, 0, sizeof(int)) != cudaSuccess)
      rc = B2G_ERR_LAUNCH;
    *code = v;
  }
  cudaSetDevice(prev);
  return rc;
}

// ---------------------------------------------------------------- allocation-free entry point
// b2g_gemm_noalloc serves callers that may not allocate device memory: a
// plugin host that hands the library only its input and output buffers and
// exposes no allocator (for instance a serving runtime whose memory pool
// already owns the GPU's free memory, where a cudaMalloc would fail or
// fragment that pool), or a latency-bound loop that cannot afford
// cudaMalloc/cudaFree, which may synchronise the device.  Operands that need
// a 16-byte-aligned staged copy are staged in this fixed file-scope array
// instead of caller workspace.  Every GPU that loads this library holds the
// array until the process exits.  All calls on a device share it and it
// keeps the last call's contents; nothing in it has to start at zero (each
// staged copy overwrites the bytes the engine reads), but calls whose work
// overlaps on the GPU (different streams, no ordering between them) race on
// it.
static __device__ __align__(256) unsigned char g_noalloc_scratch[B2G_NOALLOC_SCRATCH_BYTES];
// Device error word of this path (bounded-wait timeouts); separate from the
// word b2g_read_device_error reports, which b2g_gemm allocates on first use.
// b2g_noalloc_read_error reads and clears it without allocating.
static __device__ int g_noalloc_err;

namespace {

struct NoAllocDevice {
  bool ready = false;
  int num_sms = 0;
  void* scratch = nullptr;      // device address of g_noalloc_scratch on this device
  int* err = nullptr;           // device address of g_noalloc_err on this device
};
std::mutex g_noalloc_mu;
NoAllocDevice g_noalloc[kMaxDevices];

// Once per device, with that device current: look up the device addresses
// of the file-scope arrays.  The host-side names are only stand-ins; a
// kernel must be given these addresses.  No allocation happens here.
int noalloc_device(NoAllocDevice** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return B2G_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoAllocDevice& st = g_noalloc[dev];
  if (!st.ready) {
    int major = 0, sms = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        major != 10)
      return B2G_ERR_NO_DEVICE;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return B2G_ERR_NO_DEVICE;
    sms = std::min(sms, max_sms_override());
    void* scratch = nullptr;
    void* err = nullptr;
    if (cudaGetSymbolAddress(&scratch, g_noalloc_scratch) != cudaSuccess) return B2G_ERR_LAUNCH;
    if (cudaGetSymbolAddress(&err, g_noalloc_err) != cudaSuccess) return B2G_ERR_LAUNCH;
    st.num_sms = sms;
    st.scratch = scratch;
    st.err = static_cast<int*>(err);
    st.ready = true;
  }
  *out = &st;
  return B2G_OK;
}

}  // namespace

extern "C" int b2g_gemm_noalloc(const b2g_gemm_desc* d, b2g_stream_t stream_handle) {
  if (!valid_desc(d)) return B2G_ERR_INVALID_ARG;
  if (d->m == 0 || d->n == 0) return B2G_OK;
  NoAllocDevice* st = nullptr;
  int rc = noalloc_device(&st);
  if (rc != B2G_OK) return rc;
  b2g_gemm_plan pl;
  rc = b2g_gemm_plan_for(d, st->num_sms, &pl);
  if (rc != B2G_OK) return rc;
  if (pl.workspace_bytes > B2G_NOALLOC_SCRATCH_BYTES) return B2G_ERR_SCRATCH_LIMIT;
  if (pl.workspace_bytes + tri_gate_table_bytes(d, pl) > B2G_NOALLOC_SCRATCH_BYTES)
    return B2G_ERR_SCRATCH_LIMIT;
  return run_planned(d, pl, st->scratch, st->err, static_cast<cudaStream_t>(stream_handle),
                     nullptr, true);
}

extern "C" int b2g_noalloc_read_error(int device, int32_t* code) {
  if (!code || device < 0 || device >= kMaxDevices) return B2G_ERR_INVALID_ARG;
  *code = 0;
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return B2G_ERR_NO_DEVICE;
  if (cudaSetDevice(device) != cudaSuccess) return B2G_ERR_NO_DEVICE;
  // Both copies go through the symbol (no allocation): wait for the device's
  // work, read the word, then clear it for the next call.
  int rc = B2G_OK;
  int v = 0;
  const int zero = 0;
  if (cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpyFromSymbol(&v, g_noalloc_err, sizeof(int)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_noalloc_err, &zero, sizeof(int)) != cudaSuccess)
    rc = B2G_ERR_LAUNCH;
  *code = v;
  cudaSetDevice(prev);
  return rc;
}
