// b2g_vector.cu — the HBM-bound members of the GEMM band: matrix-vector
// product and matrix-scalar scale.  Both stream each input byte once with
// 16-byte loads and do all arithmetic in fp32 on the CUDA cores (tensor
// cores would buy nothing at one flop per loaded word).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "../../include/b2g_gemm.h"

namespace {

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// y[r] = sum_k A[r][k] x[k]: one warp per row, four independent float4
// accumulation streams per lane, then a warp reduction.
template <bool VEC>
__global__ void __launch_bounds__(256) gemv_warp_rows_kernel(const float* __restrict__ A,
                                                             int64_t lda,
                                                             const float* __restrict__ x,
                                                             float* __restrict__ y, int64_t m,
                                                             int64_t k) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= m) return;
  const float* a = A + row * lda;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  if (VEC) {
    const float4* a4 = reinterpret_cast<const float4*>(a);
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const int64_t k4 = k / 4;
    int64_t i = lane;
    for (; i + 96 < k4; i += 128) {
      float4 av[4], xv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        av[u] = __ldcs(a4 + i + 32 * u);
        xv[u] = __ldg(x4 + i + 32 * u);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        acc[u] += av[u].x * xv[u].x + av[u].y * xv[u].y + av[u].z * xv[u].z + av[u].w * xv[u].w;
    }
    for (; i < k4; i += 32) {
      const float4 av = __ldcs(a4 + i);
      const float4 xv = __ldg(x4 + i);
      acc[0] += av.x * xv.x + av.y * xv.y + av.z * xv.z + av.w * xv.w;
    }
    for (int64_t j = k4 * 4 + lane; j < k; j += 32) acc[1] += a[j] * __ldg(x + j);
  } else {
    for (int64_t j = lane; j < k; j += 32) acc[j & 3] += a[j] * __ldg(x + j);
  }
  const float s = warp_sum((acc[0] + acc[1]) + (acc[2] + acc[3]));
  if (lane == 0) y[row] = s;
}

// Few rows, long K: a 256-thread block per row, reduced through shared memory.
template <bool VEC>
__global__ void __launch_bounds__(256) gemv_block_rows_kernel(const float* __restrict__ A,
                                                              int64_t lda,
                                                              const float* __restrict__ x,
                                                              float* __restrict__ y, int64_t k) {
  __shared__ float partial[8];
  const int64_t row = blockIdx.x;
  const float* a = A + row * lda;
  float acc = 0.f;
  if (VEC) {
    const float4* a4 = reinterpret_cast<const float4*>(a);
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const int64_t k4 = k / 4;
    for (int64_t i = threadIdx.x; i < k4; i += blockDim.x) {
      const float4 av = __ldcs(a4 + i);
      const float4 xv = __ldg(x4 + i);
      acc += av.x * xv.x + av.y * xv.y + av.z * xv.z + av.w * xv.w;
    }
    for (int64_t j = k4 * 4 + threadIdx.x; j < k; j += blockDim.x) acc += a[j] * __ldg(x + j);
  } else {
    for (int64_t j = threadIdx.x; j < k; j += blockDim.x) acc += a[j] * __ldg(x + j);
  }
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? partial[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) y[row] = v;
  }
}

// out[i] = a[i] * s, one rounding per element.
// out = a * s over float4s: each thread issues kScaleUnroll independent
// 16-byte streaming loads (a block's loads cover 4 KB per step) before its
// stores, so enough bytes are in flight per SM to cover HBM latency.
constexpr int kScaleUnroll = 4;
__global__ void __launch_bounds__(256) scale_vec_kernel(const float4* __restrict__ a, float s,
                                                        float4* __restrict__ out, int64_t n4) {
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x * kScaleUnroll;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x * kScaleUnroll + threadIdx.x;
       base < n4; base += step) {
    float4 v[kScaleUnroll];
#pragma unroll
    for (int u = 0; u < kScaleUnroll; ++u) {
      const int64_t i = base + static_cast<int64_t>(u) * blockDim.x;
      if (i < n4) v[u] = __ldcs(a + i);
    }
#pragma unroll
    for (int u = 0; u < kScaleUnroll; ++u) {
      const int64_t i = base + static_cast<int64_t>(u) * blockDim.x;
      if (i < n4) __stcs(out + i, make_float4(v[u].x * s, v[u].y * s, v[u].z * s, v[u].w * s));
    }
  }
}

__global__ void scale_tail_kernel(const float* __restrict__ a, float s, float* __restrict__ out,
                                  int64_t begin, int64_t n) {
  const int64_t i = begin + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) out[i] = a[i] * s;
}

int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

}  // namespace

extern "C" int b2g_gemv(const float* a, int64_t lda, const float* x, float* y, int64_t m,
                        int64_t k, b2g_stream_t stream_handle) {
  if (m < 0 || k < 0) return B2G_ERR_INVALID_ARG;
  if (m == 0) return B2G_OK;
  if (!y || (k > 0 && (!a || !x || lda < k))) return B2G_ERR_INVALID_ARG;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_handle);
  if (k == 0) return cudaMemsetAsync(y, 0, m * sizeof(float), stream) == cudaSuccess
                         ? B2G_OK
                         : B2G_ERR_LAUNCH;
  const bool vec = (reinterpret_cast<uintptr_t>(a) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(x) % 16 == 0) && lda % 4 == 0;
  // Enough rows to give every SM 16 warps: a warp per row; else a block per row.
  if (m >= static_cast<int64_t>(sm_count()) * 16 || k < 1024) {
    const unsigned grid = static_cast<unsigned>(cdiv(m, 8));
    if (vec)
      gemv_warp_rows_kernel<true><<<grid, 256, 0, stream>>>(a, lda, x, y, m, k);
    else
      gemv_warp_rows_kernel<false><<<grid, 256, 0, stream>>>(a, lda, x, y, m, k);
  } else {
    if (m > 0x7fffffff) return B2G_ERR_UNSUPPORTED;
    if (vec)
      gemv_block_rows_kernel<true><<<static_cast<unsigned>(m), 256, 0, stream>>>(a, lda, x, y, k);
    else
      gemv_block_rows_kernel<false><<<static_cast<unsigned>(m), 256, 0, stream>>>(a, lda, x, y, k);
  }
  return cudaGetLastError() == cudaSuccess ? B2G_OK : B2G_ERR_LAUNCH;
}

extern "C" int b2g_scale(const float* a, float s, float* out, int64_t n,
                         b2g_stream_t stream_handle) {
  if (n < 0) return B2G_ERR_INVALID_ARG;
  if (n == 0) return B2G_OK;
  if (!a || !out) return B2G_ERR_INVALID_ARG;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_handle);
  const bool vec = (reinterpret_cast<uintptr_t>(a) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(out) % 16 == 0);
  const int64_t n4 = vec ? n / 4 : 0;
  if (n4 > 0) {
    const int64_t blocks = std::min<int64_t>(cdiv(n4, 256 * kScaleUnroll), int64_t{1} << 30);
    scale_vec_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
        reinterpret_cast<const float4*>(a), s, reinterpret_cast<float4*>(out), n4);
  }
  const int64_t tail = n - n4 * 4;
  if (tail > 0) {
    const int64_t blocks = cdiv(tail, 256);
    if (blocks > 0x7fffffff) return B2G_ERR_UNSUPPORTED;
    scale_tail_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(a, s, out, n4 * 4, n);
  }
  return cudaGetLastError() == cudaSuccess ? B2G_OK : B2G_ERR_LAUNCH;
}
