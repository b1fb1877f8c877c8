/*
 * b2g_gemm.h — C ABI of the B200 (sm_100a) fp32-input GEMM operator family.
 *
 * Plain pointers and sizes only; no torch types cross this boundary.  The
 * Torch C++ binding (cupilot-kernels_b200/csrc/torch_binding.cpp) and any
 * other host (ctypes, cgo, JNI) bind these symbols.
 *
 * The reference (champloo2878/cuPilot-Kernels) exposes one Part-3 host
 * function per operator, each `torch::Tensor f(torch::Tensor A, torch::Tensor B)`
 * launching a hand-written kernel.  Every one of those GEMM-band functions is
 * replaced by b2g_gemm() with a descriptor that states the operator, the
 * operand majorness and the triangle; diag_mult_cuda is replaced by
 * b2g_rowscale():
 *
 *   kernels/1_Square_matrix_multiplication_best_kernel.cu:189   matmul_cuda              -> b2g_gemm (NN)
 *   kernels/2_Standard_matrix_multiplication_best_kernel.cu:117 matmul_cuda              -> b2g_gemm (NN)
 *   kernels/3_Batched_matrix_multiplication_best_kernel.cu:113  batched_matmul_cuda      -> b2g_gemm (NN, batch)
 *   kernels/6_Matmul_with_large_K_dimension_best_kernel.cu:128  matmul_cuda              -> b2g_gemm (NN, split-K)
 *   kernels/7_Matmul_with_small_K_dimension_best_kernel.cu:80   gemm_cuda                -> b2g_gemm (NN)
 *   kernels/8_Matmul_with_irregular_shapes_best_kernel.cu:155   matmul_cuda              -> b2g_gemm (NN, staged)
 *   kernels/9_Tall_skinny_matrix_multiplication_best_kernel.cu:145 tall_skinny_matmul_cuda -> b2g_gemm (NN)
 *   kernels/10_3D_tensor_matrix_multiplication_best_kernel.cu:180 batched_matmul_cuda    -> b2g_gemm (NN, flattened)
 *   kernels/11_4D_tensor_matrix_multiplication_best_kernel.cu:132 tensor_matmul_cuda     -> b2g_gemm (NN, flattened)
 *   kernels/12_Matmul_with_diagonal_matrices_best_kernel.cu:43  diag_mult_cuda           -> b2g_rowscale
 *   kernels/13_Matmul_for_symmetric_matrices_best_kernel.cu:134 symmetric_matmul_cuda    -> b2g_gemm (NT)
 *   kernels/14_Matmul_for_upper_triangular_matrices_best_kernel.cu:135 upper_tri_matmul_cuda -> b2g_gemm (TRI_UPPER)
 *   kernels/15_Matmul_for_lower_triangular_matrices_best_kernel.cu:155 lower_tri_mul_cuda -> b2g_gemm (TRI_LOWER)
 *   kernels/16_Matmul_with_transposed_A_best_kernel.cu:124      matmul_transposed_cuda   -> b2g_gemm (TN)
 *   kernels/17_Matmul_with_transposed_B_best_kernel.cu:267      matmul_cuda              -> b2g_gemm (NT)
 *   kernels/18_Matmul_with_transposed_both_best_kernel.cu:152   matmul_transposed_cuda   -> b2g_gemm (TT)
 *   kernels/4_Matrix_vector_multiplication_best_kernel.cu:84    gemv_cuda                -> b2g_gemv
 *   kernels/5_Matrix_scalar_multiplication_best_kernel.cu:47    matrix_scalar_mult_cuda  -> b2g_scale
 *   kernels/87_conv_pointwise_2D_best_kernel.cu:451             pointwise_conv_cuda      -> b2g_pointwise_conv
 *   kernels/97_ScaledDotProductAttention_best_kernel.cu:256     fused_attention_cuda     -> b2g_sdpa
 *   kernels/6_Matmul_with_large_K_dimension_best_kernel.cu:147-200 (streams + C.add_) -> b2g_splitk_peer_reduce,
 *                                                                  or with the product: b2g_gemm_splitk_peer
 *
 * Error behaviour: every entry point returns a b2g_status; 0 is success.
 * Nothing traps or asserts on the device.  Kernel-side waits are bounded;
 * a wait that gives up writes a code into the per-device error word, which
 * b2g_read_device_error() returns (and clears).
 */
#ifndef B2G_GEMM_H
#define B2G_GEMM_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define B2G_API __attribute__((visibility("default")))
#else
#define B2G_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Opaque stream handle: a cudaStream_t (CUstream) passed through as void*. */
typedef void* b2g_stream_t;

typedef enum b2g_status {
  B2G_OK = 0,
  B2G_ERR_INVALID_ARG = 1,      /* null pointer, negative size, bad enum   */
  B2G_ERR_UNSUPPORTED = 2,      /* layout/shape the engine cannot express  */
  B2G_ERR_WORKSPACE = 3,        /* workspace missing or too small          */
  B2G_ERR_LAUNCH = 4,           /* CUDA launch / API call failed           */
  B2G_ERR_DEVICE_TIMEOUT = 5,   /* a bounded device-side wait gave up      */
  B2G_ERR_NO_DEVICE = 6,        /* no sm_100 device current                */
  B2G_ERR_SCRATCH_LIMIT = 7     /* b2g_gemm_noalloc: staging exceeds its fixed scratch */
} b2g_status;

typedef enum b2g_op {
  B2G_OP_GEMM = 0,              /* C = op(A) . op(B)                       */
  B2G_OP_TRI_UPPER = 1,         /* C = triu(triu(A) . triu(B)), square     */
  B2G_OP_TRI_LOWER = 2          /* C = tril(tril(A) . tril(B)), square     */
} b2g_op;

typedef enum b2g_precision {
  B2G_PREC_TF32 = 0,            /* one TF32 product per term               */
  B2G_PREC_3XTF32 = 1           /* hi.hi + hi.lo + lo.hi split products    */
} b2g_precision;

/*
 * One (optionally batched) GEMM, all fp32, C row-major:
 *   C[b][m][n] = sum_k opA(A)[b][m][k] * opB(B)[b][k][n]
 * trans_a == 0: A[b][m][k] at a[b*stride_a + m*lda + k]   (A stored M x K)
 * trans_a == 1: A[b][m][k] at a[b*stride_a + k*lda + m]   (A stored K x M)
 * trans_b == 0: B[b][k][n] at b[b*stride_b + k*ldb + n]   (B stored K x N)
 * trans_b == 1: B[b][k][n] at b[b*stride_b + n*ldb + k]   (B stored N x K)
 * stride_a / stride_b may be 0 (operand shared across the batch).
 * All leading dimensions and strides are in elements.
 */
typedef struct b2g_gemm_desc {
  int32_t op;                   /* b2g_op                                  */
  int32_t precision;            /* b2g_precision                           */
  int64_t m, n, k, batch;
  const float* a; int64_t lda; int64_t stride_a; int32_t trans_a;
  const float* b; int64_t ldb; int64_t stride_b; int32_t trans_b;
  float* c;       int64_t ldc; int64_t stride_c;
  void* workspace;              /* device memory, >= b2g_gemm_workspace_bytes() */
  int64_t workspace_bytes;
} b2g_gemm_desc;

/* What the host dispatcher chose for a descriptor (pure host computation). */
typedef struct b2g_gemm_plan {
  int32_t block_m, block_n, block_k;   /* block_m: output rows per work unit */
  int32_t stages;
  int32_t tiles_m, tiles_n;
  int32_t splits;               /* split-K factor; >1 accumulates into a zeroed C */
  int32_t kb_per_split;         /* K blocks of block_k per split           */
  int32_t grid;                 /* persistent CTAs launched                */
  int32_t stage_a, stage_b;     /* 1: operand copied to a 16-byte-aligned pitch in workspace */
  int32_t a_mn_major, b_mn_major;
  int32_t cluster_ctas;         /* 2: a CTA pair computes each 256-row unit (tcgen05 cta_group::2) */
  int32_t tma_store;            /* 1: C written by TMA tensor stores (C rows 16-byte aligned) */
  int32_t tri_diag;             /* 1: triangular inputs masked through diagonal-block copies in workspace */
  int32_t x3_split;             /* 1: 3xTF32 lo parts pre-split into workspace (plain GEMMs) */
  int64_t work_units;
  int64_t workspace_bytes;
} b2g_gemm_plan;

/* Compute the plan for desc on a GPU with num_sms SMs (no device access). */
B2G_API int b2g_gemm_plan_for(const b2g_gemm_desc* desc, int num_sms, b2g_gemm_plan* plan);

/* Workspace the caller must provide for desc (0 for aligned TF32 GEMMs),
 * planned for the current device's SM count (148 when no device is usable). */
B2G_API int64_t b2g_gemm_workspace_bytes(const b2g_gemm_desc* desc);

/* Launch the GEMM on stream (asynchronous; no host synchronisation). */
B2G_API int b2g_gemm(const b2g_gemm_desc* desc, b2g_stream_t stream);

/*
 * out[i][j] = d[i] * B[i][j]   — diag(d) . B, one rounding per element.
 * Replaces diag_mult_cuda (kernels/12_Matmul_with_diagonal_matrices_best_kernel.cu:43).
 */
B2G_API int b2g_rowscale(const float* d, const float* b, float* out, int64_t rows,
                 int64_t cols, int64_t ldb, int64_t ldo, b2g_stream_t stream);

/*
 * b2g_gemm_noalloc — b2g_gemm for callers that cannot allocate device memory.
 * This entry point has no counterpart in the reference.
 *
 * Who needs it: a plugin host that gives the library only its input and
 * output buffers and no allocator (e.g. a serving runtime whose memory pool
 * already owns the GPU's free memory, so a cudaMalloc would fail or fragment
 * it), or a latency-bound loop that cannot pay for cudaMalloc/cudaFree, which
 * may synchronise the device.  It makes no cudaMalloc, cudaFree or other
 * allocating call.
 *
 * Same descriptor and result as b2g_gemm; desc->workspace is ignored.
 * Everything b2g_gemm would place in caller workspace goes into one fixed
 * file-scope device array of B2G_NOALLOC_SCRATCH_BYTES (16 MiB), which every
 * GPU that loads the library holds until the process exits:
 *   - staged copies of operands whose pitch or base is not 16-byte aligned;
 *   - every 3xTF32 call on a plain GEMM, aligned or not: the lo parts of A
 *     and B (m*k + k*n floats per batch entry, rounded up to 16-byte rows),
 *     so 3xTF32 fits only while A and B together hold at most ~4 M elements;
 *   - every triangular call in TF32 on untransposed operands, aligned or
 *     not: masked copies of the diagonal blocks (2 * n * 128 floats) and the
 *     unit table (16 bytes per unit), so n is limited to about 16000; on
 *     transposed operands the unit table only (b2g_gemm keeps that one in a
 *     device cache of its own instead of the caller's workspace).
 * A descriptor needing more than that returns B2G_ERR_SCRATCH_LIMIT before
 * any work is issued; b2g_gemm_workspace_bytes() tells how much it needs.
 *
 * The first call on a device, with that device current, looks up the
 * array's device address (cudaGetSymbolAddress); make that first call before
 * any stream capture begins.  All calls on a device share the one array and
 * it keeps the last call's contents: calls whose work may overlap on the GPU
 * (unordered streams) race on it.  Bounded-wait timeouts in this path are
 * recorded in a device word of its own: read and clear it with
 * b2g_noalloc_read_error(), which allocates nothing either
 * (b2g_read_device_error does not see it).
 */
#define B2G_NOALLOC_SCRATCH_BYTES (16ll << 20)
B2G_API int b2g_gemm_noalloc(const b2g_gemm_desc* desc, b2g_stream_t stream);

/*
 * Read and clear the device error word of b2g_gemm_noalloc on `device`
 * (synchronises the device; no allocation).  0: no bounded wait gave up
 * since the last read; otherwise the code of the first wait that did (its
 * call's output is incomplete).  No counterpart in the reference.
 */
B2G_API int b2g_noalloc_read_error(int device, int32_t* code);

/*
 * y[i] = sum_k A[i][k] x[k]  (fp32 CUDA-core dot products, 16-byte streaming loads).
 * Replaces gemv_cuda (kernels/4_Matrix_vector_multiplication_best_kernel.cu:84).
 */
B2G_API int b2g_gemv(const float* a, int64_t lda, const float* x, float* y, int64_t m,
                     int64_t k, b2g_stream_t stream);

/*
 * out[i] = a[i] * s for n contiguous elements, one rounding per element.
 * Replaces matrix_scalar_mult_cuda (kernels/5_Matrix_scalar_multiplication_best_kernel.cu:47).
 */
B2G_API int b2g_scale(const float* a, float s, float* out, int64_t n, b2g_stream_t stream);

/*
 * Pointwise (1x1, stride 1, no padding) convolution over NCHW fp32 tensors:
 *   out[n][o][s] = sum_c weight[o][c] * in[n][c][s] + (bias ? bias[o] : 0)
 * with s = h * W + w running over the `spatial` = H * W positions.  Each
 * image is one GEMM of the shared weight (out_channels x in_channels) by the
 * image (in_channels x spatial); the batch runs as one batched launch and
 * the bias is added in the epilogue.  `precision` as in b2g_gemm_desc.
 * Inputs are dense (in: batch x in_channels x spatial, weight: out_channels
 * x in_channels, out: batch x out_channels x spatial).  in_channels == 0
 * writes the bias (or zeros).  The workspace size depends on the pointers'
 * alignment (unaligned operands are staged), so it takes the same pointers.
 * Replaces pointwise_conv_cuda (kernels/87_conv_pointwise_2D_best_kernel.cu:451).
 */
B2G_API int64_t b2g_pointwise_conv_workspace_bytes(const float* in, const float* weight,
                                                   const float* out, int64_t batch,
                                                   int64_t in_channels, int64_t out_channels,
                                                   int64_t spatial, int precision);
B2G_API int b2g_pointwise_conv(const float* in, const float* weight, const float* bias,
                               float* out, int64_t batch, int64_t in_channels,
                               int64_t out_channels, int64_t spatial, int precision,
                               void* workspace, int64_t workspace_bytes, b2g_stream_t stream);

/*
 * Scaled-dot-product attention, fp16 in and out, fp32 accumulation and softmax:
 *   out[b][h] = softmax(q[b][h] . k[b][h]^T * scale) . v[b][h]
 * q, k, v, out: dense (batch, heads, seq, dim) fp16 (IEEE binary16) arrays,
 * 16-byte aligned; seq <= 512, dim a multiple of 64.  scale <= 0 selects
 * 1/sqrt(dim).  One tcgen05 kernel: S = q k^T in tensor memory, the full-row
 * softmax on chip, P (fp16) . v, output scaled by 1/rowsum.
 * Replaces fused_attention_cuda (kernels/97_ScaledDotProductAttention_best_kernel.cu:256),
 * which requires seq == 512 in practice and dim == 1024 (:9-10, :267-268).
 */
B2G_API int b2g_sdpa(const void* q, const void* k, const void* v, void* out, int64_t batch,
                     int64_t heads, int64_t seq, int64_t dim, float scale, b2g_stream_t stream);

/*
 * Cross-GPU sum of a K split (one process per GPU on one node).
 *
 * Replaces the partial-sum step of the reference's large-K product, which
 * splits K over 8 streams of one GPU and adds the partials with 7 C.add_
 * calls (kernels/6_Matmul_with_large_K_dimension_best_kernel.cu:147-200).
 * Here each rank multiplies its K slice with b2g_gemm and then calls
 * b2g_splitk_peer_reduce on the same stream: a non-root rank copies its
 * partial into a landing slot of the root's mailbox through the peer
 * mapping (plain stores over NVLink, each value carrying the epoch); the
 * root waits (bounded) until every value of every rank has landed, sums
 * them in rank order and adds the sum to `out`, which already holds its
 * own partial.
 * C = sum of the partials lands on the root only.  One stream per mailbox
 * set: the root frees the previous epoch's landing slots when its next
 * epoch's kernel starts.
 *
 * Mailboxes: each rank creates one (b2g_peer_mailbox_create, device memory
 * of b2g_peer_mailbox_bytes(elems, world)), shares its IPC handle with the
 * others (any host channel), and opens theirs (b2g_peer_mailbox_open);
 * `mailboxes[r]` is rank r's mailbox as mapped in the calling process (its
 * own pointer for r == rank).  All ranks call with the same epoch, 1, 2, 3,
 * ... per mailbox set; a rank may run at most one epoch ahead of the root
 * (it waits, bounded, for the root to free the landing slot).  A wait that
 * gives up records 0x201 (slot credit) or 0x202 (values not landed) in the
 * device error word (b2g_read_device_error) and the call's output is
 * incomplete.  partial / out: elems fp32, 16-byte aligned.
 */
#define B2G_PEER_MAX_RANKS 16
typedef struct b2g_ipc_handle { unsigned char bytes[64]; } b2g_ipc_handle;
B2G_API int64_t b2g_peer_mailbox_bytes(int64_t elems, int world);
B2G_API int b2g_peer_mailbox_create(int64_t elems, int world, void** mailbox,
                                    b2g_ipc_handle* handle);
B2G_API int b2g_peer_mailbox_open(const b2g_ipc_handle* handle, void** mailbox);
B2G_API int b2g_peer_mailbox_close(void* mailbox);     /* a mailbox opened from a handle */
B2G_API int b2g_peer_mailbox_destroy(void* mailbox);   /* a mailbox this process created */
B2G_API int b2g_splitk_peer_reduce(const float* partial, float* out, int64_t elems,
                                   void* const* mailboxes, int world, int rank, int root,
                                   int64_t epoch, b2g_stream_t stream);

/*
 * The K-split product and its cross-GPU sum in ONE kernel: this rank's
 * slice C_r = A[:, K_r] B[K_r, :] (d: a plain GEMM, batch 1, C contiguous
 * M x N with ldc == n, 16-byte aligned) is computed into d->c, and once every
 * CTA's stores are complete the same kernel's epilogue warps move it over
 * NVLink: a non-root rank copies it chunk by chunk into its landing slot in
 * the root's mailbox; the root adds the landed chunks (summed in rank order) to its
 * own C.  The mailboxes, epochs and flags are those of
 * b2g_splitk_peer_reduce (mailboxes of b2g_peer_mailbox_bytes(m * n, world)),
 * and the sum is bit-identical to b2g_gemm followed by
 * b2g_splitk_peer_reduce; the two paths may alternate epoch by epoch.
 * Replaces the same reference step as b2g_splitk_peer_reduce
 * (kernels/6_Matmul_with_large_K_dimension_best_kernel.cu:147-200) together
 * with the product before it (:128).  A bounded wait that gives up records
 * 0x201 / 0x202, or 0x203 for the grid-wide arrival, in the device error
 * word.  world == 1 is b2g_gemm.
 */
B2G_API int b2g_gemm_splitk_peer(const b2g_gemm_desc* d, void* const* mailboxes, int world,
                                 int rank, int root, int64_t epoch, b2g_stream_t stream);

/* Read and clear the device-side error word of `device` (synchronises it). */
B2G_API int b2g_read_device_error(int device, int32_t* code);

/* Human-readable text for a b2g_status. */
B2G_API const char* b2g_status_string(int status);

/* Library version: major*10000 + minor*100 + patch. */
B2G_API int b2g_version(void);

#ifdef __cplusplus
}
#endif

#endif /* B2G_GEMM_H */
